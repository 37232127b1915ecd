"""The public header is plain C: a C99 program that includes include/orx.h
compiles with gcc -Wall -Werror, links against the built library and
exercises the calls that validate their arguments before touching a GPU
(defaults, bad geometry, unsupported GEMM shapes, empty inputs, last-error
text). No GPU is needed."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_DIR = os.path.join(ROOT, "orator_b200")

PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "orx.h"

static int fails = 0;
#define CHECK(c) do { if (!(c)) { printf("FAILED %s:%d %s\n", __FILE__, __LINE__, #c); ++fails; } } while (0)

int main(void) {
  orx_config c;
  orx_decoder* d = NULL;
  orx_batch* b = NULL;
  orx_layer32* l = NULL;
  CHECK(orx_version() >= 1);
  orx_config_default(&c);
  CHECK(c.hidden_size == 2048 && c.num_layers == 28 && c.num_q_heads == 16);
  CHECK(c.num_kv_heads == 8 && c.head_dim == 128 && c.intermediate_size == 6144);
  CHECK(c.vocab_size == 151936 && c.max_seq_len == 2048);
  /* geometry other than Qwen3-ASR-1.7B is rejected before any device work */
  c.hidden_size = 1024;
  CHECK(orx_decoder_create(&c, &d) == ORX_EINVAL && d == NULL);
  CHECK(strlen(orx_last_error()) > 0);
  CHECK(orx_layer32_create(&c, &l) == ORX_EINVAL && l == NULL);
  CHECK(orx_decoder_create(NULL, &d) == ORX_EINVAL);
  CHECK(orx_batch_create(NULL, 1, 1, 1, 1, &b) == ORX_EINVAL && b == NULL);
  /* free operators: empty input is a no-op; bad arguments are rejected
     before any device work */
  CHECK(orx_linear_pre(NULL, NULL, NULL, NULL, 0, 64, 128, 0, NULL) == ORX_OK);
  CHECK(orx_linear_pre((const uint16_t*)16, (const uint16_t*)16, NULL, (float*)16, 4, 64, 128,
                       3, NULL) == ORX_EINVAL);
  CHECK(orx_linear(NULL, (const uint16_t*)16, NULL, (float*)16, 4, 64, 128, 0, NULL) == ORX_EINVAL);
  CHECK(orx_rms_norm(NULL, NULL, NULL, 0, 2048, 1e-6f, NULL) == ORX_OK);
  CHECK(orx_gqa_attention((const float*)16, (const float*)16, (const float*)16, (float*)16, 2, 3,
                          2, 8, 1.0f, 1, NULL) == ORX_EINVAL);
  CHECK(orx_rope_half((float*)16, (const int*)16, 1, 1, 7, 1e6f, NULL) == ORX_EINVAL);
  CHECK(orx_argmax_banned(NULL, 10, -1, -1, (int*)16, NULL) == ORX_EINVAL);
  /* null handles */
  CHECK(orx_decoder_reset_cache(NULL) == ORX_EINVAL);
  CHECK(orx_batch_step(NULL, NULL, 0, NULL, NULL) == ORX_EINVAL);
  orx_decoder_destroy(NULL);
  orx_batch_destroy(NULL);
  orx_layer32_destroy(NULL);
  printf("%s\n", fails ? "FAIL" : "OK");
  return fails != 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_header_is_c_and_links(tmp_path):
    lib = os.path.join(LIB_DIR, "liborator_b200.so")
    if not os.path.exists(lib):
        pytest.skip("library not built")
    src = tmp_path / "abi.c"
    src.write_text(PROGRAM)
    exe = tmp_path / "abi"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-I",
                    os.path.join(ROOT, "include"), str(src), "-o", str(exe), "-L", LIB_DIR,
                    "-l:liborator_b200.so", f"-Wl,-rpath,{LIB_DIR}"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip().endswith("OK"), r.stdout + r.stderr
