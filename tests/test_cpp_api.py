"""The C++ host classes (include/orator_b200/asr_text_decoder.h), the
reference-compatible orator::model::AsrTextDecoder and the multi-session
AsrSessionPool, compiled with g++ against the built library.

CPU: the header compiles as C++17 with -Wall -Werror, the defaults match the
reference's AsrTextConfig, and argument errors surface as std::runtime_error.
GPU: a C++ program prefills seeded rows, greedy-decodes through
AsrTextDecoder::DecodeGreedy and through AsrSessionPool::StepAll, and both
token lists equal the Python path's on the same library and inputs."""
import os
import shutil
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_DIR = os.path.join(ROOT, "orator_b200")
CUDA_INC = "/usr/local/cuda/include"

CPU_PROGRAM = r"""
#include <cstdio>
#include <stdexcept>
#include "orator_b200/asr_text_decoder.h"
using orator::model::AsrTextConfig;
using orator::model::AsrTextDecoder;
using orator::model::GpuError;
int main() {
  int fails = 0;
  AsrTextConfig c;
  if (c.hidden_size != 2048 || c.num_layers != 28 || c.vocab_size != 151936 ||
      c.max_seq_len != 2048 || c.rms_norm_eps != 1e-6f || c.rope_theta != 1e6f) ++fails;
  c.num_q_heads = 8;  // not the Qwen3-ASR geometry
  try {
    AsrTextDecoder d(c);
    ++fails;
  } catch (const GpuError&) {
    ++fails;  // must be an argument error, not a device error
  } catch (const std::runtime_error& e) {
    if (std::string(e.what()).empty()) ++fails;
  }
  std::printf("%s\n", fails ? "FAIL" : "OK");
  return fails;
}
"""

GPU_PROGRAM = r"""
#include <cstdio>
#include <vector>
#include "orator_b200/asr_text_decoder.h"
using namespace orator::model;
int main(int argc, char** argv) {
  if (argc < 2) return 2;
  const int T = 24, N = 8;
  std::vector<float> x(T * 2048);
  FILE* f = std::fopen(argv[1], "rb");
  if (!f || std::fread(x.data(), 4, x.size(), f) != x.size()) return 2;
  std::fclose(f);
  AsrTextConfig c;
  c.num_layers = 2;
  c.max_seq_len = 256;
  AsrTextDecoder d(c);
  d.InitSynthetic(9);
  d.Prefill(x.data(), T);
  std::vector<int> g = d.DecodeGreedy(T, N, -1, -1, 0, 4);
  AsrSessionPool pool(d, 2, 2, 32, 16);
  int s = pool.CreateSession();
  pool.PrefillAt(s, x.data(), T);
  std::vector<int> b = pool.PendingTokens({s});
  for (int i = 1; i < N; ++i) b.push_back(pool.StepAll({s})[0]);
  for (int t : g) std::printf("%d ", t);
  std::printf("\n");
  for (int t : b) std::printf("%d ", t);
  std::printf("\n%d %d\n", d.cache_len(), pool.cache_len(s));
  return 0;
}
"""


def _compile(tmp_path, src_text, name):
    src = tmp_path / f"{name}.cc"
    src.write_text(src_text)
    exe = tmp_path / name
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-I",
                    os.path.join(ROOT, "include"), "-I", CUDA_INC, str(src), "-o", str(exe),
                    "-L", LIB_DIR, "-l:liborator_b200.so", f"-Wl,-rpath,{LIB_DIR}"], check=True)
    return exe


def _need_build():
    if shutil.which("g++") is None or not os.path.isdir(CUDA_INC):
        pytest.skip("g++ or CUDA headers not available")
    if not os.path.exists(os.path.join(LIB_DIR, "liborator_b200.so")):
        pytest.skip("library not built")


def test_cpp_header_and_errors(tmp_path):
    _need_build()
    exe = _compile(tmp_path, CPU_PROGRAM, "cpu_api")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == "OK", r.stdout + r.stderr


@pytest.mark.gpu
def test_cpp_decoder_and_pool_match_python(tmp_path, cuda):
    _need_build()
    from oracle import synth
    from orator_b200 import AsrTextConfig, AsrTextDecoder, BatchDecoder
    x = synth.audio_rows(9, 24, 2048).astype(np.float32)
    rows = tmp_path / "rows.f32"
    x.tofile(rows)
    exe = _compile(tmp_path, GPU_PROGRAM, "gpu_api")
    r = subprocess.run([str(exe), str(rows)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = r.stdout.strip().splitlines()
    cpp_greedy = [int(t) for t in lines[0].split()]
    cpp_pool = [int(t) for t in lines[1].split()]
    assert lines[2].split() == ["32", str(24 + 7)]
    d = AsrTextDecoder(AsrTextConfig(num_layers=2, max_seq_len=256))
    d.init_synthetic(9)
    d.Prefill(x)
    assert cpp_greedy == list(d.DecodeGreedy(24, 8, -1, -1, ban_steps=0, batch=4))
    bd = BatchDecoder(d, max_sessions=2, max_batch=2, pool_pages=32, max_pages_per_session=16)
    s = bd.create_session()
    bd.prefill([s], [x])
    py_pool = [int(bd.next_tokens([s])[0])] + [int(bd.step([s])[0]) for _ in range(7)]
    assert cpp_pool == py_pool
    bd.close()
    d.close()


STREAM_PROGRAM = r"""
#include <cstdio>
#include <vector>
#include "orator_b200/asr_stream.h"
using namespace orator::model;
int main(int argc, char** argv) {
  if (argc < 2) return 2;
  const int T = 20;
  std::vector<float> x(2 * T * 2048);
  FILE* f = std::fopen(argv[1], "rb");
  if (!f || std::fread(x.data(), 4, x.size(), f) != x.size()) return 2;
  std::fclose(f);
  AsrTextConfig c;
  c.num_layers = 2;
  c.max_seq_len = 256;
  AsrTextDecoder d(c);
  d.InitSynthetic(9);
  AsrSessionPool pool(d, 4, 4, 64, 16);
  AsrStreamPool s(d, pool, 10, 3);
  const int a = s.Open({1000, 1001});
  const int b = s.Open({1002});
  s.AppendAudio({a, b}, {x.data(), x.data() + T * 2048}, {T, T});
  AsrStreamPool::Request r;
  r.language = {3000};
  r.committed = {4000, 4001};
  std::map<int, AsrStreamPool::Request> req;
  req[a] = r;
  req[b] = r;
  auto out = s.Decode(req);
  for (int sid : {a, b}) {
    for (int t : out[sid]) std::printf("%d ", t);
    std::printf("\n");
  }
  std::printf("%d %d %d %d\n", s.checkpoint(a), pool.cache_len(a), s.checkpoint(b), pool.cache_len(b));
  return 0;
}
"""


@pytest.mark.gpu
def test_cpp_stream_pool_matches_python(tmp_path, cuda):
    _need_build()
    from oracle import synth
    from orator_b200 import AsrTextConfig, AsrTextDecoder, BatchDecoder
    from orator_b200 import stream as S
    x = synth.audio_rows(9, 40, 2048).astype(np.float32)
    rows = tmp_path / "rows.f32"
    x.tofile(rows)
    exe = _compile(tmp_path, STREAM_PROGRAM, "stream_api")
    r = subprocess.run([str(exe), str(rows)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = r.stdout.split("\n")
    cpp = [[int(t) for t in lines[0].split()], [int(t) for t in lines[1].split()]]
    ck = [int(v) for v in lines[2].split()]
    assert ck[0] == ck[1] and ck[2] == ck[3]
    d = AsrTextDecoder(AsrTextConfig(num_layers=2, max_seq_len=256))
    d.init_synthetic(9)
    bd = BatchDecoder(d, max_sessions=4, max_batch=4, pool_pages=64, max_pages_per_session=16)
    pool = S.AsrStreamPool(d, bd, max_new=10, ban_steps=3)
    a, b = pool.open([1000, 1001]), pool.open([1002])
    pool.append_audio([a, b], [x[:20], x[20:]])
    out = pool.decode({a: ([3000], [4000, 4001]), b: ([3000], [4000, 4001])})
    assert [out[a], out[b]] == cpp
    assert [pool.ckpt[a], pool.ckpt[b]] == [ck[0], ck[2]]
    bd.close()
    d.close()


OPS_PROGRAM = r"""
#include <cstdio>
#include <stdexcept>
#include "orator_b200/asr_text_decoder.h"
#include "orator_b200/asr_ops.h"
namespace ops = orator::model::asr_ops;
namespace gm = orator::model::asr_gemm;
int main() {
  int fails = 0;
  // empty sizes are no-ops, as in the reference
  ops::RmsNorm(nullptr, nullptr, nullptr, 0, 2048, 1e-6f);
  gm::Linear(nullptr, nullptr, nullptr, nullptr, 0, 8, 8, 0);
  // argument errors surface as std::runtime_error (not GpuError)
  try {
    ops::GqaAttention(reinterpret_cast<const float*>(16), reinterpret_cast<const float*>(16),
                      reinterpret_cast<const float*>(16), reinterpret_cast<float*>(16),
                      2, 3, 2, 8, 1.0f, true);
    ++fails;
  } catch (const orator::model::GpuError&) {
    ++fails;
  } catch (const std::runtime_error&) {
  }
  std::printf("%s\n", fails ? "FAIL" : "OK");
  return fails;
}
"""


def test_cpp_ops_header(tmp_path):
    """The asr_ops / asr_gemm shim compiles beside the decoder header with
    -Wall -Wextra -Werror, and argument errors throw std::runtime_error."""
    _need_build()
    exe = _compile(tmp_path, OPS_PROGRAM, "ops_api")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == "OK", r.stdout + r.stderr
