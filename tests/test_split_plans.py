"""Host rules of the tcgen05 GEMM planning (orator_b200/csrc/decoder.cu
proj_splits, gemm_tc.cu tc_token_tile / linear_plan), compiled with g++
against the built library: split counts divide the k-blocks, token tiles are
widths the kernel is instantiated for, and the measured choices hold (400-row
prefill projections on 144-column tiles without split K, 3200-row ones on
256-column tiles, 64-row decode steps split the short projections)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "orator_b200", "liborator_b200.so")

PROGRAM = r"""
#include <cstdio>
#include <initializer_list>
namespace orx {
int proj_splits(int N, int K, int T, int num_sms);
int tc_token_tile(int N, int T, int splits, int sms);
int linear_plan(int N, int K, int T, int sms, int* bn);
}
#define EXPECT(c) do { if (!(c)) { std::printf("FAIL line %d: %s\n", __LINE__, #c); return 1; } } while (0)
int main() {
  const int shapes[][2] = {{4096, 2048}, {2048, 2048}, {12288, 2048}, {2048, 6144}, {151936, 2048}};
  for (auto& sh : shapes)
    for (int T : {1, 7, 16, 33, 64, 100, 128, 129, 400, 800, 3200}) {
      const int sp = orx::proj_splits(sh[0], sh[1], T, 148);
      EXPECT(sp == 1 || sp == 2 || sp == 4 || sp == 8 || sp == 16);
      EXPECT(sh[1] % (64 * sp) == 0);
      const int bn = orx::tc_token_tile(sh[0], T, sp, 148);
      EXPECT(bn == 16 || bn == 32 || bn == 64 || bn == 128 || bn == 144 || bn == 256);
      EXPECT(T > 128 || bn >= (T < 16 ? 16 : T));
    }
  for (auto& sh : shapes) {
    EXPECT(orx::proj_splits(sh[0], sh[1], 400, 148) <= 4);
    EXPECT(orx::tc_token_tile(sh[0], 3200, 1, 148) == 256);
  }
  EXPECT(orx::proj_splits(4096, 2048, 400, 148) == 1);
  EXPECT(orx::tc_token_tile(4096, 400, 1, 148) == 144);
  EXPECT(orx::proj_splits(2048, 2048, 64, 148) > 1);
  EXPECT(orx::proj_splits(2048, 6144, 64, 148) > 1);
  for (int N : {4, 192, 512, 576, 1024, 1536, 2048, 12288})
    for (int K : {576, 1536, 2304, 3072, 6144, 12288})
      for (int T : {1, 50, 717, 1433, 8320}) {
        int bn = 0;
        const int sp = orx::linear_plan(N, K, T, 148, &bn);
        EXPECT(bn == 32 || bn == 64 || bn == 128 || bn == 256);
        EXPECT(sp == 1 || sp == 2 || sp == 3 || sp == 4 || sp == 6 || sp == 8);
        EXPECT(K % (64 * sp) == 0);
        EXPECT(sp == 1 || K / sp >= 128);
      }
  std::printf("ok\n");
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("g++") is None, reason="g++ not available")
def test_split_plans(tmp_path):
    if not os.path.exists(LIB):
        pytest.skip("library not built")
    src = tmp_path / "plans.cc"
    src.write_text(PROGRAM)
    exe = tmp_path / "plans"
    subprocess.run(["g++", "-std=c++17", "-O1", str(src), "-o", str(exe),
                    "-L" + os.path.dirname(LIB), "-lorator_b200",
                    "-Wl,-rpath," + os.path.dirname(LIB)], check=True, capture_output=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stdout + r.stderr
