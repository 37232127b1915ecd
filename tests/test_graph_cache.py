"""Host rules of the per-batch-size CUDA-graph cache
(orator_b200/csrc/graph_cache.h), compiled with g++ against a fake graph
handle: a graph is handed out only under the memory epoch it was captured in,
and an epoch change destroys every graph, including graphs for batch sizes
that are not looked up again (the case that once replayed a graph against a
freed split-K workspace when batch sizes went a -> c -> a)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PROGRAM = r"""
#include <cstdio>
#include <set>
#include "graph_cache.h"
static std::set<int> live;
static int destroyed = 0;
static int destroy(int h) { live.erase(h); ++destroyed; return 0; }
#define EXPECT(c) do { if (!(c)) { std::printf("FAIL line %d: %s\n", __LINE__, #c); return 1; } } while (0)
int main() {
  int next = 1;
  auto capture = [&]() { live.insert(next); return next++; };
  {
    orx::GraphCache<int, int (*)(int)> gc(destroy);
    uint64_t epoch = 0;
    // batch size 3: eager first, then captured
    EXPECT(gc.find(3, epoch) == 0 && !gc.warmed(3));
    gc.mark_warmed(3);
    const int g3 = capture();
    gc.insert(3, epoch, g3);
    EXPECT(gc.find(3, epoch) == g3);
    // batch size 8 runs eagerly and grows the workspace: the epoch moves
    EXPECT(gc.find(8, epoch) == 0);
    gc.mark_warmed(8);
    ++epoch;
    const int g8 = capture();
    gc.insert(8, epoch, g8);           // inserting under the new epoch drops g3
    EXPECT(live.count(g3) == 0);
    EXPECT(gc.find(3, epoch) == 0);    // back to 3: no stale replay ...
    EXPECT(!gc.warmed(3));             // ... and it warms up again
    EXPECT(gc.find(8, epoch) == g8);
    // a lookup alone under a newer epoch also drops everything
    ++epoch;
    EXPECT(gc.find(5, epoch) == 0 && live.empty() && gc.size() == 0);
    // same epoch, re-insert for one key destroys the old handle
    const int a = capture(), b = capture();
    gc.insert(5, epoch, a);
    gc.insert(5, epoch, b);
    EXPECT(live.count(a) == 0 && gc.find(5, epoch) == b && gc.size() == 1);
  }
  EXPECT(live.empty());  // the destructor releases what is left
  std::printf("OK %d\n", destroyed);
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("g++") is None, reason="g++ not installed")
def test_graph_cache_rules(tmp_path):
    src = tmp_path / "gc.cc"
    src.write_text(PROGRAM)
    exe = tmp_path / "gc"
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Werror", "-I",
                    os.path.join(ROOT, "orator_b200", "csrc"), str(src), "-o", str(exe)],
                   check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("OK")
