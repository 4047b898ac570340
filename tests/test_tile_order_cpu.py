"""The persistent GEMM's tile order (gemm_tile_coords in
mka_b200/csrc/fmka_internal.h), compiled from the header for the host with
nvcc and run on the CPU: for every grid shape and band height tried it visits
each (row block, column block) exactly once, and band height 1 is plain
row-major order. Every kernel derives its tile coordinates from it, so this is
what keeps each output tile computed once and every TMA coordinate inside the
operands."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SRC = r'''
#include <cstdio>
#include <vector>
#include "fmka_internal.h"
int main() {
  const int groups[] = {1, 2, 3, 8, 16};
  long checked = 0;
  for (int num_m = 1; num_m <= 70; ++num_m) {
    for (int num_n = 1; num_n <= 40; ++num_n) {
      for (int g : groups) {
        std::vector<int> seen(num_m * num_n, 0);
        for (int t = 0; t < num_m * num_n; ++t) {
          int mb = -1, nb = -1;
          fmka::gemm_tile_coords(t, num_m, num_n, g, mb, nb);
          if (mb < 0 || mb >= num_m || nb < 0 || nb >= num_n) {
            std::printf("out of range: m%d n%d g%d t%d -> %d %d\n", num_m, num_n, g, t, mb, nb);
            return 1;
          }
          if (g == 1 && (mb != t / num_n || nb != t % num_n)) {
            std::printf("not row-major: m%d n%d t%d\n", num_m, num_n, t);
            return 1;
          }
          if (seen[mb * num_n + nb]++) {
            std::printf("visited twice: m%d n%d g%d (%d, %d)\n", num_m, num_n, g, mb, nb);
            return 1;
          }
          ++checked;
        }
      }
    }
  }
  // the fused MLP's gate/up GEMM at 65536 tokens: 256 pair row blocks x 112 column blocks
  {
    const int num_m = 256, num_n = 112, g = 8;
    std::vector<int> seen(num_m * num_n, 0);
    for (int t = 0; t < num_m * num_n; ++t) {
      int mb, nb;
      fmka::gemm_tile_coords(t, num_m, num_n, g, mb, nb);
      if (mb < 0 || mb >= num_m || nb < 0 || nb >= num_n || seen[mb * num_n + nb]++) return 1;
    }
  }
  std::printf("ok %ld\n", checked);
  return 0;
}
'''


def test_tile_order_is_a_bijection(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not found")
    src = tmp_path / "tile_order.cu"
    src.write_text(SRC)
    exe = tmp_path / "tile_order"
    subprocess.check_call([nvcc, "-std=c++17", "-I", os.path.join(ROOT, "mka_b200", "csrc"), str(src), "-o", str(exe)])
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert out.stdout.startswith("ok")
