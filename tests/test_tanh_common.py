"""The epilogue's common-range tanh (tanh_f32_common, used by the tensor-core GEMM
when every value of a warp's chunk has its GELU tanh argument in [2^-25, 7.5)) is
the general glibc/fdlibm restatement tanh_f32 with the cases that range cannot take
left out.  Checked here on every f32 of the range, both signs, by compiling the
library's own arithmetic header (rustgears_b200/csrc/rg_math.cuh) for the host with
round-to-nearest and no contraction; the device self-test repeats the check with the
device's division (tests/test_gpu_transcendental.py)."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SRC = r'''
#include <math.h>
#include <stdio.h>
#include <string.h>
#include "rg_math.cuh"
using namespace rg;
int main() {
  unsigned long long bad = 0, bad_gelu = 0, outside = 0, n = 0;
  const uint32_t lo = 0x33000000u, hi = 0x40f00000u;
  #pragma omp parallel for reduction(+ : bad, n, outside) schedule(static)
  for (long long i = 0; i < 2LL * (hi - lo); ++i) {
    const uint32_t bits = (uint32_t)(lo + (uint32_t)(i >> 1)) | ((uint32_t)(i & 1) << 31);
    const float x = u2f(bits);
    if (!tanh_common_range(x)) { ++outside; continue; }
    ++n;
    bad += f2u(tanh_f32_common<false>(x)) != f2u(tanh_f32<false>(x));
  }
  /* GELU: every f32 input whose tanh argument is in range (stride over all 2^32) */
  #pragma omp parallel for reduction(+ : bad_gelu) schedule(static)
  for (long long i = 0; i < (1LL << 32); i += 7) {
    const float x = u2f((uint32_t)i);
    const float u = gelu_arg(x);
    if (!tanh_common_range(u)) continue;
    bad_gelu += f2u(gelu_from_tanh(x, tanh_f32_common<false>(u))) != f2u(gelu_f32<false>(x));
  }
  /* the range test itself: just below / at / just above each bound */
  int edges_ok = !tanh_common_range(u2f(lo - 1)) && tanh_common_range(u2f(lo)) &&
                 tanh_common_range(u2f(hi - 1)) && !tanh_common_range(u2f(hi)) &&
                 !tanh_common_range(NAN) && !tanh_common_range(INFINITY);
  printf("%llu %llu %llu %llu %d\n", n, bad, bad_gelu, outside, edges_ok);
  return 0;
}
'''


def test_tanh_common_equals_general_tanh_on_its_whole_range(tmp_path):
    src = tmp_path / "chk.cpp"
    src.write_text(SRC)
    exe = tmp_path / "chk"
    inc = os.path.join(ROOT, "rustgears_b200", "csrc")
    r = subprocess.run(["g++", "-O2", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-std=c++17", "-I", inc,
                        str(src), "-o", str(exe), "-lm"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=900,
                         env=dict(os.environ, OMP_NUM_THREADS=str(os.cpu_count() or 1)))
    assert out.returncode == 0, out.stderr
    n, bad, bad_gelu, outside, edges_ok = (int(v) for v in out.stdout.split())
    assert n == 2 * (0x40f00000 - 0x33000000) and outside == 0
    assert bad == 0 and bad_gelu == 0 and edges_ok == 1
