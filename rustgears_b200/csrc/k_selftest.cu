// k_selftest.cu -- device self-test of the fast arithmetic paths.
//
// tanh_f32, quant_scale and quant_inv divide with Markstein's reciprocal-and-
// correction sequence instead of the IEEE division, and quantization rounds with
// round_half_away instead of roundf; this kernel shows, over every f32 input, that
// tanh, GELU, the quantization scale (from every absmax), its reciprocal and the
// rounding are identical either way; and that the common-range tanh of the GEMM
// epilogue equals tanh_f32 (and GELU through it equals gelu_f32) wherever it is used,
// in its scalar form and in the packed-pair form the epilogue runs (both elements).
#include "rg_f32x2.cuh"
#include "rg_kernels.h"
#include "rg_math.cuh"

namespace rg {
namespace {

__global__ void k_selftest_fast_division(unsigned long long* counts) {
  unsigned long long bad_t = 0, bad_g = 0, bad_s = 0, bad_i = 0, bad_r = 0, bad_c = 0;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (1ull << 32); i += stride) {
    const float x = u2f((uint32_t)i);
    bad_t += f2u(tanh_f32<true>(x)) != f2u(tanh_f32<false>(x));
    bad_g += f2u(gelu_f32<true>(x)) != f2u(gelu_f32<false>(x));
    if (tanh_common_range(x)) bad_c += f2u(tanh_f32_common<true>(x)) != f2u(tanh_f32<true>(x));
    const float u = gelu_arg(x);
    if (tanh_common_range(u)) bad_c += f2u(gelu_from_tanh(x, tanh_f32_common<true>(u))) != f2u(gelu_f32<true>(x));
    if (x == x) {  // packed pairs, elements (x, -x)
      float t0, t1;
      tanh_f32_common_x2(x, -x, t0, t1);
      if (tanh_common_range(x)) {
        const float t = tanh_f32<true>(x);
        bad_c += (f2u(t0) != f2u(t)) + (f2u(t1) != f2u(tanh_f32<true>(-x)));
      }
      const f32x2 ug = gelu_arg_x2(pack2(x, -x));
      bad_c += (f2u(lo2(ug)) != f2u(u)) + (f2u(hi2(ug)) != f2u(gelu_arg(-x)));
      if (tanh_common_range(u)) {
        float g0, g1;
        tanh_f32_common_x2(lo2(ug), hi2(ug), g0, g1);
        const f32x2 g = gelu_from_tanh_x2(pack2(x, -x), pack2(g0, g1));
        bad_c += (f2u(lo2(g)) != f2u(gelu_f32<true>(x))) + (f2u(hi2(g)) != f2u(gelu_f32<true>(-x)));
      }
    }
    if (!(fabsf(x) >= 8388608.0f)) {  // |t| < 2^23 and NaN: quantization arguments
      const float r = roundf(x);
      bad_r += round_half_away(x) != (r != r ? 0 : (int32_t)r);
    }
    if (x >= 0.0f) {  // absmax values: +0 .. +inf
      const float s_ref = quant_scale<false>(x);
      bad_s += f2u(quant_scale<true>(x)) != f2u(s_ref);
      bad_i += f2u(quant_inv<true>(s_ref)) != f2u(quant_inv<false>(s_ref));
    }
  }
  if (bad_t) atomicAdd(counts, bad_t);
  if (bad_g) atomicAdd(counts + 1, bad_g);
  if (bad_s) atomicAdd(counts + 2, bad_s);
  if (bad_i) atomicAdd(counts + 3, bad_i);
  if (bad_r) atomicAdd(counts + 4, bad_r);
  if (bad_c) atomicAdd(counts + 5, bad_c);
}

}  // namespace

void launch_selftest_fast_division(unsigned long long* counts, cudaStream_t st) {
  cudaMemsetAsync(counts, 0, 6 * sizeof(unsigned long long), st);
  k_selftest_fast_division<<<148 * 8, 256, 0, st>>>(counts);
}

}  // namespace rg
