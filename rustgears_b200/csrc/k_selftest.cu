// k_selftest.cu -- device self-test of the division on the tanh / GELU path.
//
// tanh_f32 divides with Markstein's reciprocal-and-correction sequence instead of
// the IEEE division; this kernel shows, over every f32 input, that tanh and GELU
// are bit-identical either way.
#include "rg_kernels.h"
#include "rg_math.cuh"

namespace rg {
namespace {

__global__ void k_selftest_tanh_division(unsigned long long* counts) {
  unsigned long long bad_t = 0, bad_g = 0;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (1ull << 32); i += stride) {
    const float x = u2f((uint32_t)i);
    bad_t += f2u(tanh_f32<true>(x)) != f2u(tanh_f32<false>(x));
    bad_g += f2u(gelu_f32<true>(x)) != f2u(gelu_f32<false>(x));
  }
  if (bad_t) atomicAdd(counts, bad_t);
  if (bad_g) atomicAdd(counts + 1, bad_g);
}

}  // namespace

void launch_selftest_tanh_division(unsigned long long* counts, cudaStream_t st) {
  cudaMemsetAsync(counts, 0, 2 * sizeof(unsigned long long), st);
  k_selftest_tanh_division<<<148 * 8, 256, 0, st>>>(counts);
}

}  // namespace rg
