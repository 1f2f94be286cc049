// k_misc.cu -- memory-bound NpuOps: MaxPool2d, standalone Activation, Softmax, and the
// extension ops residual add (+ activation) and adaptive average pooling.
//
// Each kernel can also emit the absmax of its output (per tensor or per image)
// for the next quantizing op, so no separate absmax pass re-reads the tensor.
#include <algorithm>

#include "rg_kernels.h"
#include "rg_math.cuh"

namespace rg {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ void block_max_to(float v, unsigned* dst) {
  __shared__ float red[kThreads / 32];
  v = warp_max(v);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) red[wid] = v;
  __syncthreads();
  if (wid == 0) {
    v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
    v = warp_max(v);
    if (lane == 0 && v > 0.0f) atomicMax(dst, __float_as_uint(v));
  }
}

// max_pool2d (src/kernels.rs:165-213): pad 0, `if v > best || v.is_nan()` in window
// order.  One thread per output; K (2 and 3 as template instances, 0 = any size at
// run time) fixes the window so that all of its loads are in flight together.
// grid.y strides over the absmax slots (an image, or the whole tensor).
template <int K>
__global__ void __launch_bounds__(kThreads) k_maxpool2d(const float* __restrict__ x, int64_t planes,
                                                        int32_t h, int32_t w, int32_t kr, int32_t s,
                                                        int32_t oh, int32_t ow, float* __restrict__ y,
                                                        unsigned* amax, int64_t planes_per_slot) {
  const int32_t k = K ? K : kr;
  const int64_t slots = (planes + planes_per_slot - 1) / planes_per_slot;
  const int32_t per_plane = oh * ow;
  for (int64_t slot = blockIdx.y; slot < slots; slot += gridDim.y) {
    const int64_t p0 = slot * planes_per_slot;
    const int64_t outs = (min(planes, p0 + planes_per_slot) - p0) * per_plane;
    float m = 0.0f;
    for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < outs; i += (int64_t)gridDim.x * kThreads) {
      // 32-bit division where the slot's output count allows it (the usual case)
      const int64_t pl = outs < 0x7fffffff ? (int64_t)((uint32_t)i / (uint32_t)per_plane) : i / per_plane;
      const int32_t rem = (int32_t)(i - pl * per_plane);
      const int32_t oy = rem / ow, ox = rem - oy * ow;
      const float* xp = x + (p0 + pl) * (int64_t)h * w + (int64_t)(oy * s) * w + ox * s;
      float best = -INFINITY;
      if (K) {
        float v[K ? K * K : 1];
#pragma unroll
        for (int ki = 0; ki < K; ++ki)
#pragma unroll
          for (int kj = 0; kj < K; ++kj) v[ki * K + kj] = __ldg(xp + ki * w + kj);
#pragma unroll
        for (int t = 0; t < K * K; ++t)
          if (v[t] > best || v[t] != v[t]) best = v[t];
      } else {
        for (int32_t ki = 0; ki < k; ++ki)
          for (int32_t kj = 0; kj < k; ++kj) {
            const float v = __ldg(xp + ki * w + kj);
            if (v > best || v != v) best = v;
          }
      }
      y[(p0 + pl) * per_plane + rem] = best;
      m = fmaxf(m, fabsf(best));
    }
    if (amax) {
      block_max_to(m, amax + slot);
      __syncthreads();  // the reduction buffer is reused by the next slot
    }
  }
}

__global__ void __launch_bounds__(kThreads) k_activation(const float* __restrict__ x, int64_t n,
                                                         int32_t act, float p, float* __restrict__ y,
                                                         unsigned* amax, int64_t per_slot) {
  const int64_t slot = blockIdx.y;
  const int64_t e0 = slot * per_slot;
  const int64_t e1 = min(n, e0 + per_slot);
  float m = 0.0f;
  for (int64_t i = e0 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < e1;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = act_apply(act, p, __ldg(x + i));
    y[i] = v;
    m = fmaxf(m, fabsf(v));
  }
  if (amax) block_max_to(m, amax + slot);
}

// softmax_raw (src/tensor/ops.rs:1058-1076): serial max, exp, serial f32 sum, divide.
// One thread per row keeps the reference's summation order exactly.
__global__ void __launch_bounds__(kThreads) k_softmax(const float* __restrict__ x, int64_t outer,
                                                      int64_t last, float* __restrict__ y,
                                                      unsigned* amax) {
  float m = 0.0f;
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < outer;
       r += (int64_t)gridDim.x * blockDim.x) {
    const float* xr = x + r * last;
    float* yr = y + r * last;
    float mx = -INFINITY;
    for (int64_t j = 0; j < last; ++j) mx = fmaxf(mx, xr[j]);
    float s = 0.0f;
    for (int64_t j = 0; j < last; ++j) {
      const float e = exp_f32(__fsub_rn(xr[j], mx));
      yr[j] = e;
      s = __fadd_rn(s, e);
    }
    for (int64_t j = 0; j < last; ++j) {
      const float v = __fdiv_rn(yr[j], s);
      yr[j] = v;
      m = fmaxf(m, fabsf(v));
    }
  }
  if (amax) block_max_to(m, amax);
}

// Extension: y = act(x + s) (binary Add, tensor/ops.rs:67-76, then the block's activation).
__global__ void __launch_bounds__(kThreads) k_residual_add(const float* __restrict__ x, const float* __restrict__ sv,
                                                           int64_t n, int32_t act, float p, float* __restrict__ y,
                                                           unsigned* amax, int64_t per_slot) {
  const int64_t slot = blockIdx.y;
  const int64_t e0 = slot * per_slot;
  const int64_t e1 = min(n, e0 + per_slot);
  float m = 0.0f;
  for (int64_t i = e0 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < e1;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = act_apply(act, p, __fadd_rn(__ldg(x + i), __ldg(sv + i)));
    y[i] = v;
    m = fmaxf(m, fabsf(v));
  }
  if (amax) block_max_to(m, amax + slot);
}

// Extension: adaptive_avg_pool2d (tensor/ops.rs:994-1014): rows [y*h/oh, ceil((y+1)h/oh)),
// columns likewise; serial f32 sum in row-major order from 0, one division by the count.
__global__ void __launch_bounds__(kThreads) k_adaptive_avgpool(const float* __restrict__ x, int64_t planes,
                                                               int32_t h, int32_t w, int32_t oh, int32_t ow,
                                                               float* __restrict__ y, unsigned* amax,
                                                               int64_t planes_per_slot) {
  const int64_t slot = blockIdx.y;
  const int64_t p0 = slot * planes_per_slot;
  const int64_t p1 = min(planes, p0 + planes_per_slot);
  const int64_t per = (p1 - p0) * oh * ow;
  float m = 0.0f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < per;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = p0 * oh * ow + i;
    const int64_t plane = o / ((int64_t)oh * ow);
    const int32_t rem = (int32_t)(o - plane * oh * ow);
    const int32_t oy = rem / ow, ox = rem - oy * ow;
    const int32_t y0 = oy * h / oh, y1 = ((oy + 1) * h + oh - 1) / oh;
    const int32_t x0 = ox * w / ow, x1 = ((ox + 1) * w + ow - 1) / ow;
    const float* xp = x + plane * (int64_t)h * w;
    float sum = 0.0f;
    for (int32_t yy = y0; yy < y1; ++yy)
      for (int32_t xx = x0; xx < x1; ++xx) sum = __fadd_rn(sum, __ldg(xp + (int64_t)yy * w + xx));
    const float v = __fdiv_rn(sum, (float)((y1 - y0) * (x1 - x0)));
    y[o] = v;
    m = fmaxf(m, fabsf(v));
  }
  if (amax) block_max_to(m, amax + slot);
}

__global__ void k_fill_u32(unsigned* p, unsigned v, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    p[i] = v;
}

__global__ void k_bits_to_float(const unsigned* bits, float* out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __uint_as_float(bits[i]);
}

int grid_for(int64_t work, int64_t per_block, int cap) {
  int64_t g = (work + per_block - 1) / per_block;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return (int)g;
}

}  // namespace

void launch_maxpool2d(const float* x, int64_t n, int32_t c, int32_t h, int32_t w, int32_t k,
                      int32_t s, float* y, AmaxSink amax, cudaStream_t st) {
  const int32_t oh = (h - k) / s + 1, ow = (w - k) / s + 1;
  const int64_t planes = n * c;
  if (planes <= 0 || oh <= 0 || ow <= 0) return;
  int64_t planes_per_slot = planes;
  if (amax.ptr && amax.elems_per_slot > 0) planes_per_slot = amax.elems_per_slot / ((int64_t)oh * ow);
  if (planes_per_slot <= 0) planes_per_slot = planes;
  const int64_t slots = (planes + planes_per_slot - 1) / planes_per_slot;
  const int64_t outs_per_slot = planes_per_slot * oh * ow;
  const int64_t want = std::max<int64_t>(1, 148 * 32 / std::max<int64_t>(slots, 1));
  const unsigned bx = (unsigned)std::max<int64_t>(1, std::min<int64_t>((outs_per_slot + kThreads - 1) / kThreads, want));
  const dim3 grid(bx, (unsigned)std::min<int64_t>(slots, 65535));
  if (k == 2)
    k_maxpool2d<2><<<grid, kThreads, 0, st>>>(x, planes, h, w, k, s, oh, ow, y, amax.ptr, planes_per_slot);
  else if (k == 3)
    k_maxpool2d<3><<<grid, kThreads, 0, st>>>(x, planes, h, w, k, s, oh, ow, y, amax.ptr, planes_per_slot);
  else
    k_maxpool2d<0><<<grid, kThreads, 0, st>>>(x, planes, h, w, k, s, oh, ow, y, amax.ptr, planes_per_slot);
}

void launch_activation(const float* x, int64_t n, int32_t act, float p, float* y, AmaxSink amax,
                       cudaStream_t st) {
  if (n <= 0) return;
  int64_t per_slot = (amax.ptr && amax.elems_per_slot > 0) ? amax.elems_per_slot : n;
  const int64_t slots = (n + per_slot - 1) / per_slot;
  dim3 grid(grid_for(per_slot, kThreads * 4, slots > 1 ? 64 : 148 * 16), (unsigned)slots);
  k_activation<<<grid, kThreads, 0, st>>>(x, n, act, p, y, amax.ptr, per_slot);
}

void launch_residual_add(const float* x, const float* sv, int64_t n, int32_t act, float p, float* y,
                         AmaxSink amax, cudaStream_t st) {
  if (n <= 0) return;
  int64_t per_slot = (amax.ptr && amax.elems_per_slot > 0) ? amax.elems_per_slot : n;
  const int64_t slots = (n + per_slot - 1) / per_slot;
  dim3 grid(grid_for(per_slot, kThreads * 4, slots > 1 ? 64 : 148 * 16), (unsigned)slots);
  k_residual_add<<<grid, kThreads, 0, st>>>(x, sv, n, act, p, y, amax.ptr, per_slot);
}

void launch_adaptive_avgpool(const float* x, int64_t n, int32_t c, int32_t h, int32_t w, int32_t oh, int32_t ow,
                             float* y, AmaxSink amax, cudaStream_t st) {
  const int64_t planes = n * c;
  if (planes <= 0 || oh <= 0 || ow <= 0) return;
  int64_t planes_per_slot = planes;
  if (amax.ptr && amax.elems_per_slot > 0) planes_per_slot = amax.elems_per_slot / ((int64_t)oh * ow);
  if (planes_per_slot <= 0) planes_per_slot = planes;
  const int64_t slots = (planes + planes_per_slot - 1) / planes_per_slot;
  const int64_t per = planes_per_slot * oh * ow;
  dim3 grid(grid_for(per, kThreads, slots > 1 ? 64 : 148 * 16), (unsigned)slots);
  k_adaptive_avgpool<<<grid, kThreads, 0, st>>>(x, planes, h, w, oh, ow, y, amax.ptr, planes_per_slot);
}

void launch_softmax(const float* x, int64_t outer, int64_t last, float* y, AmaxSink amax,
                    cudaStream_t st) {
  if (outer <= 0 || last <= 0) return;
  k_softmax<<<grid_for(outer, kThreads, 148 * 8), kThreads, 0, st>>>(x, outer, last, y, amax.ptr);
}

void launch_fill_u32(unsigned* p, unsigned v, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  k_fill_u32<<<grid_for(n, kThreads, 1024), kThreads, 0, st>>>(p, v, n);
}

void launch_bits_to_float(const unsigned* bits, float* out, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  k_bits_to_float<<<grid_for(n, kThreads, 1024), kThreads, 0, st>>>(bits, out, n);
}

}  // namespace rg
