// k_quant.cu -- activation absmax and symmetric INT8 quantization kernels.
//
// Reference: QuantTensor::from_f32 / quantize_into (src/inference/quantize.rs:18-35).
// The reference folds max|v| serially over the whole tensor; max is exact and
// order-free, so a parallel reduction gives the identical value.  HBM-bound:
// 16-byte vector loads, warp-shuffle reduction, one atomic per block.
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

// Block-wide max of non-negative floats; one atomicMax on the uint bits by thread 0.
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

__global__ void __launch_bounds__(kThreads) k_absmax(const float* __restrict__ x, int64_t n,
                                                     unsigned* __restrict__ out) {
  float m = 0.0f;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    const int64_t n4 = n >> 2;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    int64_t i = tid;
    // four independent 16-byte loads in flight per thread before they are folded in
    for (; i + 3 * stride < n4; i += 4 * stride) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __ldg(x4 + i + u * stride);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        m = fmaxf(m, fabsf(v[u].x)); m = fmaxf(m, fabsf(v[u].y));
        m = fmaxf(m, fabsf(v[u].z)); m = fmaxf(m, fabsf(v[u].w));
      }
    }
    for (; i < n4; i += stride) {
      const float4 v = __ldg(x4 + i);
      m = fmaxf(m, fabsf(v.x)); m = fmaxf(m, fabsf(v.y));
      m = fmaxf(m, fabsf(v.z)); m = fmaxf(m, fabsf(v.w));
    }
    for (int64_t i = (n4 << 2) + tid; i < n; i += stride) m = fmaxf(m, fabsf(__ldg(x + i)));
  } else {
    for (int64_t i = tid; i < n; i += stride) m = fmaxf(m, fabsf(__ldg(x + i)));
  }
  block_max_to(m, out);
}

// One thread per 16 output bytes of a row.
// FROZEN: the scale is given (a calibrated scale, extension) instead of derived from
// the tensor's absmax; values beyond its range clamp to +-127 (quant1).
template <bool FROZEN>
__global__ void __launch_bounds__(kThreads) k_quantize_rows(const float* __restrict__ x, int64_t rows,
                                                            int64_t k, int64_t ldq,
                                                            const unsigned* __restrict__ amax_bits,
                                                            const float* __restrict__ frozen_scale,
                                                            int8_t* __restrict__ q,
                                                            float* __restrict__ scale_out) {
  const float scale = FROZEN ? *frozen_scale : quant_scale(__uint_as_float(*amax_bits));
  const float inv = quant_inv(scale);
  if (!FROZEN && blockIdx.x == 0 && threadIdx.x == 0 && scale_out) *scale_out = scale;
  const int64_t chunks = ldq >> 4;
  const int64_t total = rows * chunks;
  const bool vec = ((k & 3) == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = t / chunks, c0 = (t - r * chunks) << 4;
    const float* src = x + r * k + c0;
    uint32_t word[4];
    if (vec && c0 + 16 <= k) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(src) + j);
        word[j] = (uint32_t)(quant1(v.x, inv) & 0xff) | ((uint32_t)(quant1(v.y, inv) & 0xff) << 8) |
                  ((uint32_t)(quant1(v.z, inv) & 0xff) << 16) | ((uint32_t)(quant1(v.w, inv) & 0xff) << 24);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t wv = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int64_t col = c0 + j * 4 + b;
          const int32_t qv = col < k ? quant1(__ldg(src + j * 4 + b), inv) : 0;
          wv |= (uint32_t)(qv & 0xff) << (8 * b);
        }
        word[j] = wv;
      }
    }
    *reinterpret_cast<uint4*>(q + r * ldq + c0) = make_uint4(word[0], word[1], word[2], word[3]);
  }
}

// grid (blocks_per_image, n): max |x| over covered pixels of each image.
// Per-image absmax.  Without coverage masks a flat strided pass over the image; with
// them (a strided conv that skips rows / columns), a warp per (channel, row): rows
// the conv never reads are skipped whole, lanes run along the row.  grid.y strides
// over the images.
__global__ void __launch_bounds__(kThreads) k_image_absmax(const float* __restrict__ x, int64_t n, int32_t c,
                                                           int32_t h, int32_t w,
                                                           const uint8_t* __restrict__ row_cov,
                                                           const uint8_t* __restrict__ col_cov,
                                                           bool cov_smem, unsigned* __restrict__ amax) {
  const int64_t per = (int64_t)c * h * w;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int64_t img = blockIdx.y; img < n; img += gridDim.y) {
    const float* xi = x + img * per;
    float m = 0.0f;
    if (!row_cov) {
      if (((per | reinterpret_cast<uintptr_t>(x)) & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        // 16-byte loads, four in flight per thread
        const float4* x4 = reinterpret_cast<const float4*>(xi);
        const int64_t per4 = per / 4, step = (int64_t)gridDim.x * blockDim.x;
        int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
        for (; i + 3 * step < per4; i += 4 * step) {
          float4 a[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) a[k] = __ldg(x4 + i + k * step);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            m = fmaxf(fmaxf(m, fmaxf(fabsf(a[k].x), fabsf(a[k].y))), fmaxf(fabsf(a[k].z), fabsf(a[k].w)));
        }
        for (; i < per4; i += step) {
          const float4 a = __ldg(x4 + i);
          m = fmaxf(fmaxf(m, fmaxf(fabsf(a.x), fabsf(a.y))), fmaxf(fabsf(a.z), fabsf(a.w)));
        }
      } else {
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < per; i += (int64_t)gridDim.x * blockDim.x)
          m = fmaxf(m, fabsf(__ldg(xi + i)));
      }
    } else {
      // the masks in shared memory (the launcher bounds h and w); rows the conv never
      // reads are skipped whole
      extern __shared__ uint8_t cov_s[];  // [h] rows then [w] columns
      if (cov_smem) {
        for (int32_t i = threadIdx.x; i < h + w; i += kThreads) cov_s[i] = i < h ? row_cov[i] : col_cov[i - h];
        __syncthreads();
      }
      const uint8_t* rcov = cov_smem ? cov_s : row_cov;
      const uint8_t* ccov = cov_smem ? cov_s + h : col_cov;
      const int32_t rows = c * h;
      for (int32_t rr = blockIdx.x * (kThreads / 32) + wid; rr < rows; rr += gridDim.x * (kThreads / 32)) {
        if (!rcov[rr % h]) continue;  // warp-uniform
        const float* xr = xi + (int64_t)rr * w;
        for (int32_t ix = lane; ix < w; ix += 32)
          if (ccov[ix]) m = fmaxf(m, fabsf(__ldg(xr + ix)));
      }
    }
    block_max_to(m, amax + img);
    __syncthreads();  // the reduction buffer is reused by the next image
  }
}

// NCHW f32 (c <= 4 channels) -> NHWC i8 with 4-byte pixels (zero-padded channels): a
// thread per pixel, one 4-byte store; grid.y strides over the images.
__global__ void __launch_bounds__(kThreads) k_image_quantize_nhwc4(const float* __restrict__ x, int64_t n,
                                                                   int32_t c, int32_t hw,
                                                                   const unsigned* __restrict__ amax,
                                                                   int8_t* __restrict__ q,
                                                                   float* __restrict__ scales) {
  for (int64_t img = blockIdx.y; img < n; img += gridDim.y) {
    const float scale = quant_scale(__uint_as_float(amax[img]));
    const float inv = quant_inv(scale);
    if (blockIdx.x == 0 && threadIdx.x == 0 && scales) scales[img] = scale;
    const float* xi = x + img * (int64_t)c * hw;
    uint32_t* qi = reinterpret_cast<uint32_t*>(q) + img * (int64_t)hw;
    for (int32_t p = blockIdx.x * kThreads + threadIdx.x; p < hw; p += gridDim.x * kThreads) {
      uint32_t wv = 0;
      for (int32_t ch = 0; ch < c; ++ch)
        wv |= (uint32_t)(uint8_t)(int8_t)quant1(__ldg(xi + (int64_t)ch * hw + p), inv) << (8 * ch);
      qi[p] = wv;
    }
  }
}

// NCHW f32 (c <= 4 channels, even h and w) -> space-to-depth i8 pixels [n][h/2][w/2][16 B]:
// byte (dy * 2 + dx) * 4 + ch of s2d pixel (sy, sx) = channel ch of pixel (2 sy + dy,
// 2 sx + dx), zero for ch >= c.  A thread per s2d pixel, one 16-byte store; grid.y
// strides over the images.
__global__ void __launch_bounds__(kThreads) k_image_quantize_s2d(const float* __restrict__ x, int64_t n,
                                                                 int32_t c, int32_t h, int32_t w,
                                                                 const unsigned* __restrict__ amax,
                                                                 int8_t* __restrict__ q,
                                                                 float* __restrict__ scales) {
  const int32_t w2 = w / 2, hw2 = (h / 2) * w2;
  const int32_t hw = h * w;
  for (int64_t img = blockIdx.y; img < n; img += gridDim.y) {
    const float scale = quant_scale(__uint_as_float(amax[img]));
    const float inv = quant_inv(scale);
    if (blockIdx.x == 0 && threadIdx.x == 0 && scales) scales[img] = scale;
    const float* xi = x + img * (int64_t)c * hw;
    uint4* qi = reinterpret_cast<uint4*>(q) + img * (int64_t)hw2;
    for (int32_t p = blockIdx.x * kThreads + threadIdx.x; p < hw2; p += gridDim.x * kThreads) {
      const int32_t sy = p / w2, sx = p - sy * w2;
      uint32_t wv[4] = {0u, 0u, 0u, 0u};
      for (int32_t ch = 0; ch < c; ++ch) {
        const float* r0 = xi + (int64_t)ch * hw + (2 * sy) * w + 2 * sx;
        const float v00 = __ldg(r0), v01 = __ldg(r0 + 1), v10 = __ldg(r0 + w), v11 = __ldg(r0 + w + 1);
        wv[0] |= (uint32_t)(uint8_t)(int8_t)quant1(v00, inv) << (8 * ch);
        wv[1] |= (uint32_t)(uint8_t)(int8_t)quant1(v01, inv) << (8 * ch);
        wv[2] |= (uint32_t)(uint8_t)(int8_t)quant1(v10, inv) << (8 * ch);
        wv[3] |= (uint32_t)(uint8_t)(int8_t)quant1(v11, inv) << (8 * ch);
      }
      qi[p] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
  }
}

// grid-stride over (image, pixel): NCHW f32 -> NHWC i8 (pixel stride cpad).
__global__ void __launch_bounds__(kThreads) k_image_quantize_nhwc(const float* __restrict__ x, int64_t n,
                                                                  int32_t c, int32_t hw, int32_t cpad,
                                                                  const unsigned* __restrict__ amax,
                                                                  int8_t* __restrict__ q,
                                                                  float* __restrict__ scales) {
  const int64_t total = n * hw;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t img = t / hw;
    const int64_t p = t - img * hw;
    const float scale = quant_scale(__uint_as_float(amax[img]));
    const float inv = quant_inv(scale);
    if (p == 0 && scales) scales[img] = scale;
    const float* src = x + img * (int64_t)c * hw + p;
    int8_t* dst = q + t * cpad;
    for (int32_t ch = 0; ch < cpad; ++ch)
      dst[ch] = (int8_t)(ch < c ? quant1(__ldg(src + (int64_t)ch * hw), inv) : 0);
  }
}

// NCHW f32 -> 16-channel groups of i8 with the image's scale: a thread per (pixel,
// 16-channel group) loads the group's 16 values (each load instruction of a warp reads
// 32 consecutive pixels of one channel), quantizes them and stores the 16 bytes once.
// PLANAR: [img][cpad / 16][hw][16] (16-channel chunk planes); else NHWC [img][hw][cpad].
// BOUNDED: the scale came from this whole tensor (|v| <= amax), so the clamp never acts
// (quant1_bounded); else a strided conv's scale covers only the pixels it reads and
// others may exceed it (quant1).  Channels past c are written as zeros.
__device__ __forceinline__ uint32_t pack4_i8(int32_t b0, int32_t b1, int32_t b2, int32_t b3) {
  return __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
}

template <bool BOUNDED, bool PLANAR>
__global__ void __launch_bounds__(256) k_image_quantize_g16(const float* __restrict__ x, int32_t c, int32_t hw,
                                                            int32_t cpad, const unsigned* __restrict__ amax,
                                                            int8_t* __restrict__ q, float* __restrict__ scales) {
  const int64_t img = blockIdx.z;
  const int32_t g = blockIdx.y;
  const float scale = quant_scale(__uint_as_float(amax[img]));
  const float inv = quant_inv(scale);
  if (scales && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) scales[img] = scale;
  const int32_t nch = c - 16 * g;  // channels of this group that exist (<= 0: padding only)
  const float* src = x + (img * c + 16 * g) * (int64_t)hw;
  for (int32_t px = blockIdx.x * 256 + threadIdx.x; px < hw; px += gridDim.x * 256) {
    float v[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) v[k] = k < nch ? __ldg(src + (int64_t)k * hw + px) : 0.0f;
    int32_t t[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) t[k] = BOUNDED ? quant1_bounded(v[k], inv) : quant1(v[k], inv);
    const uint4 word = make_uint4(pack4_i8(t[0], t[1], t[2], t[3]), pack4_i8(t[4], t[5], t[6], t[7]),
                                  pack4_i8(t[8], t[9], t[10], t[11]), pack4_i8(t[12], t[13], t[14], t[15]));
    const int64_t off = PLANAR ? ((img * (cpad / 16) + g) * (int64_t)hw + px) * 16
                               : (img * hw + px) * (int64_t)cpad + 16 * g;
    *reinterpret_cast<uint4*>(q + off) = word;
  }
}

// The strided 1x1 conv's operand: output pixel (oy, ox) of the compact [n][oh][ow][cpad]
// NHWC tensor is input pixel (s oy, s ox); the scale's absmax covers exactly these
// pixels (no clamp).
template <bool PLANAR>
__global__ void __launch_bounds__(256) k_image_quantize_sub16(const float* __restrict__ x, int32_t c, int32_t h,
                                                              int32_t w, int32_t s, int32_t oh, int32_t ow,
                                                              int32_t cpad, const unsigned* __restrict__ amax,
                                                              int8_t* __restrict__ q, float* __restrict__ scales) {
  const int64_t img = blockIdx.z;
  const int32_t g = blockIdx.y;
  const float scale = quant_scale(__uint_as_float(amax[img]));
  const float inv = quant_inv(scale);
  if (scales && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) scales[img] = scale;
  const int32_t nch = c - 16 * g;
  const int64_t hw = (int64_t)h * w;
  const float* src = x + (img * c + 16 * g) * hw;
  const int32_t ohw = oh * ow;
  for (int32_t op = blockIdx.x * 256 + threadIdx.x; op < ohw; op += gridDim.x * 256) {
    const int32_t oy = op / ow, ox = op - oy * ow;
    const int64_t px = (int64_t)(s * oy) * w + s * ox;
    float v[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) v[k] = k < nch ? __ldg(src + (int64_t)k * hw + px) : 0.0f;
    int32_t t[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) t[k] = quant1_bounded(v[k], inv);
    const uint4 word = make_uint4(pack4_i8(t[0], t[1], t[2], t[3]), pack4_i8(t[4], t[5], t[6], t[7]),
                                  pack4_i8(t[8], t[9], t[10], t[11]), pack4_i8(t[12], t[13], t[14], t[15]));
    const int64_t off = PLANAR ? ((img * (cpad / 16) + g) * (int64_t)ohw + op) * 16 : (img * ohw + op) * (int64_t)cpad + 16 * g;
    *reinterpret_cast<uint4*>(q + off) = word;
  }
}

// The space-to-depth operand of a 3x3 / stride 2 / pad 1 conv: chunk g of s2d pixel
// (sy, sx) holds channels c0 .. c0 + 15 (16 g = dd * cpad + c0, dd = dy * 2 + dx) of
// input pixel (2 sy + dy, 2 sx + dx), zero past an odd h or w (that row / column is the
// conv's own bottom / right padding); every input pixel is read by the conv, so the
// absmax covers them all (no clamp).
__global__ void __launch_bounds__(256) k_image_quantize_s2d16(const float* __restrict__ x, int32_t c, int32_t h,
                                                              int32_t w, int32_t cpad,
                                                              const unsigned* __restrict__ amax,
                                                              int8_t* __restrict__ q, float* __restrict__ scales) {
  const int64_t img = blockIdx.z;
  const int32_t g = blockIdx.y;
  const float scale = quant_scale(__uint_as_float(amax[img]));
  const float inv = quant_inv(scale);
  if (scales && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) scales[img] = scale;
  const int32_t dd = (16 * g) / cpad, c0 = (16 * g) % cpad, dy = dd >> 1, dx = dd & 1;
  const int32_t nch = c - c0;
  const int64_t hw = (int64_t)h * w;
  const float* src = x + (img * c + c0) * hw;
  const int32_t w2 = (w + 1) / 2, hw2 = ((h + 1) / 2) * w2;
  for (int32_t sp = blockIdx.x * 256 + threadIdx.x; sp < hw2; sp += gridDim.x * 256) {
    const int32_t sy = sp / w2, sx = sp - sy * w2;
    const int32_t iy = 2 * sy + dy, ix = 2 * sx + dx;
    const int32_t nv = iy < h && ix < w ? nch : 0;  // channels present at this pixel
    const int64_t px = (int64_t)iy * w + ix;
    float v[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) v[k] = k < nv ? __ldg(src + (int64_t)k * hw + px) : 0.0f;
    int32_t t[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) t[k] = quant1_bounded(v[k], inv);
    const uint4 word = make_uint4(pack4_i8(t[0], t[1], t[2], t[3]), pack4_i8(t[4], t[5], t[6], t[7]),
                                  pack4_i8(t[8], t[9], t[10], t[11]), pack4_i8(t[12], t[13], t[14], t[15]));
    *reinterpret_cast<uint4*>(q + ((img * (4 * cpad / 16) + g) * (int64_t)hw2 + sp) * 16) = word;
  }
}

template <bool PLANAR>
void launch_g16(const float* x, int64_t n, int32_t c, int32_t hw, int32_t cpad, bool bounded, const unsigned* amax,
                int8_t* q, float* scales, cudaStream_t st) {
  const dim3 grid((unsigned)std::min<int64_t>((hw + 255) / 256, 1024), (unsigned)(cpad / 16), (unsigned)n);
  if (bounded)
    k_image_quantize_g16<true, PLANAR><<<grid, 256, 0, st>>>(x, c, hw, cpad, amax, q, scales);
  else
    k_image_quantize_g16<false, PLANAR><<<grid, 256, 0, st>>>(x, c, hw, cpad, amax, q, scales);
}

__global__ void k_nhwc_to_nchw_i8(const int8_t* __restrict__ q, int64_t n, int32_t c, int32_t cpad,
                                  int32_t hw, int8_t* __restrict__ out) {
  const int64_t total = n * (int64_t)c * hw;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t img = t / ((int64_t)c * hw);
    const int64_t rem = t - img * c * hw;
    const int32_t ch = (int32_t)(rem / hw);
    const int64_t p = rem - (int64_t)ch * hw;
    out[t] = q[(img * hw + p) * cpad + ch];
  }
}

int grid_for(int64_t work, int64_t per_block, int cap) {
  int64_t g = (work + per_block - 1) / per_block;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return (int)g;
}

}  // namespace

void launch_absmax(const float* x, int64_t n, unsigned* amax_bits, cudaStream_t st) {
  if (n <= 0) return;
  k_absmax<<<grid_for(n, kThreads * 16, 148 * 16), kThreads, 0, st>>>(x, n, amax_bits);
}

void launch_quantize_rows(const float* x, int64_t rows, int64_t k, int64_t ldq,
                          const unsigned* amax_bits, int8_t* q, float* scale_out, cudaStream_t st) {
  const int64_t work = rows * (ldq >> 4);
  if (work <= 0) return;
  k_quantize_rows<false><<<grid_for(work, kThreads, 148 * 32), kThreads, 0, st>>>(x, rows, k, ldq, amax_bits,
                                                                                  nullptr, q, scale_out);
}

void launch_quantize_rows_frozen(const float* x, int64_t rows, int64_t k, int64_t ldq, const float* scale, int8_t* q,
                                 cudaStream_t st) {
  const int64_t work = rows * (ldq >> 4);
  if (work <= 0) return;
  k_quantize_rows<true><<<grid_for(work, kThreads, 148 * 32), kThreads, 0, st>>>(x, rows, k, ldq, nullptr, scale, q,
                                                                                 nullptr);
}

// Per-image absmax over the pixels a strided conv reads, VEC consecutive columns per
// thread (w a multiple of VEC, so they share a row): lanes on rows the conv never
// reads issue no load, so only the covered rows' sectors are fetched.  grid.y strides
// over the images; the masks are staged in shared memory.
template <int VEC>
__global__ void __launch_bounds__(kThreads) k_image_absmax_cov(const float* __restrict__ x, int64_t n, int32_t c,
                                                               int32_t h, int32_t w,
                                                               const uint8_t* __restrict__ row_cov,
                                                               const uint8_t* __restrict__ col_cov,
                                                               unsigned* __restrict__ amax) {
  extern __shared__ uint8_t cov_s[];  // [h] rows then [w] columns
  for (int32_t i = threadIdx.x; i < h + w; i += kThreads) cov_s[i] = i < h ? row_cov[i] : col_cov[i - h];
  __syncthreads();
  const int32_t groups = c * h * (w / VEC);  // VEC-column groups per image
  const int32_t gpr = w / VEC;
  for (int64_t img = blockIdx.y; img < n; img += gridDim.y) {
    const float* xi = x + img * (int64_t)c * h * w;
    float m = 0.0f;
    const int32_t stride = gridDim.x * kThreads;
    for (int32_t g0 = blockIdx.x * kThreads + threadIdx.x; g0 < groups; g0 += 4 * stride) {
      // four groups' loads in flight before any of them is folded in
      float v[4][VEC];
      int32_t col[4];
      bool ok[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int32_t gi = g0 + u * stride;
        const int32_t rr = gi / gpr;
        col[u] = (gi - rr * gpr) * VEC;
        ok[u] = gi < groups && cov_s[rr % h];
        const float* p = xi + (int64_t)rr * w + col[u];
        if (!ok[u]) {
#pragma unroll
          for (int k = 0; k < VEC; ++k) v[u][k] = 0.0f;
        } else if (VEC == 4) {
          const float4 a = __ldg(reinterpret_cast<const float4*>(p));
          v[u][0] = a.x; v[u][VEC > 1 ? 1 : 0] = a.y; v[u][VEC > 2 ? 2 : 0] = a.z; v[u][VEC > 3 ? 3 : 0] = a.w;
        } else if (VEC == 2) {
          const float2 a = __ldg(reinterpret_cast<const float2*>(p));
          v[u][0] = a.x; v[u][VEC > 1 ? 1 : 0] = a.y;
        } else {
          v[u][0] = __ldg(p);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int k = 0; k < VEC; ++k)
          if (ok[u] && cov_s[h + col[u] + k]) m = fmaxf(m, fabsf(v[u][k]));
    }
    block_max_to(m, amax + img);
    __syncthreads();  // the reduction buffer is reused by the next image
  }
}

void launch_image_absmax(const float* x, int64_t n, int32_t c, int32_t h, int32_t w,
                         const uint8_t* row_cov, const uint8_t* col_cov, unsigned* amax_bits,
                         cudaStream_t st) {
  const int64_t per = (int64_t)c * h * w;
  if (n <= 0 || per <= 0) return;
  if (row_cov && h + w <= 32 * 1024 && per < ((int64_t)1 << 30)) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(x);
    const int vec = (w % 4 == 0 && (a & 15) == 0) ? 4 : (w % 2 == 0 && (a & 7) == 0) ? 2 : 1;
    const int64_t groups = per / vec;
    dim3 grid(grid_for(groups, kThreads * 4, 256), (unsigned)std::min<int64_t>(n, 65535));
    const size_t sm = (size_t)(h + w);
    if (vec == 4) k_image_absmax_cov<4><<<grid, kThreads, sm, st>>>(x, n, c, h, w, row_cov, col_cov, amax_bits);
    else if (vec == 2) k_image_absmax_cov<2><<<grid, kThreads, sm, st>>>(x, n, c, h, w, row_cov, col_cov, amax_bits);
    else k_image_absmax_cov<1><<<grid, kThreads, sm, st>>>(x, n, c, h, w, row_cov, col_cov, amax_bits);
    return;
  }
  const int64_t work = row_cov ? (int64_t)c * h * 32 : per;  // lanes in use per image
  dim3 grid(grid_for(work, kThreads * 8, 64), (unsigned)std::min<int64_t>(n, 65535));
  const bool cov_smem = row_cov && h + w <= 32 * 1024;  // the masks fit the default shared memory
  k_image_absmax<<<grid, kThreads, cov_smem ? (size_t)(h + w) : 0, st>>>(x, n, c, h, w, row_cov, col_cov,
                                                                           cov_smem, amax_bits);
}

void launch_image_quantize_planar16(const float* x, int64_t n, int32_t c, int32_t h, int32_t w, int32_t cpad,
                                    bool bounded, const unsigned* amax_bits, int8_t* q, float* scales_out,
                                    cudaStream_t st) {
  const int32_t hw = h * w;
  if (n <= 0 || hw <= 0) return;
  launch_g16<true>(x, n, c, hw, cpad, bounded, amax_bits, q, scales_out, st);
}

void launch_image_quantize_subsampled(const float* x, int64_t n, int32_t c, int32_t h, int32_t w, int32_t s,
                                      int32_t oh, int32_t ow, int32_t cpad, bool planar, const unsigned* amax_bits,
                                      int8_t* q, float* scales_out, cudaStream_t st) {
  const int32_t ohw = oh * ow;
  if (n <= 0 || ohw <= 0) return;
  const dim3 grid((unsigned)std::min<int64_t>((ohw + 255) / 256, 1024), (unsigned)(cpad / 16), (unsigned)n);
  if (planar)
    k_image_quantize_sub16<true><<<grid, 256, 0, st>>>(x, c, h, w, s, oh, ow, cpad, amax_bits, q, scales_out);
  else
    k_image_quantize_sub16<false><<<grid, 256, 0, st>>>(x, c, h, w, s, oh, ow, cpad, amax_bits, q, scales_out);
}

void launch_image_quantize_s2d_planar(const float* x, int64_t n, int32_t c, int32_t h, int32_t w, int32_t cpad,
                                      const unsigned* amax_bits, int8_t* q, float* scales_out, cudaStream_t st) {
  const int32_t hw2 = ((h + 1) / 2) * ((w + 1) / 2);
  if (n <= 0 || hw2 <= 0) return;
  const dim3 grid((unsigned)std::min<int64_t>((hw2 + 255) / 256, 1024), (unsigned)(4 * cpad / 16), (unsigned)n);
  k_image_quantize_s2d16<<<grid, 256, 0, st>>>(x, c, h, w, cpad, amax_bits, q, scales_out);
}

void launch_image_quantize_s2d(const float* x, int64_t n, int32_t c, int32_t h, int32_t w, const unsigned* amax_bits,
                               int8_t* q, float* scales_out, cudaStream_t st) {
  const int32_t hw2 = (h / 2) * (w / 2);
  if (n <= 0 || hw2 <= 0) return;
  const dim3 grid((unsigned)std::min<int64_t>((hw2 + kThreads - 1) / kThreads, 64),
                  (unsigned)std::min<int64_t>(n, 65535));
  k_image_quantize_s2d<<<grid, kThreads, 0, st>>>(x, n, c, h, w, amax_bits, q, scales_out);
}

void launch_image_quantize_nhwc(const float* x, int64_t n, int32_t c, int32_t h, int32_t w,
                                int32_t cpad, bool bounded, const unsigned* amax_bits, int8_t* q,
                                float* scales_out, cudaStream_t st) {
  const int64_t total = n * (int64_t)h * w;
  if (total <= 0) return;
  if (cpad == 4 && c <= 4) {
    const int32_t hw = h * w;
    const dim3 grid((unsigned)std::min<int64_t>((hw + kThreads - 1) / kThreads, 64),
                    (unsigned)std::min<int64_t>(n, 65535));
    k_image_quantize_nhwc4<<<grid, kThreads, 0, st>>>(x, n, c, hw, amax_bits, q, scales_out);
    return;
  }
  if ((cpad & 15) == 0 && n <= 65535) {
    launch_g16<false>(x, n, c, h * w, cpad, bounded, amax_bits, q, scales_out, st);
    return;
  }
  k_image_quantize_nhwc<<<grid_for(total, kThreads, 148 * 32), kThreads, 0, st>>>(
      x, n, c, h * w, cpad, amax_bits, q, scales_out);
}

void launch_nhwc_to_nchw_i8(const int8_t* q, int64_t n, int32_t c, int32_t cpad, int32_t h,
                            int32_t w, int8_t* out, cudaStream_t st) {
  const int64_t total = n * (int64_t)c * h * w;
  if (total <= 0) return;
  k_nhwc_to_nchw_i8<<<grid_for(total, kThreads, 148 * 32), kThreads, 0, st>>>(q, n, c, cpad, h * w, out);
}

}  // namespace rg
