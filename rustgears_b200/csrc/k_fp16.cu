// k_fp16.cu -- the FP16 arm of the NPU executor (ExecutionProvider::npu_fp16()).
//
// Reference: fp16_gemm_fused_into (src/inference/npu.rs:431-445), used by FusedLinear
// (npu.rs:317) and, over each image's transposed im2col matrix, by FusedConv2d
// (npu.rs:351-353, 372-374):
//   acc = 0; for k in order: acc += round_fp16(a[r,k]) * w[c,k]   (f32, no FMA)
//   out[r,c] = act(round_fp16(acc + bias[c]))
// with w rounded by round_fp16 at compile time (npu.rs:210, 232), except the
// diagonal Linear of a standalone ChannelAffine, whose weights stay unrounded
// (npu.rs:258-268).
//
// Exactness: two values with 11 significant bits multiply exactly in f32 (22 bits;
// round_fp16 flushes magnitudes below 2^-14 and clamps above 65504, so the product
// is a normal f32), so round(p + acc) of an FMA equals the reference's separately
// rounded product and sum.  Where the weights are fp16 values the kernel chains FMAs
// in k order; otherwise (the affine diagonal) it multiplies and adds separately.
// Zero operands (padding, K tails, flushed values) add +0 or -0 to an accumulator that
// is never -0, so they change nothing and the padded tiles stay exact.
//
// Register-tiled f32 GEMM on the CUDA cores: 64 x 64 output tiles, 256 threads with
// 4 x 4 outputs each, 16-deep K slices staged in shared memory (A rounded as it is
// staged), the next slice's global loads in flight while the current one is used.
// A convolution is the same GEMM over rows (image, oy, ox) and the reference's im2col
// order k = (c, ky, kx), gathered from the NCHW input; outputs go to NCHW.
#include <cuda_runtime.h>

#include "rg_kernels.h"
#include "rg_math.cuh"

namespace rg {
namespace {

constexpr int TM = 64, TN = 64, TK = 16, kThreads = 256;

struct Fp16Params {
  Fp16Args a;
  int64_t L;  // conv: output pixels per image
};

template <bool CONV>
__device__ __forceinline__ void load_a(const Fp16Params& P, int64_t row, int64_t k0, float (&v)[4]) {
  const Fp16Args& a = P.a;
  if (!CONV) {
    const float* src = a.x + row * a.k;
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = (row < a.m && k0 + q < a.k) ? __ldg(src + k0 + q) : 0.0f;
    return;
  }
  if (row >= a.m) {
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = 0.0f;
    return;
  }
  const int64_t img = row / P.L;
  const int32_t l = (int32_t)(row - img * P.L);
  const int32_t oy = l / a.ow, ox = l - oy * a.ow;
  const int32_t iy0 = oy * a.stride - a.pad, ix0 = ox * a.stride - a.pad;
  const float* base = a.x + img * (int64_t)a.c * a.h * a.w;
  const int32_t kk2 = a.ks * a.ks;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int64_t kk = k0 + q;
    float val = 0.0f;
    if (kk < a.k) {
      const int32_t c = (int32_t)(kk / kk2), rem = (int32_t)(kk - (int64_t)c * kk2);
      const int32_t ky = rem / a.ks, kx = rem - ky * a.ks;
      const int32_t iy = iy0 + ky, ix = ix0 + kx;
      if (iy >= 0 && iy < a.h && ix >= 0 && ix < a.w) val = __ldg(base + ((int64_t)c * a.h + iy) * a.w + ix);
    }
    v[q] = val;
  }
}

__device__ __forceinline__ void load_w(const Fp16Params& P, int64_t col, int64_t k0, float (&v)[4]) {
  const Fp16Args& a = P.a;
  const float* src = a.wt + col * a.k;
#pragma unroll
  for (int q = 0; q < 4; ++q) v[q] = (col < a.n && k0 + q < a.k) ? __ldg(src + k0 + q) : 0.0f;
}

template <bool CONV, bool EXACT>
__global__ void __launch_bounds__(kThreads) k_fp16_gemm(const Fp16Params P) {
  __shared__ __align__(16) float As[TK][TM];
  __shared__ __align__(16) float Ws[TK][TN];
  const Fp16Args& a = P.a;
  const int tid = threadIdx.x;
  const int ty = tid >> 4, tx = tid & 15;      // 4 x 4 outputs: rows 4 ty.., columns 4 tx..
  const int lr = tid & 63, lq = tid >> 6;      // staging: row / column lr, K quarter lq
  const int64_t m0 = (int64_t)blockIdx.x * TM, n0 = (int64_t)blockIdx.y * TN;
  const int64_t ktiles = (a.k + TK - 1) / TK;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
  float va[4], vw[4];
  load_a<CONV>(P, m0 + lr, lq * 4, va);
  load_w(P, n0 + lr, lq * 4, vw);
  for (int64_t t = 0; t < ktiles; ++t) {
    __syncthreads();  // the previous slice has been used
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      As[lq * 4 + q][lr] = round_fp16(va[q]);
      Ws[lq * 4 + q][lr] = vw[q];
    }
    __syncthreads();
    if (t + 1 < ktiles) {
      load_a<CONV>(P, m0 + lr, (t + 1) * TK + lq * 4, va);
      load_w(P, n0 + lr, (t + 1) * TK + lq * 4, vw);
    }
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      const float4 av = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
      const float4 wv = *reinterpret_cast<const float4*>(&Ws[kk][tx * 4]);
      const float ar[4] = {av.x, av.y, av.z, av.w}, wr[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          acc[i][j] = EXACT ? __fmaf_rn(ar[i], wr[j], acc[i][j]) : __fadd_rn(acc[i][j], __fmul_rn(ar[i], wr[j]));
    }
  }
  // epilogue: act(round_fp16(acc + bias)), row-major [m, n] or NCHW
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t row = m0 + ty * 4 + i;
    if (row >= a.m) continue;
    int64_t obase;
    int64_t cstride;
    if (CONV) {
      const int64_t img = row / P.L, l = row - img * P.L;
      obase = img * a.n * P.L + l;
      cstride = P.L;
    } else {
      obase = row * a.n;
      cstride = 1;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t col = n0 + tx * 4 + j;
      if (col >= a.n) continue;
      const float v = round_fp16(__fadd_rn(acc[i][j], __ldg(a.bias + col)));
      a.out[obase + col * cstride] = act_apply(a.act, a.act_param, v);
    }
  }
}

}  // namespace

void launch_fp16_gemm(const Fp16Args& a, cudaStream_t st) {
  if (a.m <= 0 || a.n <= 0) return;
  Fp16Params P;
  P.a = a;
  P.L = a.conv ? (int64_t)a.oh * a.ow : 0;
  const dim3 grid((unsigned)((a.m + TM - 1) / TM), (unsigned)((a.n + TN - 1) / TN));
  if (a.conv) {
    if (a.exact) k_fp16_gemm<true, true><<<grid, kThreads, 0, st>>>(P);
    else k_fp16_gemm<true, false><<<grid, kThreads, 0, st>>>(P);
  } else {
    if (a.exact) k_fp16_gemm<false, true><<<grid, kThreads, 0, st>>>(P);
    else k_fp16_gemm<false, false><<<grid, kThreads, 0, st>>>(P);
  }
}

}  // namespace rg
