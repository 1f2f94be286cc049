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
// The same kernel in its second mode runs the f32 ExecutionProvider::Cpu arm
// (run_standard, src/inference/mod.rs:260-331): the reference's CPU matmul
// (src/device/cpu.rs:43-64, 233-395) gives every output an FMA chain in k order from 0,
// except the matmul's output columns past the last full 8-wide block, which accumulate
// unfused (c += a * b); the bias is added afterwards (one rounding), no activation.
// The matmul's columns are a Linear's output features, and a conv's output pixels
// (W[O, C k k] @ cols[C k k, L] per image, src/kernels.rs:218-263).
//
// Register-tiled f32 GEMM on the CUDA cores: 256 threads with 4 x 4 outputs each,
// the tile as wide as the layer needs (16, 32 or 64 columns over 256, 128 or 64 rows),
// 16-deep K slices staged in shared memory (A rounded as it is staged), the next
// slice's global loads in flight while the current one is used.  A convolution is
// the same GEMM over rows (image, oy, ox) and the reference's im2col order
// k = (c, ky, kx), gathered from the NCHW input through a per-CTA table of the
// (c, ky, kx) offsets; a thread's rows are spread across the warp's lanes so that
// both the gathers and the NCHW stores of one instruction touch consecutive pixels.
#include <cuda_runtime.h>

#include <algorithm>

#include "rg_kernels.h"
#include "rg_math.cuh"

namespace rg {
namespace {

constexpr int TK = 16, kThreads = 256;
constexpr int64_t kMaxConvK = 16384;  // table of (c, ky, kx) offsets: 8 bytes per k in shared memory

struct Fp16Params {
  Fp16Args a;
  int64_t L;  // conv: output pixels per image
};

// MODE 0: FP16 arm (EXACT: FMA chains, else separate product and sum); MODE 1: f32 arm.
// POOL (conv): the 2 x 2 / stride 2 max-pool after the conv in the same kernel (the f32
// arm: after the conv and its standalone activation, applied to each pixel first).
// Rows are then (pool window, position): a tile holds TY windows, and the 4 rows of a
// thread (ty + TY i) are the window's pixels in the pool's scan order (dy, dx), so the
// thread finishes the window from its own accumulators: the epilogue of each pixel,
// then the reference's max (a larger value or a NaN replaces the best; first of ties).
// ACTC (POOL): the activation fixed at compile time (ReLU or none), or -1: chosen at run
// time; a fixed one keeps the 16 unrolled pooled epilogues free of the other kinds' code.
template <int TX, bool CONV, bool EXACT, int MODE = 0, bool POOL = false, int ACTC = -1>
__global__ void __launch_bounds__(kThreads) k_fp16_gemm(const Fp16Params P) {
  constexpr int TY = kThreads / TX, TM = 4 * TY, TN = 4 * TX;
  constexpr int KPT = TK * TM / kThreads;  // A values one thread stages per slice
  constexpr int WPT = TK * TN / kThreads;  // weights one thread stages per slice
  __shared__ __align__(16) float As[TK][TM];
  __shared__ __align__(16) float Ws[TK][TN];
  extern __shared__ int2 ktab[];           // conv: {c H W + ky W + kx, ky << 16 | kx} per k
  const Fp16Args& a = P.a;
  const int tid = threadIdx.x;
  const int ty = tid / TX, tx = tid % TX;
  const int lr = tid % TM, ak = (tid / TM) * KPT;  // staged A row and first k of the slice
  const int lc = tid % TN, wk = (tid / TN) * WPT;  // staged weight row (output column) and first k
  const int64_t m0 = (int64_t)blockIdx.x * TM, n0 = (int64_t)blockIdx.y * TN;
  const int64_t ktiles = (a.k + TK - 1) / TK;
  const int64_t row = m0 + lr;
  // (POOL: the staged row's window must exist; its 4 positions always do)
  const bool row_ok = POOL ? ((int64_t)blockIdx.x * TY + lr % TY) * 4 < a.m : row < a.m;
  // the staged row: a Linear row, or the output pixel whose receptive field is gathered
  const float* arow = nullptr;
  int32_t iy0 = 0, ix0 = 0;
  if (CONV) {
    for (int64_t kk = tid; kk < a.k; kk += kThreads) {
      const int32_t k2 = a.ks * a.ks;
      const int32_t c = (int32_t)(kk / k2), rem = (int32_t)(kk - (int64_t)c * k2);
      const int32_t ky = rem / a.ks, kx = rem - ky * a.ks;
      ktab[kk] = make_int2((c * a.h + ky) * a.w + kx, (ky << 16) | kx);
    }
    if (POOL && row_ok) {  // row lr of the tile: window lr % TY, position lr / TY
      const int pos = lr / TY;
      const uint32_t gw = (uint32_t)blockIdx.x * TY + (uint32_t)(lr % TY);
      const uint32_t per_img = (uint32_t)a.ph * (uint32_t)a.pw;
      const uint32_t img = gw / per_img, wr = gw - img * per_img;
      const int32_t py = (int32_t)(wr / (uint32_t)a.pw), px = (int32_t)(wr - (uint32_t)py * (uint32_t)a.pw);
      iy0 = (2 * py + (pos >> 1)) * a.stride - a.pad;
      ix0 = (2 * px + (pos & 1)) * a.stride - a.pad;
      arow = a.x + img * (int64_t)a.c * a.h * a.w;
    } else if (row_ok) {  // rows < 2^31 (checked at launch): 32-bit division
      const uint32_t img = (uint32_t)row / (uint32_t)P.L;
      const int32_t l = (int32_t)((uint32_t)row - img * (uint32_t)P.L);
      const int32_t oy = l / a.ow, ox = l - oy * a.ow;
      iy0 = oy * a.stride - a.pad;
      ix0 = ox * a.stride - a.pad;
      arow = a.x + img * (int64_t)a.c * a.h * a.w;
    }
    __syncthreads();
  } else if (row_ok) {
    arow = a.x + row * a.k;
  }
  const int64_t corner = (int64_t)iy0 * a.w + ix0;  // conv: offset of tap (0, 0) of channel 0
  auto load_a = [&](int64_t k0, float (&v)[KPT]) {
#pragma unroll
    for (int q = 0; q < KPT; ++q) {
      const int64_t kk = k0 + q;
      float val = 0.0f;
      if (row_ok && kk < a.k) {
        if (CONV) {
          const int2 e = ktab[kk];
          const int32_t iy = iy0 + (e.y >> 16), ix = ix0 + (e.y & 0xffff);
          if (iy >= 0 && iy < a.h && ix >= 0 && ix < a.w) val = __ldg(arow + corner + e.x);
        } else {
          val = __ldg(arow + kk);
        }
      }
      v[q] = val;
    }
  };
  const float* wrow = a.wt + (n0 + lc) * a.k;
  const bool col_ok = n0 + lc < a.n;
  auto load_w = [&](int64_t k0, float (&v)[WPT]) {
#pragma unroll
    for (int q = 0; q < WPT; ++q) v[q] = (col_ok && k0 + q < a.k) ? __ldg(wrow + k0 + q) : 0.0f;
  };
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
  // f32 arm: which of this thread's outputs take the FMA chain (matmul column in a full
  // 8-wide block): a Linear's columns 4 tx.. share one answer (blocks of 8 align with 4);
  // a conv's rows are pixels, each with its own
  bool fuse[4] = {true, true, true, true};
  bool all_fused = true;
  if (MODE == 1) {
    if (CONV && POOL) {  // the pixel of row ty + TY i: position i of window blockIdx.x * TY + ty
      const int64_t nvL = P.L / 8 * 8;
      const uint32_t gw = (uint32_t)blockIdx.x * TY + (uint32_t)ty;
      const uint32_t per_img = (uint32_t)a.ph * (uint32_t)a.pw;
      const uint32_t wr = gw % per_img;
      const int32_t py = (int32_t)(wr / (uint32_t)a.pw), px = (int32_t)(wr % (uint32_t)a.pw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t l = (int64_t)(2 * py + (i >> 1)) * a.ow + 2 * px + (i & 1);
        fuse[i] = l < nvL;
        all_fused = all_fused && fuse[i];
      }
    } else if (CONV) {
      const int64_t nvL = P.L / 8 * 8;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t r = m0 + ty + TY * i;
        fuse[i] = (r % P.L) < nvL;
        all_fused = all_fused && fuse[i];
      }
    } else {
      const bool f = n0 + tx * 4 < a.n / 8 * 8;
#pragma unroll
      for (int i = 0; i < 4; ++i) fuse[i] = f;
      all_fused = f;
    }
  }
  float va[KPT], vw[WPT];
  load_a(ak, va);
  load_w(wk, vw);
  for (int64_t t = 0; t < ktiles; ++t) {
    __syncthreads();  // the previous slice has been used
#pragma unroll
    for (int q = 0; q < KPT; ++q) As[ak + q][lr] = MODE == 1 ? va[q] : round_fp16(va[q]);
#pragma unroll
    for (int q = 0; q < WPT; ++q) Ws[wk + q][lc] = vw[q];
    __syncthreads();
    if (t + 1 < ktiles) {
      load_a((t + 1) * TK + ak, va);
      load_w((t + 1) * TK + wk, vw);
    }
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float ar[4];
      if (CONV) {  // rows ty + TY i: consecutive pixels across the warp
#pragma unroll
        for (int i = 0; i < 4; ++i) ar[i] = As[kk][ty + TY * i];
      } else {     // rows 4 ty + i
        const float4 av = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
        ar[0] = av.x; ar[1] = av.y; ar[2] = av.z; ar[3] = av.w;
      }
      const float4 wv = *reinterpret_cast<const float4*>(&Ws[kk][tx * 4]);
      const float wr[4] = {wv.x, wv.y, wv.z, wv.w};
      if (MODE == 1 && !all_fused) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            acc[i][j] = fuse[i] ? __fmaf_rn(ar[i], wr[j], acc[i][j]) : __fadd_rn(acc[i][j], __fmul_rn(ar[i], wr[j]));
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            acc[i][j] = EXACT ? __fmaf_rn(ar[i], wr[j], acc[i][j]) : __fadd_rn(acc[i][j], __fmul_rn(ar[i], wr[j]));
      }
    }
  }
  if (POOL) {  // the thread's window: blockIdx.x * TY + ty
    const uint32_t gw = (uint32_t)blockIdx.x * TY + (uint32_t)ty;
    if ((int64_t)gw * 4 >= a.m) return;
    const uint32_t per_img = (uint32_t)a.ph * (uint32_t)a.pw;
    const uint32_t img = gw / per_img, wr = gw - img * per_img;
    float* o = a.out + (int64_t)img * a.n * per_img + wr;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t col = n0 + tx * 4 + j;
      if (col >= a.n) continue;
      const float b = __ldg(a.bias + col);
      float best = -INFINITY;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        // the f32 arm: matmul + bias, then its activation op; the FP16 arm: its epilogue
        const float pre = MODE == 1 ? __fadd_rn(acc[i][j], b) : round_fp16(__fadd_rn(acc[i][j], b));
        const float v = act_apply(ACTC >= 0 ? ACTC : a.act, a.act_param, pre);
        if (v > best || v != v) best = v;
      }
      o[col * per_img] = best;
    }
    return;
  }
  // epilogue: act(round_fp16(acc + bias)), row-major [m, n] or NCHW
  uint32_t img_e = 0, l_e = 0;  // conv: (image, pixel) of row m0 + ty, advanced by TY per i
  if (CONV) {
    img_e = (uint32_t)(m0 + ty) / (uint32_t)P.L;
    l_e = (uint32_t)(m0 + ty) - img_e * (uint32_t)P.L;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = m0 + (CONV ? ty + TY * i : ty * 4 + i);
    if (CONV && i > 0) {
      l_e += TY;
      while (l_e >= (uint32_t)P.L) { l_e -= (uint32_t)P.L; ++img_e; }
    }
    if (r >= a.m) continue;
    int64_t obase, cstride;
    if (CONV) {
      obase = (int64_t)img_e * a.n * P.L + l_e;
      cstride = P.L;
    } else {
      obase = r * a.n;
      cstride = 1;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t col = n0 + tx * 4 + j;
      if (col >= a.n) continue;
      if (MODE == 1) {  // matmul, then `+= bias` (mod.rs:270-274, 285-291)
        a.out[obase + col * cstride] = __fadd_rn(acc[i][j], __ldg(a.bias + col));
        continue;
      }
      const float v = round_fp16(__fadd_rn(acc[i][j], __ldg(a.bias + col)));
      a.out[obase + col * cstride] = act_apply(a.act, a.act_param, v);
    }
  }
}

template <int TX, int ACTC>
void launch_pool(const Fp16Params& P, dim3 grid, size_t smem, cudaStream_t st, bool& ok) {
  const Fp16Args& a = P.a;
  auto kern = a.f32 ? k_fp16_gemm<TX, true, true, 1, true, ACTC>
              : a.exact ? k_fp16_gemm<TX, true, true, 0, true, ACTC> : k_fp16_gemm<TX, true, false, 0, true, ACTC>;
  if (smem > 48 * 1024 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
    ok = false;
    return;
  }
  kern<<<grid, kThreads, smem, st>>>(P);
}

template <int TX>
bool launch_tx(const Fp16Params& P, cudaStream_t st) {
  const Fp16Args& a = P.a;
  constexpr int TM = 4 * (kThreads / TX), TN = 4 * TX;
  const dim3 grid((unsigned)((a.m + TM - 1) / TM), (unsigned)((a.n + TN - 1) / TN));
  if (a.conv && a.pool) {
    const size_t smem = (size_t)a.k * sizeof(int2);
    bool ok = true;
    if (a.act == ACT_RELU) launch_pool<TX, ACT_RELU>(P, grid, smem, st, ok);
    else if (a.act == ACT_NONE) launch_pool<TX, ACT_NONE>(P, grid, smem, st, ok);
    else launch_pool<TX, -1>(P, grid, smem, st, ok);
    return ok;
  }
  if (a.conv) {
    const size_t smem = (size_t)a.k * sizeof(int2);
    auto kern = a.f32 ? k_fp16_gemm<TX, true, true, 1> : a.exact ? k_fp16_gemm<TX, true, true> : k_fp16_gemm<TX, true, false>;
    if (smem > 48 * 1024 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return false;
    kern<<<grid, kThreads, smem, st>>>(P);
  } else {
    auto kern = a.f32 ? k_fp16_gemm<TX, false, true, 1> : a.exact ? k_fp16_gemm<TX, false, true> : k_fp16_gemm<TX, false, false>;
    kern<<<grid, kThreads, 0, st>>>(P);
  }
  return true;
}

// ChannelAffine of the f32 arm (mod.rs:293-303): v * scale[ch] + shift[ch] over
// [n][c][inner], product and sum rounded separately.
__global__ void k_channel_affine(const float* __restrict__ x, int64_t total, int64_t c, int64_t inner,
                                 const float* __restrict__ scale, const float* __restrict__ shift, float* y) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t ch = (i / inner) % c;
    y[i] = __fadd_rn(__fmul_rn(x[i], __ldg(scale + ch)), __ldg(shift + ch));
  }
}

}  // namespace

void launch_channel_affine(const float* x, int64_t total, int64_t c, int64_t inner, const float* scale,
                           const float* shift, float* y, cudaStream_t st) {
  if (total <= 0) return;
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 16);
  k_channel_affine<<<(unsigned)blocks, 256, 0, st>>>(x, total, c, inner, scale, shift, y);
}

bool launch_fp16_gemm(const Fp16Args& a, cudaStream_t st) {
  if (a.m <= 0 || a.n <= 0) return true;
  if (a.conv && (a.k > kMaxConvK || a.h >= 65536 || a.w >= 65536 || a.ks >= 65536 ||
                 (int64_t)a.c * a.h * a.w >= ((int64_t)1 << 31) || a.m + 1024 >= ((int64_t)1 << 31)))
    return false;
  if (a.pool && (!a.conv || a.ph <= 0 || a.pw <= 0 || a.m % 4 != 0)) return false;
  Fp16Params P;
  P.a = a;
  P.L = a.conv ? (int64_t)a.oh * a.ow : 0;
  // as wide as the layer: 16, 32 or 64 output columns per tile
  if (a.n <= 16) return launch_tx<4>(P, st);
  if (a.n <= 32) return launch_tx<8>(P, st);
  return launch_tx<16>(P, st);
}

}  // namespace rg
