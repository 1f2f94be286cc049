// k_gemm_simt.cu -- i8 x i8 -> i32 GEMM on the CUDA cores (dp4a) with the fused
// dequant + bias + activation epilogue.
//
// Reference: int8_gemm_fused / int8_gemm_fused_serial / dot_i8
// (src/inference/quantize.rs:68-144).  Used for shapes too small or too
// ragged for the tensor-core kernel (K = 4, N = 3, ...) and for every Conv2d
// as an implicit GEMM: the A operand is gathered on the fly from the
// per-image-quantized NHWC i8 activation (rows = (image, oy, ox), reduction =
// (ky, kx, c)), replacing the reference's im2col + transpose + quantize.
#include <algorithm>

#include "rg_kernels.h"
#include "rg_math.cuh"

namespace rg {
namespace {

constexpr int BM = 64, BN = 64, BKW = 8;  // tile: 64 x 64 outputs, 32 bytes of K per stage
constexpr int kThreads = 256;

struct RowCtx {    // per-row gather state for the implicit-GEMM A operand
  const int8_t* base;  // image base (NHWC)
  int32_t iy0, ix0;    // top-left input coordinate of the window
  bool valid;
};

__device__ __forceinline__ RowCtx make_row(const GemmArgs& p, int64_t r) {
  RowCtx rc;
  rc.valid = r < p.m;
  if (!p.conv) {
    rc.base = p.a + (rc.valid ? r : 0) * p.lda;
    rc.iy0 = rc.ix0 = 0;
    return rc;
  }
  const int64_t L = (int64_t)p.g.oh * p.g.ow;
  const int64_t rr = rc.valid ? r : 0;
  const int64_t img = rr / L;
  const int32_t l = (int32_t)(rr - img * L);
  const int32_t oy = l / p.g.ow, ox = l - oy * p.g.ow;
  rc.base = p.a + img * (int64_t)p.g.h * p.g.w * p.g.cpad;
  rc.iy0 = oy * p.g.stride - p.g.pad;
  rc.ix0 = ox * p.g.stride - p.g.pad;
  return rc;
}

// 4 consecutive reduction bytes [kk, kk+4) of row rc.
__device__ __forceinline__ int32_t load_a_word(const GemmArgs& p, const RowCtx& rc, int64_t kk) {
  if (!rc.valid || kk >= p.k) return 0;
  if (!p.conv) return __ldg(reinterpret_cast<const int32_t*>(rc.base + kk));
  // K order (ky, kx, c) with kxp taps per kernel row (taps kx >= k are zero padding)
  const int32_t C = p.g.c, kw = p.g.k, kxp = p.g.kxp ? p.g.kxp : p.g.k;
  const int64_t kreal = (int64_t)kw * kxp * C;
  if ((C & 3) == 0) {
    if (kk >= kreal) return 0;
    const int32_t tap = (int32_t)(kk / C), ch = (int32_t)(kk - (int64_t)tap * C);
    const int32_t ky = tap / kxp, kx = tap - ky * kxp;
    const int32_t iy = rc.iy0 + ky, ix = rc.ix0 + kx;
    if (kx >= kw || iy < 0 || iy >= p.g.h || ix < 0 || ix >= p.g.w) return 0;
    return __ldg(reinterpret_cast<const int32_t*>(rc.base + ((int64_t)iy * p.g.w + ix) * p.g.cpad + ch));
  }
  uint32_t wv = 0;
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const int64_t kb = kk + b;
    if (kb >= kreal) break;
    const int32_t tap = (int32_t)(kb / C), ch = (int32_t)(kb - (int64_t)tap * C);
    const int32_t ky = tap / kxp, kx = tap - ky * kxp;
    const int32_t iy = rc.iy0 + ky, ix = rc.ix0 + kx;
    if (kx >= kw || iy < 0 || iy >= p.g.h || ix < 0 || ix >= p.g.w) continue;
    const int8_t v = rc.base[((int64_t)iy * p.g.w + ix) * p.g.cpad + ch];
    wv |= (uint32_t)(uint8_t)v << (8 * b);
  }
  return (int32_t)wv;
}

__device__ __forceinline__ void flush_max(unsigned* base, int64_t slot, float v) {
  // Warp-aggregated atomicMax when the whole warp targets the same slot.
  const int64_t s0 = __shfl_sync(0xffffffffu, slot, 0);
  if (__all_sync(0xffffffffu, slot == s0)) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0 && v > 0.0f) atomicMax(base + s0, __float_as_uint(v));
  } else if (slot >= 0 && v > 0.0f) {
    atomicMax(base + slot, __float_as_uint(v));
  }
}

template <int ACT>
__global__ void __launch_bounds__(kThreads) k_gemm_simt(const GemmArgs p) {
  __shared__ __align__(16) int32_t As[BKW][BM];
  __shared__ __align__(16) int32_t Bs[BKW][BN];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = (int64_t)blockIdx.x * BM, n0 = (int64_t)blockIdx.y * BN;

  // Each thread stages 2 A words and 2 B words per K step: rows lr and lr + 32, word lw.
  const int lr = tid >> 3, lw = tid & 7;
  const RowCtx ra0 = make_row(p, m0 + lr), ra1 = make_row(p, m0 + lr + 32);
  const bool vb0 = n0 + lr < p.n, vb1 = n0 + lr + 32 < p.n;
  const int8_t* wb0 = p.w + (vb0 ? n0 + lr : 0) * p.ldb;
  const int8_t* wb1 = p.w + (vb1 ? n0 + lr + 32 : 0) * p.ldb;

  int32_t acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0;

  for (int64_t k0 = 0; k0 < p.k; k0 += BKW * 4) {
    const int64_t kk = k0 + lw * 4;
    const int32_t a0 = load_a_word(p, ra0, kk), a1 = load_a_word(p, ra1, kk);
    const int32_t b0 = (vb0 && kk < p.k) ? __ldg(reinterpret_cast<const int32_t*>(wb0 + kk)) : 0;
    const int32_t b1 = (vb1 && kk < p.k) ? __ldg(reinterpret_cast<const int32_t*>(wb1 + kk)) : 0;
    __syncthreads();
    As[lw][lr] = a0; As[lw][lr + 32] = a1;
    Bs[lw][lr] = b0; Bs[lw][lr + 32] = b1;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < BKW; ++w) {
      const int4 av = *reinterpret_cast<const int4*>(&As[w][ty * 4]);
      const int4 bv = *reinterpret_cast<const int4*>(&Bs[w][tx * 4]);
      const int32_t a[4] = {av.x, av.y, av.z, av.w};
      const int32_t b[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __dp4a(a[i], b[j], acc[i][j]);
    }
  }

  // Fused epilogue: act((acc as f32) * (sa * sw) + bias[c]).
  float mx_lo = 0.0f, mx_hi = 0.0f;
  int64_t slot_lo = -1, slot_hi = -1;
  const int64_t L = p.out_l;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = m0 + ty * 4 + i;
    if (r >= p.m) continue;
    const float sa = p.a_scale[p.rows_per_scale ? r / p.rows_per_scale : 0];
    int64_t rowbase, colstride;
    if (L) {
      const int64_t img = r / L;
      rowbase = img * p.n * L + (r - img * L);
      colstride = L;
    } else {
      rowbase = r * p.n;
      colstride = 1;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t c = n0 + tx * 4 + j;
      if (c >= p.n) continue;
      const float sw = p.w_scale_ch ? p.w_scale_ch[c] : p.w_scale;
      const float cs = __fmul_rn(sa, sw);
      const float v = epilogue_t<ACT>(acc[i][j], cs, p.bias[c], p.act_param);
      const int64_t o = rowbase + c * colstride;
      p.out[o] = v;
      if (p.acc) p.acc[o] = acc[i][j];
      if (p.amax.ptr) {
        const int64_t slot = p.amax.elems_per_slot ? o / p.amax.elems_per_slot : 0;
        if (slot_lo < 0 || slot == slot_lo) { slot_lo = slot; mx_lo = fmaxf(mx_lo, fabsf(v)); }
        else { slot_hi = slot; mx_hi = fmaxf(mx_hi, fabsf(v)); }
      }
    }
  }
  if (p.amax.ptr) {
    flush_max(p.amax.ptr, slot_lo, mx_lo);
    flush_max(p.amax.ptr, slot_hi, mx_hi);
  }
}

constexpr int kNarrowThreads = 128;
constexpr int kNarrowMaxN = 32;

// Narrow-N Linear (N <= 32): one thread per output row, the whole weight matrix
// zero-padded to NT rows in shared memory, NT accumulators in registers (no
// predicates in the dot loop).  The accumulators are then staged through shared
// memory so that the epilogue runs once per output element, in a rolled loop
// over the block's contiguous [rows, n] output range: coalesced stores, and one
// copy of the activation code rather than NT unrolled copies.  Used for the last
// Linear layers (N = 3, 10, 32 ...) where a 128-wide tensor-core tile is mostly idle.
// Four f32 values of row `row` from column k0 (zero past af_k), quantized, packed.
__device__ __forceinline__ int32_t load_q4(const GemmArgs& p, const float* row, int64_t k0, bool vec, float inv) {
  float4 v;
  if (vec && k0 + 4 <= p.af_k) {
    v = __ldg(reinterpret_cast<const float4*>(row + k0));
  } else {
    v.x = k0 < p.af_k ? __ldg(row + k0) : 0.0f;
    v.y = k0 + 1 < p.af_k ? __ldg(row + k0 + 1) : 0.0f;
    v.z = k0 + 2 < p.af_k ? __ldg(row + k0 + 2) : 0.0f;
    v.w = k0 + 3 < p.af_k ? __ldg(row + k0 + 3) : 0.0f;
  }
  if (p.af_scale)  // a calibrated scale: values beyond its range clamp (quant1)
    return (int32_t)((uint32_t)(quant1(v.x, inv) & 0xff) | ((uint32_t)(quant1(v.y, inv) & 0xff) << 8) |
                     ((uint32_t)(quant1(v.z, inv) & 0xff) << 16) | ((uint32_t)(quant1(v.w, inv) & 0xff) << 24));
  return (int32_t)((uint32_t)(quant1_bounded(v.x, inv) & 0xff) | ((uint32_t)(quant1_bounded(v.y, inv) & 0xff) << 8) |
                   ((uint32_t)(quant1_bounded(v.z, inv) & 0xff) << 16) |
                   ((uint32_t)(quant1_bounded(v.w, inv) & 0xff) << 24));
}

template <int NT, bool QA, int TPR>
__global__ void __launch_bounds__(kNarrowThreads) k_gemm_narrow(const GemmArgs p) {
  constexpr int RPB = kNarrowThreads / TPR;  // rows per block; TPR threads share a row's K
  extern __shared__ __align__(16) int32_t sm[];
  const int kw = (int)(p.k >> 2);
  int32_t* wsm = sm;                                        // [NT][kw], rows >= n are zero
  int32_t* tile = sm + NT * kw;                             // [RPB][NT + 1]
  float* cs_sm = reinterpret_cast<float*>(tile + kNarrowThreads * (NT + 1));  // [NT]
  float* bias_sm = cs_sm + NT;                                                // [NT]
#pragma unroll 4
  for (int i = threadIdx.x; i < NT * kw; i += kNarrowThreads) {
    const int c = i / kw, w = i - c * kw;
    wsm[i] = c < (int)p.n ? __ldg(reinterpret_cast<const int32_t*>(p.w + (int64_t)c * p.ldb) + w) : 0;
  }
  float sa = 0.0f, inv = 0.0f;
  if (QA) {
    sa = p.af_scale ? *p.af_scale : quant_scale(__uint_as_float(*p.af_amax));
    inv = quant_inv(sa);
  } else {
    sa = p.a_scale[0];
  }
  if (threadIdx.x < (unsigned)p.n) {
    const float sw = p.w_scale_ch ? p.w_scale_ch[threadIdx.x] : p.w_scale;
    cs_sm[threadIdx.x] = __fmul_rn(sa, sw);
    bias_sm[threadIdx.x] = p.bias[threadIdx.x];
  }
  __syncthreads();
  const int lr = threadIdx.x / TPR, part = threadIdx.x % TPR;
  const int groups = kw / 4 / TPR;  // 16-element K groups of this thread
  const int n = (int)p.n;
  const uint32_t magic = n > 1 ? (uint32_t)((0x100000000ull + (uint64_t)n - 1) / (uint64_t)n) : 0u;
  float mx = 0.0f;
  // persistent: the block walks row tiles of RPB rows with its staged weights
  for (int64_t r0 = (int64_t)blockIdx.x * RPB; r0 < p.m; r0 += (int64_t)gridDim.x * RPB) {
    const int rows = (int)min((int64_t)RPB, p.m - r0);
    int32_t acc[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[j] = 0;
    if (lr < rows) {
      if (QA) {
        const float* row = p.af + (r0 + lr) * p.af_k;
        const bool vec = (p.af_k & 3) == 0 && (reinterpret_cast<uintptr_t>(p.af) & 15) == 0;
#pragma unroll 2
        for (int gi = 0; gi < groups; ++gi) {
          const int k4 = part * groups + gi;
          const int32_t a0 = load_q4(p, row, 16 * k4, vec, inv), a1 = load_q4(p, row, 16 * k4 + 4, vec, inv),
                        a2 = load_q4(p, row, 16 * k4 + 8, vec, inv), a3 = load_q4(p, row, 16 * k4 + 12, vec, inv);
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            const int4 wv = *reinterpret_cast<const int4*>(wsm + j * kw + 4 * k4);
            acc[j] = __dp4a(a0, wv.x, acc[j]);
            acc[j] = __dp4a(a1, wv.y, acc[j]);
            acc[j] = __dp4a(a2, wv.z, acc[j]);
            acc[j] = __dp4a(a3, wv.w, acc[j]);
          }
        }
      } else {
        const int4* arow = reinterpret_cast<const int4*>(p.a + (r0 + lr) * p.lda);
#pragma unroll 4
        for (int gi = 0; gi < groups; ++gi) {
          const int k4 = part * groups + gi;
          const int4 av = __ldg(arow + k4);
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            const int4 wv = *reinterpret_cast<const int4*>(wsm + j * kw + 4 * k4);
            acc[j] = __dp4a(av.x, wv.x, acc[j]);
            acc[j] = __dp4a(av.y, wv.y, acc[j]);
            acc[j] = __dp4a(av.z, wv.z, acc[j]);
            acc[j] = __dp4a(av.w, wv.w, acc[j]);
          }
        }
      }
    }
    // integer partial sums of one row: exact in any order
#pragma unroll
    for (int o = TPR / 2; o > 0; o >>= 1)
#pragma unroll
      for (int j = 0; j < NT; ++j) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
    if (lr < rows && part == 0)
#pragma unroll
      for (int j = 0; j < NT; ++j) tile[lr * (NT + 1) + j] = acc[j];
    __syncthreads();
    float* out = p.out + r0 * n;
    int32_t* accd = p.acc ? p.acc + r0 * n : nullptr;
#pragma unroll 4
    for (int e = threadIdx.x; e < rows * n; e += kNarrowThreads) {
      // e / n as a multiply-high by ceil(2^32 / n): exact for e < 2^16, 2 <= n <= 32
      const int rr = n == 1 ? e : (int)__umulhi((uint32_t)e, magic), j = e - rr * n;
      const int32_t a = tile[rr * (NT + 1) + j];
      const float v = epilogue(a, cs_sm[j], bias_sm[j], p.act, p.act_param);
      out[e] = v;
      if (accd) accd[e] = a;
      mx = fmaxf(mx, fabsf(v));
    }
    __syncthreads();  // the tile is rewritten by the next row tile
  }
  if (p.amax.ptr) flush_max(p.amax.ptr, 0, mx);
}

int narrow_width(int64_t n) { return n <= 4 ? 4 : n <= 8 ? 8 : n <= 16 ? 16 : 32; }
size_t narrow_smem(int nt, int64_t k) { return (size_t)nt * k + (size_t)kNarrowThreads * (nt + 1) * 4 + 8 * nt; }

}  // namespace

bool gemm_narrow_eligible(const GemmArgs& a) {
  const bool a_ok = a.af ? ((a.af_amax != nullptr || a.af_scale != nullptr) && a.af_k <= a.k)
                         : (a.lda == a.k && (reinterpret_cast<uintptr_t>(a.a) & 15) == 0);
  return a.n >= 1 && a.n <= kNarrowMaxN && narrow_smem(narrow_width(a.n), a.k) <= 48 * 1024 && !a.conv &&
         a.out_l == 0 && a.rows_per_scale == 0 && a.amax.elems_per_slot == 0 && (a.k & 15) == 0 && a_ok &&
         a.ldb >= a.k && (reinterpret_cast<uintptr_t>(a.w) & 15) == 0 && (a.ldb & 3) == 0;
}

template <int NT, bool QA, int TPR>
void launch_narrow_k(const GemmArgs& a, size_t sm, cudaStream_t st) {
  // persistent grid: as many blocks as are resident at once (at most one per row tile)
  static int per_sm = 0, num_sms = 0;
  if (per_sm == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_gemm_narrow<NT, QA, TPR>, kNarrowThreads, sm);
    if (per_sm < 1) per_sm = 1;
  }
  const int64_t rpb = kNarrowThreads / TPR, tiles = (a.m + rpb - 1) / rpb;
  const int grid = (int)std::min<int64_t>(tiles, (int64_t)per_sm * num_sms);
  k_gemm_narrow<NT, QA, TPR><<<grid, kNarrowThreads, sm, st>>>(a);
}

template <int NT, bool QA>
void launch_narrow_tpr(const GemmArgs& a, size_t sm, cudaStream_t st) {
  const int groups = (int)(a.k / 16);  // 16-element K groups per row
  const int tpr = groups % 8 == 0 ? 8 : groups % 4 == 0 ? 4 : groups % 2 == 0 ? 2 : 1;
  switch (tpr) {
    case 8: launch_narrow_k<NT, QA, 8>(a, sm, st); break;
    case 4: launch_narrow_k<NT, QA, 4>(a, sm, st); break;
    case 2: launch_narrow_k<NT, QA, 2>(a, sm, st); break;
    default: launch_narrow_k<NT, QA, 1>(a, sm, st); break;
  }
}

template <bool QA>
void launch_narrow_q(const GemmArgs& a, cudaStream_t st) {
  const int nt = narrow_width(a.n);
  const size_t sm = narrow_smem(nt, a.k);
  switch (nt) {
    case 4: launch_narrow_tpr<4, QA>(a, sm, st); break;
    case 8: launch_narrow_tpr<8, QA>(a, sm, st); break;
    case 16: launch_narrow_tpr<16, QA>(a, sm, st); break;
    default: launch_narrow_tpr<32, QA>(a, sm, st); break;
  }
}

void launch_gemm_narrow(const GemmArgs& a, cudaStream_t st) {
  if (a.m <= 0) return;
  if (a.af) launch_narrow_q<true>(a, st);
  else launch_narrow_q<false>(a, st);
}

void launch_gemm_simt(const GemmArgs& a, cudaStream_t st) {
  if (a.m <= 0 || a.n <= 0) return;
  dim3 grid((unsigned)((a.m + BM - 1) / BM), (unsigned)((a.n + BN - 1) / BN));
  switch (a.act) {
    case ACT_RELU: k_gemm_simt<ACT_RELU><<<grid, kThreads, 0, st>>>(a); break;
    case ACT_SIGMOID: k_gemm_simt<ACT_SIGMOID><<<grid, kThreads, 0, st>>>(a); break;
    case ACT_TANH: k_gemm_simt<ACT_TANH><<<grid, kThreads, 0, st>>>(a); break;
    case ACT_GELU: k_gemm_simt<ACT_GELU><<<grid, kThreads, 0, st>>>(a); break;
    case ACT_LEAKY_RELU: k_gemm_simt<ACT_LEAKY_RELU><<<grid, kThreads, 0, st>>>(a); break;
    case ACT_SILU: k_gemm_simt<ACT_SILU><<<grid, kThreads, 0, st>>>(a); break;
    default: k_gemm_simt<ACT_NONE><<<grid, kThreads, 0, st>>>(a); break;
  }
}

}  // namespace rg
