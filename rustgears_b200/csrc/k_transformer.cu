// k_transformer.cu -- the f32 parts of the transformer extension ops: token embedding
// gather, RMSNorm, non-causal multi-head attention (scores, softmax, P.V) and the
// SwiGLU gate product.  The INT8 projections around them run on the GEMM kernels.
//
// Every kernel follows the reference's f32 operation order exactly, so the INT8
// quantization of the next projection sees bit-identical activations:
//  - Embedding::forward (nn/layers.rs:438-446): row copy, id `as usize`, id >= V fails;
//  - RMSNorm::forward (nn/norm.rs:413-417): serial sum of squares (sum_dim,
//    tensor/ops.rs:715-727), times 1/d (mean_dim 755-758), + eps, sqrt, x / rms * w;
//  - attention (nn/attention.rs:178-196): bmm(q, k^T) and bmm(p, v) through the CPU
//    matmul (device/cpu.rs:234-395: per output an FMA chain over k in order from 0;
//    output columns past the last full 8-wide block accumulate unfused), scores times
//    1/sqrt(dh), softmax (tensor/ops.rs:1058-1076: max, exp(x - max), serial sum, divide);
//  - SwiGLU (nn/layers.rs:507-513): (g * sigmoid(g)) * u.
#include <algorithm>
#include <atomic>

#include "rg_kernels.h"
#include "rg_math.cuh"
#include "rg_sm100.cuh"

namespace rg {

__device__ int g_embed_error = 0;  // 1: a token id was >= V (the reference's assertion)

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide max of non-negative values into *dst (float bits, atomicMax); all threads call.
__device__ __forceinline__ void block_max_to(float v, unsigned* dst) {
  __shared__ float red[32];
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

// ---------------------------------------------------------------------------
// Embedding: one warp per token, the row copied with 16-byte accesses when d % 4 == 0.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) k_embedding(const float* __restrict__ ids, int64_t n,
                                                        const float* __restrict__ table, int64_t v, int32_t d,
                                                        float* __restrict__ y, unsigned* amax) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (kThreads / 32);
  float m = 0.0f;
  for (int64_t r = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); r < n; r += warps) {
    const float f = __ldg(ids + r);
    // f32 `as usize`: NaN and values below 1 give 0, values >= 2^64 saturate
    unsigned long long idx = 0;
    if (f >= 18446744073709551616.0f) idx = ~0ull;
    else if (f >= 1.0f) idx = __float2ull_rz(f);
    float* yr = y + r * d;
    if (idx >= (unsigned long long)v) {
      if (lane == 0) atomicExch(&g_embed_error, 1);
      for (int32_t c = lane; c < d; c += 32) yr[c] = 0.0f;
      continue;
    }
    const float* src = table + (int64_t)idx * d;
    if ((d & 3) == 0) {
      const float4* s4 = reinterpret_cast<const float4*>(src);
      float4* y4 = reinterpret_cast<float4*>(yr);
      for (int32_t c = lane; c < (d >> 2); c += 32) {
        const float4 t = __ldg(s4 + c);
        y4[c] = t;
        m = fmaxf(m, fmaxf(fmaxf(fabsf(t.x), fabsf(t.y)), fmaxf(fabsf(t.z), fabsf(t.w))));
      }
    } else {
      for (int32_t c = lane; c < d; c += 32) {
        const float t = __ldg(src + c);
        yr[c] = t;
        m = fmaxf(m, fabsf(t));
      }
    }
  }
  if (amax) block_max_to(m, amax);
}

// ---------------------------------------------------------------------------
// RMSNorm: a warp owns 32 rows.  The rows are staged through shared memory in 32x32
// tiles (coalesced loads) so that each lane can add its own row's squares serially.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) k_rmsnorm(const float* __restrict__ x, int64_t rows, int32_t d,
                                                      const float* __restrict__ w, float eps, float inv_d,
                                                      float* __restrict__ y, unsigned* amax) {
  __shared__ float tile[kThreads / 32][32][33];
  __shared__ float rms_s[kThreads / 32][32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int64_t r0 = ((int64_t)blockIdx.x * (kThreads / 32) + wid) * 32;
  float m = 0.0f;
  if (r0 < rows) {
    const int nr = rows - r0 < 32 ? (int)(rows - r0) : 32;
    float s = 0.0f;
    for (int32_t c0 = 0; c0 < d; c0 += 32) {
      const int nc = min(32, d - c0);
#pragma unroll 8
      for (int rr = 0; rr < 32; ++rr)
        tile[wid][rr][lane] = (rr < nr && lane < nc) ? __ldg(x + (r0 + rr) * d + c0 + lane) : 0.0f;
      __syncwarp();
      for (int c = 0; c < nc; ++c) {
        const float v = tile[wid][lane][c];
        s = __fadd_rn(s, __fmul_rn(v, v));
      }
      __syncwarp();
    }
    rms_s[wid][lane] = __fsqrt_rn(__fadd_rn(__fmul_rn(s, inv_d), eps));
    __syncwarp();
    for (int rr = 0; rr < nr; ++rr) {
      const float r = rms_s[wid][rr];
      const float* xr = x + (r0 + rr) * d;
      float* yr = y + (r0 + rr) * d;
      for (int32_t c = lane; c < d; c += 32) {
        const float v = __fmul_rn(__fdiv_rn(__ldg(xr + c), r), __ldg(w + c));
        yr[c] = v;
        m = fmaxf(m, fabsf(v));
      }
    }
  }
  if (amax) block_max_to(m, amax);
}

// ---------------------------------------------------------------------------
// SwiGLU gate product: gu [rows, 2h] holds g in columns [0, h) and u in [h, 2h).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) k_swiglu_mul(const float* __restrict__ gu, int64_t rows, int32_t h,
                                                         float* __restrict__ y, unsigned* amax) {
  const int64_t n = rows * h;
  float m = 0.0f;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads) {
    const int64_t r = i / h, c = i - r * h;
    const float g = __ldg(gu + r * 2 * h + c), u = __ldg(gu + r * 2 * h + h + c);
    const float v = __fmul_rn(__fmul_rn(g, act_apply(ACT_SIGMOID, 0.0f, g)), u);
    y[i] = v;
    m = fmaxf(m, fabsf(v));
  }
  if (amax) block_max_to(m, amax);
}

// ---------------------------------------------------------------------------
// Attention, any t and head size: one block per (query, batch*head); the score row
// lives in shared memory.  Used for small or irregular shapes.
// qkv [b*t, ld] with q, k, v of head hh at columns hh*dh, d + hh*dh, 2d + hh*dh.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) k_attention_row(const float* __restrict__ qkv, int64_t ld, int32_t t,
                                                       int32_t heads, int32_t dh, float scale,
                                                       float* __restrict__ out, int64_t ldo, unsigned* amax) {
  extern __shared__ __align__(16) float sc[];  // [t]
  __shared__ float red[4];
  __shared__ float total;
  const int32_t i = blockIdx.x;
  const int32_t g = blockIdx.y;
  const int32_t bi = g / heads, hh = g - bi * heads;
  const int32_t d = heads * dh;
  const int64_t base = (int64_t)bi * t;
  const float* q = qkv + (base + i) * ld + (int64_t)hh * dh;
  const int32_t nv_k = t / 8 * 8, nv_e = dh / 8 * 8;
  for (int32_t j = threadIdx.x; j < t; j += blockDim.x) {
    const float* k = qkv + (base + j) * ld + d + (int64_t)hh * dh;
    float acc = 0.0f;
    if (j < nv_k) {
      for (int32_t p = 0; p < dh; ++p) acc = fmaf(__ldg(q + p), __ldg(k + p), acc);
    } else {
      for (int32_t p = 0; p < dh; ++p) acc = __fadd_rn(acc, __fmul_rn(__ldg(q + p), __ldg(k + p)));
    }
    sc[j] = __fmul_rn(acc, scale);
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int32_t j = threadIdx.x; j < t; j += blockDim.x) mx = fmaxf(mx, sc[j]);
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  for (int32_t j = threadIdx.x; j < t; j += blockDim.x) sc[j] = exp_f32(__fsub_rn(sc[j], mx));
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.0f;
    for (int32_t j = 0; j < t; ++j) s = __fadd_rn(s, sc[j]);
    total = s;
  }
  __syncthreads();
  const float s = total;
  for (int32_t j = threadIdx.x; j < t; j += blockDim.x) sc[j] = __fdiv_rn(sc[j], s);
  __syncthreads();
  float m = 0.0f;
  for (int32_t e = threadIdx.x; e < dh; e += blockDim.x) {
    const float* v = qkv + base * ld + 2 * (int64_t)d + (int64_t)hh * dh + e;
    float acc = 0.0f;
    if (e < nv_e) {
      for (int32_t j = 0; j < t; ++j) acc = fmaf(sc[j], __ldg(v + (int64_t)j * ld), acc);
    } else {
      for (int32_t j = 0; j < t; ++j) acc = __fadd_rn(acc, __fmul_rn(sc[j], __ldg(v + (int64_t)j * ld)));
    }
    out[(base + i) * ldo + (int64_t)hh * dh + e] = acc;
    m = fmaxf(m, fabsf(acc));
  }
  if (amax) block_max_to(m, amax);
}

// ---------------------------------------------------------------------------
// Attention for head size 64 and t % 8 == 0, t <= kMaxT (every score column an FMA
// chain).  One CTA per (64 queries, batch*head), 8 warps:
//  phase 1  S = Q K^T for 128-key chunks: warp w owns queries 8w..8w+7, lane l keys
//           4l..4l+3 of the chunk, 32 FMA chains over the 64 dims;
//  softmax  per query row over all t scores in shared memory;
//  phase 2  O = P V for 128-key chunks: warp w owns queries 8w..8w+7, lane (qh, eg)
//           queries 4qh..4qh+3 x dims 4eg..4eg+3, FMA chains over the keys in order.
// K and V chunks stream through a double buffer with cp.async (K transposed by 4-byte
// copies), so the next chunk lands while the current one is used and V's first chunk
// lands during the softmax.  Shared-memory layouts (floats):
//  Qs [64 dims][64 queries], KV[2][128 x 64] (K^T [64 dims][128 keys] or V [128][64]),
//  S [t][64 queries]; Q, K^T and S rows swizzle their 16-byte groups (XOR of the group
//  index with the dim (Q, K) or key/4 (S)) to keep the transposing stores and the
//  row reads conflict-free.
// ---------------------------------------------------------------------------
constexpr int kAQ = 64, kAK = 128, kADh = 64, kAThreads = 256, kMaxT = 512;
constexpr int kAQsFloats = kADh * kAQ;     // 4096
constexpr int kAChunkFloats = kAK * kADh;  // 8192

__device__ __forceinline__ void cp_async4(float* dst, const float* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(sm100::smem_addr(dst)), "l"(src),
               "r"(valid ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async16(float* dst, const float* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sm100::smem_addr(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__global__ void __launch_bounds__(kAThreads, 1) k_attention64(const float* __restrict__ qkv, int64_t ld, int32_t t,
                                                             int32_t heads, float scale, float* __restrict__ out,
                                                             int64_t ldo, unsigned* amax) {
  extern __shared__ __align__(16) float sm[];
  float* Qs = sm;
  float* KV = sm + kAQsFloats;
  float* S = KV + 2 * kAChunkFloats;
  float* red = S + (size_t)t * kAQ;  // [4][64]
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int32_t q0 = blockIdx.x * kAQ;
  const int32_t g = blockIdx.y;
  const int32_t bi = g / heads, hh = g - bi * heads;
  const int32_t d = heads * kADh;
  const int64_t base = (int64_t)bi * t;
  const float* qg = qkv + (int64_t)hh * kADh;
  const float* kg = qkv + d + (int64_t)hh * kADh;
  const float* vg = qkv + 2 * (int64_t)d + (int64_t)hh * kADh;
  const int nk = (t + kAK - 1) / kAK;

  // 4-byte transposing copies: a warp covers 4 rows (queries or keys) x 8 dims, so the
  // global reads are whole 32-byte sectors and the swizzled stores hit 32 banks.
  auto load_q = [&]() {
#pragma unroll 4
    for (int it = 0; it < (kAQ * kADh) / kAThreads; ++it) {
      const int idx = it * kAThreads + tid;
      const int rsub = (idx >> 3) & 3, p = ((idx >> 5) & 7) * 8 + (idx & 7);
      const int row = (idx >> 8) * 4 + rsub;  // 0..63
      // idx bits: [2:0] dim low, [4:3] row low, [7:5] dim high, [11:8] row high
      const int32_t qrow = q0 + row;
      const bool ok = qrow < t;
      const float* src = qg + (base + (ok ? qrow : 0)) * ld + p;
      cp_async4(Qs + p * kAQ + ((((row >> 2) ^ (p & 7))) << 2) + (row & 3), src, ok);
    }
  };
  auto load_k = [&](int c, float* buf) {
    const int32_t k0 = c * kAK;
#pragma unroll 4
    for (int it = 0; it < kAChunkFloats / kAThreads; ++it) {
      const int idx = it * kAThreads + tid;
      const int rsub = (idx >> 3) & 3, p = ((idx >> 5) & 7) * 8 + (idx & 7);
      const int key = (idx >> 8) * 4 + rsub;  // 0..127
      const int32_t krow = k0 + key;
      const bool ok = krow < t;
      const float* src = kg + (base + (ok ? krow : 0)) * ld + p;
      cp_async4(buf + p * kAK + ((((key >> 2) ^ (p & 7))) << 2) + (key & 3), src, ok);
    }
  };
  auto load_v = [&](int c, float* buf) {
    const int32_t k0 = c * kAK;
#pragma unroll 4
    for (int it = 0; it < kAChunkFloats / 4 / kAThreads; ++it) {
      const int idx = it * kAThreads + tid;
      const int key = idx >> 4, e4 = idx & 15;
      const int32_t krow = k0 + key;
      const bool ok = krow < t;
      const float* src = vg + (base + (ok ? krow : 0)) * ld + e4 * 4;
      cp_async16(buf + key * kADh + e4 * 4, src, ok);
    }
  };
  auto issue = [&](int c) {  // chunk stream: K chunks 0..nk-1, then V chunks
    float* buf = KV + (c & 1) * kAChunkFloats;
    if (c < nk) load_k(c, buf);
    else load_v(c - nk, buf);
    cp_async_commit();
  };

  load_q();
  issue(0);
  float o[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[i][e] = 0.0f;
  const int qh = lane >> 4, eg = lane & 15;

  for (int c = 0; c < 2 * nk; ++c) {
    if (c + 1 < 2 * nk) {
      issue(c + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const float* buf = KV + (c & 1) * kAChunkFloats;
    if (c < nk) {
      // ---- phase 1: scores of queries 8w..8w+7 x keys 4*lane..4*lane+3 of chunk c ----
      float acc[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
#pragma unroll 8
      for (int p = 0; p < kADh; ++p) {
        const int sp = p & 7;
        const float4 qa = *reinterpret_cast<const float4*>(Qs + p * kAQ + (((2 * w) ^ sp) << 2));
        const float4 qb = *reinterpret_cast<const float4*>(Qs + p * kAQ + (((2 * w + 1) ^ sp) << 2));
        const float4 kv = *reinterpret_cast<const float4*>(buf + p * kAK + ((lane ^ sp) << 2));
        const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        const float kk[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(qv[i], kk[j], acc[i][j]);
      }
      const int32_t key0 = c * kAK + 4 * lane;
      if (key0 < t) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int32_t key = key0 + j;  // t % 8 == 0: a group of 4 keys is all valid or all past t
          const int s = (key >> 2) & 7;
          float* row = S + (size_t)key * kAQ;
          *reinterpret_cast<float4*>(row + (((2 * w) ^ s) << 2)) =
              make_float4(__fmul_rn(acc[0][j], scale), __fmul_rn(acc[1][j], scale), __fmul_rn(acc[2][j], scale),
                          __fmul_rn(acc[3][j], scale));
          *reinterpret_cast<float4*>(row + (((2 * w + 1) ^ s) << 2)) =
              make_float4(__fmul_rn(acc[4][j], scale), __fmul_rn(acc[5][j], scale), __fmul_rn(acc[6][j], scale),
                          __fmul_rn(acc[7][j], scale));
        }
      }
      if (c == nk - 1) {
        // ---- softmax over each query row (V's first chunk is in flight) ----
        __syncthreads();
        const int q = tid & 63, part = tid >> 6;
        const int grp = q >> 2, qe = q & 3;
        const int32_t j0 = part * (t / 4), j1 = j0 + t / 4;  // t % 8 == 0
        float mx = -INFINITY;
        for (int32_t j = j0; j < j1; ++j) mx = fmaxf(mx, S[(size_t)j * kAQ + ((grp ^ ((j >> 2) & 7)) << 2) + qe]);
        red[part * 64 + q] = mx;
        __syncthreads();
        mx = fmaxf(fmaxf(red[q], red[64 + q]), fmaxf(red[128 + q], red[192 + q]));
        for (int32_t j = j0; j < j1; ++j) {
          float* sp = S + (size_t)j * kAQ + ((grp ^ ((j >> 2) & 7)) << 2) + qe;
          *sp = exp_f32(__fsub_rn(*sp, mx));
        }
        __syncthreads();
        if (part == 0) {  // serial sum in key order
          float s = 0.0f;
          for (int32_t j = 0; j < t; ++j) s = __fadd_rn(s, S[(size_t)j * kAQ + ((grp ^ ((j >> 2) & 7)) << 2) + qe]);
          red[q] = s;
        }
        __syncthreads();
        const float s = red[q];
        for (int32_t j = j0; j < j1; ++j) {
          float* sp = S + (size_t)j * kAQ + ((grp ^ ((j >> 2) & 7)) << 2) + qe;
          *sp = __fdiv_rn(*sp, s);
        }
      }
    } else {
      // ---- phase 2: O += P V over the keys of V chunk c - nk, in key order ----
      const int32_t k0 = (c - nk) * kAK;
      const int jn = min(kAK, t - k0);
      const int qg4 = 2 * w + qh;
      for (int jl = 0; jl < jn; ++jl) {
        const int32_t j = k0 + jl;
        const float4 pv = *reinterpret_cast<const float4*>(S + (size_t)j * kAQ + ((qg4 ^ ((j >> 2) & 7)) << 2));
        const float4 vv = *reinterpret_cast<const float4*>(buf + jl * kADh + eg * 4);
        const float pp[4] = {pv.x, pv.y, pv.z, pv.w};
        const float vx[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int e = 0; e < 4; ++e) o[i][e] = fmaf(pp[i], vx[e], o[i][e]);
      }
    }
    __syncthreads();
  }
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int32_t q = q0 + 8 * w + 4 * qh + i;
    if (q < t) {
      *reinterpret_cast<float4*>(out + (base + q) * ldo + (int64_t)hh * kADh + eg * 4) =
          make_float4(o[i][0], o[i][1], o[i][2], o[i][3]);
#pragma unroll
      for (int e = 0; e < 4; ++e) m = fmaxf(m, fabsf(o[i][e]));
    }
  }
  if (amax) block_max_to(m, amax);
}

int grid_for(int64_t work, int per_block, int cap) {
  const int64_t b = (work + per_block - 1) / per_block;
  return (int)std::max<int64_t>(1, std::min<int64_t>(b, cap));
}

}  // namespace

size_t attention64_smem(int32_t t) {
  return (size_t)(kAQsFloats + 2 * kAChunkFloats + (size_t)t * kAQ + 4 * 64) * sizeof(float);
}

void launch_embedding(const float* ids, int64_t n, const float* table, int64_t v, int32_t d, float* y,
                      AmaxSink amax, cudaStream_t st) {
  if (n <= 0) return;
  k_embedding<<<grid_for(n, kThreads / 32, 148 * 16), kThreads, 0, st>>>(ids, n, table, v, d, y, amax.ptr);
}

void launch_rmsnorm(const float* x, int64_t rows, int32_t d, const float* w, float eps, float inv_d, float* y,
                    AmaxSink amax, cudaStream_t st) {
  if (rows <= 0) return;
  const int64_t blocks = (rows + kThreads - 1) / kThreads;  // 32 rows per warp, 8 warps
  k_rmsnorm<<<(unsigned)blocks, kThreads, 0, st>>>(x, rows, d, w, eps, inv_d, y, amax.ptr);
}

void launch_swiglu_mul(const float* gu, int64_t rows, int32_t h, float* y, AmaxSink amax, cudaStream_t st) {
  if (rows <= 0 || h <= 0) return;
  k_swiglu_mul<<<grid_for(rows * h, kThreads, 148 * 16), kThreads, 0, st>>>(gu, rows, h, y, amax.ptr);
}

bool attention_fast_eligible(int32_t t, int32_t dh, const float* qkv, int64_t ld, const float* out, int64_t ldo) {
  return dh == kADh && t > 0 && t % 8 == 0 && t <= kMaxT && (ld & 3) == 0 && (ldo & 3) == 0 &&
         ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
}

rg_status launch_attention(const float* qkv, int64_t ld, int64_t b, int32_t t, int32_t heads, int32_t dh,
                           float scale, float* out, int64_t ldo, AmaxSink amax, cudaStream_t st) {
  if (b <= 0 || t <= 0) return RG_OK;
  if (b * heads > 65535) return set_last_error(RG_ERR_UNSUPPORTED, "attention: batch * heads above 65535");
  if (attention_fast_eligible(t, dh, qkv, ld, out, ldo)) {
    const size_t smem = attention64_smem(t);
    static std::atomic<uint64_t> opted_in{0};  // one bit per device
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(opted_in.load() & bit)) {
      if (cudaFuncSetAttribute(k_attention64, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)attention64_smem(kMaxT)) != cudaSuccess)
        return set_last_error(RG_ERR_CUDA, "attention: shared-memory opt-in failed");
      opted_in.fetch_or(bit);
    }
    dim3 grid((unsigned)((t + kAQ - 1) / kAQ), (unsigned)(b * heads));
    k_attention64<<<grid, kAThreads, smem, st>>>(qkv, ld, t, heads, scale, out, ldo, amax.ptr);
    return RG_OK;
  }
  const size_t smem = (size_t)t * sizeof(float);
  if (smem > 200 * 1024) return set_last_error(RG_ERR_UNSUPPORTED, "attention: sequence too long");
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(k_attention_row, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return set_last_error(RG_ERR_CUDA, "attention: shared-memory opt-in failed");
  dim3 grid((unsigned)t, (unsigned)(b * heads));
  k_attention_row<<<grid, 128, smem, st>>>(qkv, ld, t, heads, dh, scale, out, ldo, amax.ptr);
  return RG_OK;
}

int embedding_take_error() {
  int v = 0, z = 0;
  cudaMemcpyFromSymbol(&v, g_embed_error, sizeof(int));
  if (v) cudaMemcpyToSymbol(g_embed_error, &z, sizeof(int));
  return v;
}

}  // namespace rg
