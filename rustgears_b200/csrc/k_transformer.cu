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
                                                        float* __restrict__ y, unsigned* amax, int* err) {
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
      if (lane == 0) atomicExch(err, 1);  // the reference's assertion (layers.rs:438-446)
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
// RMSNorm: a block stages `rpb` whole rows in shared memory (coalesced 16-byte loads
// and stores; row pitch d + 4, so that the per-row readers' 16-byte loads fall in
// distinct bank groups, or d + 1 for rows that are not whole float4s), one thread per
// row adds the squares serially, then all threads normalise from shared memory.
// Eight rows per block and several blocks per SM overlap one block's serial sums
// with the others' copies and normalisation (twice as fast as 16 or 32 rows a block).
// ---------------------------------------------------------------------------
// yq (calibration extension): instead of y, the output quantized with the frozen scale
// *q_scale into i8 rows of ldq bytes (columns d..ldq zero).
__global__ void __launch_bounds__(kThreads) k_rmsnorm(const float* __restrict__ x, int64_t rows, int32_t d,
                                                      int32_t rpb, bool vec, const float* __restrict__ w, float eps,
                                                      float inv_d, float* __restrict__ y, unsigned* amax,
                                                      int8_t* __restrict__ yq, int64_t ldq,
                                                      const float* __restrict__ q_scale) {
  const float qinv = yq ? quant_inv(*q_scale) : 0.0f;
  // [rpb][ld] staged rows; the vector path pads a row by 16 bytes (float4 rows whose
  // 16-byte columns fall in distinct bank groups across consecutive rows), the scalar
  // one by 4 bytes (distinct banks)
  extern __shared__ float4 xs4[];
  float* xs = reinterpret_cast<float*>(xs4);
  __shared__ float rms_s[32];
  const int ld = vec ? d + 4 : d + 1;
  const int d4 = d >> 2;
  float m = 0.0f;
  for (int64_t r0 = (int64_t)blockIdx.x * rpb; r0 < rows; r0 += (int64_t)gridDim.x * rpb) {
    const int nr = rows - r0 < rpb ? (int)(rows - r0) : rpb;
    const float* src = x + r0 * d;
    if (vec) {
      const float4* src4 = reinterpret_cast<const float4*>(src);
      for (int i = threadIdx.x; i < nr * d4; i += kThreads) {
        const int r = i / d4, c4 = i - r * d4;
        xs4[(r * ld >> 2) + c4] = __ldg(src4 + i);
      }
    } else {
      for (int r = 0; r < nr; ++r)
        for (int c = threadIdx.x; c < d; c += kThreads) xs[r * ld + c] = __ldg(src + (int64_t)r * d + c);
    }
    __syncthreads();
    if ((int)threadIdx.x < nr) {  // serial sum of squares in column order
      float s = 0.0f;
      if (vec) {
        const float4* row = xs4 + (threadIdx.x * ld >> 2);
#pragma unroll 4
        for (int c4 = 0; c4 < d4; ++c4) {
          const float4 v = row[c4];
          s = __fadd_rn(s, __fmul_rn(v.x, v.x));
          s = __fadd_rn(s, __fmul_rn(v.y, v.y));
          s = __fadd_rn(s, __fmul_rn(v.z, v.z));
          s = __fadd_rn(s, __fmul_rn(v.w, v.w));
        }
      } else {
        const float* row = xs + threadIdx.x * ld;
#pragma unroll 8
        for (int c = 0; c < d; ++c) s = __fadd_rn(s, __fmul_rn(row[c], row[c]));
      }
      rms_s[threadIdx.x] = __fsqrt_rn(__fadd_rn(__fmul_rn(s, inv_d), eps));
    }
    __syncthreads();
    if (vec && !yq && (reinterpret_cast<uintptr_t>(y) & 15) == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0) {
      for (int i = threadIdx.x; i < nr * d4; i += kThreads) {
        const int r = i / d4, c4 = i - r * d4;
        const float rr = rms_s[r];
        const float4 v = xs4[(r * ld >> 2) + c4];
        const float4 ww = __ldg(reinterpret_cast<const float4*>(w) + c4);
        float4 o;
        o.x = __fmul_rn(__fdiv_rn(v.x, rr), ww.x);
        o.y = __fmul_rn(__fdiv_rn(v.y, rr), ww.y);
        o.z = __fmul_rn(__fdiv_rn(v.z, rr), ww.z);
        o.w = __fmul_rn(__fdiv_rn(v.w, rr), ww.w);
        reinterpret_cast<float4*>(y + r0 * d)[i] = o;
        m = fmaxf(m, fmaxf(fmaxf(fabsf(o.x), fabsf(o.y)), fmaxf(fabsf(o.z), fabsf(o.w))));
      }
      __syncthreads();
      continue;
    }
    for (int r = 0; r < nr; ++r) {
      const float rr = rms_s[r];
      if (yq) {
        int8_t* qr = yq + (r0 + r) * ldq;
        for (int c = threadIdx.x; c < ldq; c += kThreads)
          qr[c] = c < d ? (int8_t)quant1(__fmul_rn(__fdiv_rn(xs[r * ld + c], rr), __ldg(w + c)), qinv) : 0;
        continue;
      }
      float* yr = y + (r0 + r) * d;
      for (int c = threadIdx.x; c < d; c += kThreads) {
        const float v = __fmul_rn(__fdiv_rn(xs[r * ld + c], rr), __ldg(w + c));
        yr[c] = v;
        m = fmaxf(m, fabsf(v));
      }
    }
    __syncthreads();
  }
  if (amax) block_max_to(m, amax);
}

// ---------------------------------------------------------------------------
// SwiGLU gate product: gu [rows, 2h] holds g in columns [0, h) and u in [h, 2h); one
// block per row.  sigmoid(g) = 1 / (1 + exp(-g)) (device/backend.rs:72) with the exp
// table in shared memory (the lanes of a warp index different entries).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float swiglu1(float g, float u, ExpTablePtr et) {
  const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_f32_with(-g, et)));
  return __fmul_rn(__fmul_rn(g, sig), u);
}

// yq (calibration extension): instead of y, the product quantized with the frozen
// scale *q_scale into i8 rows of ldq bytes (columns h..ldq zero).
__global__ void __launch_bounds__(kThreads) k_swiglu_mul(const float* __restrict__ gu, int64_t rows, int32_t h,
                                                         bool vec, float* __restrict__ y, unsigned* amax,
                                                         int8_t* __restrict__ yq, int64_t ldq,
                                                         const float* __restrict__ q_scale) {
  __shared__ uint64_t tab[32];
  if (threadIdx.x < 32) tab[threadIdx.x] = ExpTableConst{}(threadIdx.x);
  __syncthreads();
  const ExpTablePtr et{tab};
  const float qinv = yq ? quant_inv(*q_scale) : 0.0f;
  float m = 0.0f;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* gr = gu + r * 2 * h;
    const float* ur = gr + h;
    if (yq) {
      int8_t* qr = yq + r * ldq;
      for (int64_t c = threadIdx.x; c < ldq; c += kThreads)
        qr[c] = c < h ? (int8_t)quant1(swiglu1(__ldg(gr + c), __ldg(ur + c), et), qinv) : 0;
      continue;
    }
    float* yr = y + r * h;
    if (vec) {  // h % 4 == 0 and gu, y 16-byte aligned
      for (int32_t c = threadIdx.x; c < (h >> 2); c += kThreads) {
        const float4 g = __ldg(reinterpret_cast<const float4*>(gr) + c);
        const float4 u = __ldg(reinterpret_cast<const float4*>(ur) + c);
        const float4 v = make_float4(swiglu1(g.x, u.x, et), swiglu1(g.y, u.y, et), swiglu1(g.z, u.z, et),
                                     swiglu1(g.w, u.w, et));
        reinterpret_cast<float4*>(yr)[c] = v;
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      }
    } else {
      for (int32_t c = threadIdx.x; c < h; c += kThreads) {
        const float v = swiglu1(__ldg(gr + c), __ldg(ur + c), et);
        yr[c] = v;
        m = fmaxf(m, fabsf(v));
      }
    }
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
// chain).  One CTA per (64 queries, batch*head), 8 warps, one CTA per SM.  Shared
// memory delivers 128 B per cycle to the registers of an SM, against 128 FMAs per
// cycle, so the operand bytes per FMA decide the speed: the register tiles are
//  phase 1  S = Q K^T over 256-key chunks, lane tile 8 queries x 8 keys (64 chains
//           over the 64 dims; 1 B of operands per FMA): warp w owns keys
//           32w..32w+31 of the chunk, lane (qg, kg) queries {4qg..+3, 32+4qg..+3} x
//           keys {4kg..+3, 16+4kg..+3} of the warp's; the row maxima kept on the way;
//  softmax  exp(s - max) in parallel, the serial sum per row, the division;
//  phase 2  O = P V over 256-key chunks, lane tile 4 queries x 4 dims (2 B per FMA):
//           warp (wq, we) owns queries 32wq.. x dims 16we.., lane (qg, eg) queries
//           32wq + 4qg.. x dims 16we + 4eg..; chains over the keys in order.
// FMAs are paired (f32x2: each lane rounded once, exactly as fmaf) with the shared
// operand duplicated in registers.  Shared memory (floats): Q^T [64 dims][64
// queries] 16 KB, KV 64 KB (K^T [64 dims][256 keys] or V [256 keys][64]), S [t][64
// queries] (t = 512: 128 KB).  Q^T, K^T and S rows swizzle their 16-byte groups:
// XOR of the group index with dim & 7 (Q^T, K^T) or (key / 4) & 7 (S), so the
// transposing stores and every row read are conflict-free.
// ---------------------------------------------------------------------------
constexpr int kAQ = 64, kAK = 256, kADh = 64, kAThreads = 256, kMaxT = 512;
constexpr int kAQsFloats = kADh * kAQ;     // 4096
constexpr int kAChunkFloats = kAK * kADh;  // 16384
constexpr int kAMiscFloats = 8 * kAQ + kAQ + 64;  // per-warp maxima, row sums, the exp table

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
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// d.x = fma(a.x, b.x, c.x), d.y = fma(a.y, b.y, c.y), each rounded once as fmaf.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(d)
      : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)),
        "l"(*reinterpret_cast<uint64_t*>(&c)));
  return *reinterpret_cast<float2*>(&d);
}

__global__ void __launch_bounds__(kAThreads, 1) k_attention64(const float* __restrict__ qkv, int64_t ld, int32_t t,
                                                             int32_t heads, float scale, float* __restrict__ out,
                                                             int64_t ldo, unsigned* amax) {
  extern __shared__ __align__(16) float sm[];
  float* Qs = sm;
  float* KV = sm + kAQsFloats;
  float* S = KV + kAChunkFloats;
  float* wmax = S + (size_t)t * kAQ;  // [8 warps][64 queries]
  float* rsum = wmax + 8 * kAQ;       // [64]
  uint64_t* tab = reinterpret_cast<uint64_t*>(rsum + kAQ);
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int32_t q0 = blockIdx.x * kAQ;
  const int32_t g = blockIdx.y;
  const int32_t bi = g / heads, hh = g - bi * heads;
  const int32_t d = heads * kADh;
  const int64_t base = (int64_t)bi * t;
  const float* qsrc = qkv + (int64_t)hh * kADh;
  const float* ksrc = qkv + d + (int64_t)hh * kADh;
  const float* vsrc = qkv + 2 * (int64_t)d + (int64_t)hh * kADh;
  const int nk = (t + kAK - 1) / kAK;
  if (tid < 32) tab[tid] = ExpTableConst{}((uint32_t)tid);

  // 4-byte transposing copies: a warp covers 4 rows (queries or keys) x 8 dims (whole
  // 32-byte sectors; the swizzled stores hit 32 banks).  idx bits: [2:0] dim low,
  // [4:3] row low, [7:5] dim high, [..:8] row high.
#pragma unroll 4
  for (int it = 0; it < kAQsFloats / kAThreads; ++it) {
    const int idx = it * kAThreads + tid;
    const int p = ((idx >> 5) & 7) * 8 + (idx & 7);
    const int row = (idx >> 8) * 4 + ((idx >> 3) & 3);  // 0..63
    const bool ok = q0 + row < t;
    cp_async4(Qs + p * kAQ + (((row >> 2) ^ (p & 7)) << 2) + (row & 3), qsrc + (base + (ok ? q0 + row : 0)) * ld + p,
              ok);
  }
  auto load_chunk = [&](int c) {  // chunk stream: K chunks 0..nk-1, then V chunks
    if (c < nk) {
      const int32_t k0 = c * kAK;
#pragma unroll 8
      for (int it = 0; it < kAChunkFloats / kAThreads; ++it) {
        const int idx = it * kAThreads + tid;
        const int p = ((idx >> 5) & 7) * 8 + (idx & 7);
        const int key = (idx >> 8) * 4 + ((idx >> 3) & 3);  // 0..255
        const bool ok = k0 + key < t;
        cp_async4(KV + p * kAK + (((key >> 2) ^ (p & 7)) << 2) + (key & 3),
                  ksrc + (base + (ok ? k0 + key : 0)) * ld + p, ok);
      }
    } else {
      const int32_t k0 = (c - nk) * kAK;
#pragma unroll 4
      for (int it = 0; it < kAChunkFloats / 4 / kAThreads; ++it) {
        const int idx = it * kAThreads + tid;
        const int key = idx >> 4, e4 = idx & 15;
        const bool ok = k0 + key < t;
        cp_async16(KV + key * kADh + e4 * 4, vsrc + (base + (ok ? k0 + key : 0)) * ld + e4 * 4, ok);
      }
    }
    cp_async_commit();
  };

  // ---- phase 1 ----
  const int qg = lane >> 2, kg = lane & 3;  // phase 1 lane split
  float rmax[8];  // [query slot]: slots 0..3 = queries 4qg.., 4..7 = 32 + 4qg..
#pragma unroll
  for (int i = 0; i < 8; ++i) rmax[i] = -INFINITY;
  {
    // operand rows for dims u, u + 8, ...: the swizzle depends on dim & 7 only
    const float* qrow[8];
    const float* krow[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      qrow[u] = Qs + u * kAQ + ((qg ^ u) << 2);              // group qg; group qg + 8 at +32 floats
      krow[u] = KV + u * kAK + (((8 * w + kg) ^ u) << 2);    // group 8w + kg
    }
    for (int c = 0; c < nk; ++c) {
      load_chunk(c);  // (the first group also carries Q)
      cp_async_wait_all();
      __syncthreads();
      float2 acc[8][4];  // [query slot][key pair: (k0,k1) (k2,k3) of group kg, then of group kg + 4]
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = make_float2(0.0f, 0.0f);
#pragma unroll 8
      for (int p = 0; p < kADh; ++p) {
        const int u = p & 7;
        const float* qr = qrow[u] + (p - u) * kAQ;
        const float* kr = krow[u] + (p - u) * kAK;
        const float4 qa = *reinterpret_cast<const float4*>(qr);
        const float4 qb = *reinterpret_cast<const float4*>(qr + 32);  // group qg + 8: the XOR leaves bit 3
        const float4 ka = *reinterpret_cast<const float4*>(kr);
        // group 8w + kg + 4: its swizzled index differs in bit 2 only, by +4 or -4 groups
        const float4 kb = *reinterpret_cast<const float4*>(kr + ((u & 4) ? -16 : 16));
        const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        const float2 kp[4] = {make_float2(ka.x, ka.y), make_float2(ka.z, ka.w), make_float2(kb.x, kb.y),
                              make_float2(kb.z, kb.w)};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float2 qd = make_float2(qv[i], qv[i]);
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fma2(qd, kp[j], acc[i][j]);
        }
      }
      // scaled scores to S (rows = keys), running row maxima
#pragma unroll
      for (int kh = 0; kh < 2; ++kh) {  // key group kg, then kg + 4
        const int32_t key0 = c * kAK + 32 * w + 16 * kh + 4 * kg;
        if (key0 < t) {  // t % 8 == 0: a group of 4 keys is all valid or all past t
          const int sw = (key0 >> 2) & 7;
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            float sc[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float2 a = acc[i][2 * kh + (jj >> 1)];
              sc[i] = __fmul_rn((jj & 1) ? a.y : a.x, scale);
              rmax[i] = fmaxf(rmax[i], sc[i]);
            }
            float* row = S + (size_t)(key0 + jj) * kAQ;
            *reinterpret_cast<float4*>(row + ((qg ^ sw) << 2)) = make_float4(sc[0], sc[1], sc[2], sc[3]);
            *reinterpret_cast<float4*>(row + (((qg + 8) ^ sw) << 2)) = make_float4(sc[4], sc[5], sc[6], sc[7]);
          }
        }
      }
      __syncthreads();  // the K chunk is free
    }
  }
  load_chunk(nk);  // V's first chunk lands while the softmax runs

  // ---- softmax over each query row ----
#pragma unroll
  for (int i = 0; i < 8; ++i) {  // max over the warp's 4 key groups (lanes kg)
    rmax[i] = fmaxf(rmax[i], __shfl_xor_sync(0xffffffffu, rmax[i], 1));
    rmax[i] = fmaxf(rmax[i], __shfl_xor_sync(0xffffffffu, rmax[i], 2));
  }
  if (kg == 0) {
    *reinterpret_cast<float4*>(wmax + w * kAQ + 4 * qg) = make_float4(rmax[0], rmax[1], rmax[2], rmax[3]);
    *reinterpret_cast<float4*>(wmax + w * kAQ + 32 + 4 * qg) = make_float4(rmax[4], rmax[5], rmax[6], rmax[7]);
  }
  __syncthreads();
  {
    const int q = tid & 63, part = tid >> 6;
    const int grp = q >> 2, qe = q & 3;
    const int32_t span = t >> 2, j0 = part * span;  // t % 8 == 0
    float mx = wmax[q];
#pragma unroll
    for (int ww = 1; ww < 8; ++ww) mx = fmaxf(mx, wmax[ww * kAQ + q]);
    const ExpTablePtr et{tab};
    auto at = [&](int32_t j) { return S + (size_t)j * kAQ + ((grp ^ ((j >> 2) & 7)) << 2) + qe; };
    int32_t j = j0;
    for (; j + 4 <= j0 + span; j += 4) {  // four independent exps per step
      float v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = *at(j + u);
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = exp_f32_with(__fsub_rn(v[u], mx), et);
#pragma unroll
      for (int u = 0; u < 4; ++u) *at(j + u) = v[u];
    }
    for (; j < j0 + span; ++j) *at(j) = exp_f32_with(__fsub_rn(*at(j), mx), et);
    __syncthreads();
    if (part == 0) {  // serial sum in key order
      float sum = 0.0f;
#pragma unroll 8
      for (int32_t jj = 0; jj < t; ++jj) sum = __fadd_rn(sum, *at(jj));
      rsum[q] = sum;
    }
    __syncthreads();
    const float sum = rsum[q];
    for (j = j0; j + 4 <= j0 + span; j += 4) {
      float v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = *at(j + u);
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __fdiv_rn(v[u], sum);
#pragma unroll
      for (int u = 0; u < 4; ++u) *at(j + u) = v[u];
    }
    for (; j < j0 + span; ++j) *at(j) = __fdiv_rn(*at(j), sum);
  }

  // ---- phase 2: O += P V, keys in order ----
  const int wq = w >> 2, we = w & 3;
  const int pg = lane >> 2, eg = lane & 3;  // phase 2 lane split
  const int qgrp = 8 * wq + pg;             // this lane's group of 4 queries (0..15)
  int poff[8];  // offset of the query group in S rows j with (j / 4) & 7 == u
#pragma unroll
  for (int u = 0; u < 8; ++u) poff[u] = (qgrp ^ u) << 2;
  float2 o[2][4];  // [query pair (4qgrp, +1) / (+2, +3)][dim 16we + 4eg + e]
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[i][e] = make_float2(0.0f, 0.0f);
  const float* vcol = KV + 16 * we + 4 * eg;
  for (int c = 0; c < nk; ++c) {
    cp_async_wait_all();
    __syncthreads();
    const int32_t k0 = c * kAK;
    const int jn = min(kAK, t - k0);  // a multiple of 8
    const float* pbase = S + (size_t)k0 * kAQ;
    auto step4 = [&](const float* prow, const float* vrow) {  // one group of 4 keys, in order
      float4 pv[4], vv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        pv[u] = *reinterpret_cast<const float4*>(prow + u * kAQ);
        vv[u] = *reinterpret_cast<const float4*>(vrow + u * kADh);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float2 pp[2] = {make_float2(pv[u].x, pv[u].y), make_float2(pv[u].z, pv[u].w)};
        const float ve[4] = {vv[u].x, vv[u].y, vv[u].z, vv[u].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 vd = make_float2(ve[e], ve[e]);
          o[0][e] = fma2(pp[0], vd, o[0][e]);
          o[1][e] = fma2(pp[1], vd, o[1][e]);
        }
      }
    };
    if (jn == kAK) {  // whole chunk: 32-key blocks, the 8 swizzle offsets as constants
#pragma unroll 1
      for (int j32 = 0; j32 < kAK; j32 += 32) {
#pragma unroll
        for (int gq = 0; gq < 8; ++gq) step4(pbase + (j32 + 4 * gq) * kAQ + poff[gq], vcol + (j32 + 4 * gq) * kADh);
      }
    } else {
      for (int j4 = 0; j4 < jn; j4 += 4)
        step4(pbase + j4 * kAQ + ((qgrp ^ ((j4 >> 2) & 7)) << 2), vcol + j4 * kADh);
    }
    __syncthreads();  // the V chunk is free
    if (c + 1 < nk) load_chunk(nk + c + 1);
  }
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int32_t qa = q0 + 4 * qgrp + 2 * i;
    float* dst = out + (base + qa) * ldo + (int64_t)hh * kADh + 16 * we + 4 * eg;
    if (qa < t) {
      *reinterpret_cast<float4*>(dst) = make_float4(o[i][0].x, o[i][1].x, o[i][2].x, o[i][3].x);
#pragma unroll
      for (int e = 0; e < 4; ++e) m = fmaxf(m, fabsf(o[i][e].x));
    }
    if (qa + 1 < t) {
      *reinterpret_cast<float4*>(dst + ldo) = make_float4(o[i][0].y, o[i][1].y, o[i][2].y, o[i][3].y);
#pragma unroll
      for (int e = 0; e < 4; ++e) m = fmaxf(m, fabsf(o[i][e].y));
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
  return (size_t)(kAQsFloats + kAChunkFloats + (size_t)t * kAQ + kAMiscFloats) * sizeof(float);
}

void launch_embedding(const float* ids, int64_t n, const float* table, int64_t v, int32_t d, float* y,
                      AmaxSink amax, int* err, cudaStream_t st) {
  if (n <= 0) return;
  k_embedding<<<grid_for(n, kThreads / 32, 148 * 16), kThreads, 0, st>>>(ids, n, table, v, d, y, amax.ptr, err);
}

rg_status launch_rmsnorm(const float* x, int64_t rows, int32_t d, const float* w, float eps, float inv_d, float* y,
                         AmaxSink amax, cudaStream_t st, int8_t* yq, int64_t ldq, const float* q_scale) {
  if (rows <= 0) return RG_OK;
  // 8 rows of 1024 per block: 33 KB of shared memory, six blocks (48 serial row sums) per SM
  const int32_t rpb = (int32_t)std::max<int64_t>(1, std::min<int64_t>(8, 8192 / d));
  const size_t smem = (size_t)rpb * (d + 4) * sizeof(float);
  if (smem > 200 * 1024) return set_last_error(RG_ERR_UNSUPPORTED, "RMSNorm: rows longer than 51199 elements");
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(k_rmsnorm, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return set_last_error(RG_ERR_CUDA, "RMSNorm: shared-memory opt-in failed");
  const bool vec = (d & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  const int64_t blocks = std::min<int64_t>((rows + rpb - 1) / rpb, 148 * 32);
  k_rmsnorm<<<(unsigned)blocks, kThreads, smem, st>>>(x, rows, d, rpb, vec, w, eps, inv_d, y, amax.ptr, yq, ldq,
                                                       q_scale);
  return RG_OK;
}

void launch_swiglu_mul(const float* gu, int64_t rows, int32_t h, float* y, AmaxSink amax, cudaStream_t st,
                       int8_t* yq, int64_t ldq, const float* q_scale) {
  if (rows <= 0 || h <= 0) return;
  // the vector path needs 16-byte aligned rows; a caller's odd base takes the scalar one
  const bool vec = (h & 3) == 0 && ((reinterpret_cast<uintptr_t>(gu) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  k_swiglu_mul<<<(unsigned)std::min<int64_t>(rows, 148 * 64), kThreads, 0, st>>>(gu, rows, h, vec, y, amax.ptr, yq,
                                                                                  ldq, q_scale);
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


}  // namespace rg
