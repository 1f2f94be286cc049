// k_mlp2.cu -- a program of two narrow INT8 Linears in one cooperative launch.
//
// Reference semantics (src/inference/npu.rs:307-318, quantize.rs:18-35,93-118): each
// Linear quantizes its whole input with the scale of the batch-wide absmax, takes i8 x i8
// -> i32 dot products and applies act(f32(acc) * (sa * sw) + bias).  The two batch-wide
// reductions make three phases, separated by grid-wide barriers:
//   1. absmax of the input x [m, k1];
//   2. one thread per row: quantize the row, dot products with the n1 <= 32 rows of W1,
//      epilogue, the hidden row kept in the thread's registers, hidden absmax;
//   3. quantize the hidden row with its scale, dot products with W2, epilogue, store.
// The arithmetic is the narrow GEMM's (k_gemm_simt.cu) op for op, so the output equals
// the two-launch path bit for bit.  Every block must be resident at once, so the kernel
// is launched cooperatively with one row per thread (m <= resident threads), and every
// barrier wait is bounded: a wait that gives up sets the call's error word and the
// blocks leave.
#include <cuda_runtime.h>

#include "rg_kernels.h"
#include "rg_math.cuh"
#include "rg_sm100.cuh"

namespace rg {
namespace {

using namespace sm100;

constexpr int kMlpThreads = 256;
constexpr int kMaxK1 = 64, kMaxN = 32;

struct Mlp2Params {
  Mlp2Args a;
  unsigned* ws;      // [2] barrier arrivals, [3] abort (words 0, 1 unused)
  uint64_t wait_ns;  // limit of each barrier wait
};

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float b = 0.0f;
#pragma unroll
  for (int i = 0; i < kMlpThreads / 32; ++i) b = fmaxf(b, red[i]);
  __syncthreads();
  return b;
}

// Grid-wide barrier number `k` (1, 2): returns false when the wait gave up (or another
// block's did); the arrivals counter is zeroed before the launch.  Thread 0 then reads
// *src (the absmax the barrier completed) into *word for the block: one read per
// block, not one per warp of every block on the same address.
__device__ bool grid_barrier(unsigned* ws, unsigned k, uint64_t limit_ns, int* flag, const unsigned* src,
                             unsigned* word) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(ws + 2, 1u);
    const unsigned target = k * gridDim.x;
    volatile unsigned* cnt = ws + 2;
    volatile unsigned* abort = ws + 3;
    const uint64_t t0 = global_timer_ns();
    int ok = 1;
    while (*cnt < target) {
      if (*abort || global_timer_ns() - t0 > limit_ns) {
        ok = 0;
        atomicExch(ws + 3, 1u);
        break;
      }
      __nanosleep(32);
    }
    __threadfence();
    *flag = ok;
    *word = *(volatile const unsigned*)src;
  }
  __syncthreads();
  return *flag != 0;
}

__device__ __forceinline__ uint32_t pack4q(float a, float b, float c, float d, float inv) {
  return (uint32_t)(quant1_bounded(a, inv) & 0xff) | ((uint32_t)(quant1_bounded(b, inv) & 0xff) << 8) |
         ((uint32_t)(quant1_bounded(c, inv) & 0xff) << 16) | ((uint32_t)(quant1_bounded(d, inv) & 0xff) << 24);
}

// N1P: n1 rounded up to 4, 8, 16 or 32; KW: 4-byte words of an input row rounded up to
// 1, 4 or 16; ACT1: the first Linear's activation (or -1: chosen at run time).  The
// hidden-row loops run over these compile-time widths without early exits, so their
// iterations interleave; the weights' padded rows and columns are zero, and the padded
// hidden values are zeroed and left out of the absmax.
template <int N1P, int KW, int ACT1>
__global__ void __launch_bounds__(kMlpThreads) k_mlp2(const Mlp2Params P) {
  const Mlp2Args& a = P.a;
  __shared__ __align__(16) int32_t w1s[kMaxN][kMaxK1 / 4];
  __shared__ __align__(16) int32_t w2s[kMaxN][kMaxN / 4];
  __shared__ float cs1[kMaxN], bias1[kMaxN], cs2[kMaxN], bias2[kMaxN];
  __shared__ float red[kMlpThreads / 32];
  __shared__ int flag;
  __shared__ unsigned word;
  const int kw1 = a.kpad1 >> 2, kw2 = N1P >> 2;
  for (int i = threadIdx.x; i < N1P * KW; i += kMlpThreads) {
    const int j = i / KW, w = i % KW;
    w1s[j][w] = j < a.n1 && w < kw1 ? __ldg(reinterpret_cast<const int32_t*>(a.w1 + (int64_t)j * a.kpad1) + w) : 0;
  }
  // W2's padded columns (n1 .. N1P) hold zeros in the weights
  for (int i = threadIdx.x; i < a.n2 * kw2; i += kMlpThreads) {
    const int j = i / kw2, w = i % kw2;
    uint32_t v = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b)
      if (4 * w + b < a.n1) v |= (uint32_t)(uint8_t)a.w2[(int64_t)j * a.kpad2 + 4 * w + b] << (8 * b);
    w2s[j][w] = (int32_t)v;
  }
  if (threadIdx.x < (unsigned)kMaxN) bias1[threadIdx.x] = threadIdx.x < (unsigned)a.n1 ? a.b1[threadIdx.x] : 0.0f;
  if (threadIdx.x < (unsigned)a.n2) bias2[threadIdx.x] = a.b2[threadIdx.x];

  // ---- phase 1: absmax of the input ----
  float m1 = 0.0f;
  const int64_t total = a.m * a.k1;
  const int64_t tid = (int64_t)blockIdx.x * kMlpThreads + threadIdx.x, nth = (int64_t)gridDim.x * kMlpThreads;
  if ((total & 3) == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0) {
    const float4* x4 = reinterpret_cast<const float4*>(a.x);
    for (int64_t i = tid; i < total / 4; i += nth) {
      const float4 v = __ldg(x4 + i);
      m1 = fmaxf(m1, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
  } else {
    for (int64_t i = tid; i < total; i += nth) m1 = fmaxf(m1, fabsf(__ldg(a.x + i)));
  }
  m1 = block_max(m1, red);
  if (threadIdx.x == 0 && m1 > 0.0f) atomicMax(a.amax1, __float_as_uint(m1));
  // this thread's row (its first 16 values) is loaded before the barrier wait
  const int64_t row = tid;
  const bool has_row = row < a.m;
  const float* xr = a.x + row * a.k1;
  constexpr int kPre = KW < 4 ? 4 * KW : 16;
  float xpre[kPre];
#pragma unroll
  for (int e = 0; e < kPre; ++e) xpre[e] = has_row && e < a.k1 ? __ldg(xr + e) : 0.0f;
  if (!grid_barrier(P.ws, 1, P.wait_ns, &flag, a.amax1, &word)) {
    if (threadIdx.x == 0) atomicExch(a.err, 1);
    return;
  }

  // ---- phase 2: the first Linear, one row per thread ----
  const float sa1 = quant_scale(__uint_as_float(word)), inv1 = quant_inv(sa1);
  if (threadIdx.x < (unsigned)kMaxN) cs1[threadIdx.x] = __fmul_rn(sa1, a.w1_scale);
  __syncthreads();
  float h[N1P];
#pragma unroll
  for (int j = 0; j < N1P; ++j) h[j] = 0.0f;
  float m2 = 0.0f;
  if (has_row) {
    uint32_t q[KW];
#pragma unroll
    for (int w = 0; w < KW; ++w) {
      float v[4];
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int e = 4 * w + b;
        v[b] = e < kPre ? xpre[e < kPre ? e : 0] : (e < a.k1 ? __ldg(xr + e) : 0.0f);
      }
      q[w] = pack4q(v[0], v[1], v[2], v[3], inv1);
    }
#pragma unroll
    for (int j = 0; j < N1P; ++j) {
      int32_t acc = 0;
#pragma unroll
      for (int w = 0; w < KW; ++w) acc = __dp4a((int32_t)q[w], w1s[j][w], acc);
      const float v = ACT1 >= 0 ? epilogue_t<ACT1 >= 0 ? ACT1 : 0>(acc, cs1[j], bias1[j], a.p1)
                                : epilogue(acc, cs1[j], bias1[j], a.act1, a.p1);
      h[j] = j < a.n1 ? v : 0.0f;
      m2 = fmaxf(m2, fabsf(h[j]));
    }
  }
  m2 = block_max(m2, red);
  if (threadIdx.x == 0 && m2 > 0.0f) atomicMax(a.amax2, __float_as_uint(m2));
  if (!grid_barrier(P.ws, 2, P.wait_ns, &flag, a.amax2, &word)) {
    if (threadIdx.x == 0) atomicExch(a.err, 1);
    return;
  }

  // ---- phase 3: the second Linear on the hidden row ----
  const float sa2 = quant_scale(__uint_as_float(word)), inv2 = quant_inv(sa2);
  if (threadIdx.x < (unsigned)a.n2) cs2[threadIdx.x] = __fmul_rn(sa2, a.w2_scale);
  __syncthreads();
  float m3 = 0.0f;
  if (has_row) {
    uint32_t q[N1P / 4];
#pragma unroll
    for (int w = 0; w < N1P / 4; ++w) q[w] = pack4q(h[4 * w], h[4 * w + 1], h[4 * w + 2], h[4 * w + 3], inv2);
    float* yr = a.y + row * a.n2;
    for (int j = 0; j < a.n2; ++j) {
      int32_t acc = 0;
#pragma unroll
      for (int w = 0; w < N1P / 4; ++w) acc = __dp4a((int32_t)q[w], w2s[j][w], acc);
      const float v = epilogue(acc, cs2[j], bias2[j], a.act2, a.p2);
      yr[j] = v;
      m3 = fmaxf(m3, fabsf(v));
    }
  }
  if (a.amax) {
    m3 = block_max(m3, red);
    if (threadIdx.x == 0 && m3 > 0.0f) atomicMax(a.amax, __float_as_uint(m3));
  }
}

template <int N1P, int KW, int ACT1>
bool launch_n1(const Mlp2Args& a, unsigned* ws, cudaStream_t st) {
  static int per_sm = -1, sms = 0;
  if (per_sm < 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_mlp2<N1P, KW, ACT1>, kMlpThreads, 0) != cudaSuccess)
      per_sm = 0;
  }
  const int64_t blocks = (a.m + kMlpThreads - 1) / kMlpThreads;
  if (blocks < 1 || blocks > (int64_t)per_sm * sms) return false;
  if (cudaMemsetAsync(ws, 0, 4 * sizeof(unsigned), st) != cudaSuccess) return false;
  Mlp2Params P;
  P.a = a;
  P.ws = ws;
  P.wait_ns = 1000000000ull;
  void* args[] = {&P};
  return cudaLaunchCooperativeKernel((const void*)k_mlp2<N1P, KW, ACT1>, dim3((unsigned)blocks), dim3(kMlpThreads),
                                     args, 0, st) == cudaSuccess;
}

template <int N1P, int KW>
bool launch_act1(const Mlp2Args& a, unsigned* ws, cudaStream_t st) {
  switch (a.act1) {
    case ACT_NONE: return launch_n1<N1P, KW, ACT_NONE>(a, ws, st);
    case ACT_RELU: return launch_n1<N1P, KW, ACT_RELU>(a, ws, st);
    case ACT_LEAKY_RELU: return launch_n1<N1P, KW, ACT_LEAKY_RELU>(a, ws, st);
    default: return launch_n1<N1P, KW, -1>(a, ws, st);  // transcendental activations: chosen at run time
  }
}

template <int N1P>
bool launch_kw(const Mlp2Args& a, unsigned* ws, cudaStream_t st) {
  const int kwu = (a.k1 + 3) / 4;
  if (kwu <= 1) return launch_act1<N1P, 1>(a, ws, st);
  if (kwu <= 4) return launch_act1<N1P, 4>(a, ws, st);
  return launch_act1<N1P, 16>(a, ws, st);
}

}  // namespace

bool mlp2_eligible(const Mlp2Args& a) {
  return a.m > 0 && a.k1 >= 1 && a.k1 <= kMaxK1 && a.kpad1 >= a.k1 && (a.kpad1 & 15) == 0 && a.kpad1 <= kMaxK1 &&
         a.n1 >= 1 && a.n1 <= kMaxN && a.n2 >= 1 && a.n2 <= kMaxN && a.kpad2 >= a.n1 && a.err && a.amax1 && a.amax2 &&
         (reinterpret_cast<uintptr_t>(a.w1) & 3) == 0;
}

bool launch_mlp2(const Mlp2Args& a, unsigned* ws, cudaStream_t st) {
  if (!mlp2_eligible(a)) return false;
  const int n1p = (a.n1 + 3) / 4 * 4;
  if (n1p <= 4) return launch_kw<4>(a, ws, st);
  if (n1p <= 8) return launch_kw<8>(a, ws, st);
  if (n1p <= 16) return launch_kw<16>(a, ws, st);
  return launch_kw<32>(a, ws, st);
}

}  // namespace rg
