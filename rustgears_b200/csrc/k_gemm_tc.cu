// k_gemm_tc.cu -- i8 x i8 -> i32 GEMM on the 5th-generation tensor cores (tcgen05
// kind::i8) with the fused dequant + bias + activation epilogue.
//
// Reference: int8_gemm_fused (src/inference/quantize.rs:93-118):
//   out[r, c] = act(f32(sum_k A[r,k] * W[c,k]) * (sa * sw) + bias[c]).
//
// Persistent, warp-specialised, one CTA per SM:
//   warp 0      TMA producer: A [128 x 128 B] and W [BN x 128 B] tiles into a
//               STAGES-deep ring of 128-byte-swizzled shared-memory buffers;
//   warp 1      MMA issuer: 4 x tcgen05.mma (K = 32 each) per stage into a TMEM
//               accumulator; two accumulators (2 x BN columns) so the epilogue
//               of one tile overlaps the main loop of the next;
//   warps 2-17  epilogue: tcgen05.ld (32 lanes x 16 columns), exact f32 epilogue,
//               16-byte stores, running absmax for the next layer's scale.
// Every mbarrier wait is bounded: on timeout the CTA raises an abort flag, the
// roles leave their loops, in-flight copies and MMAs are drained (bounded), TMEM
// is freed and a device error word is set for the host to report.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>

#include "rg_kernels.h"
#include "rg_math.cuh"
#include "rg_sm100.cuh"

namespace rg {
namespace {

using namespace sm100;

constexpr int BM = 128;          // rows per tile (TMEM lanes)
constexpr int BK = 128;          // K bytes per stage (one 128-byte swizzle row)
constexpr int kEpiWarps = 16;   // 4 per SM sub-partition: the exact GELU epilogue is long
constexpr int kThreads = 64 + 32 * kEpiWarps;

template <int BN>
struct Cfg {
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kABytes = BM * BK;
  static constexpr int kBBytes = BN * BK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kBarBytes = 256;
  static constexpr int kSmem = 1024 /*align slack*/ + kStages * kStageBytes + kBarBytes;
};

struct TcParams {
  int64_t m, n, k;          // k: padded reduction length (row stride of A and W)
  const float* a_scale;
  float w_scale;
  const float* w_scale_ch;
  const float* bias;
  int32_t act;
  float act_param;
  float* out;               // [m, n] row-major
  int32_t* acc;             // optional [m, n]
  unsigned* amax;           // optional: max |out| (float bits)
  int32_t tiles_m, tiles_n;
};

__device__ int g_tc_error;  // set when a bounded wait gave up (read by the host)

// Grouped tile order: 16 M-tiles sweep all N-tiles so the W panel stays in L2.
__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int& mb, int& nb) {
  constexpr int G = 16;
  const int per_group = G * tiles_n;
  const int group = tile / per_group;
  const int first_m = group * G;
  const int gm = min(G, tiles_m - first_m);
  const int in = tile - group * per_group;
  mb = first_m + in % gm;
  nb = in / gm;
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
              const TcParams p) {
  using C = Cfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_base = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* full = bars;                       // [kStages]
  uint64_t* empty = bars + C::kStages;         // [kStages]
  uint64_t* tfull = bars + 2 * C::kStages;     // [2]
  uint64_t* tempty = tfull + 2;                // [2]
  uint64_t* done = tempty + 2;                 // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = p.tiles_m * p.tiles_n;
  const int num_kb = (int)((p.k + BK - 1) / BK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);
    }
    mbar_init(done, 1);
    *abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_w);
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_parity[C::kStages];
      bool issued[C::kStages];
      for (int s = 0; s < C::kStages; ++s) issued[s] = false;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, p.tiles_m, p.tiles_n, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort)) { ok = false; break; }
          uint8_t* sa = stage_base + stage * C::kStageBytes;
          uint8_t* sb = sa + C::kABytes;
          mbar_arrive_expect_tx(&full[stage], C::kStageBytes);
          tma_load_2d(sa, &map_a, &full[stage], kb * BK, mb * BM);
          tma_load_2d(sb, &map_w, &full[stage], kb * BK, nb * BN);
          issued[stage] = true;
          issued_parity[stage] = phase;
          if (++stage == C::kStages) { stage = 0; phase ^= 1; }
        }
      }
      // Drain: every issued copy must have landed before the CTA may exit.
      volatile int never = 0;
      for (int s = 0; s < C::kStages; ++s)
        if (issued[s]) mbar_wait(&full[s], issued_parity[s], &never, 200000000ull);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int iter = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++iter) {
        const int buf = iter & 1;
        const uint32_t aphase = (iter >> 1) & 1;
        if (!mbar_wait(&tempty[buf], aphase ^ 1, abort)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_addr(stage_base + stage * C::kStageBytes);
          const uint32_t sb = sa + C::kABytes;
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk)
            mma_i8(d_tmem, desc_kmajor_sw128(sa + kk * 32), desc_kmajor_sw128(sb + kk * 32), idesc,
                   (kb | kk) != 0);
          mma_commit(&empty[stage]);
          if (++stage == C::kStages) { stage = 0; phase ^= 1; }
        }
        if (ok) mma_commit(&tfull[buf]);
      }
      // Drain: all MMAs this thread issued complete before TMEM is freed.
      mma_commit(done);
      volatile int never = 0;
      mbar_wait(done, 0, &never, 200000000ull);
    }
  } else {
    // ---------------- epilogue ----------------
    const int q = warp & 3;                 // TMEM lane quadrant this warp may access
    const int part = (warp - 2) >> 2;       // which quarter of the BN columns
    constexpr int kCols = BN / (kEpiWarps / 4);
    const float sa = p.a_scale[0];
    const float cs_tensor = __fmul_rn(sa, p.w_scale);
    float amax = 0.0f;
    int iter = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++iter) {
      int mb, nb;
      tile_coords(tile, p.tiles_m, p.tiles_n, mb, nb);
      const int buf = iter & 1;
      const uint32_t aphase = (iter >> 1) & 1;
      // every lane waits; the vote keeps the warp converged for the warp-wide tcgen05.ld
      const bool got = mbar_wait(&tfull[buf], aphase, abort);
      if (!__all_sync(0xffffffffu, got)) { *abort = 1; break; }
      tc_fence_after();
      const int64_t row = (int64_t)mb * BM + q * 32 + lane;
      const bool row_ok = row < p.m;
#pragma unroll 1
      for (int c0 = part * kCols; c0 < (part + 1) * kCols; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN + c0), v);
        tmem_ld_wait();
        const int64_t col0 = (int64_t)nb * BN + c0;
        if (row_ok && col0 < p.n) {
          float o[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int64_t c = col0 + j;
            const int64_t cc = c < p.n ? c : p.n - 1;
            const float cs = p.w_scale_ch ? __fmul_rn(sa, __ldg(p.w_scale_ch + cc)) : cs_tensor;
            o[j] = epilogue((int32_t)v[j], cs, __ldg(p.bias + cc), p.act, p.act_param);
            if (c < p.n) amax = fmaxf(amax, fabsf(o[j]));
          }
          float* dst = p.out + row * p.n + col0;
          if (col0 + 16 <= p.n && (p.n & 3) == 0) {
#pragma unroll
            for (int j = 0; j < 16; j += 4)
              *reinterpret_cast<float4*>(dst + j) = make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]);
            if (p.acc) {
              int32_t* ad = p.acc + row * p.n + col0;
#pragma unroll
              for (int j = 0; j < 16; j += 4)
                *reinterpret_cast<int4*>(ad + j) = make_int4((int)v[j], (int)v[j + 1], (int)v[j + 2], (int)v[j + 3]);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (col0 + j < p.n) {
                dst[j] = o[j];
                if (p.acc) p.acc[row * p.n + col0 + j] = (int32_t)v[j];
              }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
    if (p.amax) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if (lane == 0 && amax > 0.0f) atomicMax(p.amax, __float_as_uint(amax));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *abort) atomicExch(&g_tc_error, 1);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t ld, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)ld, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN>
bool launch_bn(const GemmArgs& a, int num_sms, cudaStream_t st) {
  using C = Cfg<BN>;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncSetAttribute(k_gemm_tc<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  });
  CUtensorMap ma, mw;
  if (!make_map(&ma, a.a, a.m, a.lda, BM) || !make_map(&mw, a.w, a.n, a.ldb, BN)) return false;
  TcParams p;
  p.m = a.m; p.n = a.n; p.k = a.k;
  p.a_scale = a.a_scale; p.w_scale = a.w_scale; p.w_scale_ch = a.w_scale_ch; p.bias = a.bias;
  p.act = a.act; p.act_param = a.act_param; p.out = a.out; p.acc = a.acc; p.amax = a.amax.ptr;
  p.tiles_m = (int)((a.m + BM - 1) / BM);
  p.tiles_n = (int)((a.n + BN - 1) / BN);
  const int tiles = p.tiles_m * p.tiles_n;
  const int grid = tiles < num_sms ? tiles : num_sms;
  k_gemm_tc<BN><<<grid, kThreads, C::kSmem, st>>>(ma, mw, p);
  return true;
}

}  // namespace

bool gemm_tc_eligible(const GemmArgs& a) {
  if (a.conv || a.out_l != 0 || a.rows_per_scale != 0 || a.amax.elems_per_slot != 0) return false;
  if (a.m <= 0 || a.n < 16 || a.k < 32 || (a.k & 15) || a.lda != a.k || a.ldb != a.k) return false;
  if ((reinterpret_cast<uintptr_t>(a.a) | reinterpret_cast<uintptr_t>(a.w)) & 15) return false;
  if (a.m * a.n * a.k < (int64_t)1 << 22) return false;
  return encode_fn() != nullptr;
}

bool launch_gemm_tc(const GemmArgs& a, int num_sms, cudaStream_t st) {
  return a.n >= 256 ? launch_bn<256>(a, num_sms, st) : launch_bn<128>(a, num_sms, st);
}

int gemm_tc_take_error() {
  int h = 0, z = 0;
  if (cudaMemcpyFromSymbol(&h, g_tc_error, sizeof h) != cudaSuccess) return -1;
  if (h) cudaMemcpyToSymbol(g_tc_error, &z, sizeof z);
  return h;
}

}  // namespace rg
