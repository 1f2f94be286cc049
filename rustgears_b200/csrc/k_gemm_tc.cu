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
//               the 32 x 16 f32 result staged in shared memory (64-byte swizzle:
//               lane = row writes conflict-free) and written by one TMA tile store,
//               running absmax for the next layer's scale.
// Every mbarrier wait is bounded: on timeout the CTA raises an abort flag, the
// roles leave their loops, in-flight copies and MMAs are drained (bounded), TMEM
// is freed and a device error word is set for the host to report.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "rg_kernels.h"
#include "rg_math.cuh"
#include "rg_f32x2.cuh"
#include "rg_sm100.cuh"

namespace rg {
namespace {

using namespace sm100;

constexpr int BM = 128;          // rows per tile (TMEM lanes)
constexpr int BK = 128;          // K bytes per stage (one 128-byte swizzle row)
constexpr int kEpiWarps = 16;   // 4 per SM sub-partition: the exact GELU epilogue is long
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr uint64_t kDefaultWaitNs = 2000000000ull;  // pipeline waits give up after 2 s

template <int BN>
struct Cfg {
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kABytes = BM * BK;
  static constexpr int kBBytes = BN * BK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kBarBytes = 256;
  static constexpr int kStgBytes = kEpiWarps * 32 * 16 * 4;  // one 32 x 16 f32 tile per epilogue warp
  static constexpr int kSmem = 1024 /*align slack*/ + kStages * kStageBytes + kStgBytes + kBarBytes;
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
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
  int32_t tma_store;        // out written through map_o (n % 4 == 0, 16-byte aligned base)
  int32_t vec_cols;         // bias / w_scale_ch 16-byte aligned and n % 4 == 0: vector loads
  int* err;                 // this call's error word: set to 1 when a bounded wait gave up
  uint64_t wait_ns;         // limit of every pipeline wait
  int32_t starve;           // test hook: the producer issues no loads (the MMA's waits run out)
};

// Grouped tile order: 32 M-tiles sweep all N-tiles, so the 32 A panels in flight and the
// W panel stay in L2 (with 148 CTAs the wave spans about 5 N-tiles of one group).  At
// 65536 x 4096 x 14336 this read 1.46 GB from DRAM per launch against 2.47 GB with 16.
__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int& mb, int& nb) {
  constexpr int G = 32;
  const int per_group = G * tiles_n;
  const int group = tile / per_group;
  const int first_m = group * G;
  const int gm = min(G, tiles_m - first_m);
  const int in = tile - group * per_group;
  mb = first_m + in % gm;
  nb = in / gm;
}

// FULL: every tile is whole (m % BM == 0, n % BN == 0), the output leaves through TMA
// tile stores, bias loads are 16-byte vectors, the weight scale is per tensor, and
// no absmax or accumulator dump is asked for.  The epilogue then has no per-chunk
// branch besides the out-of-range tanh loop (each one a branch-resolution stall of
// every epilogue warp).
template <int BN, int ACT, bool FULL>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
              const __grid_constant__ CUtensorMap map_o, const TcParams p) {
  using C = Cfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_base = smem;
  float* stg_base = reinterpret_cast<float*>(smem + C::kStages * C::kStageBytes);  // 1024-aligned
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes + C::kStgBytes);
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
    if (p.tma_store) tma_prefetch_desc(&map_o);
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
          if (!mbar_wait(&empty[stage], phase ^ 1, abort, p.wait_ns)) { ok = false; break; }
          uint8_t* sa = stage_base + stage * C::kStageBytes;
          uint8_t* sb = sa + C::kABytes;
          if (p.starve) {  // nothing arrives on full[stage]: the MMA issuer's wait runs out
            if (++stage == C::kStages) { stage = 0; phase ^= 1; }
            continue;
          }
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
        if (!mbar_wait(&tempty[buf], aphase ^ 1, abort, p.wait_ns)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort, p.wait_ns)) { ok = false; break; }
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
    float* stg = stg_base + (warp - 2) * (32 * 16);
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
      const bool got = mbar_wait(&tfull[buf], aphase, abort, p.wait_ns);
      if (!__all_sync(0xffffffffu, got)) { *abort = 1; break; }
      tc_fence_after();
      const int64_t row0 = (int64_t)mb * BM + q * 32;
      const int64_t row = row0 + lane;
      const bool row_ok = FULL || row < p.m;
#pragma unroll 1
      for (int c0 = part * kCols; c0 < (part + 1) * kCols; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN + c0), v);
        tmem_ld_wait();
        const int64_t col0 = (int64_t)nb * BN + c0;
        if (!FULL && (col0 >= p.n || row0 >= p.m)) continue;  // warp-uniform
        float o[16];  // (acc as f32) * cs + bias, then the activation in place
        if (FULL || (p.vec_cols && col0 + 16 <= p.n)) {
          // Full chunk: scale and bias as 16-byte loads.
          const float4* bp = reinterpret_cast<const float4*>(p.bias + col0);
          const float4* sp = reinterpret_cast<const float4*>(p.w_scale_ch + col0);
#pragma unroll
          for (int j4 = 0; j4 < 4; ++j4) {
            const float4 b = __ldg(bp + j4);
            float4 cs = make_float4(cs_tensor, cs_tensor, cs_tensor, cs_tensor);
            if (!FULL && p.w_scale_ch) {
              const float4 sw = __ldg(sp + j4);
              cs = make_float4(__fmul_rn(sa, sw.x), __fmul_rn(sa, sw.y), __fmul_rn(sa, sw.z), __fmul_rn(sa, sw.w));
            }
            o[4 * j4] = dequant((int32_t)v[4 * j4], cs.x, b.x);
            o[4 * j4 + 1] = dequant((int32_t)v[4 * j4 + 1], cs.y, b.y);
            o[4 * j4 + 2] = dequant((int32_t)v[4 * j4 + 2], cs.z, b.z);
            o[4 * j4 + 3] = dequant((int32_t)v[4 * j4 + 3], cs.w, b.w);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int64_t c = col0 + j;
            const int64_t cc = c < p.n ? c : p.n - 1;
            const float cs = p.w_scale_ch ? __fmul_rn(sa, __ldg(p.w_scale_ch + cc)) : cs_tensor;
            o[j] = dequant((int32_t)v[j], cs, __ldg(p.bias + cc));
          }
        }
        if constexpr (ACT == ACT_GELU) {
          // Every value takes the restatement with only the common range's cases
          // (bit-identical to the general one there), two values per packed f32x2
          // instruction; the values whose tanh argument lies outside it (|u| >= 7.5,
          // |u| < 2^-25, non-finite) are recomputed with the general restatement, one
          // value per lane per round, in a loop holding a single copy of it.
          float t[16];
          uint32_t redo = 0;
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            const f32x2 u = gelu_arg_x2(pack2(o[j], o[j + 1]));
            tanh_f32_common_x2(lo2(u), hi2(u), t[j], t[j + 1]);
            redo |= (uint32_t)!tanh_common_range(lo2(u)) << j;
            redo |= (uint32_t)!tanh_common_range(hi2(u)) << (j + 1);
          }
          while (__any_sync(0xffffffffu, redo != 0)) {
            const int jr = redo ? __ffs(redo) - 1 : 0;
            float xr = o[0];
#pragma unroll
            for (int j = 1; j < 16; ++j) xr = jr == j ? o[j] : xr;
            const float tr = tanh_f32(gelu_arg(xr));
#pragma unroll
            for (int j = 0; j < 16; ++j) t[j] = (redo && jr == j) ? tr : t[j];
            redo &= redo - 1;
          }
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            const f32x2 g = gelu_from_tanh_x2(pack2(o[j], o[j + 1]), pack2(t[j], t[j + 1]));
            o[j] = lo2(g);
            o[j + 1] = hi2(g);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] = act_apply(ACT, p.act_param, o[j]);
        }
        if (!FULL && p.amax && row_ok) {  // (a consumer quantizes this output: its absmax)
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (col0 + j < p.n) amax = fmaxf(amax, fabsf(o[j]));
        }
        if (FULL || p.tma_store) {
          // The previous chunk's store must have finished reading the staging tile.
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 4; ++j)  // 16-byte chunk j of row `lane`, 64-byte swizzle
            *reinterpret_cast<float4*>(stg + lane * 16 + ((j ^ ((lane >> 1) & 3)) << 2)) =
                make_float4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d_evict_first(&map_o, stg, (int32_t)col0, (int32_t)row0);
            bulk_commit();
          }
        } else if (row_ok) {
          float* dst = p.out + row * p.n + col0;
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (col0 + j < p.n) dst[j] = o[j];
        }
        if (!FULL && p.acc && row_ok) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (col0 + j < p.n) p.acc[row * p.n + col0 + j] = (int32_t)v[j];
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
    if (p.tma_store && lane == 0) bulk_wait_all();
    if (p.amax) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if (lane == 0 && amax > 0.0f) atomicMax(p.amax, __float_as_uint(amax));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *abort) atomicExch(p.err, 1);
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

// Output map: f32 [rows, cols] row-major, 32 x 16 boxes, 64-byte swizzle.
bool make_out_map(CUtensorMap* map, float* base, int64_t rows, int64_t cols) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 4};
  cuuint32_t box[2] = {16, 32};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
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

template <int BN, int ACT, bool FULL>
bool launch_inst(const GemmArgs& a, int num_sms, cudaStream_t st) {
  using C = Cfg<BN>;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncSetAttribute(k_gemm_tc<BN, ACT, FULL>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  });
  CUtensorMap ma, mw, mo;
  if (!make_map(&ma, a.a, a.m, a.lda, BM) || !make_map(&mw, a.w, a.n, a.ldb, BN)) return false;
  memset(&mo, 0, sizeof mo);
  const bool tma_store = (a.n & 3) == 0 && (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 &&
                         make_out_map(&mo, a.out, a.m, a.n);
  TcParams p;
  p.m = a.m; p.n = a.n; p.k = a.k;
  p.a_scale = a.a_scale; p.w_scale = a.w_scale; p.w_scale_ch = a.w_scale_ch; p.bias = a.bias;
  p.act = a.act; p.act_param = a.act_param; p.out = a.out; p.acc = a.acc; p.amax = a.amax.ptr;
  p.tiles_m = (int)((a.m + BM - 1) / BM);
  p.tiles_n = (int)((a.n + BN - 1) / BN);
  p.tma_store = tma_store ? 1 : 0;
  p.vec_cols = (a.n & 3) == 0 &&
               ((reinterpret_cast<uintptr_t>(a.bias) | reinterpret_cast<uintptr_t>(a.w_scale_ch)) & 15) == 0;
  p.err = a.err;
  p.wait_ns = a.wait_ns ? a.wait_ns : kDefaultWaitNs;
  p.starve = a.starve;
  const int tiles = p.tiles_m * p.tiles_n;
  const int grid = tiles < num_sms ? tiles : num_sms;
  if (FULL && !(tma_store && p.vec_cols)) return false;
  k_gemm_tc<BN, ACT, FULL><<<grid, kThreads, C::kSmem, st>>>(ma, mw, mo, p);
  return true;
}

template <int BN, int ACT>
bool launch_bn(const GemmArgs& a, int num_sms, cudaStream_t st) {
  const bool full = a.m % BM == 0 && a.n % BN == 0 && (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(a.bias) & 15) == 0 && a.w_scale_ch == nullptr &&
                    a.amax.ptr == nullptr && a.acc == nullptr && a.out_l == 0;
  return full ? launch_inst<BN, ACT, true>(a, num_sms, st) : launch_inst<BN, ACT, false>(a, num_sms, st);
}

template <int BN>
bool launch_act(const GemmArgs& a, int num_sms, cudaStream_t st) {
  switch (a.act) {
    case ACT_NONE: return launch_bn<BN, ACT_NONE>(a, num_sms, st);
    case ACT_RELU: return launch_bn<BN, ACT_RELU>(a, num_sms, st);
    case ACT_SIGMOID: return launch_bn<BN, ACT_SIGMOID>(a, num_sms, st);
    case ACT_TANH: return launch_bn<BN, ACT_TANH>(a, num_sms, st);
    case ACT_GELU: return launch_bn<BN, ACT_GELU>(a, num_sms, st);
    case ACT_LEAKY_RELU: return launch_bn<BN, ACT_LEAKY_RELU>(a, num_sms, st);
    case ACT_SILU: return launch_bn<BN, ACT_SILU>(a, num_sms, st);
    default: return false;
  }
}

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 tma_encode_fn() { return encode_fn(); }

bool gemm_tc_eligible(const GemmArgs& a) {
  if (a.conv || a.out_l != 0 || a.rows_per_scale != 0 || a.amax.elems_per_slot != 0) return false;
  if (a.m <= 0 || a.n < 16 || a.k < 32 || (a.k & 15) || a.lda != a.k || a.ldb != a.k) return false;
  if ((reinterpret_cast<uintptr_t>(a.a) | reinterpret_cast<uintptr_t>(a.w)) & 15) return false;
  if (a.m * a.n * a.k < (int64_t)1 << 22) return false;
  return encode_fn() != nullptr;
}

bool launch_gemm_tc(const GemmArgs& a, int num_sms, cudaStream_t st) {
  if (!a.err) return false;
  return a.n >= 256 ? launch_act<256>(a, num_sms, st) : launch_act<128>(a, num_sms, st);
}

}  // namespace rg
