// k_conv_tc.cu -- Conv2d as an implicit GEMM on the 5th-generation tensor cores
// (tcgen05 kind::i8), in place of the reference's im2col + GEMM.
//
// Reference: the FusedConv2d arm of NpuProgram::execute (src/inference/npu.rs:319-383):
// per image, im2col (kernels.rs:28-96) -> quantize with the image's own scale ->
// int8_gemm_fused (quantize.rs:93-144) -> NCHW f32.  Here the GEMM rows are the
// output pixels (image, oy, ox) of the whole batch, the reduction runs over
// (ky, kx, c) with c padded to a multiple of 16, and the A operand is gathered
// on the fly from the per-image-quantized NHWC i8 activation:
//
//   warps 0-3   producers: thread r owns row r of the 128-row A tile; per stage it
//               loads the 8 16-byte channel chunks of its output pixel's taps
//               (zero for padding) and stores them in the no-swizzle K-major core-
//               matrix layout (8 rows x 16 B per core matrix); lane 0 of warp 0
//               also loads the weight tile [BN x 128 B] by TMA (128-byte swizzle);
//   warp 4      MMA issuer: 4 x tcgen05.mma (K = 32) per stage into a TMEM
//               accumulator, two accumulators so the epilogue overlaps;
//   warps 5-12  epilogue: tcgen05.ld, act(f32(acc) * (s_img * s_w) + bias), NCHW
//               f32 stores (consecutive lanes are consecutive pixels), per-image
//               absmax for the next conv's scale.
// Every mbarrier wait is bounded; on timeout the CTA raises an abort flag, the roles
// leave their loops, in-flight copies and MMAs are drained, TMEM is freed and a
// device error word is set for the host.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "rg_kernels.h"
#include "rg_math.cuh"
#include "rg_sm100.cuh"

namespace rg {

PFN_cuTensorMapEncodeTiled_v12000 tma_encode_fn();  // k_gemm_tc.cu

namespace {

using namespace sm100;

constexpr int BM = 128;           // output pixels per tile (TMEM lanes)
constexpr int BK = 128;           // reduction bytes per stage: 8 chunks of 16 channels
constexpr int kProdWarps = 4;     // one thread per A row
constexpr int kEpiWarps = 8;      // 2 per TMEM lane quadrant
constexpr int kWarpMma = kProdWarps;
constexpr int kWarpEpi0 = kProdWarps + 1;
constexpr int kThreads = (kProdWarps + 1 + kEpiWarps) * 32;
constexpr int kASbo = 8 * 128;    // 8-row groups of the A tile: 8 chunks x 128 B apart

template <int BN>
struct Cfg {
  static constexpr int kStages = BN == 256 ? 4 : BN == 128 ? 6 : 8;
  static constexpr int kABytes = BM * BK;
  static constexpr int kBBytes = BN * BK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kBarBytes = 256;
  static constexpr int kSmem = 1024 /*align slack*/ + kStages * kStageBytes + kBarBytes;
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
};

struct ConvTcParams {
  const int8_t* a;          // NHWC i8 [n_img, h, w, cpad]
  int32_t n_img, h, w, cpad, k, stride, pad, oh, ow;
  int32_t kxp;              // narrow operand (cpad 4): taps per kernel row, a multiple of 4
  int64_t m;                // n_img * oh * ow
  int32_t n;                // output channels
  int32_t kdim;             // k * k * cpad (multiple of 16)
  const float* a_scale;     // per image
  float w_scale;
  const float* w_scale_ch;
  const float* bias;
  float act_param;
  float* out;               // NCHW [n_img, n, oh, ow]
  const float* residual;    // optional, same layout: out = res_act(epilogue + residual)
  int32_t res_act;
  float res_param;
  int32_t* acc;             // optional, same layout
  unsigned* amax;           // optional absmax sink
  int64_t amax_per_slot;    // 0: one slot; else elements per slot (n * oh * ow: per image)
  int32_t tiles_m, tiles_n;
  int* err;                 // this call's error word: set to 1 when a bounded wait gave up
};

__device__ __forceinline__ uint64_t desc_noswz(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version; layout type 0 = no swizzle
  return d;
}

__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int& mb, int& nb) {
  constexpr int G = 16;  // 16 M-tiles sweep all N-tiles: the weights stay in L2
  const int per_group = G * tiles_n;
  const int group = tile / per_group;
  const int first_m = group * G;
  const int gm = min(G, tiles_m - first_m);
  const int in = tile - group * per_group;
  mb = first_m + in % gm;
  nb = in / gm;
}

__device__ __forceinline__ void flush_slot_max(unsigned* base, int64_t slot, float v) {
  const int64_t s0 = __shfl_sync(0xffffffffu, slot, 0);
  if (__all_sync(0xffffffffu, slot == s0)) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0 && v > 0.0f) atomicMax(base + s0, __float_as_uint(v));
  } else if (slot >= 0 && v > 0.0f) {
    atomicMax(base + slot, __float_as_uint(v));
  }
}

// NARROW: a 4-byte operand pixel (up to 4 channels, e.g. an RGB stem); a 16-byte K
// chunk then holds 4 consecutive taps of one kernel row, loaded as 4 pixel words.
template <int BN, int ACT, bool NARROW>
__global__ void __launch_bounds__(kThreads, 1)
    k_conv_tc(const __grid_constant__ CUtensorMap map_w, const ConvTcParams p) {
  using C = Cfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* full = bars;                    // [kStages]
  uint64_t* empty = bars + C::kStages;      // [kStages]
  uint64_t* tfull = bars + 2 * C::kStages;  // [2]
  uint64_t* tempty = tfull + 2;             // [2]
  uint64_t* done = tempty + 2;              // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = p.tiles_m * p.tiles_n;
  const int num_kb = (p.kdim + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], kProdWarps);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);
    }
    mbar_init(done, 1);
    *abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_w);
  }
  if (warp == kWarpMma) tmem_alloc(tmem_slot, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < kProdWarps) {
    // ---------------- producers: A gather (+ weight TMA) ----------------
    const int r = threadIdx.x;  // this thread's row of the A tile
    const uint32_t a_off = (uint32_t)((r & 7) * 16 + (r >> 3) * kASbo);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    // stages whose weight copy this thread (warp 0 lane 0) issued and that were not consumed
    uint32_t issued_parity[C::kStages];
    bool issued[C::kStages];
    for (int s = 0; s < C::kStages; ++s) issued[s] = false;
    const int64_t hw_out = (int64_t)p.oh * p.ow;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      int mb, nb;
      tile_coords(tile, p.tiles_m, p.tiles_n, mb, nb);
      const int64_t row = (int64_t)mb * BM + r;
      const bool valid = row < p.m;
      int32_t img = 0, iy0 = 0, ix0 = 0;
      if (valid) {
        img = (int32_t)(row / hw_out);
        const int32_t rem = (int32_t)(row - (int64_t)img * hw_out);
        const int32_t oy = rem / p.ow, ox = rem - oy * p.ow;
        iy0 = oy * p.stride - p.pad;
        ix0 = ox * p.stride - p.pad;
      }
      const int8_t* base = p.a + (int64_t)img * p.h * p.w * p.cpad;
      // (tap, channel) of the next chunk to load, advanced incrementally; the loads of
      // stage kb + 1 are in flight while stage kb waits for its slot and is stored
      int32_t c0 = 0, kx = 0, ky = 0, k0 = 0;
      auto load_stage = [&](uint4 (&v)[8]) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          v[j] = make_uint4(0u, 0u, 0u, 0u);
          const int32_t iy = iy0 + ky;
          if (NARROW) {  // taps kx..kx+3 of kernel row ky: 4 pixel words
            if (valid && k0 < p.kdim && iy >= 0 && iy < p.h) {
              const uint32_t* rowp = reinterpret_cast<const uint32_t*>(base + (int64_t)iy * p.w * 4);
              uint32_t wv[4];
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                const int32_t ix = ix0 + kx + t;
                wv[t] = (kx + t < p.k && ix >= 0 && ix < p.w) ? __ldg(rowp + ix) : 0u;
              }
              v[j] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
            }
            k0 += 16;
            kx += 4;
            if (kx == p.kxp) { kx = 0; ++ky; }
          } else {
            const int32_t ix = ix0 + kx;
            if (valid && k0 < p.kdim && iy >= 0 && iy < p.h && ix >= 0 && ix < p.w)
              v[j] = __ldg(reinterpret_cast<const uint4*>(base + ((int64_t)iy * p.w + ix) * p.cpad + c0));
            k0 += 16;
            c0 += 16;
            if (c0 == p.cpad) {
              c0 = 0;
              if (++kx == p.k) { kx = 0; ++ky; }
            }
          }
        }
      };
      uint4 cur[8], nxt[8];
      load_stage(nxt);
      for (int kb = 0; kb < num_kb; ++kb) {
#pragma unroll
        for (int j = 0; j < 8; ++j) cur[j] = nxt[j];
        if (kb + 1 < num_kb) load_stage(nxt);
        const bool got = mbar_wait(&empty[stage], phase ^ 1, abort);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
        uint8_t* sa = smem + stage * C::kStageBytes;
#pragma unroll
        for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(sa + a_off + j * 128) = cur[j];
        fence_async_smem();  // generic-proxy stores -> visible to the tensor core
        __syncwarp();
        if (lane == 0) {
          if (warp == 0) {
            mbar_arrive_expect_tx(&full[stage], C::kBBytes);
            tma_load_2d(sa + C::kABytes, &map_w, &full[stage], kb * BK, nb * BN);
            issued[stage] = true;
            issued_parity[stage] = phase;
          } else {
            mbar_arrive(&full[stage]);
          }
        }
        if (++stage == C::kStages) { stage = 0; phase ^= 1; }
      }
    }
    if (!ok) *abort = 1;
    if (warp == 0 && lane == 0) {  // every issued weight copy must land before the CTA exits
      volatile int never = 0;
      for (int s = 0; s < C::kStages; ++s)
        if (issued[s]) mbar_wait(&full[s], issued_parity[s], &never, 200000000ull);
    }
  } else if (warp == kWarpMma) {
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
          const uint32_t sa = smem_addr(smem + stage * C::kStageBytes);
          const uint32_t sb = sa + C::kABytes;
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk)
            mma_i8(d_tmem, desc_noswz(sa + kk * 256, 128, kASbo), desc_kmajor_sw128(sb + kk * 32), idesc,
                   (kb | kk) != 0);
          mma_commit(&empty[stage]);
          if (++stage == C::kStages) { stage = 0; phase ^= 1; }
        }
        if (ok) mma_commit(&tfull[buf]);
      }
      mma_commit(done);
      volatile int never = 0;
      mbar_wait(done, 0, &never, 200000000ull);
    }
  } else {
    // ---------------- epilogue ----------------
    const int e = warp - kWarpEpi0;
    const int q = warp & 3;           // TMEM lane quadrant this warp may access
    const int part = e >> 2;          // which half of the BN columns
    constexpr int kCols = BN / 2;
    const int64_t hw_out = (int64_t)p.oh * p.ow;
    int iter = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++iter) {
      int mb, nb;
      tile_coords(tile, p.tiles_m, p.tiles_n, mb, nb);
      const int buf = iter & 1;
      const uint32_t aphase = (iter >> 1) & 1;
      const bool got = mbar_wait(&tfull[buf], aphase, abort);
      if (!__all_sync(0xffffffffu, got)) { *abort = 1; break; }
      tc_fence_after();
      const int64_t row = (int64_t)mb * BM + q * 32 + lane;
      const bool row_ok = row < p.m;
      int64_t img = 0, pix = 0;
      if (row_ok) {
        img = row / hw_out;
        pix = row - img * hw_out;
      }
      const float sa = row_ok ? p.a_scale[img] : 0.0f;
      const float cs_tensor = __fmul_rn(sa, p.w_scale);
      float* obase = p.out + img * (int64_t)p.n * hw_out + pix;
      const float* rbase = p.residual ? p.residual + img * (int64_t)p.n * hw_out + pix : nullptr;
      float mx = 0.0f;
#pragma unroll 1
      for (int c0 = part * kCols; c0 < (part + 1) * kCols; c0 += 16) {
        uint32_t v[16];
        __syncwarp();  // the warp-wide TMEM load runs converged
        tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN + c0), v);
        tmem_ld_wait();
        const int64_t col0 = (int64_t)nb * BN + c0;
        if (row_ok && col0 < p.n) {
          // the residual values first: all 16 loads in flight before the stores
          float res[16];
          if (rbase) {
#pragma unroll
            for (int j = 0; j < 16; ++j) res[j] = col0 + j < p.n ? __ldg(rbase + (col0 + j) * hw_out) : 0.0f;
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int64_t c = col0 + j;
            if (c < p.n) {
              const float cs = p.w_scale_ch ? __fmul_rn(sa, __ldg(p.w_scale_ch + c)) : cs_tensor;
              float o = epilogue_t<ACT>((int32_t)v[j], cs, __ldg(p.bias + c), p.act_param);
              if (rbase) {  // the block's activation: none, ReLU or LeakyReLU (the fusable ones)
                o = __fadd_rn(o, res[j]);
                if (p.res_act == ACT_RELU) o = fmaxf(o, 0.0f);
                else if (p.res_act == ACT_LEAKY_RELU) o = o > 0.0f ? o : __fmul_rn(p.res_param, o);
              }
              obase[c * hw_out] = o;
              if (p.acc) p.acc[img * (int64_t)p.n * hw_out + c * hw_out + pix] = (int32_t)v[j];
              mx = fmaxf(mx, fabsf(o));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
      if (p.amax) flush_slot_max(p.amax, row_ok ? (p.amax_per_slot ? img : 0) : -1, mx);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *abort) atomicExch(p.err, 1);
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

bool make_w_map(CUtensorMap* map, const void* base, int64_t rows, int64_t ld, int box_rows) {
  auto fn = tma_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)ld, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int ACT, bool NARROW>
bool launch_bn(const GemmArgs& a, int num_sms, cudaStream_t st) {
  using C = Cfg<BN>;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncSetAttribute(k_conv_tc<BN, ACT, NARROW>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  });
  CUtensorMap mw;
  if (!make_w_map(&mw, a.w, a.n, a.ldb, BN)) return false;
  ConvTcParams p;
  p.a = a.a;
  p.n_img = (int32_t)(a.m / a.out_l);
  p.h = a.g.h; p.w = a.g.w; p.cpad = a.g.cpad; p.k = a.g.k; p.stride = a.g.stride; p.pad = a.g.pad;
  p.oh = a.g.oh; p.ow = a.g.ow;
  p.kxp = a.g.kxp ? a.g.kxp : a.g.k;
  p.m = a.m; p.n = (int32_t)a.n; p.kdim = (int32_t)a.k;
  p.a_scale = a.a_scale; p.w_scale = a.w_scale; p.w_scale_ch = a.w_scale_ch; p.bias = a.bias;
  p.act_param = a.act_param; p.out = a.out; p.acc = a.acc;
  p.residual = a.residual; p.res_act = a.res_act; p.res_param = a.res_param;
  p.amax = a.amax.ptr; p.amax_per_slot = a.amax.elems_per_slot;
  p.tiles_m = (int)((a.m + BM - 1) / BM);
  p.tiles_n = (int)((a.n + BN - 1) / BN);
  p.err = a.err;
  const int tiles = p.tiles_m * p.tiles_n;
  const int grid = tiles < num_sms ? tiles : num_sms;
  k_conv_tc<BN, ACT, NARROW><<<grid, kThreads, C::kSmem, st>>>(mw, p);
  return true;
}

template <int BN, bool NARROW = false>
bool launch_act(const GemmArgs& a, int num_sms, cudaStream_t st) {
  switch (a.act) {
    case ACT_NONE: return launch_bn<BN, ACT_NONE, NARROW>(a, num_sms, st);
    case ACT_RELU: return launch_bn<BN, ACT_RELU, NARROW>(a, num_sms, st);
    case ACT_SIGMOID: return launch_bn<BN, ACT_SIGMOID, NARROW>(a, num_sms, st);
    case ACT_TANH: return launch_bn<BN, ACT_TANH, NARROW>(a, num_sms, st);
    case ACT_GELU: return launch_bn<BN, ACT_GELU, NARROW>(a, num_sms, st);
    case ACT_LEAKY_RELU: return launch_bn<BN, ACT_LEAKY_RELU, NARROW>(a, num_sms, st);
    case ACT_SILU: return launch_bn<BN, ACT_SILU, NARROW>(a, num_sms, st);
    default: return false;
  }
}

}  // namespace

// Convs the kernel takes: channels padded to a multiple of 16 in the NHWC operand and the
// weights, NCHW output, per-image activation scales, and enough work for the tensor cores.
bool conv_tc_eligible(const GemmArgs& a) {
  if (!a.conv || a.out_l <= 0 || a.rows_per_scale != a.out_l) return false;
  const bool narrow = a.g.cpad == 4;
  const int32_t kxp = a.g.kxp ? a.g.kxp : a.g.k;
  if (narrow ? (kxp & 3) || kxp < a.g.k || a.k != (int64_t)a.g.k * kxp * 4
             : (a.g.cpad & 15) || kxp != a.g.k || a.k != (int64_t)a.g.k * a.g.k * a.g.cpad)
    return false;
  if (a.g.c != a.g.cpad || a.n < 16 || (a.k & 15) || a.ldb != a.k) return false;
  if (a.amax.ptr && a.amax.elems_per_slot != 0 && a.amax.elems_per_slot != a.n * a.out_l) return false;
  if ((reinterpret_cast<uintptr_t>(a.a) | reinterpret_cast<uintptr_t>(a.w)) & 15) return false;
  if (a.m * a.n * a.k < (int64_t)1 << 22) return false;
  return tma_encode_fn() != nullptr;
}

bool launch_conv_tc(const GemmArgs& a, int num_sms, cudaStream_t st) {
  if (!a.err) return false;
  if (a.g.cpad == 4) return launch_act<64, true>(a, num_sms, st);
  if (a.n >= 256) return launch_act<256>(a, num_sms, st);
  if (a.n >= 128) return launch_act<128>(a, num_sms, st);
  return launch_act<64>(a, num_sms, st);
}


}  // namespace rg
