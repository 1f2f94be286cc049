// k_conv3x3.cu -- 3x3 / stride 1 / pad 1 Conv2d on the tcgen05 tensor cores as a direct
// convolution over zero-padded input tiles (no im2col gather).
//
// Reference: the FusedConv2d arm of NpuProgram::execute (src/inference/npu.rs:319-383):
// per image, im2col (kernels.rs:28-96), quantize with the image's scale, int8 GEMM with
// the fused epilogue, NCHW f32.  The i32 sums do not depend on the reduction order, so
// the taps may be accumulated one after the other.
//
// Index the zero-padded image by flat positions f = py * (W + 2) + px (py, px in the
// padded (H + 2) x (W + 2) grid).  The output pixel centred at f reads, for tap
// (ky, kx), the padded pixel f + (ky - 1) (W + 2) + (kx - 1): every tap's A operand is
// the same run of 128 consecutive positions shifted by a constant.  So a CTA tile is
// 128 consecutive centre positions of one image; the operand is stored as 16-channel
// chunk planes [img][chunk][h][w][16 B], so per 64-channel stage 4 TMA loads (rows of
// 16 (W + 2) contiguous bytes) bring the padded input rows the tile needs as 4 planes
// [rows][W + 2][16 B] (out-of-range rows and columns read as zeros: the padding), and
// the MMA warp issues 9 taps x 2 MMAs whose A descriptors point into the planes at
// the tap's row offset (no-swizzle K-major layout with 16-byte rows: an 8-row group is
// 128 contiguous bytes, so any row offset is a valid start).  Positions on the padding
// columns are computed and discarded (2 of W + 2 per row).  Weights for the stage
// arrive by one bulk copy, pre-arranged by the host in the same core-matrix layout.
//
//   warp 0     producer (lane 0): 4 TMA tile loads + 1 weight bulk copy per stage
//   warp 1     MMA issuer (lane 0): 18 tcgen05.mma (M 128, K 32) per stage into one
//              of two TMEM accumulators
//   warps 2-17 epilogue: tcgen05.ld, act(f32(acc) * (s_img * s_w) + bias), optional
//              fused residual add, NCHW stores, per-image absmax for the next conv
//              (and, optionally, over the pixels a later strided 1x1 conv reads)
// Every mbarrier wait is bounded; on timeout the CTA raises an abort flag, the roles
// leave their loops, copies and MMAs in flight are drained, TMEM is freed and a device
// error word is set for the host.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "rg_kernels.h"
#include "rg_math.cuh"
#include "rg_sm100.cuh"

namespace rg {

PFN_cuTensorMapEncodeTiled_v12000 tma_encode_fn();  // k_gemm_tc.cu

namespace {

using namespace sm100;

constexpr int BM = 128;         // centre positions per tile (TMEM lanes)
constexpr int kCS = 64;         // channels per stage (4 chunk planes of 16 bytes)
constexpr int kEpiWarps = 16;   // 4 per TMEM lane quadrant (the stores and residual loads are latency-bound)
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kBarBytes = 256;
// Four TMEM accumulators: an epilogue warp may run up to three tiles ahead of the
// slowest one, so the warps drift out of step and one's global stores overlap
// another's TMEM loads and arithmetic (the store path is the epilogue's bound).
constexpr int kAccBufs = 4;

struct C3Params {
  int32_t n_img, h, w, cpad, n;    // n: output channels
  int32_t n_pad;                   // n rounded up to BN (staged per-channel constants)
  int32_t tiles_m, tiles_n, stages_k;  // tiles per image, N tiles, 64-channel stages
  int32_t rbox;                    // padded rows per TMA box
  int32_t wp, pad_t, pad_l;        // padded row length; zero rows / columns before the image
  int32_t f0;                      // flat position of output (0, 0): pad_t * wp + pad_l
  int32_t min_off;                 // smallest tap offset (flat positions)
  int32_t toff[9];                 // tap offsets relative to the centre, dy * wp + dx
  int32_t plane_bytes;             // rbox * (w + 2) * 16: what one TMA load writes
  int32_t plane_stride;            // plane_bytes rounded up to 128 (TMA destination alignment)
  int32_t stage_bytes, ring;       // bytes per ring slot (A planes + weights), slots
  int32_t resident;                // one K stage and one N tile: the weights are loaded once
                                   // into their own region, the ring slots hold A only
  const int8_t* wd;                // weights [tiles_n][stages_k][9][4][BN][16]
  const float* a_scale;            // per image
  float w_scale;
  const float* w_scale_ch;
  const float* bias;
  float act_param;
  float* out;                      // NCHW [n_img, n, h, w]
  const float* residual;           // optional: out = res_act(epilogue + residual)
  int32_t res_act;
  float res_param;
  int32_t* acc;                    // optional i32 dump, NCHW
  unsigned* amax;                  // optional absmax sink
  int64_t amax_per_slot;           // 0: one slot; else n * h * w (per image)
  unsigned* amax2;                 // optional per-image absmax over the pixels a later
  int32_t cov_s, cov_oh, cov_ow;   // 1x1 / pad 0 / stride cov_s conv reads
  int* err;                        // this call's error word: set to 1 when a bounded wait gave up
};

__device__ __forceinline__ uint64_t desc_rows16(uint32_t saddr, uint32_t lbo) {
  // no-swizzle K-major: rows 16 bytes apart (8-row groups 128 B apart), K chunks `lbo` apart
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(128 >> 4) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version; layout type 0 = no swizzle
  return d;
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t c0,
                                            int32_t c1, int32_t c2, int32_t c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, "
      "%6}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// tile -> (image, centre tile within the image, N tile); N tiles vary fastest so the
// CTAs working on one image's input tile run close together (L2 reuse).  A CTA's tiles
// are blockIdx.x + k gridDim.x: the walk adds gridDim.x's decomposition with carries
// instead of dividing every tile index (the tile count is below 2^31).
struct TileWalk {
  int32_t img, mt, nb;        // current tile
  int32_t d_img, d_mt, d_nb;  // gridDim.x decomposed
  int32_t tiles_m, tiles_n;
  __device__ void start(const C3Params& p, uint32_t first) {
    tiles_m = p.tiles_m;
    tiles_n = p.tiles_n;
    const uint32_t g = gridDim.x;
    d_nb = (int32_t)(g % (uint32_t)tiles_n);
    d_mt = (int32_t)((g / (uint32_t)tiles_n) % (uint32_t)tiles_m);
    d_img = (int32_t)((g / (uint32_t)tiles_n) / (uint32_t)tiles_m);
    nb = (int32_t)(first % (uint32_t)tiles_n);
    mt = (int32_t)((first / (uint32_t)tiles_n) % (uint32_t)tiles_m);
    img = (int32_t)((first / (uint32_t)tiles_n) / (uint32_t)tiles_m);
  }
  __device__ void advance() {
    nb += d_nb;
    int32_t c = 0;
    if (nb >= tiles_n) { nb -= tiles_n; c = 1; }
    mt += d_mt + c;
    c = 0;
    if (mt >= tiles_m) { mt -= tiles_m; c = 1; }
    img += d_img + c;
  }
};

__device__ __forceinline__ void flush_slot_max(unsigned* base, int64_t slot, float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0 && v > 0.0f && slot >= 0) atomicMax(base + slot, __float_as_uint(v));
}

template <int BN, int ACT, int TAPS>
__global__ void __launch_bounds__(kThreads, 1)
    k_conv3x3(const __grid_constant__ CUtensorMap map_in, const C3Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)p.ring * p.stage_bytes);
  uint64_t* full = bars;              // [ring]
  uint64_t* empty = bars + p.ring;    // [ring]
  uint64_t* tfull = empty + p.ring;   // [kAccBufs]
  uint64_t* tempty = tfull + kAccBufs;  // [kAccBufs]
  uint64_t* done = tempty + kAccBufs;   // [1]
  uint64_t* wbar = done + 1;          // [1] resident weights landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(wbar + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // per-channel bias and weight scales, [n_pad] each (n_pad = n rounded up to BN)
  float* bias_s = reinterpret_cast<float*>(smem + (size_t)p.ring * p.stage_bytes + kBarBytes);
  float* wsc_s = bias_s + p.n_pad;
  uint8_t* wres = reinterpret_cast<uint8_t*>(wsc_s + p.n_pad);  // resident weights
  constexpr int kBBytes = TAPS * 4 * BN * 16;
  constexpr int kTmemCols = kAccBufs * BN;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t num_tiles = (int64_t)p.n_img * p.tiles_m * p.tiles_n;
  const int32_t wp = p.wp;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.ring; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kAccBufs; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);
    }
    mbar_init(done, 1);
    mbar_init(wbar, 1);
    *abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_in);
  }
  for (int32_t i = threadIdx.x; i < p.n_pad; i += kThreads) {
    bias_s[i] = i < p.n ? p.bias[i] : 0.0f;
    wsc_s[i] = i < p.n && p.w_scale_ch ? p.w_scale_ch[i] : 0.0f;
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const uint32_t a_bytes = 4u * (uint32_t)p.plane_bytes;
      const uint32_t a_span = 4u * (uint32_t)p.plane_stride;
      if (p.resident) {
        mbar_arrive_expect_tx(wbar, kBBytes);
        bulk_load(wres, p.wd, kBBytes, wbar);
      }
      uint32_t issued_parity[8];
      bool issued[8];
      for (int s = 0; s < 8; ++s) issued[s] = false;
      TileWalk tw;
      tw.start(p, blockIdx.x);
      for (int64_t tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, tw.advance()) {
        const int32_t img = tw.img, mt = tw.mt, nb = tw.nb;
        const int32_t r_lo = (p.f0 + BM * mt + p.min_off) / wp;  // first padded row the tile reads
        for (int s = 0; s < p.stages_k; ++s) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort)) { ok = false; break; }
          uint8_t* sa = smem + (size_t)stage * p.stage_bytes;
          mbar_arrive_expect_tx(&full[stage], a_bytes + (p.resident ? 0u : (uint32_t)kBBytes));
#pragma unroll
          for (int j = 0; j < 4; ++j)  // chunk plane j: channels s*64 + 16j .. +15; x from pixel -pad_l
            tma_load_4d(sa + j * p.plane_stride, &map_in, &full[stage], -2 * p.pad_l, r_lo - p.pad_t, s * 4 + j, img);
          if (!p.resident)
            bulk_load(sa + a_span, p.wd + ((int64_t)nb * p.stages_k + s) * kBBytes, kBBytes, &full[stage]);
          issued[stage] = true;
          issued_parity[stage] = phase;
          if (++stage == p.ring) { stage = 0; phase ^= 1; }
        }
      }
      // drain: every copy issued must have landed before the CTA exits
      volatile int never = 0;
      if (p.resident) mbar_wait(wbar, 0, &never, 200000000ull);
      for (int s = 0; s < p.ring; ++s)
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
      if (p.resident) {
        ok = mbar_wait(wbar, 0, abort);
        tc_fence_after();
      }
      TileWalk tw;
      tw.start(p, blockIdx.x);
      for (int64_t tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++iter, tw.advance()) {
        const int32_t mt = tw.mt;
        const int32_t r_lo = (p.f0 + BM * mt + p.min_off) / wp;
        const int32_t a_row0 = p.f0 + BM * mt - r_lo * wp;  // the tile's first centre in its loaded rows
        const int buf = iter & (kAccBufs - 1);
        const uint32_t aphase = (iter / kAccBufs) & 1;
        if (!mbar_wait(&tempty[buf], aphase ^ 1, abort)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * BN);
        for (int s = 0; s < p.stages_k; ++s) {
          if (!mbar_wait(&full[stage], phase, abort)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_addr(smem + (size_t)stage * p.stage_bytes);
          const uint32_t sb = p.resident ? smem_addr(wres) : sa + 4u * (uint32_t)p.plane_stride;
#pragma unroll
          for (int t = 0; t < TAPS; ++t) {
            const int32_t row = a_row0 + p.toff[t];
#pragma unroll
            for (int kk = 0; kk < 2; ++kk)
              mma_i8(d_tmem, desc_rows16(sa + (uint32_t)(2 * kk * p.plane_stride + row * 16), (uint32_t)p.plane_stride),
                     desc_rows16(sb + (uint32_t)((t * 4 + 2 * kk) * BN * 16), BN * 16), idesc,
                     (s | t | kk) != 0);
          }
          mma_commit(&empty[stage]);
          if (++stage == p.ring) { stage = 0; phase ^= 1; }
        }
        if (ok) mma_commit(&tfull[buf]);
      }
      mma_commit(done);
      volatile int never = 0;
      mbar_wait(done, 0, &never, 200000000ull);
    }
  } else {
    // ---------------- epilogue ----------------
    const int e = warp - 2;
    const int q = warp & 3;           // TMEM lane quadrant this warp may access
    const int part = e >> 2;          // which quarter of the BN columns
    constexpr int kCols = BN / (kEpiWarps / 4);
    const int32_t hw = p.h * p.w;     // n * hw < 2^31 (conv3x3_eligible)
    const int64_t img_stride = (int64_t)p.n * hw;
    // Per tile and lane: the centre position, whether it is an image pixel, its pixel index.
    auto lane_pixel = [&](const TileWalk& t, int32_t& img, int32_t& nb, bool& valid, int32_t& pix, int32_t& iy,
                          int32_t& ix) {
      img = t.img;
      nb = t.nb;
      const int32_t mt = t.mt;
      const int32_t f = p.f0 + BM * mt + q * 32 + lane;  // this lane's centre position
      const int32_t py = f / wp;
      iy = py - p.pad_t;
      ix = f - py * wp - p.pad_l;
      valid = iy >= 0 && iy < p.h && ix >= 0 && ix < p.w;
      pix = valid ? iy * p.w + ix : 0;
    };
    // The residual block's add: res[] holds the residual of the tile being processed; as
    // each value is used, the load of the same channel for the CTA's next tile is issued
    // in its place, so the loads are in flight for a whole tile.
    float res[kCols];
    TileWalk tw;  // this tile
    tw.start(p, blockIdx.x);
    if (p.residual) {
      int32_t img, nb, pix, iy, ix;
      bool valid;
      lane_pixel(tw, img, nb, valid, pix, iy, ix);
      const int32_t colw = nb * BN + part * kCols;
      const float* rb = p.residual + (int64_t)img * img_stride + pix;
#pragma unroll
      for (int j = 0; j < kCols; ++j) res[j] = valid && colw + j < p.n ? __ldg(rb + (colw + j) * hw) : 0.0f;
    }
    int iter = 0;
    for (int64_t tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++iter, tw.advance()) {
      int32_t img, nb, pix, iy, ix;
      bool valid;
      lane_pixel(tw, img, nb, valid, pix, iy, ix);
      const int buf = iter & (kAccBufs - 1);
      const uint32_t aphase = (iter / kAccBufs) & 1;
      // read by the later strided 1x1 conv: rows and columns cov_s * i, i < cov_oh / cov_ow
      const bool cov2 = valid && p.amax2 && iy % p.cov_s == 0 && ix % p.cov_s == 0 && iy / p.cov_s < p.cov_oh &&
                        ix / p.cov_s < p.cov_ow;
      const int32_t colw = nb * BN + part * kCols;  // this warp's first column
      const float sa = p.a_scale[img];
      const float cs_tensor = __fmul_rn(sa, p.w_scale);
      float* ob = p.out + (int64_t)img * img_stride + colw * hw + pix;
      // the next tile's residual (rolling prefetch)
      const float* rn = nullptr;
      int32_t ncols = 0;
      if (p.residual && tile + gridDim.x < num_tiles) {
        int32_t img2, nb2, pix2, iy2, ix2;
        bool valid2;
        TileWalk tn = tw;
        tn.advance();
        lane_pixel(tn, img2, nb2, valid2, pix2, iy2, ix2);
        const int32_t colw2 = nb2 * BN + part * kCols;
        rn = p.residual + (int64_t)img2 * img_stride + colw2 * hw + pix2;
        ncols = valid2 ? p.n - colw2 : 0;  // columns of the next tile this lane loads
      }
      const bool got = mbar_wait(&tfull[buf], aphase, abort);
      if (!__all_sync(0xffffffffu, got)) { *abort = 1; break; }
      tc_fence_after();
      const bool fast = !p.acc && colw + kCols <= p.n;  // every column exists, no i32 dump
      float mx = 0.0f, mx2 = 0.0f;
#pragma unroll
      for (int cc = 0; cc < kCols; cc += 16) {
        uint32_t v[16];
        __syncwarp();  // the warp-wide TMEM load runs converged
        tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN + part * kCols + cc), v);
        tmem_ld_wait();
        if (fast) {
          // per-channel constants from shared memory (16-byte loads, all lanes the same address)
          float bz[16];
#pragma unroll
          for (int j4 = 0; j4 < 16; j4 += 4) {
            const float4 b4 = *reinterpret_cast<const float4*>(bias_s + colw + cc + j4);
            bz[j4] = b4.x; bz[j4 + 1] = b4.y; bz[j4 + 2] = b4.z; bz[j4 + 3] = b4.w;
          }
          float o[16];
          if (p.w_scale_ch) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              o[j] = epilogue_t<ACT>((int32_t)v[j], __fmul_rn(sa, wsc_s[colw + cc + j]), bz[j], p.act_param);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) o[j] = epilogue_t<ACT>((int32_t)v[j], cs_tensor, bz[j], p.act_param);
          }
          if (p.residual) {  // the residual block's activation: none, ReLU or LeakyReLU
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              o[j] = __fadd_rn(o[j], res[cc + j]);
              res[cc + j] = cc + j < ncols ? __ldg(rn + (cc + j) * hw) : 0.0f;
            }
            if (p.res_act == ACT_RELU) {
#pragma unroll
              for (int j = 0; j < 16; ++j) o[j] = fmaxf(o[j], 0.0f);
            } else if (p.res_act == ACT_LEAKY_RELU) {
#pragma unroll
              for (int j = 0; j < 16; ++j) o[j] = o[j] > 0.0f ? o[j] : __fmul_rn(p.res_param, o[j]);
            }
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (valid) ob[(cc + j) * hw] = o[j];
            mx = fmaxf(mx, fabsf(o[j]));
          }
          if (p.amax2) {
#pragma unroll
            for (int j = 0; j < 16; ++j) mx2 = fmaxf(mx2, fabsf(o[j]));
          }
        } else {
          const int32_t col0 = colw + cc;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int32_t c = col0 + j;
            if (c < p.n) {
              const float cs = p.w_scale_ch ? __fmul_rn(sa, __ldg(p.w_scale_ch + c)) : cs_tensor;
              float o = epilogue_t<ACT>((int32_t)v[j], cs, __ldg(p.bias + c), p.act_param);
              if (p.residual) {
                o = __fadd_rn(o, res[cc + j]);
                if (p.res_act == ACT_RELU) o = fmaxf(o, 0.0f);
                else if (p.res_act == ACT_LEAKY_RELU) o = o > 0.0f ? o : __fmul_rn(p.res_param, o);
              }
              if (valid) {
                ob[(cc + j) * hw] = o;
                if (p.acc) p.acc[(int64_t)img * img_stride + (int64_t)c * hw + pix] = (int32_t)v[j];
              }
              mx = fmaxf(mx, fabsf(o));
              mx2 = fmaxf(mx2, fabsf(o));
            }
            if (p.residual) res[cc + j] = cc + j < ncols ? __ldg(rn + (cc + j) * hw) : 0.0f;
          }
        }
      }
      if (!valid) mx = 0.0f;   // padding positions: computed, not part of the output
      if (!cov2) mx2 = 0.0f;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
      if (p.amax) flush_slot_max(p.amax, p.amax_per_slot ? img : 0, mx);
      if (p.amax2) flush_slot_max(p.amax2, img, mx2);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *abort) atomicExch(p.err, 1);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// Input map: chunk-planar i8 [n][cpad / 16][h][w][16 B] as 4 dims of 8-byte elements
// (2w, h, chunks, n); boxes of one chunk plane x rbox rows x wp pixels, starting pad_l
// pixels left of the image.
bool make_in_map(CUtensorMap* map, const void* base, int32_t n, int32_t h, int32_t w, int32_t cpad, int32_t wp,
                 int32_t rbox) {
  auto fn = tma_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {(cuuint64_t)2 * w, (cuuint64_t)h, (cuuint64_t)(cpad / 16), (cuuint64_t)n};
  cuuint64_t strides[3] = {(cuuint64_t)16 * w, (cuuint64_t)16 * w * h, (cuuint64_t)16 * w * h * (cpad / 16)};
  cuuint32_t box[4] = {(cuuint32_t)(2 * wp), (cuuint32_t)rbox, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 4, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The tap geometry of a mode over an h x w operand grid (= the output grid).
struct TapGeom {
  int taps = 0, pad_t = 0, pad_l = 0, wp = 0, f0 = 0, min_off = 0, max_off = 0, rbox = 0, tiles_m = 0;
  int toff[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
};

TapGeom tap_geom(int mode, int32_t h, int32_t w) {
  TapGeom g;
  if (mode == DCONV_3X3) {
    g.taps = 9; g.pad_t = 1; g.pad_l = 1; g.wp = w + 2;
    for (int t = 0; t < 9; ++t) g.toff[t] = (t / 3 - 1) * g.wp + (t % 3 - 1);
  } else if (mode == DCONV_S2D) {  // taps (ay, ax) in {-1, 0}^2 over 2x2 pixel blocks
    g.taps = 4; g.pad_t = 1; g.pad_l = 1; g.wp = w + 1;
    for (int t = 0; t < 4; ++t) g.toff[t] = (t / 2 - 1) * g.wp + (t % 2 - 1);
  } else {
    g.taps = 1; g.wp = w;
  }
  g.f0 = g.pad_t * g.wp + g.pad_l;
  g.min_off = g.max_off = g.toff[0];
  for (int t = 1; t < g.taps; ++t) {
    g.min_off = std::min(g.min_off, g.toff[t]);
    g.max_off = std::max(g.max_off, g.toff[t]);
  }
  // 128 consecutive centres from any start span at most this many padded rows
  g.rbox = (g.wp + 126 + (g.max_off - g.min_off)) / g.wp + 1;
  g.tiles_m = (int)(((int64_t)(h - 1) * g.wp + w + BM - 1) / BM);
  return g;
}

template <int BN, int ACT, int TAPS>
bool launch_bn(const GemmArgs& a, int mode, int32_t H, int32_t W, int32_t cpad, const int8_t* wd, int num_sms,
               cudaStream_t st) {
  const TapGeom tg = tap_geom(mode, H, W);
  C3Params p;
  p.n_img = (int32_t)(a.m / ((int64_t)H * W));
  p.h = H; p.w = W; p.cpad = cpad; p.n = (int32_t)a.n;
  p.tiles_m = tg.tiles_m;
  p.tiles_n = (int32_t)((a.n + BN - 1) / BN);
  p.stages_k = cpad / kCS;
  p.rbox = tg.rbox;
  p.wp = tg.wp; p.pad_t = tg.pad_t; p.pad_l = tg.pad_l; p.f0 = tg.f0; p.min_off = tg.min_off;
  for (int t = 0; t < 9; ++t) p.toff[t] = tg.toff[t];
  p.plane_bytes = p.rbox * tg.wp * 16;
  p.plane_stride = (p.plane_bytes + 127) / 128 * 128;
  const int a_bytes = 4 * p.plane_stride;
  p.resident = p.stages_k == 1 && p.tiles_n == 1;
  const int wres_bytes = p.resident ? TAPS * 4 * BN * 16 : 0;
  p.stage_bytes = (a_bytes + (p.resident ? 0 : TAPS * 4 * BN * 16) + 1023) / 1024 * 1024;
  p.ring = (227 * 1024 - 1024 - kBarBytes - 2 * p.tiles_n * BN * 4 - wres_bytes) / p.stage_bytes;
  if (p.ring > 8) p.ring = 8;
  if (p.ring < 2) return false;
  p.n_pad = p.tiles_n * BN;
  const int smem = 1024 + p.ring * p.stage_bytes + kBarBytes + 2 * p.n_pad * 4 + wres_bytes;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncSetAttribute(k_conv3x3<BN, ACT, TAPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  CUtensorMap mi;
  if (!make_in_map(&mi, a.a, p.n_img, H, W, cpad, tg.wp, p.rbox)) return false;
  p.wd = wd;
  p.a_scale = a.a_scale; p.w_scale = a.w_scale; p.w_scale_ch = a.w_scale_ch; p.bias = a.bias;
  p.act_param = a.act_param; p.out = a.out; p.acc = a.acc;
  p.residual = a.residual; p.res_act = a.res_act; p.res_param = a.res_param;
  p.amax = a.amax.ptr; p.amax_per_slot = a.amax.elems_per_slot;
  p.amax2 = a.amax2; p.cov_s = a.cov_s > 0 ? a.cov_s : 1; p.cov_oh = a.cov_oh; p.cov_ow = a.cov_ow;
  p.err = a.err;
  const int64_t tiles = (int64_t)p.n_img * p.tiles_m * p.tiles_n;
  const int grid = tiles < num_sms ? (int)tiles : num_sms;
  k_conv3x3<BN, ACT, TAPS><<<grid, kThreads, smem, st>>>(mi, p);
  return true;
}

template <int BN, int TAPS>
bool launch_act(const GemmArgs& a, int mode, int32_t h, int32_t w, int32_t cpad, const int8_t* wd, int num_sms,
                cudaStream_t st) {
  switch (a.act) {
    case ACT_NONE: return launch_bn<BN, ACT_NONE, TAPS>(a, mode, h, w, cpad, wd, num_sms, st);
    case ACT_RELU: return launch_bn<BN, ACT_RELU, TAPS>(a, mode, h, w, cpad, wd, num_sms, st);
    case ACT_SIGMOID: return launch_bn<BN, ACT_SIGMOID, TAPS>(a, mode, h, w, cpad, wd, num_sms, st);
    case ACT_TANH: return launch_bn<BN, ACT_TANH, TAPS>(a, mode, h, w, cpad, wd, num_sms, st);
    case ACT_GELU: return launch_bn<BN, ACT_GELU, TAPS>(a, mode, h, w, cpad, wd, num_sms, st);
    case ACT_LEAKY_RELU: return launch_bn<BN, ACT_LEAKY_RELU, TAPS>(a, mode, h, w, cpad, wd, num_sms, st);
    case ACT_SILU: return launch_bn<BN, ACT_SILU, TAPS>(a, mode, h, w, cpad, wd, num_sms, st);
    default: return false;
  }
}

int mode_taps(int mode) { return mode == DCONV_3X3 ? 9 : mode == DCONV_S2D ? 4 : 1; }

}  // namespace

int conv3x3_bn(int32_t out_channels) { return out_channels >= 128 ? 128 : 64; }

bool dconv_shape_ok(int mode, int64_t n_img, int32_t h, int32_t w, int32_t cpad, int32_t out_channels) {
  if (mode < DCONV_3X3 || mode > DCONV_1X1) return false;
  if ((cpad & 63) || out_channels < 16 || n_img < 1 || n_img > 65535 || h < 1 || w < 1) return false;
  const TapGeom tg = tap_geom(mode, h, w);
  if (2 * tg.wp > 256 || tg.rbox > 256) return false;  // TMA box extents
  if (n_img * h * w * (int64_t)out_channels * tg.taps * cpad < (int64_t)1 << 22) return false;
  return tma_encode_fn() != nullptr;
}

bool conv3x3_shape_ok(int64_t n_img, int32_t h, int32_t w, int32_t cpad, int32_t k, int32_t stride, int32_t pad,
                      int32_t out_channels) {
  return k == 3 && stride == 1 && pad == 1 && dconv_shape_ok(DCONV_3X3, n_img, h, w, cpad, out_channels);
}

bool dconv_eligible(const GemmArgs& a, int mode, int32_t h, int32_t w, int32_t cpad) {
  if (!a.conv || a.out_l <= 0 || a.out_l != (int64_t)h * w || a.rows_per_scale != a.out_l) return false;
  if (!dconv_shape_ok(mode, a.m / a.out_l, h, w, cpad, (int32_t)a.n)) return false;
  if (a.amax.ptr && a.amax.elems_per_slot != 0 && a.amax.elems_per_slot != a.n * a.out_l) return false;
  if (a.n * a.out_l >= ((int64_t)1 << 31)) return false;  // per-image offsets in 32 bits
  if ((a.m / a.out_l) * tap_geom(mode, h, w).tiles_m * ((a.n + 63) / 64) >= ((int64_t)1 << 31))
    return false;  // tile indices in 32 bits
  if (reinterpret_cast<uintptr_t>(a.a) & 15) return false;
  return tma_encode_fn() != nullptr;
}

bool conv3x3_eligible(const GemmArgs& a) {
  if (a.g.c != a.g.cpad || a.g.oh != a.g.h || a.g.ow != a.g.w || a.g.k != 3 || a.g.stride != 1 || a.g.pad != 1)
    return false;
  return dconv_eligible(a, DCONV_3X3, a.g.h, a.g.w, a.g.cpad);
}

// Host-side weight arrangement: w [N][C][k][k] quantized (reference layout) ->
// [tiles_n][cpad_op / 64][taps][4 chunks][BN rows][16 B], zero where no weight applies.
// Operand channel sc of tap t:
//   3x3: channel sc, kernel (t / 3, t % 3);            1x1: channel sc;
//   s2d: sc = (dy * 2 + dx) * cpad + c, tap (ay, ax) = (t / 2 - 1, t % 2 - 1), kernel
//        (2 ay + dy + 1, 2 ax + dx + 1) when inside 0..2 (pixel 2 oy - 1 + ky of the
//        stride-2 / pad-1 conv is s2d row oy + ay, sub-row dy).
void dconv_arrange_weights(int mode, const int8_t* wq, int32_t n, int32_t c, int32_t k, int32_t cpad, int8_t* out) {
  const int32_t bn = conv3x3_bn(n), tiles_n = (n + bn - 1) / bn;
  const int taps = mode_taps(mode);
  const int32_t cop = mode == DCONV_S2D ? 4 * cpad : cpad, sk = cop / kCS;
  const size_t per = (size_t)taps * 4 * bn * 16;
  memset(out, 0, per * sk * tiles_n);
  for (int32_t o = 0; o < n; ++o) {
    const int32_t nb = o / bn, r = o % bn;
    for (int32_t sc = 0; sc < cop; ++sc) {
      const int32_t s = sc / kCS, j = (sc % kCS) / 16, b = sc % 16;
      for (int t = 0; t < taps; ++t) {
        int32_t ch = sc, ky = 0, kx = 0;
        if (mode == DCONV_3X3) {
          ky = t / 3; kx = t % 3;
        } else if (mode == DCONV_S2D) {
          const int32_t dd = sc / cpad, dy = dd / 2, dx = dd % 2;
          ch = sc % cpad;
          ky = 2 * (t / 2 - 1) + dy + 1;
          kx = 2 * (t % 2 - 1) + dx + 1;
          if (ky < 0 || ky > 2 || kx < 0 || kx > 2) continue;
        }
        if (ch >= c) continue;
        out[((size_t)nb * sk + s) * per + (((size_t)t * 4 + j) * bn + r) * 16 + b] =
            wq[(((size_t)o * c + ch) * k + ky) * k + kx];
      }
    }
  }
}

size_t dconv_weight_bytes(int mode, int32_t n, int32_t cpad) {
  const int32_t bn = conv3x3_bn(n);
  const int32_t cop = mode == DCONV_S2D ? 4 * cpad : cpad;
  return (size_t)((n + bn - 1) / bn) * (cop / kCS) * mode_taps(mode) * 4 * bn * 16;
}

void conv3x3_arrange_weights(const int8_t* wq, int32_t n, int32_t c, int32_t cpad, int8_t* out) {
  dconv_arrange_weights(DCONV_3X3, wq, n, c, 3, cpad, out);
}

size_t conv3x3_weight_bytes(int32_t n, int32_t cpad) { return dconv_weight_bytes(DCONV_3X3, n, cpad); }

bool launch_dconv(const GemmArgs& a, int mode, int32_t h, int32_t w, int32_t cpad, const int8_t* wd, int num_sms,
                  cudaStream_t st) {
  if (!a.err) return false;
  const bool b128 = conv3x3_bn((int32_t)a.n) == 128;
  switch (mode) {
    case DCONV_3X3:
      return b128 ? launch_act<128, 9>(a, mode, h, w, cpad, wd, num_sms, st)
                  : launch_act<64, 9>(a, mode, h, w, cpad, wd, num_sms, st);
    case DCONV_S2D:
      return b128 ? launch_act<128, 4>(a, mode, h, w, cpad, wd, num_sms, st)
                  : launch_act<64, 4>(a, mode, h, w, cpad, wd, num_sms, st);
    case DCONV_1X1:
      return b128 ? launch_act<128, 1>(a, mode, h, w, cpad, wd, num_sms, st)
                  : launch_act<64, 1>(a, mode, h, w, cpad, wd, num_sms, st);
    default: return false;
  }
}

bool launch_conv3x3(const GemmArgs& a, const int8_t* wd, int num_sms, cudaStream_t st) {
  return launch_dconv(a, DCONV_3X3, a.g.h, a.g.w, a.g.cpad, wd, num_sms, st);
}


}  // namespace rg
