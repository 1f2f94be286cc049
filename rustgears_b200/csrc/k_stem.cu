// k_stem.cu -- the ResNet stem, Conv2d(C <= 4 -> 64, k 7, stride 2, pad 3) + activation
// followed by MaxPool2d(3, 2), as one tcgen05 kernel: the conv's f32 output never goes
// to memory, only the pooled tensor does.
//
// Reference: the FusedConv2d arm of NpuProgram::execute (src/inference/npu.rs:319-383:
// per-image im2col, quantize with the image's scale, int8 GEMM, fused epilogue) and
// max_pool2d (src/tensor/conv.rs, window scanned row by row, `v > best || v.is_nan()`).
//
// Space-to-depth: a stride-2 conv is a stride-1 conv over the 2x2 pixel blocks of its
// input.  The quantized input is stored as s2d pixels [img][h/2][w/2][16 B], byte
// (dy * 2 + dx) * 4 + c = pixel (2 sy + dy, 2 sx + dx), channel c.  Output (oy, ox)
// reads s2d pixels (oy + ay, ox + ax), ay, ax in -2..1 (ky = 2 ay + dy + 3): a 4 x 4
// stride-1 conv over 16-byte pixels whose weights are zero where ky or kx falls outside
// 0..6.  The i32 sums are those of the reference's im2col GEMM (the extra products are
// zero, integer addition is exact in any order).
//
// A tile is one conv output row (M = 128 TMEM lanes, ox = lane, w/2 <= 125 valid): a
// TMA load brings the padded s2d rows oy - 2 .. (zero rows and columns outside the
// image), and 8 MMAs (K 32: two vertically adjacent taps, LBO = one padded row) read
// the taps at constant offsets.  Each CTA owns a contiguous range of pool rows and
// computes the conv rows they need in order; the epilogue folds each pooling window's
// three columns of the conv row (the reference's scan order within the row; the
// neighbouring columns come from the neighbouring TMEM lanes by warp shuffles), then
// folds the rows into the running window (row order) -- the same
// result as the reference's row-major scan, NaN and signed zeros included: the scan
// returns the last NaN, else the first maximal element in row-major order, and
// folding per-row results in row order preserves both.
//
//   warp 0     producer (lane 0): one TMA load per conv row; the weights once
//   warp 1     MMA issuer (lane 0): 8 tcgen05.mma per conv row into one of two
//              TMEM accumulators
//   warps 2-17 epilogue: tcgen05.ld, act(f32(acc) * (s_img * s_w) + bias), the
//              pooling folds in registers, NCHW pool stores and the per-image absmax
//              of the pooled tensor
// Every mbarrier wait is bounded; on timeout the CTA raises an abort flag, the roles
// leave their loops together, copies and MMAs in flight are drained, TMEM is freed and
// a device error word is set for the host.
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

constexpr int BM = 128;          // conv output columns per tile (TMEM lanes)
constexpr int BN = 64;           // output channels
constexpr int kEpiWarps = 16;    // 4 per TMEM lane quadrant, 16 channels each
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kThreads = 64 + kEpiThreads;
constexpr int kTaps = 8;         // MMAs per tile: (ay pair, ax)
constexpr int kWBytes = kTaps * 2 * BN * 16;  // 16 KB of arranged weights
constexpr int kRing = 6;
constexpr int kBarBytes = 256;

struct StemParams {
  int32_t n_img, h2, w2;           // s2d grid = conv output grid
  int32_t ph, pw;                  // pool output
  int32_t rbox;                    // padded s2d rows per TMA box
  int32_t slot_bytes;              // ring slot (rbox * (w2 + 3) * 16, rounded to 128)
  int64_t pool_rows;               // n_img * ph
  const int8_t* wd;                // [8 taps][2 K chunks][64 rows][16 B]
  const float* a_scale;            // per image
  float w_scale;
  const float* w_scale_ch;
  const float* bias;
  float act_param;
  float* out;                      // NCHW [n_img, 64, ph, pw]
  unsigned* amax;                  // optional absmax sink of out
  int32_t amax_per_image;
};

__device__ int g_stem_error;

__device__ __forceinline__ uint64_t desc_rows16(uint32_t saddr, uint32_t lbo) {
  // no-swizzle K-major: rows 16 bytes apart (8-row groups 128 B apart), K chunks `lbo` apart
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(128 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t c0,
                                            int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// The conv rows a CTA computes, in order: for each image its pool rows [ra, rb) need
// conv rows 2 ra .. 2 rb (pool row r reads conv rows 2r, 2r + 1, 2r + 2).
struct RowIter {
  int64_t g, g_end;   // global pool rows img * ph + r still to finish
  int32_t img, ra, rb, y;
  __device__ void start(int64_t g0, int64_t g1, int32_t ph) {
    g = g0;
    g_end = g1;
    if (g < g_end) seg(ph);
  }
  __device__ void seg(int32_t ph) {
    img = (int32_t)(g / ph);
    ra = (int32_t)(g - (int64_t)img * ph);
    const int64_t left = g_end - g;
    rb = left < (int64_t)(ph - ra) ? ra + (int32_t)left : ph;
    y = 2 * ra;
  }
  __device__ bool valid() const { return g < g_end; }
  __device__ void next(int32_t ph) {
    if (y < 2 * rb) {
      ++y;
      return;
    }
    g += rb - ra;
    if (g < g_end) seg(ph);
  }
};

// One step of the reference's window scan, best = (v > best || v is NaN) ? v : best, as
// predicated selects (no branch).
__device__ __forceinline__ float pool_fold(float best, float v) {
  float r;
  asm("{\n .reg .pred p, q;\n setp.gt.f32 p, %2, %1;\n setp.nan.f32 q, %2, %2;\n or.pred p, p, q;\n"
      " selp.f32 %0, %2, %1, p;\n}"
      : "=f"(r)
      : "f"(best), "f"(v));
  return r;
}

template <int ACT>
__global__ void __launch_bounds__(kThreads, 1)
    k_stem_pool(const __grid_constant__ CUtensorMap map_in, const StemParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;                                            // [kRing][slot_bytes]
  uint8_t* wsm = ring + (size_t)kRing * p.slot_bytes;              // [kWBytes]
  float* xch = reinterpret_cast<float*>(wsm + kWBytes);            // [2][4 parts][4 quadrants][16]
  uint64_t* bars = reinterpret_cast<uint64_t*>(xch + 2 * 4 * 4 * 16);
  uint64_t* full = bars;              // [kRing]
  uint64_t* empty = full + kRing;     // [kRing]
  uint64_t* tfull = empty + kRing;    // [2]
  uint64_t* tempty = tfull + 2;       // [2]
  uint64_t* wbar = tempty + 2;        // weights landed
  uint64_t* done = wbar + 1;          // every MMA retired
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  constexpr int kTmemCols = 2 * BN;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int32_t wp = p.w2 + 3;  // 2 zero columns left, 1 right
  const int64_t g0 = p.pool_rows * blockIdx.x / gridDim.x;
  const int64_t g1 = p.pool_rows * (blockIdx.x + 1) / gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);
    }
    mbar_init(wbar, 1);
    mbar_init(done, 1);
    *abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_in);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      mbar_arrive_expect_tx(wbar, kWBytes);
      bulk_load(wsm, p.wd, kWBytes, wbar);
      const uint32_t a_bytes = (uint32_t)(p.rbox * wp * 16);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_parity[kRing];
      bool issued[kRing];
      for (int s = 0; s < kRing; ++s) issued[s] = false;
      RowIter it;
      for (it.start(g0, g1, p.ph); it.valid(); it.next(p.ph)) {
        if (!mbar_wait(&empty[stage], phase ^ 1, abort)) break;
        mbar_arrive_expect_tx(&full[stage], a_bytes);
        // padded rows y - 2 .. y - 2 + rbox - 1, columns from s2d pixel -2 (x = -4 eight-byte elements)
        tma_load_3d(ring + (size_t)stage * p.slot_bytes, &map_in, &full[stage], -4, it.y - 2, it.img);
        issued[stage] = true;
        issued_parity[stage] = phase;
        if (++stage == kRing) { stage = 0; phase ^= 1; }
      }
      // drain: every copy issued must have landed before the CTA exits
      volatile int never = 0;
      mbar_wait(wbar, 0, &never, 200000000ull);
      for (int s = 0; s < kRing; ++s)
        if (issued[s]) mbar_wait(&full[s], issued_parity[s], &never, 200000000ull);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(BM, BN);
      const uint32_t sw = smem_addr(wsm);
      int stage = 0;
      uint32_t phase = 0;
      int iter = 0;
      bool ok = mbar_wait(wbar, 0, abort);
      if (ok) tc_fence_after();
      RowIter it;
      for (it.start(g0, g1, p.ph); ok && it.valid(); it.next(p.ph), ++iter) {
        const int buf = iter & 1;
        const uint32_t aphase = (iter >> 1) & 1;
        if (!mbar_wait(&tempty[buf], aphase ^ 1, abort)) break;
        if (!mbar_wait(&full[stage], phase, abort)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * BN);
        const uint32_t sa = smem_addr(ring + (size_t)stage * p.slot_bytes);
#pragma unroll
        for (int t = 0; t < kTaps; ++t) {
          // taps (ay, ax) and (ay + 1, ax), ay = 2 (t / 4) - 2, ax = t % 4 - 2: padded row
          // 2 (t / 4), padded column ox + t % 4
          const uint32_t pos = (uint32_t)((t / 4) * 2 * wp + (t % 4));
          mma_i8(d_tmem, desc_rows16(sa + pos * 16u, (uint32_t)wp * 16u), desc_rows16(sw + t * 2 * BN * 16, BN * 16),
                 idesc, t != 0);
        }
        mma_commit(&empty[stage]);
        mma_commit(&tfull[buf]);
        if (++stage == kRing) { stage = 0; phase ^= 1; }
      }
      mma_commit(done);
      volatile int never = 0;
      mbar_wait(done, 0, &never, 200000000ull);
    }
  } else {
    // ---------------- epilogue ----------------
    // Lane ox holds conv column ox of its 16 channels; the pool window's columns ox + 1
    // and ox + 2 come from the neighbouring lanes (lane 30's ox + 2 from lane 0 of the
    // next quadrant's warp, through shared memory); the row folds run in registers.
    const int e = warp - 2;
    const int q = warp & 3;                 // TMEM lane quadrant this warp may access
    const int part = e >> 2;                // channels part * 16 .. + 15
    const int32_t ox = q * 32 + lane;       // conv output column of this lane
    const int32_t px = ox >> 1;
    const bool centre = (ox & 1) == 0 && px < p.pw;  // the first column of pool window px
    const int32_t plane = p.ph * p.pw;
    float bias_r[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) bias_r[j] = __ldg(p.bias + part * 16 + j);
    int32_t cs_img = -1;
    float sa = 0.0f, cs_t = 0.0f;           // the image's scale, times the tensor weight scale
    float vs[16];                           // running window fold per channel (pool column px)
    float mx = 0.0f;
    int iter = 0;
    RowIter it;
    for (it.start(g0, g1, p.ph); it.valid(); it.next(p.ph), ++iter) {
      const int buf = iter & 1;
      const uint32_t aphase = (iter >> 1) & 1;
      float o[16];
      const bool got = mbar_wait(&tfull[buf], aphase, abort);
      if (__all_sync(0xffffffffu, got)) {
        tc_fence_after();
        uint32_t v[16];
        tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN + part * 16), v);
        tmem_ld_wait();
        if (it.img != cs_img) {
          cs_img = it.img;
          sa = p.a_scale[it.img];
          cs_t = __fmul_rn(sa, p.w_scale);
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float cs = p.w_scale_ch ? __fmul_rn(sa, __ldg(p.w_scale_ch + part * 16 + j)) : cs_t;
          o[j] = epilogue_t<ACT>((int32_t)v[j], cs, bias_r[j], p.act_param);
        }
        tc_fence_before();
        if (lane == 0) {
          float* xs = xch + ((buf * 4 + part) * 4 + q) * 16;
#pragma unroll
          for (int j = 0; j < 16; ++j) xs[j] = o[j];
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
      // the part's four quadrant warps: exchange published, accumulators all received
      if (!bar_and(2 + part, 128, got)) {
        *abort = 1;
        break;
      }
      const bool first = it.y == 2 * it.ra;
      const bool closes = !first && (it.y & 1) == 0;  // completes pool row y / 2 - 1
      const float* xn = xch + ((buf * 4 + part) * 4 + ((q + 1) & 3)) * 16;
      float* orow = p.out + ((int64_t)it.img * BN + part * 16) * plane + (it.y / 2 - 1) * p.pw + px;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float n1 = __shfl_down_sync(0xffffffffu, o[j], 1);
        float n2 = __shfl_down_sync(0xffffffffu, o[j], 2);
        if (lane == 30) n2 = xn[j];
        // the window's row: columns 2 px, 2 px + 1, 2 px + 2 in the reference's order
        const float h = pool_fold(pool_fold(o[j], n1), n2);
        if (first) {
          vs[j] = h;
        } else if (!closes) {
          vs[j] = pool_fold(vs[j], h);
        } else {
          const float best = pool_fold(vs[j], h);
          if (centre) {
            orow[(int64_t)j * plane] = best;
            mx = fmaxf(mx, fabsf(best));
          }
          vs[j] = h;
        }
      }
      if (it.y == 2 * it.rb) {  // the image's last conv row in this CTA: flush its absmax
        if (p.amax) {
          float m = mx;
#pragma unroll
          for (int k = 16; k > 0; k >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, k));
          if (lane == 0 && m > 0.0f) atomicMax(p.amax + (p.amax_per_image ? it.img : 0), __float_as_uint(m));
        }
        mx = 0.0f;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *abort) atomicExch(&g_stem_error, 1);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// s2d operand [n][h2][w2][16 B] as 3 dims of 8-byte elements (2 w2, h2, n); boxes of
// rbox rows x (w2 + 3) pixels starting two pixels left of the image.
bool make_s2d_map(CUtensorMap* map, const void* base, int32_t n, int32_t h2, int32_t w2, int32_t rbox) {
  auto fn = tma_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)2 * w2, (cuuint64_t)h2, (cuuint64_t)n};
  cuuint64_t strides[2] = {(cuuint64_t)16 * w2, (cuuint64_t)16 * w2 * h2};
  cuuint32_t box[3] = {(cuuint32_t)(2 * (w2 + 3)), (cuuint32_t)rbox, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int32_t stem_rbox(int32_t w2) {
  const int32_t wp = w2 + 3;
  // the last tap pair's second row, read at column up to 127 + 3 (positions past the
  // image row are discarded), must stay inside the box
  const int32_t need = 3 * wp + BM + 3;
  const int32_t r = (need + wp - 1) / wp;
  return r < 5 ? 5 : r;
}

template <int ACT>
bool launch_t(const StemPoolArgs& a, int num_sms, cudaStream_t st) {
  StemParams p;
  p.n_img = (int32_t)a.n;
  p.h2 = a.h / 2;
  p.w2 = a.w / 2;
  p.ph = (p.h2 - 3) / 2 + 1;
  p.pw = (p.w2 - 3) / 2 + 1;
  p.rbox = stem_rbox(p.w2);
  p.slot_bytes = (p.rbox * (p.w2 + 3) * 16 + 127) / 128 * 128;
  p.pool_rows = a.n * p.ph;
  p.wd = a.wd;
  p.a_scale = a.a_scale; p.w_scale = a.w_scale; p.w_scale_ch = a.w_scale_ch; p.bias = a.bias;
  p.act_param = a.act_param; p.out = a.out;
  p.amax = a.amax.ptr;
  p.amax_per_image = a.amax.ptr && a.amax.elems_per_slot > 0;
  const int smem = 1024 + kRing * p.slot_bytes + kWBytes + 2 * 4 * 4 * 16 * 4 + kBarBytes;
  if (smem > 227 * 1024) return false;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncSetAttribute(k_stem_pool<ACT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  CUtensorMap mi;
  if (!make_s2d_map(&mi, a.q, p.n_img, p.h2, p.w2, p.rbox)) return false;
  const int64_t grid = p.pool_rows < num_sms ? p.pool_rows : num_sms;
  k_stem_pool<ACT><<<(unsigned)grid, kThreads, smem, st>>>(mi, p);
  return true;
}

}  // namespace

bool stem_pool_shape_ok(int64_t n_img, int32_t c, int32_t h, int32_t w, int32_t k, int32_t stride, int32_t pad,
                        int32_t out_channels, int32_t pool_k, int32_t pool_s) {
  if (k != 7 || stride != 2 || pad != 3 || c < 1 || c > 4 || out_channels != BN) return false;
  if (pool_k != 3 || pool_s != 2 || (h & 1) || (w & 1) || h < 6 || w < 6) return false;
  if (w / 2 > 125 || n_img < 1 || n_img > 65535) return false;  // the M tile and the TMA box width
  if (n_img * (int64_t)((h / 2 - 3) / 2 + 1) > ((int64_t)1 << 40)) return false;
  return tma_encode_fn() != nullptr;
}

size_t stem_weight_bytes() { return (size_t)kWBytes; }

// w [64][C][7][7] quantized (reference layout) -> [8 taps][2 K chunks][64 rows][16 B]:
// tap t = (ay pair t / 4, ax = t % 4 - 2), chunk kc: ay = 2 (t / 4) - 2 + kc; byte
// (dy * 2 + dx) * 4 + c holds w[o][c][2 ay + dy + 3][2 ax + dx + 3] (zero outside 0..6).
void stem_arrange_weights(const int8_t* wq, int32_t c, int8_t* out) {
  memset(out, 0, kWBytes);
  for (int t = 0; t < kTaps; ++t)
    for (int kc = 0; kc < 2; ++kc) {
      const int ay = 2 * (t / 4) - 2 + kc, ax = t % 4 - 2;
      for (int o = 0; o < BN; ++o)
        for (int dy = 0; dy < 2; ++dy)
          for (int dx = 0; dx < 2; ++dx) {
            const int ky = 2 * ay + dy + 3, kx = 2 * ax + dx + 3;
            if (ky < 0 || ky > 6 || kx < 0 || kx > 6) continue;
            for (int ch = 0; ch < c; ++ch)
              out[((t * 2 + kc) * BN + o) * 16 + (dy * 2 + dx) * 4 + ch] = wq[((o * c + ch) * 7 + ky) * 7 + kx];
          }
    }
}

bool launch_stem_pool(const StemPoolArgs& a, int num_sms, cudaStream_t st) {
  if (a.n <= 0) return true;
  if ((reinterpret_cast<uintptr_t>(a.q) & 15) || (reinterpret_cast<uintptr_t>(a.wd) & 15)) return false;
  switch (a.act) {
    case ACT_NONE: return launch_t<ACT_NONE>(a, num_sms, st);
    case ACT_RELU: return launch_t<ACT_RELU>(a, num_sms, st);
    case ACT_SIGMOID: return launch_t<ACT_SIGMOID>(a, num_sms, st);
    case ACT_TANH: return launch_t<ACT_TANH>(a, num_sms, st);
    case ACT_GELU: return launch_t<ACT_GELU>(a, num_sms, st);
    case ACT_LEAKY_RELU: return launch_t<ACT_LEAKY_RELU>(a, num_sms, st);
    default: return false;
  }
}

int stem_take_error() {
  int h = 0, z = 0;
  if (cudaMemcpyFromSymbol(&h, g_stem_error, sizeof h) != cudaSuccess) return -1;
  if (h) cudaMemcpyToSymbol(g_stem_error, &z, sizeof z);
  return h;
}

}  // namespace rg
