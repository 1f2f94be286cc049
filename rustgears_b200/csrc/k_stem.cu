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
// A tile is two conv output rows y, y + 1 (y even).  The weights are the MMA's A operand
// (M = 128: rows 0-63 the 64 channels of row y, rows 64-127 the same channels of row
// y + 1, their taps shifted by one s2d row), the s2d positions its B operand (N = the
// row's w/2 columns, rows 16 bytes apart): a TMA load brings the padded s2d rows y - 2 ..
// y + 3 (zero rows and columns outside the image) and 12 MMAs (K 32 = two vertically
// adjacent s2d rows; 3 row pairs x 4 column shifts) accumulate the tile in TMEM with a
// channel per lane and a conv column per TMEM column.  So an epilogue thread holds 32
// consecutive conv columns of one channel and row in registers: the pooling window's
// three columns fold there (the reference's scan order within a row), the row y + 1
// thread hands its folded row to the row y thread through shared memory, and the row
// folds run in row order across tiles -- the same result as the reference's row-major
// scan, NaN and signed zeros included: the scan returns the last NaN, else the first
// maximal element in row-major order, and folding per-row results in row order
// preserves both.  Each CTA owns a contiguous range of pool rows.
//
//   warp 0     producer (lane 0): one TMA load per tile; the weights once
//   warp 1     MMA issuer (lane 0): 12 tcgen05.mma per tile into one of two TMEM
//              accumulators
//   warps 2-17 epilogue: warp w reads TMEM lane quadrant w % 4 (channel half, row of
//              the tile) and conv columns 28 (w - 2) / 4 ..; act(f32(acc) * (s_img *
//              s_w) + bias), the window folds, the pooled row staged in shared memory
//              and stored a channel row at a time, the per-image absmax of the pooled
//              tensor
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

constexpr int BN = 64;           // output channels
constexpr int kEpiWarps = 16;    // 4 per TMEM lane quadrant, one column range each
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kThreads = 64 + kEpiThreads;
constexpr int kMmas = 12;        // per tile: (s2d row pair 0..2) x (column shift 0..3)
constexpr int kWBytes = kMmas * 2 * 128 * 16;  // 48 KB of arranged weights
constexpr int kXchBytes = 4 * 16 * BN * 4;     // [4 column ranges][16 px][64 channels] f32
constexpr int kStgPitch = 57;                  // staged pool row: [64 channels][57] f32 (odd pitch)
constexpr int kStgBytes = BN * kStgPitch * 4;
constexpr int kRbox = 6;         // padded s2d rows per tile: y - 2 .. y + 3
constexpr int kTmemCols = 256;   // two accumulators of up to 112 columns
constexpr int kMaxW2 = 112;
constexpr int kRing = 6;
constexpr int kBarBytes = 256;

struct StemParams {
  int32_t n_img, h2, w2;           // s2d grid = conv output grid
  int32_t ph, pw;                  // pool output
  int32_t n_mma;                   // MMA N: w2 rounded up to 16
  int32_t span;                    // pool columns per epilogue column range: ceil(pw / 4)
  int32_t slot_bytes;              // ring slot (kRbox * (w2 + 3) * 16 + read-past margin, rounded to 128)
  int64_t pool_rows;               // n_img * ph
  const int8_t* wd;                // [12 MMAs][2 K chunks][128 rows][16 B]
  const float* a_scale;            // per image
  float w_scale;
  const float* w_scale_ch;
  const float* bias;
  float act_param;
  float* out;                      // NCHW [n_img, 64, ph, pw]
  unsigned* amax;                  // optional absmax sink of out
  int32_t amax_per_image;
  int* err;                        // this call's error word: set to 1 when a bounded wait gave up
};

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

// The tiles a CTA computes, in order: for each image its pool rows [ra, rb) need conv
// rows 2 ra .. 2 rb (pool row r reads conv rows 2r, 2r + 1, 2r + 2), i.e. the tiles
// (2r, 2r + 1) for r = ra .. rb (the last tile's second row is not used).
struct TileIter {
  int64_t g, g_end;   // global pool rows img * ph + r still to finish
  int32_t img, ra, rb, r;
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
    r = ra;
  }
  __device__ bool valid() const { return g < g_end; }
  __device__ void next(int32_t ph) {
    if (r < rb) {
      ++r;
      return;
    }
    g += rb - ra;
    if (g < g_end) seg(ph);
  }
};

// One step of the reference's window scan, best = (v > best || v is NaN) ? v : best, as
// predicated selects (no branch).
__device__ __forceinline__ void named_bar(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ float pool_fold(float best, float v) {
  float r;
  asm("{\n .reg .pred p, q;\n setp.nan.f32 q, %2, %2;\n setp.gt.or.f32 p, %2, %1, q;\n"
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
  float* xch = reinterpret_cast<float*>(wsm + kWBytes);            // [4][16][64]
  float* stg = xch + kXchBytes / 4;                                // [64][kStgPitch]
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(stg) + kStgBytes);
  uint64_t* full = bars;              // [kRing]
  uint64_t* empty = full + kRing;     // [kRing]
  uint64_t* tfull = empty + kRing;    // [2]
  uint64_t* tempty = tfull + 2;       // [2]
  uint64_t* wbar = tempty + 2;        // weights landed
  uint64_t* done = wbar + 1;          // every MMA retired
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

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
      const uint32_t a_bytes = (uint32_t)(kRbox * wp * 16);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_parity[kRing];
      bool issued[kRing];
      for (int s = 0; s < kRing; ++s) issued[s] = false;
      TileIter it;
      for (it.start(g0, g1, p.ph); it.valid(); it.next(p.ph)) {
        if (!mbar_wait(&empty[stage], phase ^ 1, abort)) break;
        mbar_arrive_expect_tx(&full[stage], a_bytes);
        // padded s2d rows 2r - 2 .. 2r + 3, columns from s2d pixel -2 (x = -4 eight-byte elements)
        tma_load_3d(ring + (size_t)stage * p.slot_bytes, &map_in, &full[stage], -4, 2 * it.r - 2, it.img);
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
      const uint32_t idesc = idesc_i8(128, p.n_mma);
      const uint32_t sw = smem_addr(wsm);
      int stage = 0;
      uint32_t phase = 0;
      int iter = 0;
      bool ok = mbar_wait(wbar, 0, abort);
      if (ok) tc_fence_after();
      TileIter it;
      for (it.start(g0, g1, p.ph); ok && it.valid(); it.next(p.ph), ++iter) {
        const int buf = iter & 1;
        const uint32_t aphase = (iter >> 1) & 1;
        if (!mbar_wait(&tempty[buf], aphase ^ 1, abort)) break;
        if (!mbar_wait(&full[stage], phase, abort)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * p.n_mma);
        const uint32_t sa = smem_addr(ring + (size_t)stage * p.slot_bytes);
#pragma unroll
        for (int t = 0; t < kMmas; ++t) {
          // s2d rows 2r - 2 + 2 (t / 4) and the next one (K chunks one padded row apart),
          // columns shifted by t % 4 - 2
          const uint32_t pos = (uint32_t)((t / 4) * 2 * wp + (t % 4));
          mma_i8(d_tmem, desc_rows16(sw + t * 2 * 128 * 16, 128 * 16), desc_rows16(sa + pos * 16u, (uint32_t)wp * 16u),
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
    // Per tile: (A) every warp folds its 32 columns' windows; the row-(y + 1) warps
    // publish theirs; (B) the row-y warps fold the rows and stage the finished pool row
    // r - 1 in shared memory as [channel][column]; (C) all warps store it, a channel row
    // per store instruction (coalesced).
    const int q = warp & 3;                 // TMEM lane quadrant: channel half q & 1, tile row q >> 1
    const int k = (warp - 2) >> 2;          // column range: pool columns k * span .. + span - 1
    const bool row0 = q < 2;                // this thread holds row y (else y + 1)
    const int32_t c = (q & 1) * 32 + lane;  // channel
    const int32_t px0 = k * p.span;
    const int32_t npx = min(p.span, p.pw - px0);  // pool columns of this range (may be <= 0)
    const int32_t plane = p.ph * p.pw;
    const float bias_c = __ldg(p.bias + c);
    const float wsc = p.w_scale_ch ? __ldg(p.w_scale_ch + c) : p.w_scale;
    float* xb = xch + (size_t)(k * 16) * BN + c;  // [j][channel]
    int32_t cs_img = -1;
    float cs = 0.0f;
    float part[16];                         // fold of pool row r's first two rows (row y threads)
    float mx = 0.0f;
    int iter = 0;
    TileIter it;
    for (it.start(g0, g1, p.ph); it.valid(); it.next(p.ph), ++iter) {
      const int buf = iter & 1;
      const uint32_t aphase = (iter >> 1) & 1;
      float h[16];                          // the window's row folded, per pool column
      const bool got = mbar_wait(&tfull[buf], aphase, abort);
      if (__all_sync(0xffffffffu, got)) {
        tc_fence_after();
        uint32_t v[32];
        const uint32_t ta = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * p.n_mma + 2 * px0);
        tmem_ld16(ta, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
        tmem_ld16(ta + 16, *reinterpret_cast<uint32_t(*)[16]>(&v[16]));
        tmem_ld_wait();
        tc_fence_before();
        if (it.img != cs_img) {
          cs_img = it.img;
          cs = __fmul_rn(p.a_scale[it.img], wsc);
        }
        // |acc| <= 147 taps x 127 x 127 < 2^22
        float o[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = epilogue_small_t<ACT>((int32_t)v[i], cs, bias_c, p.act_param);
        // the window's columns 2 px, 2 px + 1, 2 px + 2 in the reference's order
#pragma unroll
        for (int j = 0; j < 15; ++j) h[j] = pool_fold(pool_fold(o[2 * j], o[2 * j + 1]), o[2 * j + 2]);
        h[15] = o[30];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
      if (!row0) {
#pragma unroll
        for (int j = 0; j < 16; ++j) xb[j * BN] = h[j];
      }
      // (A) done everywhere: the row-(y + 1) folds are published, every accumulator read
      if (!bar_and(1, kEpiThreads, got)) {
        *abort = 1;
        break;
      }
      const bool emits = it.r > it.ra;   // completes pool row r - 1 with row 2r
      const bool starts = it.r < it.rb;  // pool row r: rows 2r, 2r + 1 folded here
      if (row0) {
        // all shared-memory loads first: the stores below may not be reordered above them
        float hn[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) hn[j] = xb[j * BN];
        if (emits) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float best = pool_fold(part[j], h[j]);
            if (j < npx) {
              stg[c * kStgPitch + px0 + j] = best;
              mx = fmaxf(mx, fabsf(best));
            }
          }
        }
        if (starts) {
#pragma unroll
          for (int j = 0; j < 16; ++j) part[j] = pool_fold(h[j], hn[j]);
        }
      }
      // (B) done: pool row r - 1 staged, the row-(y + 1) folds read (the exchange buffer
      // is free for the next tile)
      named_bar(2, kEpiThreads);
      if (emits) {
        // (C) warp e stores channels 4e .. 4e + 3 of pool row r - 1
        const int e = warp - 2;
        float* orow = p.out + ((int64_t)it.img * BN + 4 * e) * plane + (int64_t)(it.r - 1) * p.pw;
        // columns lane and lane + 32 (pw <= 56 < 64), staged rows are kStgPitch = 57 wide
        float sv[8];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          sv[2 * cc] = stg[(4 * e + cc) * kStgPitch + lane];
          sv[2 * cc + 1] = lane + 32 < kStgPitch ? stg[(4 * e + cc) * kStgPitch + lane + 32] : 0.0f;
        }
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          if (lane < p.pw) orow[(int64_t)cc * plane + lane] = sv[2 * cc];
          if (lane + 32 < p.pw) orow[(int64_t)cc * plane + lane + 32] = sv[2 * cc + 1];
        }
      }
      if (it.r == it.rb) {  // the image's last tile in this CTA: flush its absmax
        if (p.amax) {
          float m = mx;
#pragma unroll
          for (int o2 = 16; o2 > 0; o2 >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o2));
          if (lane == 0 && m > 0.0f) atomicMax(p.amax + (p.amax_per_image ? it.img : 0), __float_as_uint(m));
        }
        mx = 0.0f;
      }
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

template <int ACT>
bool launch_t(const StemPoolArgs& a, int num_sms, cudaStream_t st) {
  StemParams p;
  p.n_img = (int32_t)a.n;
  p.h2 = a.h / 2;
  p.w2 = a.w / 2;
  p.ph = (p.h2 - 3) / 2 + 1;
  p.pw = (p.w2 - 3) / 2 + 1;
  p.n_mma = (p.w2 + 15) / 16 * 16;
  p.span = (p.pw + 3) / 4;
  // the last MMA's B rows reach n_mma - 1 + 3 columns into the sixth row
  p.slot_bytes = (kRbox * (p.w2 + 3) * 16 + (p.n_mma - p.w2) * 16 + 127) / 128 * 128;
  p.pool_rows = a.n * p.ph;
  p.wd = a.wd;
  p.a_scale = a.a_scale; p.w_scale = a.w_scale; p.w_scale_ch = a.w_scale_ch; p.bias = a.bias;
  p.act_param = a.act_param; p.out = a.out;
  p.amax = a.amax.ptr;
  p.amax_per_image = a.amax.ptr && a.amax.elems_per_slot > 0;
  p.err = a.err;
  if (!p.err) return false;
  const int smem = 1024 + kRing * p.slot_bytes + kWBytes + kXchBytes + kStgBytes + kBarBytes;
  if (smem > 227 * 1024) return false;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncSetAttribute(k_stem_pool<ACT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  CUtensorMap mi;
  if (!make_s2d_map(&mi, a.q, p.n_img, p.h2, p.w2, kRbox)) return false;
  const int64_t grid = p.pool_rows < num_sms ? p.pool_rows : num_sms;
  k_stem_pool<ACT><<<(unsigned)grid, kThreads, smem, st>>>(mi, p);
  return true;
}

}  // namespace

bool stem_pool_shape_ok(int64_t n_img, int32_t c, int32_t h, int32_t w, int32_t k, int32_t stride, int32_t pad,
                        int32_t out_channels, int32_t pool_k, int32_t pool_s) {
  if (k != 7 || stride != 2 || pad != 3 || c < 1 || c > 4 || out_channels != BN) return false;
  if (pool_k != 3 || pool_s != 2 || (h & 1) || (w & 1) || h < 6 || w < 6) return false;
  // two accumulators of w/2 columns in TMEM (each epilogue warp reads 32 columns from
  // 2 x ceil(pw / 4) x 3), 16 pool columns per range at most
  if (w / 2 > kMaxW2 || n_img < 1 || n_img > 65535) return false;
  return tma_encode_fn() != nullptr;
}

size_t stem_weight_bytes() { return (size_t)kWBytes; }

// w [64][C][7][7] quantized (reference layout) -> [12 MMAs][2 K chunks][128 rows][16 B]:
// MMA t reads s2d rows 2r - 2 + 2 (t / 4) + kc (kc = K chunk) at column shift
// ax = t % 4 - 2; row m < 64 is channel m of conv row 2r (tap ay = 2 (t / 4) - 2 + kc),
// row m >= 64 channel m - 64 of conv row 2r + 1 (tap ay - 1); byte (dy * 2 + dx) * 4 + c
// holds w[o][c][2 ay + dy + 3][2 ax + dx + 3], zero where a tap index leaves -2..1 or a
// kernel index leaves 0..6.
void stem_arrange_weights(const int8_t* wq, int32_t c, int8_t* out) {
  memset(out, 0, kWBytes);
  for (int t = 0; t < kMmas; ++t)
    for (int kc = 0; kc < 2; ++kc)
      for (int m = 0; m < 128; ++m) {
        const int o = m % BN, ay = 2 * (t / 4) - 2 + kc - m / BN, ax = t % 4 - 2;
        if (ay < -2 || ay > 1) continue;
        for (int dy = 0; dy < 2; ++dy)
          for (int dx = 0; dx < 2; ++dx) {
            const int ky = 2 * ay + dy + 3, kx = 2 * ax + dx + 3;
            if (ky < 0 || ky > 6 || kx < 0 || kx > 6) continue;
            for (int ch = 0; ch < c; ++ch)
              out[((t * 2 + kc) * 128 + m) * 16 + (dy * 2 + dx) * 4 + ch] = wq[((o * c + ch) * 7 + ky) * 7 + kx];
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
    case ACT_SILU: return launch_t<ACT_SILU>(a, num_sms, st);
    default: return false;
  }
}

}  // namespace rg
