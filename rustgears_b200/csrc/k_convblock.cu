// k_convblock.cu -- one kernel for the CNN block
//   FusedConv2d(1->16, k3 s1 p1, act) -> MaxPool2d(2,2) -> FusedConv2d(16->C2, k3 s1 p1, act) -> MaxPool2d(2,2)
// on 28x28 images, every intermediate of an image kept in shared memory, TMEM or registers.
//
// Reference semantics (src/inference/npu.rs:319-383, kernels.rs:28-96,165-213,
// quantize.rs:27-35,122-144):
//   * each conv quantizes ITS OWN INPUT per image (absmax over the image's im2col,
//     which for a stride-1/pad-1 conv is every pixel), i8 x i8 -> i32, epilogue
//     act(f32(acc) * (s_img * s_w) + bias[c]);
//   * the pool takes the window max of the f32 activations.
// Max pooling is taken on the i32 accumulators and the epilogue applied once per
// window: f32(acc), *cs (cs > 0), +bias and a non-decreasing activation are each
// monotone under round-to-nearest, so max(f(acc_i)) == f(max(acc_i)) exactly.  When
// an image's scale is not finite (an inf in the input) the kernel falls back to the
// reference order (activation per pixel, NaN-propagating max), uniformly per image.
//
// Persistent, one CTA per SM, warp-specialised; images flow through a pipeline whose
// stages hand over through mbarrier rings (every wait bounded):
//   warp 0      loader: bulk-copies each f32 image into a 4-slot shared-memory ring;
//   warps 1-4   quantizer: image absmax -> scale -> padded i8 rows -> conv1 im2col
//               tile, one pool window (its 4 pixels) per thread, double-buffered;
//   warp 5      conv1 MMA issuer, warp 6 conv2 MMA issuer (descriptors precomputed),
//               each into double-buffered TMEM accumulators;
//   warps 7-14  conv1 epilogue: window max over the 4 window positions, epilogue,
//               image absmax -> conv2 scale -> requantized interleaved map;
//   warps 15-18 conv2 epilogue: window max, epilogue, f32 stores, output absmax.
// Groups of warps that reduce together use named barriers whose AND-vote also
// carries "every wait succeeded", so a timeout makes a whole group leave its loop
// together; the teardown drains in-flight copies and MMAs before TMEM is freed.
//
// Tensor-core operands (tcgen05.mma kind::i8, K-major, no swizzle: 8-row x 16-byte
// core matrices, SBO between 8-row groups, LBO between the two 16-byte K halves):
//   conv1: an im2col tile built per image, taps packed as 4*ky + kx (three 4-byte runs
//          of the padded input row) in 16 bytes.  Row w of tile (g, pp) holds pool
//          window 128g + w: its pixel at position 2pp (dy = pp, dx = 0) in the first 16
//          bytes of K and its pixel at position 2pp + 1 in the second; the weights are
//          the block-diagonal 32 x 32 tile [W1 0; 0 W1], so one MMA (N = 32) yields both
//          positions and the 4 pixels of a window land in one TMEM lane, 16 columns
//          apart.
//   conv2: no im2col.  The quantized 16-channel map is stored padded (16 x 16 pixels
//          of 16 bytes) with each row column-interleaved: the 8 even columns, then the
//          8 odd ones.  For output column parity dx, the operand rows (y, j) of tap
//          (ky, kx) -- input column 2j + dx + kx -- are then 8 consecutive 16-byte
//          pixels of one half row (a core matrix) and 8-row groups are image rows
//          (SBO = 256): each MMA K step reads the map in place.  The two dx tiles
//          go to two TMEM column blocks, so the horizontal pool max is in-thread and
//          the vertical one is a single shuffle (rows y, y+1 are lanes l, l^8).
//          K steps pair taps in the order of their offsets for that dx (LBO > 0);
//          the weights are staged once per order.
#include <cuda_runtime.h>

#include "rg_kernels.h"
#include "rg_math.cuh"
#include "rg_sm100.cuh"

namespace rg {
namespace {

using namespace sm100;

constexpr int H = 28, W = 28, C1 = 16;
constexpr int P1 = 14;                 // pooled conv1 map is 14 x 14 (16 x 16 padded)
constexpr int P2 = 7;                  // pooled conv2 map is 7 x 7
constexpr int Rows1 = H * W;           // 784 conv1 output pixels
constexpr int MT1 = 4;                 // conv1 tiles: 2 groups of 128 windows x 2 position pairs
constexpr int Q1P = 40;                // padded conv1 input row pitch (bytes): pixel x of a row at byte 4 + x
constexpr int Q1BYTES = 30 * Q1P;      // 30 padded rows
constexpr int SBO1 = 256;              // conv1 tile: 2 chunks x 128 B per 8-row group
constexpr int Q2ROW = 256;             // conv2 map row: 16 pixels x 16 B (even half, odd half)
constexpr int kImgBytes = H * W * 4;   // one f32 input image
constexpr int kInSlots = 4;            // input ring depth
constexpr int kA1Bytes = MT1 * 128 * 32;
constexpr int kQ2Bytes = 19 * Q2ROW;
constexpr int kTmemCols = 512;         // conv1: 2 x 128 columns at 0; conv2: 2 x 2*C2 at 256

// roles (warp indices)
constexpr int kWarpLoad = 0, kWarpQ = 1, kQWarps = 4, kWarpMma1 = 5, kWarpMma2 = 6, kWarpE1 = 7,
              kE1Warps = 8, kWarpE2 = 15, kE2Warps = 4;
constexpr int kThreads = (kWarpE2 + kE2Warps) * 32;
constexpr int kBarQ = 1, kBarE1 = 2, kBarE2 = 3;  // named barriers (0 is __syncthreads)
constexpr uint64_t kWaitNs = 1000000000ull;      // limit of every pipeline wait

// Tap order per output-column parity dx: the taps of each kernel row sorted by their
// byte offset in the interleaved row, so every K-step pair has a positive LBO.
// dx = 0: kx offsets 0 (kx0), 16 (kx2), 128 (kx1); dx = 1: 16 (kx1), 128 (kx0), 144 (kx2).
__host__ __device__ constexpr int tap_order(int dx, int i) {
  return (i / 3) * 3 + (dx == 0 ? (i % 3 == 0 ? 0 : i % 3 == 1 ? 2 : 1) : (i % 3 == 0 ? 1 : i % 3 == 1 ? 0 : 2));
}
__host__ __device__ constexpr int tap_offset(int dx, int tap) {  // bytes from the (row 0, j 0) pixel
  return (tap / 3) * Q2ROW + ((dx + tap % 3) & 1) * 128 + ((dx + tap % 3) >> 1) * 16;
}

template <int C2>
struct Lay {
  static constexpr int K2P = 160, SBO2W = 10 * 128;             // W2 tile: 10 chunks per 8-row group
  static constexpr int OFF_IN = 0;                               // kInSlots f32 images
  static constexpr int OFF_Q1 = OFF_IN + kInSlots * kImgBytes;   // i8 [30][40] padded rows (+2 spare words)
  static constexpr int OFF_A1 = OFF_Q1 + Q1BYTES + 16;           // 2 conv1 im2col tiles: 8 x 128 rows x 32 B
  static constexpr int OFF_W1 = OFF_A1 + 2 * kA1Bytes;           // W1 as a 32 x 32 B block-diagonal tile
  static constexpr int OFF_Q2 = OFF_W1 + 2 * C1 * 32;            // 2 x i8 [19 rows][256 B], interleaved
  static constexpr int OFF_W2 = OFF_Q2 + 2 * kQ2Bytes;           // W2 in the dx = 0 and dx = 1 tap orders
  static constexpr int OFF_BIAS = OFF_W2 + 2 * C2 * K2P;         // b1[16], b2[C2]
  static constexpr int OFF_MISC = OFF_BIAS + (C1 + C2) * 4;      // barriers, scales, reductions
  static constexpr int SMEM = OFF_MISC + 512;
  static_assert(OFF_A1 % 16 == 0 && OFF_Q2 % 16 == 0 && OFF_W2 % 16 == 0 && OFF_MISC % 8 == 0, "alignment");
};

struct Misc {  // shared-memory control block
  uint64_t full_in[kInSlots], empty_in[kInSlots];
  uint64_t full_a1[2], empty_a1[2], t1_full[2], t1_empty[2];
  uint64_t full_q2[2], empty_q2[2], t2_full[2], t2_empty[2];
  uint64_t done1, done2;
  uint32_t tmem_slot;
  int abort;
  float scale1[2], scale2[2];
  float red_q[kQWarps];
  float red_e1[2][kE1Warps];
  float red_e2[2][kE2Warps];
};
static_assert(sizeof(Misc) <= 512, "control block");

struct CBParams {
  const float* x;          // [n, 1, 28, 28]
  int64_t n;
  const int8_t* w1;        // [16, kpad1], reduction order (ky, kx)
  int32_t kpad1;
  const int8_t* w2;        // [C2, kpad2], reduction order (ky, kx, c)
  int32_t kpad2;
  float w1_scale, w2_scale;
  const float* b1;
  const float* b2;
  float p1, p2;            // LeakyReLU slopes
  float* out;              // [n, C2, 7, 7]
  unsigned* amax;          // optional sink of the output's absmax
  int64_t amax_per_image;
  int* err;                // this call's error word: set to 1 when a bounded wait gave up
  int8_t* out_q;           // calibration extension: i8 output [n, C2 * 49] with the frozen scale
  const float* q_scale;
};

__device__ __forceinline__ uint64_t desc_noswz(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version; layout type 0 = no swizzle
  return d;
}

__host__ __device__ __forceinline__ int canon(int r, int j, int sbo) { return (r & 7) * 16 + (r >> 3) * sbo + j * 128; }

// Max over the warp of absolute values (NaN ignored, as f32::max): non-negative floats
// order like their bit patterns, so one redux.sync on the bits replaces five shuffle
// rounds; fmaxf(v, 0) first turns a NaN (a thread whose values were all NaN) into 0.
__device__ __forceinline__ float warp_max(float v) {
  return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fmaxf(v, 0.0f))));
}

template <int ACT>
__device__ __forceinline__ float epi(int32_t acc, float cs, float bias, float p) {
  const float v = __fadd_rn(__fmul_rn(__int2float_rn(acc), cs), bias);
  if (ACT == ACT_RELU) return fmaxf(v, 0.0f);
  if (ACT == ACT_LEAKY_RELU) return v > 0.0f ? v : __fmul_rn(p, v);
  return v;
}

// Four values of a tensor quantized with the scale of its own absmax, packed little-endian.
__device__ __forceinline__ uint32_t pack4(float a, float b, float c, float d, float inv) {
  return (uint32_t)(quant1_bounded(a, inv) & 0xff) | ((uint32_t)(quant1_bounded(b, inv) & 0xff) << 8) |
         ((uint32_t)(quant1_bounded(c, inv) & 0xff) << 16) | ((uint32_t)(quant1_bounded(d, inv) & 0xff) << 24);
}
__device__ __forceinline__ uint32_t pack4b(float4 v, float inv) { return pack4(v.x, v.y, v.z, v.w, inv); }

__device__ __forceinline__ void fence_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <int C2, int ACT1, int ACT2>
__global__ void __launch_bounds__(kThreads, 1) k_convblock(const CBParams p) {
  using L = Lay<C2>;
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* in = sm + L::OFF_IN;
  uint8_t* q1 = sm + L::OFF_Q1;
  uint8_t* a1 = sm + L::OFF_A1;
  uint8_t* w1s = sm + L::OFF_W1;
  uint8_t* q2 = sm + L::OFF_Q2;
  uint8_t* w2s = sm + L::OFF_W2;
  float* b1s = reinterpret_cast<float*>(sm + L::OFF_BIAS);
  float* b2s = b1s + C1;
  Misc& ms = *reinterpret_cast<Misc*>(sm + L::OFF_MISC);
  volatile int* abort = &ms.abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x;
  const int n_it = p.n > (int64_t)blockIdx.x ? (int)((p.n - 1 - blockIdx.x) / G + 1) : 0;

  // ---- one-time set-up: zero the padded staging areas, stage weights, biases, table ----
  for (int i = L::OFF_Q1 + tid * 16; i < L::OFF_W1; i += kThreads * 16) *reinterpret_cast<uint4*>(sm + i) = make_uint4(0, 0, 0, 0);
  for (int i = L::OFF_Q2 + tid * 16; i < L::OFF_W2 + 2 * C2 * L::K2P; i += kThreads * 16)
    *reinterpret_cast<uint4*>(sm + i) = make_uint4(0, 0, 0, 0);
  for (int i = L::OFF_W1 + tid * 16; i < L::OFF_Q2; i += kThreads * 16) *reinterpret_cast<uint4*>(sm + i) = make_uint4(0, 0, 0, 0);
  __syncthreads();
  for (int i = tid; i < C1 * 12; i += kThreads) {  // W1 byte 4*ky + kx <- reference column 3*ky + kx
    const int n = i / 12, b = i % 12, ky = b >> 2, kx = b & 3;
    if (kx < 3) {
      const uint8_t v = (uint8_t)p.w1[(int64_t)n * p.kpad1 + 3 * ky + kx];
      w1s[canon(n, 0, SBO1) + b] = v;        // rows 0-15: first K half
      w1s[canon(C1 + n, 1, SBO1) + b] = v;   // rows 16-31: second K half
    }
  }
  for (int i = tid; i < 2 * C2 * 144; i += kThreads) {  // W2 chunk k holds tap tap_order(dx, k); 144.. stay 0
    const int dx = i / (C2 * 144), rem = i % (C2 * 144), n = rem / 144, b = rem % 144;
    const int k = b >> 4, tap = tap_order(dx, k);
    w2s[dx * C2 * L::K2P + canon(n, k, L::SBO2W) + (b & 15)] = (uint8_t)p.w2[(int64_t)n * p.kpad2 + tap * 16 + (b & 15)];
  }
  if (tid < C1) b1s[tid] = p.b1[tid];
  if (tid < C2) b2s[tid] = p.b2[tid];
  if (tid == 0) {
    for (int s = 0; s < kInSlots; ++s) {
      mbar_init(&ms.full_in[s], 1);
      mbar_init(&ms.empty_in[s], kQWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ms.full_a1[b], kQWarps);
      mbar_init(&ms.empty_a1[b], 2);            // conv1 MMAs done + conv1 epilogue read the scale
      mbar_init(&ms.t1_full[b], 1);
      mbar_init(&ms.t1_empty[b], kE1Warps);
      mbar_init(&ms.full_q2[b], kE1Warps);
      mbar_init(&ms.empty_q2[b], 1 + kE2Warps);  // conv2 MMAs done + conv2 epilogue read the scale
      mbar_init(&ms.t2_full[b], 1);
      mbar_init(&ms.t2_empty[b], kE2Warps);
    }
    mbar_init(&ms.done1, 1);
    mbar_init(&ms.done2, 1);
    ms.abort = 0;
    fence_mbar_init();
  }
  if (warp == kWarpMma1) tmem_alloc(&ms.tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ms.tmem_slot;

  if (warp == kWarpLoad) {
    // ---------------- loader ----------------
    if (lane == 0) {
      int it = 0;
      for (; it < n_it; ++it) {
        const int s = it % kInSlots;
        if (!mbar_wait(&ms.empty_in[s], ((it / kInSlots) & 1) ^ 1, abort, kWaitNs)) break;
        mbar_arrive_expect_tx(&ms.full_in[s], kImgBytes);
        bulk_load(in + s * kImgBytes, p.x + (blockIdx.x + (int64_t)it * G) * (H * W), kImgBytes, &ms.full_in[s]);
      }
      // Drain: the last copies of each slot must have landed before the CTA may exit.
      volatile int never = 0;
      for (int j = it - kInSlots < 0 ? 0 : it - kInSlots; j < it; ++j)
        mbar_wait(&ms.full_in[j % kInSlots], (j / kInSlots) & 1, &never, 200000000ull);
    }
  } else if (warp < kWarpQ + kQWarps) {
    // ---------------- quantizer: image -> scale -> padded rows -> conv1 im2col ----------------
    const int tq = tid - kWarpQ * 32, qw = warp - kWarpQ;
    const bool two = tq < H * W / 4 - 128;     // this thread also owns float4 tq + 128
    const bool win2 = tq + 128 < P1 * P1;      // ... and pool window tq + 128
    // Pool window w = 14 wy + wx needs padded rows 2wy .. 2wy+3, bytes 3+2wx .. 6+2wx
    // (columns 2wx-1 .. 2wx+2): two words per row.  Its pixel (dy, dx) goes to tile
    // 2*(w/128) + dy, row w % 128, K half dx.
    int wsrc[2], wdst[2];
    uint32_t wsh[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int w = tq + 128 * k, wy = w / P1, wx = w % P1;
      const int byte = 2 * wy * Q1P + 3 + 2 * wx;
      wsrc[k] = byte >> 2;
      wsh[k] = 8u * (uint32_t)(byte & 3);
      wdst[k] = canon(2 * (w >> 7) * 128 + (w & 127), 0, SBO1);
    }
    for (int it = 0; it < n_it; ++it) {
      const int s = it % kInSlots, b = it & 1;
      const uint32_t ph = (it >> 1) & 1;
      bool ok = mbar_wait(&ms.full_in[s], (it / kInSlots) & 1, abort, kWaitNs);
      float4 va = make_float4(0.f, 0.f, 0.f, 0.f), vb = va;
      float m = 0.0f;
      if (ok) {
        const float4* src = reinterpret_cast<const float4*>(in + s * kImgBytes);
        va = src[tq];
        m = fmaxf(fmaxf(fabsf(va.x), fabsf(va.y)), fmaxf(fabsf(va.z), fabsf(va.w)));
        if (two) {
          vb = src[tq + 128];
          m = fmaxf(m, fmaxf(fmaxf(fabsf(vb.x), fabsf(vb.y)), fmaxf(fabsf(vb.z), fabsf(vb.w))));
        }
      }
      m = warp_max(m);
      if (lane == 0) ms.red_q[qw] = m;
      __syncwarp();
      if (lane == 0 && ok) mbar_arrive(&ms.empty_in[s]);  // the image now lives in registers
      ok = ok && mbar_wait(&ms.empty_a1[b], ph ^ 1, abort, kWaitNs);
      if (!bar_and(kBarQ, kQWarps * 32, ok)) { *abort = 1; break; }
      const float s1 = quant_scale(fmaxf(fmaxf(ms.red_q[0], ms.red_q[1]), fmaxf(ms.red_q[2], ms.red_q[3])));
      const float inv1 = quant_inv(s1);
      uint32_t* q1w = reinterpret_cast<uint32_t*>(q1);
      {  // 4 pixels of one row -> one aligned word
        const int f = tq, y = (4 * f) / W, x = (4 * f) % W;
        q1w[((y + 1) * Q1P + 4 + x) >> 2] = pack4b(va, inv1);
        if (two) {
          const int f2 = tq + 128, y2 = (4 * f2) / W, x2 = (4 * f2) % W;
          q1w[((y2 + 1) * Q1P + 4 + x2) >> 2] = pack4b(vb, inv1);
        }
      }
      bar_and(kBarQ, kQWarps * 32, true);
      // conv1 im2col, one window per step: 4 rows x 2 words -> 4 tile rows of bytes 4*ky + kx
      uint8_t* a1b = a1 + b * kA1Bytes;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        if (k == 0 || win2) {
          uint32_t lo[4], hi[4];
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            lo[r] = q1w[wsrc[k] + r * (Q1P / 4)];
            hi[r] = q1w[wsrc[k] + r * (Q1P / 4) + 1];
          }
#pragma unroll
          for (int pos = 0; pos < 4; ++pos) {
            const int dy = pos >> 1;
            const uint32_t sh = wsh[k] + 8u * (uint32_t)(pos & 1);
            *reinterpret_cast<uint4*>(a1b + wdst[k] + (pos >> 1) * 16 * SBO1 + (pos & 1) * 128) =
                make_uint4(__funnelshift_rc(lo[dy], hi[dy], sh), __funnelshift_rc(lo[dy + 1], hi[dy + 1], sh),
                           __funnelshift_rc(lo[dy + 2], hi[dy + 2], sh), 0u);
          }
        }
      }
      if (tq == 0) ms.scale1[b] = __fmul_rn(s1, p.w1_scale);
      fence_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ms.full_a1[b]);
    }
  } else if (warp == kWarpMma1) {
    // ---------------- conv1 MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc1 = idesc_i8(128, 2 * C1);
      const uint64_t a1d = desc_noswz(smem_addr(a1), 128, SBO1), w1d = desc_noswz(smem_addr(w1s), 128, SBO1);
      bool ok = true;
      for (int it = 0; it < n_it && ok; ++it) {
        const int b = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        ok = mbar_wait(&ms.full_a1[b], ph, abort, kWaitNs) && mbar_wait(&ms.t1_empty[b], ph ^ 1, abort, kWaitNs);
        if (!ok) break;
        tc_fence_after();
        const uint64_t ad = a1d + (uint64_t)((b * kA1Bytes) >> 4);
#pragma unroll
        for (int t = 0; t < MT1; ++t)
          mma_i8(tmem + (uint32_t)(b * 128 + t * 2 * C1), ad + (uint64_t)((t * 16 * SBO1) >> 4), w1d, idesc1, 0);
        mma_commit(&ms.t1_full[b]);
        mma_commit(&ms.empty_a1[b]);
      }
      if (!ok) *abort = 1;
      // Drain: every MMA this thread issued completes before TMEM is freed.
      mma_commit(&ms.done1);
      volatile int never = 0;
      mbar_wait(&ms.done1, 0, &never, 200000000ull);
    }
  } else if (warp == kWarpMma2) {
    // ---------------- conv2 MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc2 = idesc_i8(128, C2);
      const uint64_t q2d = desc_noswz(smem_addr(q2), 0, Q2ROW), w2d = desc_noswz(smem_addr(w2s), 128, L::SBO2W);
      bool ok = true;
      for (int it = 0; it < n_it && ok; ++it) {
        const int b = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        ok = mbar_wait(&ms.full_q2[b], ph, abort, kWaitNs) && mbar_wait(&ms.t2_empty[b], ph ^ 1, abort, kWaitNs);
        if (!ok) break;
        tc_fence_after();
        const uint64_t qd = q2d + (uint64_t)((b * kQ2Bytes) >> 4);
#pragma unroll
        for (int dx = 0; dx < 2; ++dx)
#pragma unroll
          for (int s = 0; s < 5; ++s) {
            const uint32_t oa = (uint32_t)tap_offset(dx, tap_order(dx, 2 * s));
            const uint32_t ob = s < 4 ? (uint32_t)tap_offset(dx, tap_order(dx, 2 * s + 1)) : oa + 16u;  // zero weights
            mma_i8(tmem + (uint32_t)(256 + b * 2 * C2 + dx * C2), qd + (uint64_t)(oa >> 4) + ((uint64_t)((ob - oa) >> 4) << 16),
                   w2d + (uint64_t)((dx * C2 * L::K2P + s * 256) >> 4), idesc2, s > 0);
          }
        mma_commit(&ms.t2_full[b]);
        mma_commit(&ms.empty_q2[b]);
      }
      if (!ok) *abort = 1;
      mma_commit(&ms.done2);
      volatile int never = 0;
      mbar_wait(&ms.done2, 0, &never, 200000000ull);
    }
  } else if (warp < kWarpE1 + kE1Warps) {
    // ---------------- conv1 epilogue: lane = pool window, max over the 4 position tiles ----------------
    const int e = warp - kWarpE1, q = warp & 3, g = e >> 2;
    const int win = 128 * g + 32 * q + lane;  // this lane's pool window
    const bool win_ok = win < P1 * P1;
    const bool busy = 128 * g + 32 * q < P1 * P1;  // a warp with no valid window only hands over
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    const int q2off = (win / P1 + 1) * Q2ROW + ((win % P1 + 1) & 1) * 128 + ((win % P1 + 1) >> 1) * 16;
    for (int it = 0; it < n_it; ++it) {
      const int b = it & 1;
      const uint32_t ph = (it >> 1) & 1;
      bool ok = mbar_wait(&ms.t1_full[b], ph, abort, kWaitNs) && mbar_wait(&ms.full_a1[b], ph, abort, kWaitNs);
      ok = __all_sync(0xffffffffu, ok);
      const float cs1 = ms.scale1[b];
      float v[16];
      float m2 = 0.0f;
      if (ok && busy) {
        tc_fence_after();
        const uint32_t tb = lane_base + (uint32_t)(b * 128 + 4 * g * C1);
        if (isfinite(cs1)) {
          // the window's four positions in one TMEM round trip; biases broadcast from smem
          uint32_t acc[16], acc2[16], acc3[16], acc4[16];
          tmem_ld16(tb, acc);
          tmem_ld16(tb + (uint32_t)C1, acc2);
          tmem_ld16(tb + (uint32_t)(2 * C1), acc3);
          tmem_ld16(tb + (uint32_t)(3 * C1), acc4);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int32_t mx = max(max((int32_t)acc[j], (int32_t)acc2[j]), max((int32_t)acc3[j], (int32_t)acc4[j]));
            v[j] = epi<ACT1>(mx, cs1, b1s[j], p.p1);
          }
        } else {  // reference order: activation per pixel, NaN-propagating max in (dy, dx) order
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = -INFINITY;
#pragma unroll 1
          for (int pos = 0; pos < 4; ++pos) {
            uint32_t acc[16];
            tmem_ld16(tb + (uint32_t)(pos * C1), acc);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float ev = epi<ACT1>((int32_t)acc[j], cs1, b1s[j], p.p1);
              if (ev > v[j] || ev != ev) v[j] = ev;
            }
          }
        }
        if (win_ok)
#pragma unroll
          for (int j = 0; j < 16; ++j) m2 = fmaxf(m2, fabsf(v[j]));
      }
      m2 = warp_max(m2);
      if (lane == 0) ms.red_e1[b][e] = m2;
      tc_fence_before();
      if (!bar_and(kBarE1, kE1Warps * 32, ok)) { *abort = 1; break; }
      // every conv1-epilogue thread has read scale1[b] and finished its TMEM loads
      if (e == 0 && lane == 0) mbar_arrive(&ms.empty_a1[b]);
      if (lane == 0) mbar_arrive(&ms.t1_empty[b]);
      float amax = 0.0f;
#pragma unroll
      for (int i = 0; i < kE1Warps; ++i) amax = fmaxf(amax, ms.red_e1[b][i]);
      const float s2 = quant_scale(amax), inv2 = quant_inv(s2);
      // requantize from registers into the interleaved padded map: one 16-B store per window
      ok = mbar_wait(&ms.empty_q2[b], ph ^ 1, abort, kWaitNs);
      if (ok) {
        if (win_ok)
          *reinterpret_cast<uint4*>(q2 + b * kQ2Bytes + q2off) =
              make_uint4(pack4(v[0], v[1], v[2], v[3], inv2), pack4(v[4], v[5], v[6], v[7], inv2),
                         pack4(v[8], v[9], v[10], v[11], inv2), pack4(v[12], v[13], v[14], v[15], inv2));
        if (e == 0 && lane == 0) ms.scale2[b] = __fmul_rn(s2, p.w2_scale);
        fence_async();
      }
      __syncwarp();
      if (lane == 0 && ok) mbar_arrive(&ms.full_q2[b]);
    }
  } else {
    // ---------------- conv2 epilogue: lane (y, j) = 8*y + j; window (y/2, j) = lanes l, l ^ 8 ----------------
    const int e = warp - kWarpE2, q = warp & 3;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    const int y = 4 * q + (lane >> 3), j = lane & 7;
    const int py = y >> 1, half = y & 1;  // half: which 8 of 16 channels this lane finishes
    const bool pos_ok = py < P2 && j < P2;
    float feat_amax = 0.0f;
    const float q_inv = p.out_q ? quant_inv(*p.q_scale) : 0.0f;
    for (int it = 0; it < n_it; ++it) {
      const int b = it & 1;
      const uint32_t ph = (it >> 1) & 1;
      const int64_t img = blockIdx.x + (int64_t)it * G;
      bool ok = mbar_wait(&ms.t2_full[b], ph, abort, kWaitNs) && mbar_wait(&ms.full_q2[b], ph, abort, kWaitNs);
      ok = __all_sync(0xffffffffu, ok);
      const float cs2 = ms.scale2[b];
      __syncwarp();
      if (lane == 0 && ok) mbar_arrive(&ms.empty_q2[b]);
      float mo = 0.0f;
      if (ok) {
        tc_fence_after();
        const bool fast2 = isfinite(cs2);
#pragma unroll 1
        for (int c0 = 0; c0 < C2; c0 += 16) {
          uint32_t a0[16], a1v[16];
          const uint32_t tb = lane_base + (uint32_t)(256 + b * 2 * C2 + c0);
          tmem_ld16(tb, a0);
          tmem_ld16(tb + (uint32_t)C2, a1v);
          tmem_ld_wait();
          float out[8];
          if (fast2) {
            int32_t mx[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              const int32_t h = max((int32_t)a0[k], (int32_t)a1v[k]);
              mx[k] = max(h, __shfl_xor_sync(0xffffffffu, h, 8));
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) out[k] = epi<ACT2>(half ? mx[8 + k] : mx[k], cs2, b2s[c0 + half * 8 + k], p.p2);
          } else {  // reference order (dy, dx): (y0,dx0), (y0,dx1), (y1,dx0), (y1,dx1)
            float best[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              const float bk = b2s[c0 + k];
              const float e0 = epi<ACT2>((int32_t)a0[k], cs2, bk, p.p2);
              const float e1 = epi<ACT2>((int32_t)a1v[k], cs2, bk, p.p2);
              const float f0 = __shfl_sync(0xffffffffu, e0, lane & ~8);
              const float f1 = __shfl_sync(0xffffffffu, e1, lane & ~8);
              const float f2 = __shfl_sync(0xffffffffu, e0, lane | 8);
              const float f3 = __shfl_sync(0xffffffffu, e1, lane | 8);
              float bb = -INFINITY;
              if (f0 > bb || f0 != f0) bb = f0;
              if (f1 > bb || f1 != f1) bb = f1;
              if (f2 > bb || f2 != f2) bb = f2;
              if (f3 > bb || f3 != f3) bb = f3;
              best[k] = bb;
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) out[k] = half ? best[8 + k] : best[k];
          }
          if (pos_ok) {
            const int64_t o0 = img * (int64_t)(C2 * P2 * P2) + (int64_t)(c0 + half * 8) * (P2 * P2) + py * P2 + j;
            if (p.out_q) {  // the next Linear's operand, quantized with its calibrated scale
#pragma unroll
              for (int k = 0; k < 8; ++k) p.out_q[o0 + k * (P2 * P2)] = (int8_t)quant1(out[k], q_inv);
            } else {
              float* og = p.out + o0;
#pragma unroll
              for (int k = 0; k < 8; ++k) {
                og[k * (P2 * P2)] = out[k];
                mo = fmaxf(mo, fabsf(out[k]));
              }
            }
          }
        }
        tc_fence_before();
      }
      __syncwarp();
      if (lane == 0 && ok) mbar_arrive(&ms.t2_empty[b]);
      if (p.amax_per_image) {
        const float mw = warp_max(mo);
        if (lane == 0) ms.red_e2[b][e] = mw;
        if (!bar_and(kBarE2, kE2Warps * 32, ok)) { *abort = 1; break; }
        if (e == 0 && lane == 0) {
          const float mi = fmaxf(fmaxf(ms.red_e2[b][0], ms.red_e2[b][1]), fmaxf(ms.red_e2[b][2], ms.red_e2[b][3]));
          if (mi > 0.0f) atomicMax(p.amax + img, __float_as_uint(mi));
        }
      } else {
        feat_amax = fmaxf(feat_amax, mo);
        if (!bar_and(kBarE2, kE2Warps * 32, ok)) { *abort = 1; break; }
      }
    }
    if (p.amax && !p.amax_per_image) {
      feat_amax = warp_max(feat_amax);
      if (lane == 0 && feat_amax > 0.0f) atomicMax(p.amax, __float_as_uint(feat_amax));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (tid == 0 && ms.abort) atomicExch(p.err, 1);
  if (warp == kWarpMma1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int C2, int ACT1, int ACT2>
void launch_cfg(const ConvBlockArgs& a, int num_sms, cudaStream_t st) {
  using L = Lay<C2>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_convblock<C2, ACT1, ACT2>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
    attr = true;
  }
  CBParams p;
  p.x = a.x; p.n = a.n; p.w1 = a.w1; p.kpad1 = a.kpad1; p.w2 = a.w2; p.kpad2 = a.kpad2;
  p.w1_scale = a.w1_scale; p.w2_scale = a.w2_scale; p.b1 = a.b1; p.b2 = a.b2; p.p1 = a.p1; p.p2 = a.p2;
  p.out = a.out; p.amax = a.amax; p.amax_per_image = a.amax_per_image;
  p.err = a.err;
  p.out_q = a.out_q; p.q_scale = a.q_scale;
  const int grid = (int)(a.n < num_sms ? a.n : num_sms);
  k_convblock<C2, ACT1, ACT2><<<grid, kThreads, L::SMEM, st>>>(p);
}

template <int C2>
void launch_c2(const ConvBlockArgs& a, int num_sms, cudaStream_t st) {
  const int k = a.act1 * 8 + a.act2;
  switch (k) {
    case ACT_RELU * 8 + ACT_RELU: launch_cfg<C2, ACT_RELU, ACT_RELU>(a, num_sms, st); break;
    case ACT_NONE * 8 + ACT_NONE: launch_cfg<C2, ACT_NONE, ACT_NONE>(a, num_sms, st); break;
    case ACT_RELU * 8 + ACT_NONE: launch_cfg<C2, ACT_RELU, ACT_NONE>(a, num_sms, st); break;
    case ACT_NONE * 8 + ACT_RELU: launch_cfg<C2, ACT_NONE, ACT_RELU>(a, num_sms, st); break;
    default: launch_cfg<C2, ACT_LEAKY_RELU, ACT_LEAKY_RELU>(a, num_sms, st); break;
  }
}

}  // namespace

// Shapes and activations with an instantiated kernel: 28x28 single-channel images,
// 16 channels after the first conv, 16 or 32 after the second; ReLU / none, or
// LeakyReLU (slope >= 0) on both convs.
bool convblock_supported(int c0, int c1, int c2, int h, int w, int act1, int act2) {
  if (c0 != 1 || c1 != C1 || h != H || w != W || (c2 != 16 && c2 != 32)) return false;
  auto simple = [](int a) { return a == ACT_NONE || a == ACT_RELU; };
  return (simple(act1) && simple(act2)) || (act1 == ACT_LEAKY_RELU && act2 == ACT_LEAKY_RELU);
}

void launch_convblock(const ConvBlockArgs& a, int num_sms, cudaStream_t st) {
  if (a.n <= 0 || !a.err) return;
  if (a.c2 == 32) launch_c2<32>(a, num_sms, st);
  else launch_c2<16>(a, num_sms, st);
}

}  // namespace rg
