// k_convblock.cu -- one kernel for the CNN block
//   FusedConv2d(1->16, k3 s1 p1, act) -> MaxPool2d(2,2) -> FusedConv2d(16->C2, k3 s1 p1, act) -> MaxPool2d(2,2)
// on 28x28 images, every intermediate of an image kept in shared memory or registers.
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
// Tensor-core operands (tcgen05.mma kind::i8, K-major, no swizzle: 8-row x 16-byte
// core matrices, SBO between 8-row groups, LBO between the two 16-byte K halves):
//   conv1: an im2col tile built per image, K packed as 4*ky + kx (three 4-byte runs of
//          the padded input row, 12 of 32 bytes used).  Tile (g, pos) holds window
//          position pos = dy*2 + dx of pool windows 128g..128g+127, so the 4 pixels of
//          a window land in one TMEM lane, 4 column blocks apart.
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

__device__ int g_cb_error;  // set when an MMA-completion wait gave up (read by the host)

constexpr int kThreads = 256;
constexpr int H = 28, W = 28, C1 = 16;
constexpr int P1 = 14;                 // pooled conv1 map is 14 x 14 (16 x 16 padded)
constexpr int P2 = 7;                  // pooled conv2 map is 7 x 7
constexpr int Rows1 = H * W;           // 784 conv1 output pixels
constexpr int MT1 = 8;                 // conv1 tiles: 2 groups of 128 windows x 4 window positions
constexpr int Q1W = 32;                // padded conv1 input row pitch (bytes)
constexpr int SBO1 = 256;              // conv1 tile: 2 chunks x 128 B per 8-row group
constexpr int Q2ROW = 256;             // conv2 map row: 16 pixels x 16 B (even half, odd half)

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
  static constexpr int K2P = 160, SBO2W = 10 * 128;            // W2 tile: 10 chunks per 8-row group
  static constexpr int OFF_Q1 = 0;                              // i8 [30][32] (+1 spare word row)
  static constexpr int OFF_A1 = OFF_Q1 + 1024;                  // conv1 im2col: 8 x 128 rows x 32 B
  static constexpr int OFF_W1 = OFF_A1 + MT1 * 128 * 32;        // W1: 16 rows x 32 B
  static constexpr int OFF_Q2 = OFF_W1 + C1 * 32;               // i8 [19 rows][256 B], interleaved
  static constexpr int OFF_W2 = OFF_Q2 + 19 * Q2ROW;            // W2 in the dx = 0 and dx = 1 tap orders
  static constexpr int OFF_MISC = OFF_W2 + 2 * C2 * K2P;
  static constexpr int SMEM = OFF_MISC + 128;
  static constexpr int TMEM_COLS = 128;  // conv1: 8 x 16 columns; conv2 reuses 0 .. 2*C2
};

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
};

__device__ __forceinline__ uint64_t desc_noswz(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version; layout type 0 = no swizzle
  return d;
}

__device__ __forceinline__ int canon(int r, int j, int sbo) { return (r & 7) * 16 + (r >> 3) * sbo + j * 128; }

__device__ __forceinline__ float block_max(float v, float* red, int tid) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((tid & 31) == 0) red[tid >> 5] = v;
  __syncthreads();
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) m = fmaxf(m, red[i]);
  return m;
}

template <int ACT>
__device__ __forceinline__ float epi(int32_t acc, float cs, float bias, float p) {
  const float v = __fadd_rn(__fmul_rn(__int2float_rn(acc), cs), bias);
  if (ACT == ACT_RELU) return fmaxf(v, 0.0f);
  if (ACT == ACT_LEAKY_RELU) return v > 0.0f ? v : __fmul_rn(p, v);
  return v;
}

__device__ __forceinline__ uint32_t pack4(float a, float b, float c, float d, float inv) {
  return (uint32_t)(quant1(a, inv) & 0xff) | ((uint32_t)(quant1(b, inv) & 0xff) << 8) |
         ((uint32_t)(quant1(c, inv) & 0xff) << 16) | ((uint32_t)(quant1(d, inv) & 0xff) << 24);
}

template <int C2, int ACT1, int ACT2>
__global__ void __launch_bounds__(kThreads, 3) k_convblock(const CBParams p) {
  using L = Lay<C2>;
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* q1 = sm + L::OFF_Q1;
  uint8_t* a1 = sm + L::OFF_A1;
  uint8_t* w1s = sm + L::OFF_W1;
  uint8_t* q2 = sm + L::OFF_Q2;
  uint8_t* w2s = sm + L::OFF_W2;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L::OFF_MISC);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L::OFF_MISC + 8);
  float* red = reinterpret_cast<float*>(sm + L::OFF_MISC + 16);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // ---- one-time set-up: zero the staging areas, stage weights in canonical layout ----
  for (int i = tid * 16; i < L::OFF_MISC; i += kThreads * 16) *reinterpret_cast<uint4*>(sm + i) = make_uint4(0, 0, 0, 0);
  __syncthreads();
  for (int i = tid; i < C1 * 12; i += kThreads) {  // W1 byte 4*ky + kx <- reference column 3*ky + kx
    const int n = i / 12, b = i % 12, ky = b >> 2, kx = b & 3;
    if (kx < 3) w1s[canon(n, 0, SBO1) + b] = (uint8_t)p.w1[(int64_t)n * p.kpad1 + 3 * ky + kx];
  }
  for (int i = tid; i < 2 * C2 * 144; i += kThreads) {  // W2 chunk k holds tap tap_order(dx, k); 144.. stay 0
    const int dx = i / (C2 * 144), rem = i % (C2 * 144), n = rem / 144, b = rem % 144;
    const int k = b >> 4, tap = tap_order(dx, k);
    w2s[dx * C2 * L::K2P + canon(n, k, L::SBO2W) + (b & 15)] =
        (uint8_t)p.w2[(int64_t)n * p.kpad2 + tap * 16 + (b & 15)];
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  uint32_t phase = 0;
  constexpr uint32_t idesc1 = idesc_i8(128, C1);
  constexpr uint32_t idesc2 = idesc_i8(128, C2);
  float feat_amax = 0.0f;
  const int q = warp & 3;  // TMEM lane quadrant of this warp
  const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);

  // Each thread < 196 owns 4 pixels of the image; the next image's pixels are fetched
  // while the current one is being processed.
  float4 v4_next = make_float4(0.f, 0.f, 0.f, 0.f);
  if (tid < H * W / 4 && (int64_t)blockIdx.x < p.n)
    v4_next = __ldg(reinterpret_cast<const float4*>(p.x + (int64_t)blockIdx.x * (H * W)) + tid);

  for (int64_t img = blockIdx.x; img < p.n; img += gridDim.x) {
    // ---- 1. image -> absmax -> scale -> padded i8 rows (pitch 32) ----------------------
    const float4 v4 = v4_next;
    float m = 0.0f;
    if (tid < H * W / 4) m = fmaxf(fmaxf(fabsf(v4.x), fabsf(v4.y)), fmaxf(fabsf(v4.z), fabsf(v4.w)));
    if (tid < H * W / 4 && img + gridDim.x < p.n)
      v4_next = __ldg(reinterpret_cast<const float4*>(p.x + (img + gridDim.x) * (int64_t)(H * W)) + tid);
    const float s1 = quant_scale(block_max(m, red, tid)), inv1 = quant_inv(s1);
    const float cs1 = __fmul_rn(s1, p.w1_scale);
    if (tid < H * W / 4) {
      const int y = (tid * 4) / W, x = (tid * 4) % W;
      uint8_t* dst = q1 + (y + 1) * Q1W + (x + 1);
      dst[0] = (uint8_t)quant1(v4.x, inv1);
      dst[1] = (uint8_t)quant1(v4.y, inv1);
      dst[2] = (uint8_t)quant1(v4.z, inv1);
      dst[3] = (uint8_t)quant1(v4.w, inv1);
    }
    __syncthreads();
    // ---- 2. conv1 im2col: pixel (window w, position pos) -> tile 4*(w/128) + pos, row w%128;
    //         bytes 4*ky + kx ------------------------------------------------------------
    const uint32_t* q1w = reinterpret_cast<const uint32_t*>(q1);
    for (int r = tid; r < Rows1; r += kThreads) {
      const int w = r >> 2, pos = r & 3;
      const int oy = 2 * (w / P1) + (pos >> 1), ox = 2 * (w % P1) + (pos & 1);
      const int row = (4 * (w >> 7) + pos) * 128 + (w & 127);
      uint32_t word[3];
#pragma unroll
      for (int ky = 0; ky < 3; ++ky) {
        const int byte = (oy + ky) * Q1W + ox;
        word[ky] = __funnelshift_r(q1w[byte >> 2], q1w[(byte >> 2) + 1], 8 * (byte & 3));
      }
      *reinterpret_cast<uint4*>(a1 + canon(row, 0, SBO1)) = make_uint4(word[0], word[1], word[2], 0u);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    // ---- 3. conv1: 8 MMAs 128 x 16 x 32 -------------------------------------------------
    if (tid == 0) {
      tc_fence_after();
      const uint32_t a1a = smem_addr(a1), w1a = smem_addr(w1s);
#pragma unroll
      for (int t = 0; t < MT1; ++t)
        mma_i8(tmem + (uint32_t)(t * C1), desc_noswz(a1a + t * 16 * SBO1, 128, SBO1), desc_noswz(w1a, 128, SBO1),
               idesc1, 0);
      mma_commit(bar);
    }
    if (!mbar_wait_sleep(bar, phase, 4000000000ull) && tid == 0) atomicExch(&g_cb_error, 1);
    phase ^= 1;
    tc_fence_after();
    // ---- 4. conv1 epilogue: lane = pool window, max over the 4 position tiles ----------
    const bool fast1 = isfinite(cs1);
    const int g = warp >> 2, win = 128 * g + 32 * q + lane;  // this lane's pool window
    float v[16];
    if (fast1) {
      int32_t mx[16];
      uint32_t acc[16];
      tmem_ld16(lane_base + (uint32_t)((4 * g) * C1), acc);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; ++j) mx[j] = (int32_t)acc[j];
#pragma unroll
      for (int pos = 1; pos < 4; ++pos) {
        tmem_ld16(lane_base + (uint32_t)((4 * g + pos) * C1), acc);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) mx[j] = max(mx[j], (int32_t)acc[j]);
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = epi<ACT1>(mx[j], cs1, __ldg(p.b1 + j), p.p1);
    } else {  // reference order: activation per pixel, NaN-propagating max in (dy, dx) order
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = -INFINITY;
#pragma unroll 1
      for (int pos = 0; pos < 4; ++pos) {
        uint32_t acc[16];
        tmem_ld16(lane_base + (uint32_t)((4 * g + pos) * C1), acc);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float e = epi<ACT1>((int32_t)acc[j], cs1, __ldg(p.b1 + j), p.p1);
          if (e > v[j] || e != e) v[j] = e;
        }
      }
    }
    const bool win_ok = win < P1 * P1;
    float m2 = 0.0f;
    if (win_ok)
#pragma unroll
      for (int j = 0; j < 16; ++j) m2 = fmaxf(m2, fabsf(v[j]));
    tc_fence_before();
    const float s2 = quant_scale(block_max(m2, red, tid)), inv2 = quant_inv(s2);
    const float cs2 = __fmul_rn(s2, p.w2_scale);
    // ---- 5. requantize from registers into the interleaved padded map: one 16-B store ---
    if (win_ok) {
      const int py = win / P1 + 1, px = win % P1 + 1;  // padded coordinates
      *reinterpret_cast<uint4*>(q2 + py * Q2ROW + (px & 1) * 128 + (px >> 1) * 16) =
          make_uint4(pack4(v[0], v[1], v[2], v[3], inv2), pack4(v[4], v[5], v[6], v[7], inv2),
                     pack4(v[8], v[9], v[10], v[11], inv2), pack4(v[12], v[13], v[14], v[15], inv2));
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    // ---- 6. conv2 straight from the map: 2 column parities x 5 K steps ------------------
    if (tid == 0) {
      tc_fence_after();
      const uint32_t q2a = smem_addr(q2), w2a = smem_addr(w2s);
#pragma unroll
      for (int dx = 0; dx < 2; ++dx)
#pragma unroll
        for (int s = 0; s < 5; ++s) {
          const uint32_t oa = (uint32_t)tap_offset(dx, tap_order(dx, 2 * s));
          const uint32_t ob = s < 4 ? (uint32_t)tap_offset(dx, tap_order(dx, 2 * s + 1)) : oa + 16u;  // zero weights
          mma_i8(tmem + (uint32_t)(dx * C2), desc_noswz(q2a + oa, ob - oa, Q2ROW),
                 desc_noswz(w2a + (uint32_t)(dx * C2 * L::K2P + s * 256), 128, L::SBO2W), idesc2, s > 0);
        }
      mma_commit(bar);
    }
    if (!mbar_wait_sleep(bar, phase, 4000000000ull) && tid == 0) atomicExch(&g_cb_error, 1);
    phase ^= 1;
    tc_fence_after();
    // ---- 7. conv2 epilogue: lane (y, j) = 8*y + j; window (y/2, j) = lanes l, l ^ 8 -----
    const bool fast2 = isfinite(cs2);
    {
      const int c0 = (warp >> 2) * 16;            // channel chunk of this warp
      const int y = 4 * q + (lane >> 3), j = lane & 7;
      const int py = y >> 1, half = y & 1;        // half: which 8 of the 16 channels this lane finishes
      const bool ok = c0 < C2 && py < P2 && j < P2;
      float mo = 0.0f;
      if (c0 < C2) {
        uint32_t a0[16], a1v[16];
        tmem_ld16(lane_base + (uint32_t)(c0), a0);
        tmem_ld16(lane_base + (uint32_t)(C2 + c0), a1v);
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
          for (int k = 0; k < 8; ++k)
            out[k] = epi<ACT2>(half ? mx[8 + k] : mx[k], cs2, __ldg(p.b2 + c0 + half * 8 + k), p.p2);
        } else {  // reference order (dy, dx): (y0,dx0), (y0,dx1), (y1,dx0), (y1,dx1)
          float best[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const float bk = __ldg(p.b2 + c0 + k);
            const float e0 = epi<ACT2>((int32_t)a0[k], cs2, bk, p.p2);
            const float e1 = epi<ACT2>((int32_t)a1v[k], cs2, bk, p.p2);
            const float f0 = __shfl_sync(0xffffffffu, e0, lane & ~8);
            const float f1 = __shfl_sync(0xffffffffu, e1, lane & ~8);
            const float f2 = __shfl_sync(0xffffffffu, e0, lane | 8);
            const float f3 = __shfl_sync(0xffffffffu, e1, lane | 8);
            float b = -INFINITY;
            if (f0 > b || f0 != f0) b = f0;
            if (f1 > b || f1 != f1) b = f1;
            if (f2 > b || f2 != f2) b = f2;
            if (f3 > b || f3 != f3) b = f3;
            best[k] = b;
          }
#pragma unroll
          for (int k = 0; k < 8; ++k) out[k] = half ? best[8 + k] : best[k];
        }
        if (ok) {
          float* og = p.out + img * (int64_t)(C2 * P2 * P2) + (int64_t)(c0 + half * 8) * (P2 * P2) + py * P2 + j;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            og[k * (P2 * P2)] = out[k];
            mo = fmaxf(mo, fabsf(out[k]));
          }
        }
      }
      if (p.amax_per_image) {
        const float mi = block_max(mo, red, tid);
        if (tid == 0 && mi > 0.0f) atomicMax(p.amax + img, __float_as_uint(mi));
      } else {
        feat_amax = fmaxf(feat_amax, mo);
      }
    }
    tc_fence_before();
    __syncthreads();
  }

  if (p.amax && !p.amax_per_image) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) feat_amax = fmaxf(feat_amax, __shfl_xor_sync(0xffffffffu, feat_amax, o));
    if (lane == 0 && feat_amax > 0.0f) atomicMax(p.amax, __float_as_uint(feat_amax));
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
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
  const int64_t want = 3LL * num_sms;
  const int grid = (int)(a.n < want ? a.n : want);
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

int convblock_take_error() {
  int h = 0, z = 0;
  if (cudaMemcpyFromSymbol(&h, g_cb_error, sizeof h) != cudaSuccess) return -1;
  if (h) cudaMemcpyToSymbol(g_cb_error, &z, sizeof z);
  return h;
}

void launch_convblock(const ConvBlockArgs& a, int num_sms, cudaStream_t st) {
  if (a.n <= 0) return;
  if (a.c2 == 32) launch_c2<32>(a, num_sms, st);
  else launch_c2<16>(a, num_sms, st);
}

}  // namespace rg
