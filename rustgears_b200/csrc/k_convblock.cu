// k_convblock.cu -- one kernel for the CNN block
//   FusedConv2d(1->16, k3 s1 p1, act) -> MaxPool2d(2,2) -> FusedConv2d(16->C2, k3 s1 p1, act) -> MaxPool2d(2,2)
// on 28x28 images, every intermediate of an image kept in shared memory.
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
//          a window land in one TMEM lane, 4 column blocks apart: the window max is
//          3 register max ops per channel;
//   conv2: no im2col at all.  With 16 channels (16 bytes) per pixel, the operand rows
//          of one tap are consecutive pixels of the padded 16-wide NHWC map, so each
//          MMA K step (two taps) reads the quantized map in place: rows 16 B apart
//          (SBO = 128), the second tap LBO bytes after the first.  Output rows are
//          pixels on the 16-wide grid (columns 14, 15 computed and dropped); a 2x2
//          window is lanes {x, x^1, x^16, x^17} of one warp.
#include <cuda_runtime.h>

#include "rg_kernels.h"
#include "rg_math.cuh"
#include "rg_sm100.cuh"

namespace rg {
namespace {

using namespace sm100;

constexpr int kThreads = 256;
constexpr int H = 28, W = 28, C1 = 16;
constexpr int P1 = 14;                 // pooled conv1 map is 14 x 14
constexpr int WP = 16;                 // padded width of that map (14 + 2)
constexpr int P2 = 7;                  // pooled conv2 map is 7 x 7
constexpr int Rows1 = H * W;           // 784 conv1 output pixels
constexpr int MT1 = 8;                 // conv1 tiles: 2 groups of 128 windows x 4 window positions
constexpr int MT2 = 2;                 // conv2 rows: 16 output rows x 16 = 256
constexpr int Q1W = 32;                // padded conv1 input row pitch (bytes)
constexpr int SBO1 = 256;              // conv1 tile: 2 chunks x 128 B per 8-row group

__host__ __device__ constexpr int rup(int v, int m) { return (v + m - 1) / m * m; }

template <int C2>
struct Lay {
  static constexpr int K2P = 160, CH2 = 10, SBO2W = CH2 * 128;  // W2 tile: 10 chunks per 8-row group
  static constexpr int OFF_Q1 = 0;                              // i8 [30][32] (+1 spare word row)
  static constexpr int OFF_A1 = OFF_Q1 + 1024;                  // conv1 im2col: 8 x 128 rows x 32 B
  static constexpr int OFF_W1 = OFF_A1 + MT1 * 128 * 32;        // W1: 16 rows x 32 B
  static constexpr int OFF_P1 = OFF_W1 + C1 * 32;               // f32 [196][16] pooled conv1
  static constexpr int OFF_Q2 = OFF_P1 + P1 * P1 * C1 * 4;      // i8 [19][16][16] padded NHWC
  static constexpr int OFF_W2 = OFF_Q2 + 19 * WP * C1;          // W2: C2 rows x 160 B
  static constexpr int OFF_MISC = OFF_W2 + C2 * K2P;
  static constexpr int SMEM = OFF_MISC + 128;
  static constexpr int TMEM_COLS = 128;  // conv1: 8 x 16 columns; conv2 reuses 0..2*C2
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

// 2x2 window of 16 accumulator columns held by lanes {l, l^m1, l^m2, l^(m1|m2)}; every lane
// of the window ends with the 4 channels c0 + s + 4k (k = 0..3, s = this lane's slot).
template <int ACT, int M1, int M2>
__device__ __forceinline__ void window4(const uint32_t (&acc)[16], bool fast, float cs, const float* bias, int c0,
                                        float p, int slot, float (&out)[4]) {
  const int lane = threadIdx.x & 31;
  if (fast) {
    int32_t m[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      int32_t v = (int32_t)acc[j];
      v = max(v, __shfl_xor_sync(0xffffffffu, v, M1));
      v = max(v, __shfl_xor_sync(0xffffffffu, v, M2));
      m[j] = v;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int32_t a = slot == 0 ? m[4 * k] : slot == 1 ? m[4 * k + 1] : slot == 2 ? m[4 * k + 2] : m[4 * k + 3];
      out[k] = epi<ACT>(a, cs, __ldg(bias + c0 + 4 * k + slot), p);
    }
  } else {
    // reference order: epilogue per pixel, then max over the window in (dy, dx) order
    const int base = lane & ~(M1 | M2);
    float best[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float v = epi<ACT>((int32_t)acc[j], cs, __ldg(bias + c0 + j), p);
      float b = -INFINITY;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int src = base | ((q >> 1) ? M2 : 0) | ((q & 1) ? M1 : 0);
        const float vq = __shfl_sync(0xffffffffu, v, src);
        if (vq > b || vq != vq) b = vq;
      }
      best[j] = b;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k)
      out[k] = slot == 0 ? best[4 * k] : slot == 1 ? best[4 * k + 1] : slot == 2 ? best[4 * k + 2] : best[4 * k + 3];
  }
}

template <int C2, int ACT1, int ACT2>
__global__ void __launch_bounds__(kThreads, 3) k_convblock(const CBParams p) {
  using L = Lay<C2>;
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* q1 = sm + L::OFF_Q1;
  uint8_t* a1 = sm + L::OFF_A1;
  uint8_t* w1s = sm + L::OFF_W1;
  float* p1s = reinterpret_cast<float*>(sm + L::OFF_P1);
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
  for (int i = tid; i < C2 * 144; i += kThreads) {  // W2 bytes (ky, kx, c); bytes 144..159 stay zero
    const int n = i / 144, b = i % 144;
    w2s[canon(n, b >> 4, L::SBO2W) + (b & 15)] = (uint8_t)p.w2[(int64_t)n * p.kpad2 + b];
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
    mbar_wait_sleep(bar, phase, 4000000000ull);
    phase ^= 1;
    tc_fence_after();
    // ---- 4. conv1 epilogue: lane = pool window, max over the 4 position tiles ----------
    const bool fast1 = isfinite(cs1);
    float m2 = 0.0f;
    {
      const int g = warp >> 2, w = 128 * g + 32 * q + lane;  // this lane's pool window
      const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
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
      if (w < P1 * P1) {
        float4* dst = reinterpret_cast<float4*>(p1s + w * C1);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          dst[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
          m2 = fmaxf(m2, fmaxf(fmaxf(fabsf(v[4 * k]), fabsf(v[4 * k + 1])), fmaxf(fabsf(v[4 * k + 2]), fabsf(v[4 * k + 3]))));
        }
      }
    }
    tc_fence_before();
    const float s2 = quant_scale(block_max(m2, red, tid)), inv2 = quant_inv(s2);
    const float cs2 = __fmul_rn(s2, p.w2_scale);
    // ---- 5. requantize into the padded 16-wide NHWC map (4 channels per thread step) -----
    for (int i = tid; i < P1 * P1 * (C1 / 4); i += kThreads) {
      const int w = i >> 2, c4 = i & 3, py = w / P1, px = w % P1;
      const float4 f = *reinterpret_cast<const float4*>(p1s + w * C1 + c4 * 4);
      const uint32_t word = (uint32_t)(quant1(f.x, inv2) & 0xff) | ((uint32_t)(quant1(f.y, inv2) & 0xff) << 8) |
                            ((uint32_t)(quant1(f.z, inv2) & 0xff) << 16) | ((uint32_t)(quant1(f.w, inv2) & 0xff) << 24);
      *reinterpret_cast<uint32_t*>(q2 + ((py + 1) * WP + (px + 1)) * C1 + c4 * 4) = word;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    // ---- 6. conv2 straight from the map: 2 M-tiles x 5 K steps (tap pairs) ---------------
    if (tid == 0) {
      tc_fence_after();
      const uint32_t q2a = smem_addr(q2), w2a = smem_addr(w2s);
#pragma unroll
      for (int t = 0; t < MT2; ++t)
#pragma unroll
        for (int s = 0; s < 5; ++s) {
          const int ta = 2 * s, tb = 2 * s + 1;  // tap 9 (s = 4) meets zero weights
          const uint32_t off_a = (uint32_t)(((8 * t + ta / 3) * WP + ta % 3) * C1);
          const uint32_t off_b = tb < 9 ? (uint32_t)(((8 * t + tb / 3) * WP + tb % 3) * C1) : off_a + 16u;
          mma_i8(tmem + (uint32_t)(t * C2), desc_noswz(q2a + off_a, off_b - off_a, 128),
                 desc_noswz(w2a + s * 256, 128, L::SBO2W), idesc2, s > 0);
        }
      mma_commit(bar);
    }
    mbar_wait_sleep(bar, phase, 4000000000ull);
    phase ^= 1;
    tc_fence_after();
    // ---- 7. conv2 epilogue: window = lanes {x, x^1, x^16, x^17}, features to global -----
    const bool fast2 = isfinite(cs2);
    {
      const int t = warp >> 2;
      const int py = 4 * t + q;            // pooled row of this warp
      const int px = (lane & 15) >> 1;     // pooled column of this lane's window
      const int slot = (lane & 1) | ((lane >> 4) << 1);
      const bool ok = py < P2 && px < P2;
      float* og = p.out + img * (int64_t)(C2 * P2 * P2) + py * P2 + px;
      float mo = 0.0f;
#pragma unroll 1
      for (int c0 = 0; c0 < C2; c0 += 16) {
        uint32_t acc[16];
        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(t * C2 + c0), acc);
        tmem_ld_wait();
        float v[4];
        window4<ACT2, 1, 16>(acc, fast2, cs2, p.b2, c0, p.p2, slot, v);
        if (ok) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            og[(c0 + 4 * k + slot) * (P2 * P2)] = v[k];
            mo = fmaxf(mo, fabsf(v[k]));
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

void launch_convblock(const ConvBlockArgs& a, int num_sms, cudaStream_t st) {
  if (a.n <= 0) return;
  if (a.c2 == 32) launch_c2<32>(a, num_sms, st);
  else launch_c2<16>(a, num_sms, st);
}

}  // namespace rg
