// rg_kernels.h -- launchers of the device kernels (internal to librg_npu.so).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/rg_npu.h"

namespace rg {

// Sets the calling thread's rg_last_error() message; returns st.
rg_status set_last_error(rg_status st, const char* msg);

// Where the absmax of an op's output goes (the next quantizing op's input scale).
struct AmaxSink {
  unsigned* ptr = nullptr;   // float bits of max|x| (non-negative floats order like uints)
  int64_t elems_per_slot = 0;  // 0: one slot for the whole tensor; else slot = elem / elems_per_slot
};

// ---- quantization (k_quant.cu) ------------------------------------------------
// amax_bits[0] = max |x| (NaN ignored). Caller zeroes amax_bits first.
void launch_absmax(const float* x, int64_t n, unsigned* amax_bits, cudaStream_t st);
// x [rows,k] f32 -> q [rows,ldq] i8 with the per-tensor scale from amax_bits; scale_out[0] = scale.
void launch_quantize_rows(const float* x, int64_t rows, int64_t k, int64_t ldq,
                          const unsigned* amax_bits, int8_t* q, float* scale_out, cudaStream_t st);
// The same with a given (calibrated) scale *scale; values beyond its range clamp to +-127.
void launch_quantize_rows_frozen(const float* x, int64_t rows, int64_t k, int64_t ldq, const float* scale, int8_t* q,
                                 cudaStream_t st);
// Per-image absmax over the pixels a conv actually reads (row/col coverage masks; NULL = all).
void launch_image_absmax(const float* x, int64_t n, int32_t c, int32_t h, int32_t w,
                         const uint8_t* row_cov, const uint8_t* col_cov, unsigned* amax_bits,
                         cudaStream_t st);
// NCHW f32 -> NHWC i8 (channels padded to cpad with zeros) with per-image scales.
// bounded: the scale's absmax covers every element quantized (no strided-conv coverage
// mask), so the clamp to +-127 can be left out.
void launch_image_quantize_nhwc(const float* x, int64_t n, int32_t c, int32_t h, int32_t w,
                                int32_t cpad, bool bounded, const unsigned* amax_bits, int8_t* q,
                                float* scales_out, cudaStream_t st);
// The same scale, written as 16-channel chunk planes [n][cpad / 16][h * w][16] (cpad a
// multiple of 16, n <= 65535): the input layout of the direct 3x3 conv.
void launch_image_quantize_planar16(const float* x, int64_t n, int32_t c, int32_t h, int32_t w, int32_t cpad,
                                    bool bounded, const unsigned* amax_bits, int8_t* q, float* scales_out,
                                    cudaStream_t st);
// NCHW f32 (c <= 4, even h, w) -> space-to-depth i8 pixels [n][h/2][w/2][16 B] (byte
// (dy * 2 + dx) * 4 + ch), per-image scales: the input layout of the fused stem.
void launch_image_quantize_s2d(const float* x, int64_t n, int32_t c, int32_t h, int32_t w, const unsigned* amax_bits,
                               int8_t* q, float* scales_out, cudaStream_t st);
// The pixels a 1x1 / pad 0 / stride s conv reads, (s * oy, s * ox) for oy < oh, ox < ow,
// quantized with the per-image scale of their own absmax into a compact NHWC operand
// [n][oh][ow][cpad] (cpad a multiple of 16, n <= 65535): the conv becomes a 1x1
// stride-1 conv over it.
void launch_image_quantize_subsampled(const float* x, int64_t n, int32_t c, int32_t h, int32_t w, int32_t s,
                                      int32_t oh, int32_t ow, int32_t cpad, bool planar, const unsigned* amax_bits,
                                      int8_t* q, float* scales_out, cudaStream_t st);
// NCHW f32 -> the space-to-depth operand of a 3x3 / stride 2 / pad 1 conv as 16-channel
// chunk planes [n][4 cpad / 16][ceil(h / 2)][ceil(w / 2)][16 B]: channel (dy * 2 + dx) *
// cpad + c of s2d pixel (sy, sx) = channel c of pixel (2 sy + dy, 2 sx + dx), zero for
// c >= c_in and past an odd h or w.
void launch_image_quantize_s2d_planar(const float* x, int64_t n, int32_t c, int32_t h, int32_t w, int32_t cpad,
                                      const unsigned* amax_bits, int8_t* q, float* scales_out, cudaStream_t st);
// NHWC i8 (cpad) -> NCHW i8 (c) for traces.
void launch_nhwc_to_nchw_i8(const int8_t* q, int64_t n, int32_t c, int32_t cpad, int32_t h,
                            int32_t w, int8_t* out, cudaStream_t st);

// ---- GEMM (k_gemm_simt.cu, k_gemm_tc.cu) ---------------------------------------
struct ConvGeom {      // implicit-GEMM A operand: rows = (img, oy, ox), k = (ky, kx, c)
  int32_t h = 0, w = 0, c = 0, cpad = 0, k = 0, stride = 1, pad = 0, oh = 0, ow = 0;
  int32_t kxp = 0;     // taps per kernel row in the K order (0: k); narrow operands (cpad 4)
                       // pad it to a multiple of 4 so that a 16-byte K chunk is 4 taps
};

struct GemmArgs {
  // A: dense i8 [m, lda] (conv == false) or gathered from NHWC i8 (conv == true)
  const int8_t* a = nullptr;
  int64_t lda = 0;
  // ... or f32 [m, af_k] row-major, quantized while it is loaded with the per-tensor
  // scale of absmax *af_amax (kernels that support it; a and a_scale are then unused)
  const float* af = nullptr;
  int64_t af_k = 0;
  const unsigned* af_amax = nullptr;
  // ... or with a given (calibrated) scale *af_scale, values beyond its range clamping
  const float* af_scale = nullptr;
  bool conv = false;
  ConvGeom g;
  // B: weights [n, ldb] i8, K-contiguous (ldb multiple of 16, zero-padded)
  const int8_t* w = nullptr;
  int64_t ldb = 0;
  int64_t m = 0, n = 0, k = 0;   // k = padded reduction length (multiple of 16)
  // epilogue
  const float* a_scale = nullptr;  // device; index = row / rows_per_scale
  int64_t rows_per_scale = 0;      // 0: one scale for all rows
  float w_scale = 1.0f;
  const float* w_scale_ch = nullptr;  // per-output-channel weight scales (extension), or NULL
  const float* bias = nullptr;
  int32_t act = 0;
  float act_param = 0.0f;
  float* out = nullptr;
  int64_t out_l = 0;               // 0: row-major [m,n]; L>0: NCHW out[(r/L)*n*L + c*L + r%L]
  int32_t* acc = nullptr;          // optional i32 dump, same layout as out
  AmaxSink amax;                   // optional absmax of out
  // tcgen05 conv only: out = res_act(epilogue + residual), residual in out's layout
  // (a residual block's closing add fused into the conv before it)
  const float* residual = nullptr;
  int32_t res_act = 0;
  float res_param = 0.0f;
  // direct 3x3 conv only: a second per-image absmax of out over the pixels a later
  // 1x1 / pad 0 / stride cov_s conv reads (rows and columns cov_s * i, i < cov_oh / cov_ow)
  unsigned* amax2 = nullptr;
  int32_t cov_s = 1, cov_oh = 0, cov_ow = 0;
  // tensor-core kernels: this call's device error word (required; set to 1 when a
  // bounded wait gave up) and the limit of their pipeline waits (0: the default)
  int* err = nullptr;
  uint64_t wait_ns = 0;
  int32_t starve = 0;  // test hook (k_gemm_tc): issue no operand loads, so the waits run out
};

// FP16 arm (fp16_gemm_fused_into, npu.rs:431-445) on the CUDA cores: out =
// act(round_fp16(sum_k round_fp16(a) * w + bias)) with the sum in k order, bit-exact.
struct Fp16Args {
  const float* x = nullptr;     // Linear: [m, k] row-major; conv: NCHW input
  const float* wt = nullptr;    // weights [n, k] row-major (reference layout; conv k = (c, ky, kx))
  const float* bias = nullptr;  // [n]
  float* out = nullptr;         // Linear: [m, n]; conv: NCHW
  int64_t m = 0, n = 0, k = 0;  // conv: m = images * oh * ow
  int32_t act = 0;
  float act_param = 0.0f;
  int32_t exact = 1;            // every weight is an fp16 value (FMA chain is exact)
  int32_t f32 = 0;              // the f32 arm instead (ExecutionProvider::Cpu, run_standard): no
                                // rounding, FMA chains except past the matmul's last full
                                // 8-wide column block, out = acc + bias
  int32_t conv = 0, c = 0, h = 0, w = 0, ks = 0, stride = 1, pad = 0, oh = 0, ow = 0;
  // FP16 conv only: the MaxPool2d(2, 2) that follows, fused (out is then the pooled
  // [images, n, ph, pw] map and m = images * ph * pw * 4)
  int32_t pool = 0, ph = 0, pw = 0;
};
// false: a conv whose reduction (C k k > 16384) or geometry the kernel does not take
bool launch_fp16_gemm(const Fp16Args& a, cudaStream_t st);
// ChannelAffine of the f32 arm: y = x * scale[ch] + shift[ch], ch = (i / inner) % c.
void launch_channel_affine(const float* x, int64_t total, int64_t c, int64_t inner, const float* scale,
                           const float* shift, float* y, cudaStream_t st);

void launch_gemm_simt(const GemmArgs& a, cudaStream_t st);
// Narrow dense GEMM (N <= 32) on the CUDA cores: one thread per output row; takes an
// i8 A, or an f32 A (af) that it quantizes on the fly.
bool gemm_narrow_eligible(const GemmArgs& a);
void launch_gemm_narrow(const GemmArgs& a, cudaStream_t st);
// tcgen05 path.  eligible(): shape/alignment/driver checks.  launch() returns false
// when the TMA descriptors could not be encoded (nothing was launched).
bool gemm_tc_eligible(const GemmArgs& a);
bool launch_gemm_tc(const GemmArgs& a, int num_sms, cudaStream_t st);
// tcgen05 implicit-GEMM conv (A gathered from the NHWC i8 operand, channels padded to
// a multiple of 16, g.c == g.cpad; NCHW output, per-image scales).
bool conv_tc_eligible(const GemmArgs& a);
bool launch_conv_tc(const GemmArgs& a, int num_sms, cudaStream_t st);
// 3x3 / stride 1 / pad 1 convs (channels padded to a multiple of 64) as a direct
// convolution over zero-padded TMA input tiles of the chunk-planar operand
// (launch_image_quantize_planar16); weights pre-arranged by
// conv3x3_arrange_weights into conv3x3_weight_bytes(n, cpad) bytes.  launch() returns
// false when the tensor map could not be encoded (nothing was launched).
bool conv3x3_eligible(const GemmArgs& a);
// The same kernel over other tap sets (the operand: 16-channel chunk planes of an h x w
// grid equal to the output grid, cpad a multiple of 64):
//   DCONV_3X3  3x3 / stride 1 / pad 1;
//   DCONV_S2D  3x3 / stride 2 / pad 1 over the space-to-depth operand
//              (launch_image_quantize_s2d_planar, 4 x the conv's channels): 2x2 taps;
//   DCONV_1X1  1x1 over the operand (a strided 1x1 conv's compact operand,
//              launch_image_quantize_subsampled with planar output).
enum { DCONV_3X3 = 0, DCONV_S2D = 1, DCONV_1X1 = 2 };
bool dconv_shape_ok(int mode, int64_t n_img, int32_t h, int32_t w, int32_t cpad, int32_t out_channels);
bool dconv_eligible(const GemmArgs& a, int mode, int32_t h, int32_t w, int32_t cpad);
// weights [n][c][k][k] quantized; cpad = the conv's padded channel count (the s2d operand has 4 x cpad)
size_t dconv_weight_bytes(int mode, int32_t n, int32_t cpad);
void dconv_arrange_weights(int mode, const int8_t* wq, int32_t n, int32_t c, int32_t k, int32_t cpad, int8_t* out);
bool launch_dconv(const GemmArgs& a, int mode, int32_t h, int32_t w, int32_t cpad, const int8_t* wd, int num_sms,
                  cudaStream_t st);
// The shape test of conv3x3_eligible, before the operand is quantized (which layout).
bool conv3x3_shape_ok(int64_t n_img, int32_t h, int32_t w, int32_t cpad, int32_t k, int32_t stride, int32_t pad,
                      int32_t out_channels);
size_t conv3x3_weight_bytes(int32_t n, int32_t cpad);
void conv3x3_arrange_weights(const int8_t* wq, int32_t n, int32_t c, int32_t cpad, int8_t* out);
bool launch_conv3x3(const GemmArgs& a, const int8_t* wd, int num_sms, cudaStream_t st);

// ---- fused stem (k_stem.cu) ------------------------------------------------------
// Conv2d(c <= 4 -> 64, k 7, s 2, p 3) + act, then MaxPool2d(3, 2), one kernel over the
// space-to-depth operand (launch_image_quantize_s2d); weights pre-arranged by
// stem_arrange_weights into stem_weight_bytes() bytes.  Output NCHW [n, 64, ph, pw].
struct StemPoolArgs {
  const int8_t* q = nullptr;       // s2d operand
  int64_t n = 0;
  int32_t h = 0, w = 0;            // conv input size (even)
  const int8_t* wd = nullptr;
  const float* a_scale = nullptr;  // per image
  float w_scale = 1.0f;
  const float* w_scale_ch = nullptr;
  const float* bias = nullptr;
  int32_t act = 0;
  float act_param = 0.0f;
  float* out = nullptr;
  AmaxSink amax;                   // of the pooled output
  int* err = nullptr;              // this call's error word (required)
};
bool stem_pool_shape_ok(int64_t n_img, int32_t c, int32_t h, int32_t w, int32_t k, int32_t stride, int32_t pad,
                        int32_t out_channels, int32_t pool_k, int32_t pool_s);
size_t stem_weight_bytes();
void stem_arrange_weights(const int8_t* wq, int32_t c, int8_t* out);
bool launch_stem_pool(const StemPoolArgs& a, int num_sms, cudaStream_t st);

// ---- fused CNN block (k_convblock.cu) ------------------------------------------
// Conv(C0->C1,k3,s1,p1)+act -> MaxPool(2,2) -> Conv(C1->C2,k3,s1,p1)+act -> MaxPool(2,2),
// per-image quantization of each conv input, all intermediates in shared memory.
// A program of two INT8 Linears, both narrow (k1 <= 64 inputs, n1 and n2 <= 32 outputs,
// per-tensor weights), in one cooperative launch (k_mlp2.cu): input absmax, the first
// Linear with the hidden row in registers and the hidden absmax, the second Linear.
struct Mlp2Args {
  const float* x = nullptr;  // [m, k1]
  int64_t m = 0;
  int32_t k1 = 0, kpad1 = 0, n1 = 0, kpad2 = 0, n2 = 0;
  const int8_t* w1 = nullptr;  // [n1, kpad1]
  const int8_t* w2 = nullptr;  // [n2, kpad2]
  float w1_scale = 1.0f, w2_scale = 1.0f;
  const float* b1 = nullptr;
  const float* b2 = nullptr;
  int32_t act1 = 0, act2 = 0;
  float p1 = 0.0f, p2 = 0.0f;
  float* y = nullptr;        // [m, n2]
  unsigned* amax = nullptr;  // optional absmax sink of y
  unsigned* amax1 = nullptr;  // absmax of x, then of the hidden rows (float bits; zeroed by the caller)
  unsigned* amax2 = nullptr;
  int* err = nullptr;        // this call's error word (a barrier wait gave up)
};
bool mlp2_eligible(const Mlp2Args& a);
// false (nothing launched) when the rows exceed one per resident thread or the
// cooperative launch is refused; ws: 4 words of device scratch owned by the caller
bool launch_mlp2(const Mlp2Args& a, unsigned* ws, cudaStream_t st);

struct ConvBlockArgs {
  const float* x = nullptr;          // [n, c0, h, w] f32
  int64_t n = 0;
  int32_t c0 = 0, c1 = 0, c2 = 0, h = 0, w = 0;
  const int8_t* w1 = nullptr;        // [c1, kpad1], reduction order (ky, kx, c)
  int32_t kpad1 = 0;
  const int8_t* w2 = nullptr;        // [c2, kpad2]
  int32_t kpad2 = 0;
  float w1_scale = 1.0f, w2_scale = 1.0f;
  const float* b1 = nullptr;
  const float* b2 = nullptr;
  int32_t act1 = 0, act2 = 0;        // non-decreasing activations only (see convblock_supported)
  float p1 = 0.0f, p2 = 0.0f;
  float* out = nullptr;              // [n, c2, h/4, w/4]
  unsigned* amax = nullptr;          // optional absmax sink of out
  int64_t amax_per_image = 0;
  int* err = nullptr;                // this call's error word (required)
  // calibration extension: out_q non-null writes the output quantized with the frozen
  // scale *q_scale as i8 [n, c2 * (h/4) * (w/4)] instead of the f32 out
  int8_t* out_q = nullptr;
  const float* q_scale = nullptr;
};
bool convblock_supported(int c0, int c1, int c2, int h, int w, int act1, int act2);
void launch_convblock(const ConvBlockArgs& a, int num_sms, cudaStream_t st);

// ---- misc (k_misc.cu) ----------------------------------------------------------
void launch_maxpool2d(const float* x, int64_t n, int32_t c, int32_t h, int32_t w, int32_t k,
                      int32_t s, float* y, AmaxSink amax, cudaStream_t st);
// Counts f32 inputs where a fast path changes a result, over all 2^32 bit patterns
// (zeroed first): counts[0] tanh, [1] GELU, [2] quant_scale, [3] quant_inv,
// [4] round_half_away, [5] tanh_f32_common / GELU through it on its range.
void launch_selftest_fast_division(unsigned long long* counts, cudaStream_t st);
// Extensions: y = act(x + s) elementwise; adaptive average pooling to oh x ow.
void launch_residual_add(const float* x, const float* s, int64_t n, int32_t act, float p, float* y,
                         AmaxSink amax, cudaStream_t st);
void launch_adaptive_avgpool(const float* x, int64_t n, int32_t c, int32_t h, int32_t w, int32_t oh, int32_t ow,
                             float* y, AmaxSink amax, cudaStream_t st);
void launch_activation(const float* x, int64_t n, int32_t act, float p, float* y, AmaxSink amax,
                       cudaStream_t st);
void launch_softmax(const float* x, int64_t outer, int64_t last, float* y, AmaxSink amax,
                    cudaStream_t st);
// Transformer extension (k_transformer.cu).  Token ids are f32 values; an id >= v sets
// the caller's device error word *err to 1.
void launch_embedding(const float* ids, int64_t n, const float* table, int64_t v, int32_t d, float* y,
                      AmaxSink amax, int* err, cudaStream_t st);
// yq non-null (calibration extension): the output is written quantized with the frozen
// scale *q_scale into i8 rows of ldq bytes (zero-padded) instead of y.
rg_status launch_rmsnorm(const float* x, int64_t rows, int32_t d, const float* w, float eps, float inv_d, float* y,
                         AmaxSink amax, cudaStream_t st, int8_t* yq = nullptr, int64_t ldq = 0,
                         const float* q_scale = nullptr);
// gu [rows, 2h] = [g | u] -> y [rows, h] = (g * sigmoid(g)) * u (or yq, as for RMSNorm)
void launch_swiglu_mul(const float* gu, int64_t rows, int32_t h, float* y, AmaxSink amax, cudaStream_t st,
                       int8_t* yq = nullptr, int64_t ldq = 0, const float* q_scale = nullptr);
// qkv [b*t, ld] (q, k, v of head hh at columns hh*dh, d + hh*dh, 2d + hh*dh) ->
// out [b*t, ldo] with the heads merged; scores scaled by `scale` before the softmax.
rg_status launch_attention(const float* qkv, int64_t ld, int64_t b, int32_t t, int32_t heads, int32_t dh,
                           float scale, float* out, int64_t ldo, AmaxSink amax, cudaStream_t st);
bool attention_fast_eligible(int32_t t, int32_t dh, const float* qkv, int64_t ld, const float* out, int64_t ldo);
void launch_fill_u32(unsigned* p, unsigned v, int64_t n, cudaStream_t st);
void launch_bits_to_float(const unsigned* bits, float* out, int64_t n, cudaStream_t st);

}  // namespace rg
