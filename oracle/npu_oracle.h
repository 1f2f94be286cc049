/*
 * npu_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the RustGears Npu(Int8) inference path, used as the parity
 * checker for the CUDA execution provider and as the timed CPU baseline.  Nothing
 * in the product library links or calls this code.
 *
 * Every function cites the reference file:line it restates (paths relative to
 * the RustGears project root).  Parity status: the reference cannot be compiled
 * in this image (no Rust toolchain), so this restatement is pinned by the
 * reference's known answers (tests/integration.rs:128-164 structure,
 * docs/USAGE.md:376-380 byte and MAC counts) and by self-generated golden
 * vectors; see tests/golden/.
 */
#ifndef RG_NPU_ORACLE_H
#define RG_NPU_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- SplitMix64 generator: src/rng.rs:10-58 ---------------------------- */
typedef struct { uint64_t state; } og_rng;

void og_rng_seed(og_rng* r, uint64_t seed);                 /* rng.rs:16-18, manual_seed 71-73 */
uint64_t og_rng_next_u64(og_rng* r);                        /* rng.rs:21-27 */
float og_rng_uniform(og_rng* r);                            /* rng.rs:30-32 */
float og_rng_uniform_range(og_rng* r, float lo, float hi);  /* rng.rs:35-37 */
float og_rng_normal(og_rng* r);                             /* rng.rs:40-44 */
void og_fill_uniform_range(og_rng* r, float* out, int64_t n, float lo, float hi); /* tensor/mod.rs:128-131 */
void og_fill_normal(og_rng* r, float* out, int64_t n);      /* tensor/mod.rs:116-119 */
void og_fill_normal_scaled(og_rng* r, float* out, int64_t n, float std); /* nn/init.rs:18-20,30-32 */
void og_fill_below(og_rng* r, int64_t* out, int64_t n, uint64_t bound);  /* rng.rs:47-49 */
float og_kaiming_bound(int64_t fan_in);                     /* nn/init.rs:6-9 */
float og_bias_bound(int64_t fan_in);                        /* nn/init.rs:23-26 */

/* ---- IR: src/inference/mod.rs:24-100 ----------------------------------- */
enum {
  OG_LAYER_LINEAR = 1, OG_LAYER_CONV2D = 2, OG_LAYER_CHANNEL_AFFINE = 3,
  OG_LAYER_MAXPOOL2D = 4, OG_LAYER_FLATTEN = 5, OG_LAYER_ACTIVATION = 6,
  OG_LAYER_SOFTMAX = 7,
  /* extensions (see include/rg_npu.h): residual blocks, adaptive average pooling */
  OG_LAYER_RESIDUAL_BEGIN = 8, OG_LAYER_RESIDUAL_END = 9, OG_LAYER_SHORTCUT_CONV2D = 10,
  OG_LAYER_ADAPTIVE_AVGPOOL2D = 11,
  /* extensions for the transformer configuration (see include/rg_npu.h) */
  OG_LAYER_EMBEDDING = 12, OG_LAYER_RMSNORM = 13, OG_LAYER_ATTENTION = 14, OG_LAYER_SWIGLU = 15
};
enum { OG_ACT_NONE = 0, OG_ACT_RELU = 1, OG_ACT_SIGMOID = 2, OG_ACT_TANH = 3,
       OG_ACT_GELU = 4, OG_ACT_LEAKY_RELU = 5, OG_ACT_SILU = 6 /* extension */ };
enum { OG_PREC_INT8 = 0, OG_PREC_FP16 = 1 };

typedef struct {
  int32_t kind;
  int32_t in_features, out_features;                 /* Linear */
  int32_t in_channels, out_channels, kernel, stride, padding; /* Conv2d; MaxPool uses kernel/stride */
  const float* weight; int64_t weight_len;           /* Linear [in,out]; Conv [O,C,k,k]; Affine: scale */
  const float* bias; int64_t bias_len;               /* bias; Affine: shift */
  int32_t act; float act_param;                      /* Activation */
} og_layer;

/* Compiled program: src/inference/npu.rs:43-79 (NpuOp), 179-185 (NpuProgram). */
typedef struct og_op {
  int32_t kind;           /* OG_LAYER_LINEAR / CONV2D / MAXPOOL2D / FLATTEN / ACTIVATION / SOFTMAX */
  int32_t in_features, out_features;
  int32_t in_channels, out_channels, kernel, stride, padding;
  int8_t* wq; int64_t wq_len; float w_scale;   /* Linear: [out,in]; Conv: [O, C*k*k] */
  float* bias; int64_t bias_len;
  int32_t act; float act_param;
  /* extensions: the INT8 Linears inside an attention block (q, k, v, o) or a SwiGLU
   * (gate, up, down), and an f32 array (embedding table [V, d], RMSNorm weight [d]) */
  struct og_op* sub; int32_t n_sub, _pad2;
  float* extra; int64_t extra_len;
  /* FP16 arm (npu.rs:207-210, 231-232, 258-268): the weights in the reference layout
   * rounded by round_fp16 (a standalone ChannelAffine keeps its unrounded diagonal) */
  float* wh; int64_t wh_len;
  /* per-output-channel weight scales (NULL: per-tensor, the reference's only mode;
   * the extension quantizes each row of the [out, in] / [O, C*k*k] matrix with
   * QuantTensor::from_f32's arithmetic, quantize.rs:18-24) */
  float* w_scale_ch;
  /* static-calibration extension (no counterpart in the reference): with `frozen` set,
   * a Linear quantizes its input with frozen_scale instead of the scale of the input's
   * own absmax (values beyond the calibrated range clamp to +-127); seen_scale is the
   * scale the last run quantized with (how a calibration run records it) */
  int32_t frozen; float frozen_scale; float seen_scale; int32_t _pad3;
} og_op;

typedef struct {
  int32_t precision, original_layers, n_ops, _pad;
  og_op* ops;
  int64_t fp32_bytes, npu_bytes;
} og_program;

float og_act_apply(int32_t act, float param, float x);      /* mod.rs:38-53 + device/backend.rs:61-78 */
float og_quant_scale(const float* v, int64_t n);            /* quantize.rs:19-20 */
float og_quantize_into(const float* v, int64_t n, int8_t* out); /* quantize.rs:27-35 */
float og_round_fp16(float x);                               /* quantize.rs:50-64 */

og_program* og_compile(const og_layer* layers, int32_t n_layers, int32_t precision); /* npu.rs:188-276 */
/* og_compile with the weight-quantization mode: 0 per-tensor (the reference), 1 per
 * output channel (extension; byte accounting 4 B per scale, as quantize.rs:43-45). */
og_program* og_compile_ex(const og_layer* layers, int32_t n_layers, int32_t precision,
                          int32_t weight_quant);
/* The f32 ExecutionProvider::Cpu arm: fold_batch_norm then run_standard (mod.rs:162-166,
 * 260-331) over the reference's layer kinds 1-7.  Returns 0, -1 (bad input rank), -2
 * (shape mismatch), -3 (output capacity) or -5 (a layer kind outside 1-7). */
int32_t og_run_standard(const og_layer* layers, int32_t n_layers, const float* x, const int64_t* shape,
                        int32_t ndim, float* y, int64_t y_cap, int64_t* y_shape, int32_t* y_ndim);
void og_program_free(og_program* p);
/* NpuOp::label (npu.rs:83-104); returns bytes written (excluding NUL). */
int32_t og_op_label(const og_op* op, char* buf, int32_t cap);
/* NpuProgram::summary (npu.rs:280-293). */
int32_t og_program_summary(const og_program* p, int32_t raw_count, char* buf, int32_t cap);

/* ---- per-op execution (npu.rs:296-421) ---------------------------------- */
/* FusedLinear Int8 arm (npu.rs:307-318).  aq [rows,in] and acc [rows,out] are optional dumps. */
void og_op_linear(const og_op* op, const float* x, int64_t rows, float* y,
                  float* a_scale, int8_t* aq, int32_t* acc, int32_t nthreads);
/* Same with the activation absmax given by the caller (max over all batch shards). */
void og_op_linear_with_amax(const og_op* op, const float* x, int64_t rows, float amax, float* y,
                            int32_t nthreads);
/* Same, restricted to rows [r0, r1) with the scale taken over all `rows` (row sampling for huge M). */
void og_op_linear_rows(const og_op* op, const float* x, int64_t rows, int64_t r0, int64_t r1,
                       float* y, float* a_scale, int32_t* acc, int32_t nthreads);
/* FusedConv2d Int8 arm (npu.rs:319-383).  y [n,O,oh,ow].  a_scales [n].  aq [n,C,H,W] (every pixel
 * quantized with its image's scale) and acc [n,O,oh*ow] are optional dumps. */
void og_op_conv2d(const og_op* op, const float* x, int64_t n, int32_t h, int32_t w, float* y,
                  float* a_scales, int8_t* aq, int32_t* acc, int32_t nthreads);
void og_maxpool2d(const float* x, int64_t n, int32_t c, int32_t h, int32_t w, int32_t k,
                  int32_t stride, float* y, int32_t nthreads);          /* kernels.rs:165-213 */
void og_activation(const float* x, int64_t n, int32_t act, float param, float* y); /* npu.rs:395-399 */
/* extensions: adaptive average pooling (tensor/ops.rs:994-1014) and y = act(x + s) */
void og_adaptive_avgpool2d(const float* x, int64_t n, int32_t c, int32_t h, int32_t w, int32_t oh,
                           int32_t ow, float* y);
void og_residual_add(const float* x, const float* s, int64_t n, int32_t act, float param, float* y);
/* transformer extensions: 0 on success, -6 for an embedding id out of range */
int32_t og_embedding(const og_op* op, const float* ids, int64_t n, float* y);
void og_rmsnorm(const og_op* op, const float* x, int64_t rows, float* y);
void og_attention(const og_op* op, const float* x, int64_t b, int64_t t, float* y, int32_t nthreads);
void og_swiglu(const og_op* op, const float* x, int64_t rows, float* y, int32_t nthreads);
void og_bmm_fma(const float* a, const float* bm, int64_t batch, int64_t m, int64_t k, int64_t n, float* c);
void og_softmax(const float* x, int64_t outer, int64_t last, float* y); /* tensor/ops.rs:1058-1076 */
int64_t og_out_size(int64_t input, int64_t k, int64_t stride, int64_t pad); /* kernels.rs:10-15 */
void og_im2col(const float* x, int32_t c, int32_t h, int32_t w, int32_t k, int32_t stride,
               int32_t pad, int32_t oh, int32_t ow, float* cols);       /* kernels.rs:28-96 */
void og_transpose2d(const float* x, int64_t rows, int64_t cols, float* out); /* shape.rs:105-123 */
void og_fold_batch_norm_count(const og_layer* layers, int32_t n, int32_t* out_count);

/* Whole-program execute (npu.rs:296-421).  y_cap elements; out shape written to y_shape/y_ndim.
 * op_ns / op_macs receive the per-op OpRecord durations (ns) and MACs (n_ops entries each). */
int32_t og_execute(const og_program* p, const float* x, const int64_t* shape, int32_t ndim,
                   float* y, int64_t y_cap, int64_t* y_shape, int32_t* y_ndim,
                   int32_t nthreads, int64_t* op_ns, int64_t* op_macs);

#ifdef __cplusplus
}
#endif
#endif
