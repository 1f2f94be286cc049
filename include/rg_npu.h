/*
 * rg_npu.h -- C ABI of the B200 INT8 execution provider (librg_npu.so).
 *
 * The library replaces the CPU executor behind RustGears'
 * `ExecutionProvider::npu_int8()` (src/inference/npu.rs).  A host binding
 * (Rust FFI, ctypes, C++) keeps the reference surface --
 * `InferenceSession::from_layers / from_module / run / last_npu_profile /
 * compilation_report` -- and forwards to these entry points.  All pointers
 * are plain host or device pointers; no framework types cross the boundary.
 *
 * Errors: every entry point returns an rg_status; the message of the last
 * failure on the calling thread is available from rg_last_error().  There is
 * no CPU fallback: without a usable CUDA device the calls fail with
 * RG_ERR_NO_DEVICE.
 */
#ifndef RG_NPU_H
#define RG_NPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RG_NPU_ABI_VERSION 1

typedef enum rg_status {
  RG_OK = 0,
  RG_ERR_INVALID_ARG = 1,   /* bad pointer, size or enum value */
  RG_ERR_SHAPE = 2,         /* input shape does not match the program */
  RG_ERR_CUDA = 3,          /* CUDA runtime/driver error */
  RG_ERR_NCCL = 4,          /* NCCL error (multi-GPU) */
  RG_ERR_TIMEOUT = 5,       /* a bounded device wait gave up */
  RG_ERR_UNSUPPORTED = 6,   /* layer or precision this provider does not run */
  RG_ERR_IO = 7,            /* .rtim read failure / bad file */
  RG_ERR_OOM = 8,           /* device allocation failed */
  RG_ERR_NO_DEVICE = 9,     /* no sm_100 device visible */
  RG_ERR_NO_PROFILE = 10    /* last_profile before any run */
} rg_status;

/* Thread-local message of the last failure (never NULL). */
const char* rg_last_error(void);
/* Library version string, e.g. "rustgears-b200 0.1.0 (sm_100a)". */
const char* rg_version(void);
/* Number of visible sm_100 devices (0 when none). */
int32_t rg_device_count(void);

/* ---------------------------------------------------------------------------
 * IR: one entry per reference `LayerSpec` (src/inference/mod.rs:70-100).
 * `kind` uses the .rtim tags (src/save.rs:172-224); `act` uses the .rtim
 * activation codes (src/save.rs:206-214).
 * ------------------------------------------------------------------------- */
typedef enum rg_layer_kind {
  RG_LAYER_LINEAR = 1,          /* weight [in,out] row-major, bias [out] */
  RG_LAYER_CONV2D = 2,          /* weight [O,C,k,k], bias [O] */
  RG_LAYER_CHANNEL_AFFINE = 3,  /* weight = scale [C], bias = shift [C] (exported BatchNorm) */
  RG_LAYER_MAXPOOL2D = 4,       /* kernel, stride; no padding */
  RG_LAYER_FLATTEN = 5,
  RG_LAYER_ACTIVATION = 6,      /* act, act_param */
  RG_LAYER_SOFTMAX = 7,
  /* Extensions (no reference LayerSpec or .rtim tag): residual blocks and adaptive
   * average pooling, for ResNet-style networks.  A block is
   *   RESIDUAL_BEGIN, <main-path layers>, [SHORTCUT_CONV2D, ChannelAffine], RESIDUAL_END
   * and computes y = act(main(x) + shortcut(x)) with shortcut = identity or the conv. */
  RG_LAYER_RESIDUAL_BEGIN = 8,        /* saves the current activation as the block input */
  RG_LAYER_RESIDUAL_END = 9,          /* y = act(x + saved) with act, act_param; pops the saved input */
  RG_LAYER_SHORTCUT_CONV2D = 10,      /* Conv2d fields; applied to the saved input, replacing it */
  RG_LAYER_ADAPTIVE_AVGPOOL2D = 11,   /* output size: kernel = height, stride = width */
  /* Extensions for the transformer configuration (no reference LayerSpec; the blocks
   * compose the reference's Embedding, RMSNorm, MultiHeadAttention and SwiGLU with
   * their Linears on the INT8 path).  Weights are [in,out] row-major like Linear. */
  RG_LAYER_EMBEDDING = 12,  /* in_features = vocabulary V, out_features = d; weight [V, d];
                               input: token ids (f32 values), output [.., d] */
  RG_LAYER_RMSNORM = 13,    /* in_features = d; weight [d]; act_param = eps */
  RG_LAYER_ATTENTION = 14,  /* non-causal multi-head attention: in_features = d, out_features =
                               heads; weight = [Wq; Wk; Wv; Wo] (4 x [d, d]); bias = [bq; bk; bv; bo] */
  RG_LAYER_SWIGLU = 15      /* in_features = d, out_features = hidden h; weight = [Wgate [d,h];
                               Wup [d,h]; Wdown [h,d]]; no bias */
} rg_layer_kind;

typedef enum rg_activation {
  RG_ACT_NONE = 0, RG_ACT_RELU = 1, RG_ACT_SIGMOID = 2, RG_ACT_TANH = 3,
  RG_ACT_GELU = 4, RG_ACT_LEAKY_RELU = 5,
  /* Extension (no reference Activation variant or .rtim code): SiLU x * sigmoid(x), the
   * reference's nn::Silu forward (src/nn/layers.rs:337-346: x.mul(x.sigmoid())) */
  RG_ACT_SILU = 6
} rg_activation;

/* RG_PREC_F32: the f32 ExecutionProvider::Cpu arm (run_standard, src/inference/mod.rs:260-331):
 * BatchNorm folded, no fusion, f32 matmuls in the reference CPU matmul's FMA order; its
 * sessions record no NpuProfile (rg_session_last_profile returns RG_ERR_NO_PROFILE). */
typedef enum rg_precision { RG_PREC_INT8 = 0, RG_PREC_FP16 = 1, RG_PREC_F32 = 2 } rg_precision;

typedef struct rg_layer_spec {
  int32_t kind;
  int32_t in_features, out_features;
  int32_t in_channels, out_channels, kernel, stride, padding;
  const float* weight; int64_t weight_len;
  const float* bias; int64_t bias_len;
  int32_t act; float act_param;
} rg_layer_spec;

/* ---------------------------------------------------------------------------
 * Sessions: InferenceSession over ExecutionProvider::Npu(Int8).
 * ------------------------------------------------------------------------- */
typedef struct rg_session rg_session;

typedef struct rg_session_options {
  int32_t device;        /* CUDA ordinal */
  int32_t precision;     /* RG_PREC_INT8, or RG_PREC_FP16 (NpuPrecision::Fp16, npu.rs:425-445:
                            fp16-rounded operands, f32 sums in k order; attention and SwiGLU
                            blocks are INT8 only), or RG_PREC_F32 (the Cpu provider: the
                            reference's layer kinds 1-7 only) */
  int32_t weight_quant;  /* 0 = per-tensor (reference, quantize.rs:18-24); 1 = per-output-channel (extension) */
  int32_t flags;         /* RG_SESSION_* bits */
} rg_session_options;

#define RG_SESSION_NO_PROFILE 1   /* skip per-op CUDA events (records carry 0 durations) */
#define RG_SESSION_NO_FUSION 2    /* disable multi-op kernels (each NpuOp runs on its own) */
#define RG_SESSION_NO_GRAPH 4     /* do not replay repeated device-buffer runs from a CUDA graph */

/* Replaces `InferenceSession::from_layers(layers, ExecutionProvider::npu_int8())`
 * (src/inference/mod.rs:162-180) and `npu::compile` (src/inference/npu.rs:188-276):
 * folds ChannelAffine into the preceding Linear/Conv2d, fuses the following
 * Activation, quantizes weights (symmetric i8) and uploads them to the device. */
rg_status rg_session_create(const rg_layer_spec* layers, int32_t n_layers,
                            const rg_session_options* opts, rg_session** out);

/* Replaces `load_inference_layers(path)` (src/save.rs:227-279) followed by
 * `InferenceSession::from_layers`: the .rtim file drops in unchanged. */
rg_status rg_session_create_from_rtim(const char* path, const rg_session_options* opts,
                                      rg_session** out);

void rg_session_destroy(rg_session* s);

/* Output shape `run` would produce for an input shape (no device work). */
rg_status rg_session_output_shape(rg_session* s, const int64_t* shape, int32_t ndim,
                                  int64_t* y_shape, int32_t* y_ndim);

/* Replaces `InferenceSession::run` (src/inference/mod.rs:212-221) ->
 * `NpuProgram::execute` (src/inference/npu.rs:296-421).  x and y are HOST
 * buffers (pinned or pageable); the copies are part of the call.  y_cap is
 * the capacity of y in elements.  Calls on one session are serialised. */
rg_status rg_session_run(rg_session* s, const float* x, const int64_t* shape, int32_t ndim,
                         float* y, int64_t y_cap, int64_t* y_shape, int32_t* y_ndim);

/* Same program on DEVICE buffers of the session's device; enqueued on
 * `stream` (a cudaStream_t, NULL = the session's own stream) and
 * synchronised before return unless RG_RUN_ASYNC is passed in `flags`.  An
 * asynchronous run records no per-op timing (last_profile keeps the previous
 * synchronous run's) and its device error words are checked by the next
 * synchronous run.  Repeated runs with the same shape and buffers replay a
 * CUDA graph of the program (see RG_SESSION_NO_GRAPH). */
#define RG_RUN_ASYNC 1
rg_status rg_session_run_device(rg_session* s, const float* x_dev, const int64_t* shape,
                                int32_t ndim, float* y_dev, int64_t y_cap, int64_t* y_shape,
                                int32_t* y_ndim, void* stream, int32_t flags);

/* Replaces `InferenceSession::compilation_report` (src/inference/mod.rs:198-209,
 * npu.rs:280-293).  Writes at most cap bytes (NUL-terminated); *needed
 * receives the full length + 1. */
rg_status rg_session_compilation_report(rg_session* s, char* buf, int64_t cap, int64_t* needed);

/* `NpuProfile` / `OpRecord` (src/inference/npu.rs:107-176). */
typedef struct rg_profile {
  int32_t precision, original_layers, fused_ops, n_records;
  int64_t fp32_weight_bytes, npu_weight_bytes;
  uint64_t total_macs;
  int64_t total_time_ns;
  int32_t kernel_launches;  /* device kernels the last run launched (this library's own) */
  int32_t _reserved;
} rg_profile;

typedef struct rg_op_record {
  char op[96];          /* NpuOp::label (npu.rs:83-104) */
  uint64_t macs;
  int64_t duration_ns;  /* CUDA-event time of the op's kernels */
} rg_op_record;

/* Replaces `InferenceSession::last_npu_profile` (src/inference/mod.rs:193-195).
 * Returns RG_ERR_NO_PROFILE before the first run. */
rg_status rg_session_last_profile(rg_session* s, rg_profile* prof, rg_op_record* records,
                                  int32_t cap);

/* Introspection of the compiled program (tests and tools). */
typedef struct rg_op_info {
  int32_t kind, in_features, out_features, in_channels, out_channels, kernel, stride, padding;
  int32_t act; float act_param;
  float w_scale;          /* per-tensor weight scale (0 when per-channel) */
  int64_t wq_len, bias_len;
  char label[96];
} rg_op_info;
rg_status rg_session_num_ops(rg_session* s, int32_t* n_ops);
rg_status rg_session_op_info(rg_session* s, int32_t op, rg_op_info* info);
/* Copies the op's quantized weights in the reference layout ([out,in] for
 * Linear, [O, C*k*k] for Conv2d) to host memory. */
rg_status rg_session_op_weights(rg_session* s, int32_t op, int8_t* wq, int64_t cap, float* bias,
                                int64_t bias_cap);

/* ---------------------------------------------------------------------------
 * Static calibration (extension; no counterpart in the reference, whose every
 * Linear quantizes its input with the absmax of the batch it is given,
 * src/inference/npu.rs:312).  A calibrated session quantizes each Linear input
 * with a frozen per-tensor scale instead: no absmax pass and, across GPUs, no
 * all-reduce; the producers that can (the fused CNN block, RMSNorm, the SwiGLU
 * gate product) write the Linear's i8 operand directly instead of f32.  Values
 * beyond a frozen scale's range clamp to +-127.  Conv inputs keep their per-image
 * scales.  One target per Linear; two per attention / SwiGLU block (its input,
 * and the inner activation its second projection reads), in op order.
 * ------------------------------------------------------------------------- */
rg_status rg_session_calibration_targets(rg_session* s, int32_t* n);
/* Runs x (host buffer) with the reference's dynamic scales and freezes the scale
 * each target quantized with (QuantTensor::from_f32's absmax / 127, over every
 * rank's shard when a communicator is attached: a collective call then). */
rg_status rg_session_calibrate(rg_session* s, const float* x, const int64_t* shape, int32_t ndim);
/* Installs n frozen scales (finite, positive; n = the target count), or with
 * n = 0 returns to the reference's dynamic scales. */
rg_status rg_session_set_calibration(rg_session* s, const float* scales, int32_t n);
/* The frozen scales (RG_ERR_INVALID_ARG when the session is not calibrated). */
rg_status rg_session_get_calibration(rg_session* s, float* scales, int32_t cap);

/* Per-op trace for parity tests: when enabled, `run` keeps every op's
 * activation scale(s), i8 input, i32 accumulators and f32 output. */
typedef enum rg_trace_item {
  RG_TRACE_SCALES = 0,  /* f32: 1 (Linear) or n images (Conv2d) */
  RG_TRACE_AQ = 1,      /* i8: [rows,in] (Linear) or [n,C,H,W] (Conv2d) */
  RG_TRACE_ACC = 2,     /* i32: [rows,out] (Linear) or [n,O,OH,OW] (Conv2d) */
  RG_TRACE_OUT = 3      /* f32: op output */
} rg_trace_item;
rg_status rg_session_set_trace(rg_session* s, int32_t enable);
rg_status rg_session_trace_get(rg_session* s, int32_t op, int32_t item, void* buf,
                               int64_t cap_bytes, int64_t* n_bytes);

/* ---------------------------------------------------------------------------
 * Multi-GPU (one process per GPU).  The batch is split across ranks; every
 * Linear's activation absmax is max-all-reduced (4 bytes over NCCL) so each
 * rank quantizes with the scale a single device would use.
 * ------------------------------------------------------------------------- */
rg_status rg_nccl_unique_id(uint8_t id[128]);
rg_status rg_session_attach_comm(rg_session* s, const uint8_t id[128], int32_t rank,
                                 int32_t world);
/* All-gather of equal-sized f32 shards (device buffers) over the session's
 * communicator: recv holds world * count elements in rank order.  With a NULL
 * stream it runs on the session's stream and returns when done; on a caller's
 * stream it is enqueued there and returns at once (every rank must enqueue it). */
rg_status rg_session_allgather(rg_session* s, const float* send_dev, float* recv_dev,
                               int64_t count, void* stream);

/* ---------------------------------------------------------------------------
 * Kernel-level entry points (device pointers, enqueued on `stream`).
 * ------------------------------------------------------------------------- */
/* max |x| over n f32 (NaN ignored, as `fold(0, f32::max)`), written to *amax. */
rg_status rg_absmax_f32(const float* x, int64_t n, float* amax, void* stream);
/* QuantTensor::from_f32 (src/inference/quantize.rs:18-24) given a
 * precomputed absmax: x [rows,k] -> q [rows,ldq] (columns k..ldq zero),
 * *scale = absmax < 1e-12 ? 1 : absmax / 127. */
rg_status rg_quantize_f32_i8(const float* x, int64_t rows, int64_t k, int64_t ldq,
                             const float* amax, int8_t* q, float* scale, void* stream);
/* int8_gemm_fused (src/inference/quantize.rs:93-118): a [m,ld] i8, w [n,ld] i8
 * ("B transposed"), ld a multiple of 16 with zero padding beyond k;
 * out[r,c] = act(f32(sum_k a*w) * (a_scale*w_scale) + bias[c]).  acc (i32
 * [m,n]) and out_amax (max |out|, accumulated with max into *out_amax) are
 * optional (NULL).
 * Shapes that run on the tensor cores (m*n*k >= 2^22, n >= 16, k >= 32) use a
 * kernel whose pipeline waits are bounded: the call waits for it on `stream`
 * and returns RG_ERR_TIMEOUT if a wait gave up (its output is then invalid).
 * The word that reports it belongs to this call alone (a slot of a static
 * device array held for the call).  Inside a stream capture the call is
 * recorded without that check.  Other shapes run on the CUDA cores, have no
 * waits, and the call returns once they are enqueued. */
rg_status rg_gemm_i8_fused(const int8_t* a, const int8_t* w, int64_t m, int64_t n, int64_t ld,
                           const float* a_scale, float w_scale, const float* bias, int32_t act,
                           float act_param, float* out, int32_t* acc, float* out_amax,
                           void* stream);
/* One FusedLinear op (npu.rs:307-318): absmax + quantize of x [m,k] f32 and
 * the fused GEMM against w [n,ld] i8.  `workspace` must hold
 * rg_linear_i8_workspace_size(m, ld) bytes of device memory.  Timeouts are
 * reported as by rg_gemm_i8_fused. */
int64_t rg_linear_i8_workspace_size(int64_t m, int64_t ld);
rg_status rg_linear_i8(const float* x, int64_t m, int64_t k, const int8_t* w, int64_t n,
                       int64_t ld, float w_scale, const float* bias, int32_t act,
                       float act_param, float* out, void* workspace, void* stream);
/* rg_linear_i8 without the workspace argument, for callers that cannot
 * allocate device memory (a host that owns every byte of device memory
 * through its own pool, or a hot loop that must not call cudaMalloc).  No
 * counterpart in the reference.  Scratch is a static device array inside the
 * library (RG_LINEAR_NOALLOC_MAX_BYTES of quantized activations, i.e.
 * m * ld <= 16 MiB; larger calls fail with RG_ERR_INVALID_ARG), held by every
 * GPU that loads the library until exit.  All calls on a device share it:
 * calls that overlap on the GPU race.  The first call on a device looks up
 * the scratch address and should come before any stream capture; the address
 * is kept for the life of the process, so a process that resets a device
 * (cudaDeviceReset) must not call this entry point on it afterwards.
 * Timeouts are reported as by rg_gemm_i8_fused. */
#define RG_LINEAR_NOALLOC_MAX_BYTES (16u << 20)
rg_status rg_linear_i8_noalloc(const float* x, int64_t m, int64_t k, const int8_t* w, int64_t n,
                               int64_t ld, float w_scale, const float* bias, int32_t act,
                               float act_param, float* out, void* stream);
/* The status a run reports for its device error words (no counterpart in the
 * reference): words[0] set -> RG_ERR_TIMEOUT (a tensor-core kernel gave up on a
 * bounded wait), words[1] set -> RG_ERR_INVALID_ARG (an embedding id not below
 * the vocabulary size), else RG_OK.  Host-only; every run and kernel-level call
 * maps its words through it. */
rg_status rg_status_from_error_words(const int32_t words[2]);
/* Test hook of the bounded-wait failure path (no counterpart in the reference):
 * tcgen05 GEMM launches that follow bound every pipeline wait by wait_ns
 * (0 restores the 2 s default), and with starve_loads != 0 issue no operand
 * loads, so the first wait on them runs out and the call reports
 * RG_ERR_TIMEOUT.  Launch parameters are fixed when a session captures its
 * CUDA graph: test on host-buffer runs or RG_SESSION_NO_GRAPH sessions. */
void rg_debug_set_tc_wait(uint64_t wait_ns, int32_t starve_loads);
/* max_pool2d (src/kernels.rs:165-213), NCHW f32, no padding. */
rg_status rg_maxpool2d_f32(const float* x, int64_t n, int32_t c, int32_t h, int32_t w,
                           int32_t k, int32_t stride, float* y, void* stream);
/* softmax_raw over the last dim (src/tensor/ops.rs:1058-1076). */
rg_status rg_softmax_f32(const float* x, int64_t outer, int64_t last, float* y, void* stream);
/* Activation::apply elementwise (src/inference/mod.rs:38-53). */
rg_status rg_activation_f32(const float* x, int64_t n, int32_t act, float act_param, float* y,
                            void* stream);
/* Extension (the transformer layer kind RG_LAYER_ATTENTION): non-causal multi-head
 * attention core in f32 (src/nn/attention.rs:178-196): qkv [batch*t, ld] holds q, k,
 * v of head h at columns h*dh, d + h*dh, 2d + h*dh (d = heads*dh); out [batch*t, ldo]
 * receives softmax(q k^T * (1/sqrt(dh))) v with the heads merged.  Both matmuls
 * follow the reference CPU matmul's FMA order (src/device/cpu.rs:234-395). */
rg_status rg_attention_f32(const float* qkv, int64_t ld, int64_t batch, int32_t t, int32_t heads,
                           int32_t head_dim, float* out, int64_t ldo, void* stream);
/* Device self-test of the fast arithmetic the kernels use (no counterpart in the
 * reference): for every one of the 2^32 f32 bit patterns, evaluates each fast path
 * and the plain IEEE / libdevice form and counts the inputs whose results differ:
 * mismatches[0] tanh, [1] GELU (division), [2] the quantization scale from an
 * absmax (non-negative inputs), [3] its reciprocal, [4] the rounding of a
 * quantization argument (|t| < 2^23 and NaN), [5] the GEMM epilogue's
 * common-range tanh (and GELU through it) against the general one, on every
 * input where the epilogue uses it.  Synchronous, current device, ~0.3 s. */
rg_status rg_selftest_fast_paths(uint64_t mismatches[6]);

/* ---------------------------------------------------------------------------
 * Deterministic generator used by the benchmark configurations: SplitMix64
 * with the reference's f32 draws (src/rng.rs:10-58, tensor/mod.rs:116-131).
 * ------------------------------------------------------------------------- */
typedef struct rg_rng { uint64_t state; } rg_rng;
void rg_rng_seed(rg_rng* r, uint64_t seed);
uint64_t rg_rng_next_u64(rg_rng* r);
void rg_rng_fill_uniform(rg_rng* r, float* out, int64_t n, float lo, float hi);
void rg_rng_fill_normal(rg_rng* r, float* out, int64_t n, float std_scale);
void rg_rng_fill_below(rg_rng* r, int64_t* out, int64_t n, uint64_t bound);
float rg_kaiming_bound(int64_t fan_in);
float rg_bias_bound(int64_t fan_in);

#ifdef __cplusplus
}
#endif
#endif /* RG_NPU_H */
