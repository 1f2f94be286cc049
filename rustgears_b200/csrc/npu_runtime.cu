// npu_runtime.cu -- host runtime of the B200 INT8 execution provider and its C ABI.
//
// Replaces the CPU `NpuProgram` of RustGears:
//   * compile (src/inference/npu.rs:188-276, mod.rs:225-257): BatchNorm folding,
//     Linear/Conv2d + next-Activation fusion, symmetric per-tensor i8 weights,
//     byte accounting; weights are uploaded once;
//   * execute (npu.rs:296-421): one device program per call, ops launched on
//     the session's stream, per-op CUDA events filling the OpRecord durations.
// Each quantizing op's input absmax (per tensor for Linear, per image for
// Conv2d) is produced in the epilogue of the kernel that writes that tensor,
// so no op re-reads its input just to find the scale.
#include <cuda_runtime.h>
#include <nccl.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/rg_npu.h"
#include "rg_kernels.h"
#include "rg_math.cuh"

namespace rg {

// ----------------------------------------------------------------------------
// errors
// ----------------------------------------------------------------------------
static thread_local std::string g_err = "ok";

// Test hook state (rg_debug_set_tc_wait): copied into every tcgen05 GEMM launch.
static std::atomic<uint64_t> g_tc_wait_ns{0};
static std::atomic<int32_t> g_tc_starve{0};

static rg_status fail(rg_status st, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return st;
}

rg_status set_last_error(rg_status st, const char* msg) {
  g_err = msg;
  return st;
}

#define RG_CUDA_TRY(expr)                                                                   \
  do {                                                                                      \
    cudaError_t e_ = (expr);                                                                \
    if (e_ != cudaSuccess)                                                                  \
      return fail(e_ == cudaErrorMemoryAllocation ? RG_ERR_OOM : RG_ERR_CUDA, "%s: %s (%s:%d)", \
                  #expr, cudaGetErrorString(e_), __FILE__, __LINE__);                       \
  } while (0)

#define RG_NCCL_TRY(expr)                                                                   \
  do {                                                                                      \
    ncclResult_t r_ = (expr);                                                               \
    if (r_ != ncclSuccess)                                                                  \
      return fail(RG_ERR_NCCL, "%s: %s", #expr, ncclGetErrorString(r_));                    \
  } while (0)

#define RG_LAUNCHED(name)                                                                   \
  do {                                                                                      \
    cudaError_t e_ = cudaGetLastError();                                                    \
    if (e_ != cudaSuccess)                                                                  \
      return fail(RG_ERR_CUDA, "launch of %s failed: %s", name, cudaGetErrorString(e_));    \
  } while (0)

#define RG_PENDING(where)                                                                   \
  do {                                                                                      \
    cudaError_t e_ = cudaGetLastError();                                                    \
    if (e_ != cudaSuccess)                                                                  \
      return fail(RG_ERR_CUDA, "pending CUDA error before %s: %s", where, cudaGetErrorString(e_)); \
  } while (0)

#define RG_TRY(expr)                 \
  do {                               \
    rg_status s_ = (expr);           \
    if (s_ != RG_OK) return s_;      \
  } while (0)

static int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

static int64_t out_size(int64_t input, int64_t k, int64_t stride, int64_t pad) {  // kernels.rs:10-15
  const int64_t padded = input + 2 * pad;
  if (k <= 0 || stride <= 0 || padded < k) return -1;
  return (padded - k) / stride + 1;
}

// ----------------------------------------------------------------------------
// device buffer
// ----------------------------------------------------------------------------
struct DevBuf {  // owning, move-only device allocation
  void* p = nullptr;
  size_t bytes = 0;
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  DevBuf(DevBuf&& o) noexcept : p(o.p), bytes(o.bytes) { o.p = nullptr; o.bytes = 0; }
  DevBuf& operator=(DevBuf&& o) noexcept {
    if (this != &o) {
      if (p) cudaFree(p);
      p = o.p; bytes = o.bytes;
      o.p = nullptr; o.bytes = 0;
    }
    return *this;
  }
  ~DevBuf() { if (p) cudaFree(p); }
  rg_status ensure(size_t n) {
    if (n <= bytes) return RG_OK;
    if (p) { cudaFree(p); p = nullptr; bytes = 0; }
    const size_t want = std::max<size_t>(n, 256);
    RG_CUDA_TRY(cudaMalloc(&p, want));
    bytes = want;
    return RG_OK;
  }
  template <class T> T* as() const { return reinterpret_cast<T*>(p); }
};

// ----------------------------------------------------------------------------
// compiled program
// ----------------------------------------------------------------------------
struct HostLayer {
  int32_t kind = 0, in_f = 0, out_f = 0, in_c = 0, out_c = 0, k = 0, stride = 0, pad = 0;
  int32_t act = 0;
  float param = 0.0f;
  std::vector<float> w, b;
};

struct Op {
  int32_t kind = 0;  // RG_LAYER_LINEAR / CONV2D / MAXPOOL2D / FLATTEN / ACTIVATION / SOFTMAX
  int32_t in_f = 0, out_f = 0, in_c = 0, out_c = 0, k = 0, stride = 0, pad = 0;
  int32_t act = 0;
  float param = 0.0f;
  float w_scale = 0.0f;          // per-tensor weight scale
  std::vector<float> w_scale_ch;  // per-output-channel scales (extension)
  std::vector<int8_t> wq;        // reference layout: Linear [out,in]; Conv [O, C*k*k]
  std::vector<float> bias;
  int64_t kdim = 0, kpad = 0;     // GEMM reduction length and its padded device stride
  int32_t cpad = 0;               // conv: channels per tap in the device layouts (16-aligned, 4, or 1)
  int32_t kxp = 0;                // conv: taps per kernel row in the K order (k; with cpad 4: a multiple of 4)
  DevBuf d_w, d_bias, d_wsc;     // device weights [N, kpad] (conv: (ky,kx,c) order)
  DevBuf d_w3;                   // direct-conv weight arrangement for mode dmode
  int32_t dmode = -1;            // DCONV_3X3 / DCONV_S2D / DCONV_1X1, or -1 (implicit GEMM only)
  DevBuf d_ws;                   // 7x7 / stride 2 stems (<= 4 channels -> 64): the fused stem's arrangement
  DevBuf d_wh;                   // FP16 arm: f32 weights rounded by round_fp16, reference layout [N, K]
  bool wh_exact = true;          // every d_wh value is an fp16 value (not the affine diagonal)
  bool bias_finite = true;
  std::string label;
  // transformer extension: the INT8 Linears inside an op (attention: fused QKV
  // [3d, d] with per-column scales, then Wo; SwiGLU: fused gate|up [2h, d], then
  // Wdown) and an f32 array (embedding table [V, d], RMSNorm weight [d])
  std::vector<Op> subs;
  DevBuf d_ext;
};

struct TraceRec {
  std::vector<float> scales;
  std::vector<int8_t> aq;
  std::vector<int32_t> acc;
  std::vector<float> out;
};

struct Profile {
  bool valid = false;
  int32_t launches = 0;
  uint64_t total_macs = 0;
  int64_t total_ns = 0;
  std::vector<uint64_t> macs;
  std::vector<int64_t> ns;
};

struct Session {
  int device = 0;
  int precision = RG_PREC_INT8;
  int weight_quant = 0;
  int flags = 0;
  int num_sms = 148;
  int original_layers = 0;
  int64_t fp32_bytes = 0, npu_bytes = 0;
  std::vector<Op> ops;
  cudaStream_t stream = nullptr;
  cudaStream_t copy_stream = nullptr;      // host copies that overlap the first / last op
  std::vector<cudaEvent_t> chunk_events;   // one per input chunk (timing disabled)
  std::vector<cudaEvent_t> drain_events;   // one per output chunk (timing disabled)
  cudaEvent_t drain_done = nullptr;        // the last output chunk has reached the host
  std::vector<cudaEvent_t> events;
  std::vector<int> ev_of;  // ev_of[i]: event marking the start of op i (ops that launch nothing share one)
  std::mutex mu;
  // workspace
  DevBuf act0, act1, act2, act3, qbuf, amax, scales, accbuf, xin, yout, covbuf, mlpws;
  // This session's device error words, set by its kernels and read (and cleared) by
  // the host after a synchronous run: [0] a tensor-core kernel gave up on a bounded
  // wait; [1] an embedding id was not below the vocabulary size.  Per session, so a
  // failure is reported to the run it happened in and to no other session.
  DevBuf errw;
  DevBuf ext0, ext1;  // attention / SwiGLU intermediates (QKV or gate|up, merged heads or g*u)
  // profile + trace
  Profile last;
  bool trace = false;
  std::vector<TraceRec> traces;
  bool used_tc = false;  // a tcgen05 kernel ran since the last error-word check
  bool used_embed = false;  // an embedding gather ran since the last error-word check
  // Static calibration (extension, no counterpart in the reference): one frozen
  // per-tensor scale per Linear input -- a Linear has one; an attention or SwiGLU block
  // two (its input, and the inner activation its second projection reads).  With
  // scales installed, those Linears quantize with them (clamping beyond the calibrated
  // range) instead of the batch absmax, need no absmax pass or all-reduce, and the
  // producers that can (the fused CNN block, RMSNorm, the SwiGLU gate product) write
  // the Linear's i8 operand directly.
  std::vector<int32_t> calib_off;  // per op: index of its first scale, or -1
  int32_t calib_targets = 0;
  bool calibrated = false;
  std::vector<float> calib;
  DevBuf d_calib;
  // multi-GPU
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  // Repeated device-buffer runs (same shape, same input and output pointers) replay the
  // program from a CUDA graph captured on the second such run: one launch instead of
  // the host planning and per-kernel launches.
  struct Graph {
    std::vector<int64_t> shape;
    const void* x = nullptr;
    void* y = nullptr;
    bool events = false;
    int seen = 0;                    // identical runs so far (capture on the second)
    bool off = false;                // capture failed or not applicable: run directly
    cudaGraphExec_t exec = nullptr;
    int32_t launches = 0;
    bool used_tc = false, used_embed = false;
    std::vector<int> ev_of;
    std::shared_ptr<void> plan;      // the RunPlan the graph was captured with
  } graph;
  bool capturing = false;
  cudaEvent_t t0 = nullptr, t1 = nullptr;  // whole-run timing
  ~Session() {
    if (graph.exec) cudaGraphExecDestroy(graph.exec);
  }
};

static void act_name(int32_t act, float p, char* out, size_t cap) {
  switch (act) {
    case RG_ACT_NONE: snprintf(out, cap, "none"); break;
    case RG_ACT_RELU: snprintf(out, cap, "ReLU"); break;
    case RG_ACT_SIGMOID: snprintf(out, cap, "Sigmoid"); break;
    case RG_ACT_TANH: snprintf(out, cap, "Tanh"); break;
    case RG_ACT_GELU: snprintf(out, cap, "GELU"); break;
    case RG_ACT_LEAKY_RELU: {
      // Rust `{}` of an f32: shortest decimal that round-trips, no exponent.
      char num[64];
      for (int prec = 0; prec <= 60; ++prec) {
        snprintf(num, sizeof num, "%.*f", prec, (double)p);
        if (strtof(num, nullptr) == p) break;
      }
      snprintf(out, cap, "LeakyReLU(%s)", num);
      break;
    }
    case RG_ACT_SILU: snprintf(out, cap, "SiLU"); break;  // extension: nn::Silu
    default: snprintf(out, cap, "?"); break;
  }
}

static std::string make_label(const Op& op) {  // NpuOp::label (npu.rs:83-104)
  char a[96], buf[192];
  act_name(op.act, op.param, a, sizeof a);
  switch (op.kind) {
    case RG_LAYER_LINEAR:
      if (op.act == RG_ACT_NONE) snprintf(buf, sizeof buf, "NPU::Gemm(%d->%d)", op.in_f, op.out_f);
      else snprintf(buf, sizeof buf, "NPU::FusedGemmAct(%d->%d, %s)", op.in_f, op.out_f, a);
      break;
    case RG_LAYER_CONV2D:
      if (op.act == RG_ACT_NONE) snprintf(buf, sizeof buf, "NPU::Conv2d(%d->%d, k=%d)", op.in_c, op.out_c, op.k);
      else snprintf(buf, sizeof buf, "NPU::FusedConv2dAct(%d->%d, k=%d, %s)", op.in_c, op.out_c, op.k, a);
      break;
    case RG_LAYER_MAXPOOL2D: snprintf(buf, sizeof buf, "NPU::MaxPool2d(k=%d)", op.k); break;
    case RG_LAYER_FLATTEN: snprintf(buf, sizeof buf, "NPU::Flatten"); break;
    case RG_LAYER_ACTIVATION: snprintf(buf, sizeof buf, "NPU::Act(%s)", a); break;
    case RG_LAYER_SOFTMAX: snprintf(buf, sizeof buf, "NPU::Softmax"); break;
    // extension ops
    case RG_LAYER_RESIDUAL_BEGIN: snprintf(buf, sizeof buf, "NPU::ResidualBegin"); break;
    case RG_LAYER_RESIDUAL_END:
      if (op.act == RG_ACT_NONE) snprintf(buf, sizeof buf, "NPU::ResidualAdd");
      else snprintf(buf, sizeof buf, "NPU::ResidualAdd(%s)", a);
      break;
    case RG_LAYER_SHORTCUT_CONV2D:
      snprintf(buf, sizeof buf, "NPU::ShortcutConv2d(%d->%d, k=%d)", op.in_c, op.out_c, op.k);
      break;
    case RG_LAYER_ADAPTIVE_AVGPOOL2D: snprintf(buf, sizeof buf, "NPU::AdaptiveAvgPool2d(%dx%d)", op.k, op.stride); break;
    case RG_LAYER_EMBEDDING: snprintf(buf, sizeof buf, "NPU::Embedding(%d, %d)", op.in_f, op.out_f); break;
    case RG_LAYER_RMSNORM: snprintf(buf, sizeof buf, "NPU::RMSNorm(%d)", op.in_f); break;
    case RG_LAYER_ATTENTION: snprintf(buf, sizeof buf, "NPU::Attention(d=%d, heads=%d)", op.in_f, op.out_f); break;
    case RG_LAYER_SWIGLU: snprintf(buf, sizeof buf, "NPU::SwiGLU(%d->%d->%d)", op.in_f, op.out_f, op.in_f); break;
    default: snprintf(buf, sizeof buf, "NPU::?"); break;
  }
  return buf;
}

// Symmetric i8 quantization (quantize.rs:18-24) of n values; returns the scale.
static float quantize_host(const float* v, int64_t n, int8_t* out) {
  float m = 0.0f;
  for (int64_t i = 0; i < n; ++i) m = fmaxf(m, fabsf(v[i]));
  const float scale = quant_scale(m);
  const float inv = quant_inv(scale);
  for (int64_t i = 0; i < n; ++i) out[i] = (int8_t)quant1(v[i], inv);
  return scale;
}

static rg_status validate_layer(const rg_layer_spec& l, int idx) {
  switch (l.kind) {
    case RG_LAYER_LINEAR:
      if (l.in_features <= 0 || l.out_features <= 0 ||
          l.weight_len != (int64_t)l.in_features * l.out_features || l.bias_len != l.out_features ||
          !l.weight || !l.bias)
        return fail(RG_ERR_INVALID_ARG, "layer %d: Linear(%d, %d) needs weight [in,out] and bias [out]", idx,
                    l.in_features, l.out_features);
      return RG_OK;
    case RG_LAYER_CONV2D:
    case RG_LAYER_SHORTCUT_CONV2D:
      if (l.in_channels <= 0 || l.out_channels <= 0 || l.kernel <= 0 || l.stride <= 0 || l.padding < 0 ||
          l.weight_len != (int64_t)l.out_channels * l.in_channels * l.kernel * l.kernel ||
          l.bias_len != l.out_channels || !l.weight || !l.bias)
        return fail(RG_ERR_INVALID_ARG, "layer %d: Conv2d(%d, %d, k=%d) has inconsistent weights", idx,
                    l.in_channels, l.out_channels, l.kernel);
      return RG_OK;
    case RG_LAYER_CHANNEL_AFFINE:
      if (l.weight_len <= 0 || l.bias_len != l.weight_len || !l.weight || !l.bias)
        return fail(RG_ERR_INVALID_ARG, "layer %d: ChannelAffine needs scale and shift of equal length", idx);
      return RG_OK;
    case RG_LAYER_MAXPOOL2D:
      if (l.kernel <= 0 || l.stride <= 0)
        return fail(RG_ERR_INVALID_ARG, "layer %d: kernel and stride must be positive", idx);
      return RG_OK;
    case RG_LAYER_FLATTEN:
    case RG_LAYER_SOFTMAX:
    case RG_LAYER_RESIDUAL_BEGIN:
      return RG_OK;
    case RG_LAYER_ADAPTIVE_AVGPOOL2D:
      if (l.kernel <= 0 || l.stride <= 0)
        return fail(RG_ERR_INVALID_ARG, "layer %d: adaptive pool output size must be positive", idx);
      return RG_OK;
    case RG_LAYER_RESIDUAL_END:
    case RG_LAYER_ACTIVATION:
      if (l.act < RG_ACT_NONE || l.act > RG_ACT_SILU)
        return fail(RG_ERR_INVALID_ARG, "layer %d: unknown activation tag %d", idx, l.act);
      return RG_OK;
    case RG_LAYER_EMBEDDING:
      if (l.in_features <= 0 || l.out_features <= 0 || !l.weight ||
          l.weight_len != (int64_t)l.in_features * l.out_features)
        return fail(RG_ERR_INVALID_ARG, "layer %d: Embedding(%d, %d) needs a table [V, d]", idx, l.in_features,
                    l.out_features);
      return RG_OK;
    case RG_LAYER_RMSNORM:
      if (l.in_features <= 0 || !l.weight || l.weight_len != l.in_features)
        return fail(RG_ERR_INVALID_ARG, "layer %d: RMSNorm(%d) needs a weight [d]", idx, l.in_features);
      return RG_OK;
    case RG_LAYER_ATTENTION:
      if (l.in_features <= 0 || l.out_features <= 0 || l.in_features % l.out_features != 0 || !l.weight ||
          !l.bias || l.weight_len != 4 * (int64_t)l.in_features * l.in_features || l.bias_len != 4 * (int64_t)l.in_features)
        return fail(RG_ERR_INVALID_ARG,
                    "layer %d: Attention(d=%d, heads=%d) needs heads | d, weight 4 x [d, d] and bias 4 x [d]", idx,
                    l.in_features, l.out_features);
      return RG_OK;
    case RG_LAYER_SWIGLU:
      if (l.in_features <= 0 || l.out_features <= 0 || !l.weight ||
          l.weight_len != 3 * (int64_t)l.in_features * l.out_features)
        return fail(RG_ERR_INVALID_ARG, "layer %d: SwiGLU(%d->%d) needs weight [d,h] [d,h] [h,d]", idx,
                    l.in_features, l.out_features);
      return RG_OK;
    default:
      return fail(RG_ERR_INVALID_ARG, "layer %d: unknown layer tag %d", idx, l.kind);
  }
}

// fold_batch_norm (src/inference/mod.rs:225-257): w *= s, b = b * s + shift (two roundings).
static std::vector<HostLayer> fold(const rg_layer_spec* L, int32_t n) {
  std::vector<HostLayer> out;
  for (int32_t i = 0; i < n; ++i) {
    const rg_layer_spec& l = L[i];
    if (l.kind == RG_LAYER_CHANNEL_AFFINE && !out.empty()) {
      HostLayer& p = out.back();
      const int64_t c = l.weight_len;
      if (p.kind == RG_LAYER_LINEAR && p.out_f == c) {
        for (int64_t r = 0; r < p.in_f; ++r)
          for (int64_t j = 0; j < p.out_f; ++j) p.w[r * p.out_f + j] = p.w[r * p.out_f + j] * l.weight[j];
        for (int64_t j = 0; j < p.out_f; ++j) { const float t = p.b[j] * l.weight[j]; p.b[j] = t + l.bias[j]; }
        continue;
      }
      if ((p.kind == RG_LAYER_CONV2D || p.kind == RG_LAYER_SHORTCUT_CONV2D) && p.out_c == c) {
        const int64_t plane = (int64_t)p.in_c * p.k * p.k;
        for (int64_t o = 0; o < p.out_c; ++o) {
          for (int64_t j = 0; j < plane; ++j) p.w[o * plane + j] = p.w[o * plane + j] * l.weight[o];
          const float t = p.b[o] * l.weight[o];
          p.b[o] = t + l.bias[o];
        }
        continue;
      }
    }
    HostLayer h;
    h.kind = l.kind; h.in_f = l.in_features; h.out_f = l.out_features; h.in_c = l.in_channels;
    h.out_c = l.out_channels; h.k = l.kernel; h.stride = l.stride; h.pad = l.padding;
    h.act = l.act; h.param = l.act_param;
    if (l.weight_len > 0) h.w.assign(l.weight, l.weight + l.weight_len);
    if (l.bias_len > 0) h.b.assign(l.bias, l.bias + l.bias_len);
    out.push_back(std::move(h));
  }
  return out;
}

static rg_status upload_op(Op& op) {
  // Device layout [N, kpad], K-contiguous, zero padded; conv reduction order (ky, kx, c).
  const int64_t N = op.kind == RG_LAYER_LINEAR ? op.out_f : op.out_c;
  std::vector<int8_t> dev((size_t)(N * op.kpad), 0);
  if (op.kind == RG_LAYER_LINEAR) {
    for (int64_t n = 0; n < N; ++n)
      memcpy(&dev[(size_t)(n * op.kpad)], &op.wq[(size_t)(n * op.in_f)], (size_t)op.in_f);
  } else {  // reduction order (ky, kx, c), c padded to cpad with zeros
    const int64_t C = op.in_c, K = op.k, CP = op.cpad;
    for (int64_t o = 0; o < N; ++o)
      for (int64_t c = 0; c < C; ++c)
        for (int64_t ky = 0; ky < K; ++ky)
          for (int64_t kx = 0; kx < K; ++kx)
            dev[(size_t)(o * op.kpad + (ky * op.kxp + kx) * CP + c)] = op.wq[(size_t)(((o * C + c) * K + ky) * K + kx)];
  }
  RG_TRY(op.d_w.ensure(dev.size()));
  RG_CUDA_TRY(cudaMemcpy(op.d_w.p, dev.data(), dev.size(), cudaMemcpyHostToDevice));
  // the direct (tap-shifted) conv kernel: 3x3 / stride 1 / pad 1, 3x3 / stride 2 / pad 1
  // (space-to-depth), 1x1 / pad 0 (any stride, over the compact operand)
  op.dmode = -1;
  if (op.kind == RG_LAYER_CONV2D || op.kind == RG_LAYER_SHORTCUT_CONV2D) {
    if (op.kind == RG_LAYER_CONV2D && op.k == 3 && op.stride == 1 && op.pad == 1 && op.cpad % 64 == 0)
      op.dmode = DCONV_3X3;
    else if (op.k == 3 && op.stride == 2 && op.pad == 1 && op.cpad % 16 == 0)
      op.dmode = DCONV_S2D;
    else if (op.k == 1 && op.pad == 0 && op.cpad % 64 == 0)
      op.dmode = DCONV_1X1;
  }
  if (op.dmode >= 0) {
    std::vector<int8_t> w3(dconv_weight_bytes(op.dmode, op.out_c, op.cpad));
    dconv_arrange_weights(op.dmode, op.wq.data(), op.out_c, op.in_c, op.k, op.cpad, w3.data());
    RG_TRY(op.d_w3.ensure(w3.size()));
    RG_CUDA_TRY(cudaMemcpy(op.d_w3.p, w3.data(), w3.size(), cudaMemcpyHostToDevice));
  }
  if (op.kind == RG_LAYER_CONV2D && op.k == 7 && op.stride == 2 && op.pad == 3 && op.in_c <= 4 && op.out_c == 64) {
    std::vector<int8_t> ws(stem_weight_bytes());
    stem_arrange_weights(op.wq.data(), op.in_c, ws.data());
    RG_TRY(op.d_ws.ensure(ws.size()));
    RG_CUDA_TRY(cudaMemcpy(op.d_ws.p, ws.data(), ws.size(), cudaMemcpyHostToDevice));
  }
  RG_TRY(op.d_bias.ensure(op.bias.size() * sizeof(float)));
  RG_CUDA_TRY(cudaMemcpy(op.d_bias.p, op.bias.data(), op.bias.size() * sizeof(float), cudaMemcpyHostToDevice));
  if (!op.w_scale_ch.empty()) {
    RG_TRY(op.d_wsc.ensure(op.w_scale_ch.size() * sizeof(float)));
    RG_CUDA_TRY(cudaMemcpy(op.d_wsc.p, op.w_scale_ch.data(), op.w_scale_ch.size() * sizeof(float),
                           cudaMemcpyHostToDevice));
  }
  return RG_OK;
}

static void quantize_weights(Op& op, const float* w_ref_layout, int64_t rows, int64_t cols, int per_channel) {
  op.wq.resize((size_t)(rows * cols));
  if (!per_channel) {
    op.w_scale = quantize_host(w_ref_layout, rows * cols, op.wq.data());
  } else {
    op.w_scale = 0.0f;
    op.w_scale_ch.resize((size_t)rows);
    for (int64_t r = 0; r < rows; ++r)
      op.w_scale_ch[(size_t)r] = quantize_host(w_ref_layout + r * cols, cols, op.wq.data() + r * cols);
  }
}

// Linears that read the same input, each weight [in, out_each] row-major with its own
// per-tensor scale (Linear::new / Linear::no_bias on the INT8 path, a-7/a-9 semantics),
// quantized into one fused Op whose output columns hold the parts side by side: the
// parts' scales become per-column scales.  Byte accounting per part as for a Linear.
static rg_status fuse_linears(Session& s, int32_t in, int32_t out_each, const std::vector<const float*>& ws,
                              const std::vector<const float*>& bs, Op& op) {
  const int64_t parts = (int64_t)ws.size(), n = out_each * parts;
  op.kind = RG_LAYER_LINEAR; op.in_f = in; op.out_f = (int32_t)n; op.act = RG_ACT_NONE;
  op.kdim = in; op.kpad = round_up(in, 16);
  op.wq.assign((size_t)(n * in), 0);
  op.bias.assign((size_t)n, 0.0f);
  if (parts > 1) op.w_scale_ch.assign((size_t)n, 0.0f);
  std::vector<float> wt((size_t)in * out_each);
  for (int64_t j = 0; j < parts; ++j) {
    const float* w = ws[(size_t)j];
    for (int64_t r = 0; r < in; ++r)  // transpose2d [in,out] -> [out,in] (npu.rs:208)
      for (int64_t c = 0; c < out_each; ++c) wt[(size_t)(c * in + r)] = w[r * out_each + c];
    const float sc = quantize_host(wt.data(), (int64_t)in * out_each, op.wq.data() + j * out_each * in);
    if (parts > 1) {
      for (int64_t c = 0; c < out_each; ++c) op.w_scale_ch[(size_t)(j * out_each + c)] = sc;
    } else {
      op.w_scale = sc;
    }
    if (bs[(size_t)j]) memcpy(op.bias.data() + j * out_each, bs[(size_t)j], sizeof(float) * (size_t)out_each);
    s.fp32_bytes += ((int64_t)in * out_each + (bs[(size_t)j] ? out_each : 0)) * 4;
    s.npu_bytes += ((int64_t)in * out_each + 4) + (bs[(size_t)j] ? (int64_t)out_each * 4 : 0);
  }
  op.label = make_label(op);
  return upload_op(op);
}

// The FP16 arm's weights (npu.rs:210, 232): round_fp16 of the reference-layout f32
// weights, kept in f32 on the device; `round` false keeps them as given (the
// diagonal of a standalone ChannelAffine, npu.rs:258-268).
static rg_status upload_fp16(Op& op, const std::vector<float>& w, bool round) {
  std::vector<float> h(w.size());
  for (size_t j = 0; j < w.size(); ++j) h[j] = round ? round_fp16(w[j]) : w[j];
  op.wh_exact = round;
  RG_TRY(op.d_wh.ensure(h.size() * sizeof(float)));
  if (!h.empty()) RG_CUDA_TRY(cudaMemcpy(op.d_wh.p, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice));
  return RG_OK;
}

// npu::compile (npu.rs:188-276).
static rg_status compile(Session& s, const rg_layer_spec* layers, int32_t n) {
  for (int32_t i = 0; i < n; ++i) RG_TRY(validate_layer(layers[i], i));
  int depth = 0;  // residual blocks must nest and close
  for (int32_t i = 0; i < n; ++i) {
    const int32_t k = layers[i].kind;
    if (k == RG_LAYER_RESIDUAL_BEGIN) ++depth;
    if ((k == RG_LAYER_RESIDUAL_END || k == RG_LAYER_SHORTCUT_CONV2D) && depth == 0)
      return fail(RG_ERR_INVALID_ARG, "layer %d: %s outside a residual block", i,
                  k == RG_LAYER_RESIDUAL_END ? "ResidualEnd" : "ShortcutConv2d");
    if (k == RG_LAYER_RESIDUAL_END) --depth;
  }
  if (depth != 0) return fail(RG_ERR_INVALID_ARG, "%d residual block(s) not closed", depth);
  std::vector<HostLayer> f = fold(layers, n);
  s.original_layers = n;
  for (size_t i = 0; i < f.size(); ++i) {
    HostLayer& l = f[i];
    // an Activation after a shortcut conv belongs to the main path: not fused into it;
    // the f32 provider fuses nothing (run_standard walks the folded layers one by one)
    const bool f32 = s.precision == RG_PREC_F32;
    if (f32 && l.kind > RG_LAYER_SOFTMAX)
      return fail(RG_ERR_UNSUPPORTED, "layer %zu: the f32 provider runs the reference's layer kinds 1-7 only", i);
    const bool next_act = !f32 && i + 1 < f.size() && f[i + 1].kind == RG_LAYER_ACTIVATION &&
                          l.kind != RG_LAYER_SHORTCUT_CONV2D;
    Op op;
    if (l.kind == RG_LAYER_LINEAR || l.kind == RG_LAYER_CONV2D || l.kind == RG_LAYER_SHORTCUT_CONV2D) {
      op.kind = l.kind;
      op.act = next_act ? f[i + 1].act : RG_ACT_NONE;
      op.param = next_act ? f[i + 1].param : 0.0f;
      if (l.kind == RG_LAYER_LINEAR) {
        op.in_f = l.in_f; op.out_f = l.out_f;
        std::vector<float> wt((size_t)l.w.size());
        for (int64_t r = 0; r < l.in_f; ++r)  // transpose2d [in,out] -> [out,in] (npu.rs:208)
          for (int64_t c = 0; c < l.out_f; ++c) wt[(size_t)(c * l.in_f + r)] = l.w[(size_t)(r * l.out_f + c)];
        quantize_weights(op, wt.data(), l.out_f, l.in_f, s.weight_quant);
        op.kdim = l.in_f;
        if (s.precision == RG_PREC_FP16) RG_TRY(upload_fp16(op, wt, true));  // npu.rs:210
        if (f32) RG_TRY(upload_fp16(op, wt, false));  // f32 weights, [out, in] for the kernel
      } else {
        op.in_c = l.in_c; op.out_c = l.out_c; op.k = l.k; op.stride = l.stride; op.pad = l.pad;
        // channels padded to 16 per tap so the tensor-core conv gathers 16-byte chunks
        // (a single channel stays unpadded: the fused CNN block reads it directly)
        // (2-4 channels, e.g. an RGB stem: a 4-byte pixel, taps per kernel row padded to a
        // multiple of 4 so that a 16-byte chunk holds 4 taps)
        op.cpad = l.in_c == 1 ? 1 : l.in_c <= 4 ? 4 : (int32_t)round_up(l.in_c, 16);
        op.kxp = op.cpad == 4 ? (int32_t)round_up(l.k, 4) : l.k;
        quantize_weights(op, l.w.data(), l.out_c, (int64_t)l.in_c * l.k * l.k, s.weight_quant);
        op.kdim = (int64_t)op.cpad * l.k * op.kxp;
        if (s.precision == RG_PREC_FP16) RG_TRY(upload_fp16(op, l.w, true));  // npu.rs:232
        if (f32) RG_TRY(upload_fp16(op, l.w, false));
      }
      op.kpad = round_up(op.kdim, 16);
      op.bias = l.b;
      s.fp32_bytes += (int64_t)(l.w.size() + l.b.size()) * 4;
      // 4 bytes per weight scale (quantize.rs:43-45): one per tensor, or one per output channel
      const int64_t n_scales = op.w_scale_ch.empty() ? 1 : (int64_t)op.w_scale_ch.size();
      s.npu_bytes += s.precision == RG_PREC_INT8 ? ((int64_t)op.wq.size() + 4 * n_scales) + (int64_t)l.b.size() * 4
                                                 : (int64_t)l.w.size() * 2 + (int64_t)l.b.size() * 2;
      if (next_act) ++i;
    } else if (l.kind == RG_LAYER_CHANNEL_AFFINE && f32) {
      // the f32 provider applies a standalone affine elementwise (mod.rs:293-303)
      op.kind = RG_LAYER_CHANNEL_AFFINE; op.in_f = (int32_t)l.w.size();
      op.bias = l.b;
      RG_TRY(upload_fp16(op, l.w, false));
      RG_TRY(op.d_bias.ensure(op.bias.size() * sizeof(float)));
      if (!op.bias.empty())
        RG_CUDA_TRY(cudaMemcpy(op.d_bias.p, op.bias.data(), op.bias.size() * sizeof(float), cudaMemcpyHostToDevice));
    } else if (l.kind == RG_LAYER_CHANNEL_AFFINE) {
      // standalone affine -> diagonal FusedLinear (npu.rs:254-270), no byte accounting
      const int64_t c = (int64_t)l.w.size();
      std::vector<float> w((size_t)(c * c), 0.0f);
      for (int64_t j = 0; j < c; ++j) w[(size_t)(j * c + j)] = l.w[(size_t)j];
      op.kind = RG_LAYER_LINEAR; op.in_f = (int32_t)c; op.out_f = (int32_t)c;
      quantize_weights(op, w.data(), c, c, s.weight_quant);
      op.kdim = c; op.kpad = round_up(c, 16);
      if (s.precision == RG_PREC_FP16) RG_TRY(upload_fp16(op, w, false));  // npu.rs:266: unrounded
      op.bias = l.b;
      op.act = RG_ACT_NONE;
    } else if ((l.kind == RG_LAYER_ATTENTION || l.kind == RG_LAYER_SWIGLU) && s.precision != RG_PREC_INT8) {
      return fail(RG_ERR_UNSUPPORTED, "layer %zu: attention and SwiGLU blocks run on the INT8 arm only", i);
    } else if (l.kind == RG_LAYER_ATTENTION) {
      const int32_t d = l.in_f;
      op.kind = l.kind; op.in_f = d; op.out_f = l.out_f;  // out_f = heads
      const int64_t dd = (int64_t)d * d;
      op.subs.resize(2);
      RG_TRY(fuse_linears(s, d, d, {l.w.data(), l.w.data() + dd, l.w.data() + 2 * dd},
                          {l.b.data(), l.b.data() + d, l.b.data() + 2 * d}, op.subs[0]));
      RG_TRY(fuse_linears(s, d, d, {l.w.data() + 3 * dd}, {l.b.data() + 3 * d}, op.subs[1]));
    } else if (l.kind == RG_LAYER_SWIGLU) {
      const int32_t d = l.in_f, hd = l.out_f;
      op.kind = l.kind; op.in_f = d; op.out_f = hd;
      const int64_t dh = (int64_t)d * hd;
      op.subs.resize(2);
      RG_TRY(fuse_linears(s, d, hd, {l.w.data(), l.w.data() + dh}, {nullptr, nullptr}, op.subs[0]));
      RG_TRY(fuse_linears(s, hd, d, {l.w.data() + 2 * dh}, {nullptr}, op.subs[1]));
    } else if (l.kind == RG_LAYER_EMBEDDING || l.kind == RG_LAYER_RMSNORM) {
      op.kind = l.kind; op.in_f = l.in_f; op.out_f = l.out_f; op.param = l.param;
      RG_TRY(op.d_ext.ensure(l.w.size() * sizeof(float)));
      RG_CUDA_TRY(cudaMemcpy(op.d_ext.p, l.w.data(), l.w.size() * sizeof(float), cudaMemcpyHostToDevice));
      s.fp32_bytes += (int64_t)l.w.size() * 4;  // kept in f32 on both paths
      s.npu_bytes += (int64_t)l.w.size() * 4;
    } else {
      op.kind = l.kind; op.k = l.k; op.stride = l.stride; op.act = l.act; op.param = l.param;
    }
    op.label = make_label(op);
    for (float b : op.bias)
      if (!std::isfinite(b)) op.bias_finite = false;
    if (op.kind == RG_LAYER_LINEAR || op.kind == RG_LAYER_CONV2D || op.kind == RG_LAYER_SHORTCUT_CONV2D)
      RG_TRY(upload_op(op));
    s.ops.push_back(std::move(op));
  }
  return RG_OK;
}

// ----------------------------------------------------------------------------
// run planning
// ----------------------------------------------------------------------------
struct OpShape {
  std::vector<int64_t> in, out;
  int64_t in_elems = 0, out_elems = 0;
  uint64_t macs = 0;
};

static rg_status plan_shapes(const Session& s, const int64_t* shape, int32_t ndim, std::vector<OpShape>& out) {
  if (ndim < 1 || ndim > 8) return fail(RG_ERR_SHAPE, "input rank %d not supported", ndim);
  std::vector<int64_t> sh(shape, shape + ndim);
  for (int64_t d : sh)
    if (d < 0) return fail(RG_ERR_SHAPE, "negative dimension in input shape");
  auto numel = [](const std::vector<int64_t>& v) {
    int64_t n = 1;
    for (int64_t d : v) n *= d;
    return n;
  };
  out.clear();
  std::vector<std::vector<int64_t>> saved;  // residual block inputs
  for (size_t i = 0; i < s.ops.size(); ++i) {
    const Op& op = s.ops[i];
    OpShape os;
    os.in = sh;
    os.in_elems = numel(sh);
    if (op.kind == RG_LAYER_SHORTCUT_CONV2D) {  // works on the saved block input, not the main path
      std::vector<int64_t>& ss = saved.back();
      if (ss.size() != 4 || ss[1] != op.in_c)
        return fail(RG_ERR_SHAPE, "op %zu (%s): expected a saved [N,%d,H,W] block input", i, op.label.c_str(),
                    op.in_c);
      const int64_t oh = out_size(ss[2], op.k, op.stride, op.pad), ow = out_size(ss[3], op.k, op.stride, op.pad);
      if (oh <= 0 || ow <= 0)
        return fail(RG_ERR_SHAPE, "op %zu (%s): kernel %d larger than padded input", i, op.label.c_str(), op.k);
      os.in = ss;
      os.in_elems = numel(ss);
      os.macs = (uint64_t)ss[0] * op.out_c * op.in_c * op.k * op.k * oh * ow;
      ss = {ss[0], op.out_c, oh, ow};
      os.out = ss;
      os.out_elems = numel(ss);
      out.push_back(std::move(os));
      continue;
    }
    switch (op.kind) {
      case RG_LAYER_LINEAR: {
        if (sh.back() != op.in_f)
          return fail(RG_ERR_SHAPE, "op %zu (%s): last dim %lld != in_features %d", i, op.label.c_str(),
                      (long long)sh.back(), op.in_f);
        const int64_t rows = os.in_elems / op.in_f;
        os.macs = (uint64_t)rows * op.in_f * op.out_f;
        sh.back() = op.out_f;
        break;
      }
      case RG_LAYER_CONV2D: {
        if (sh.size() != 4 || sh[1] != op.in_c)
          return fail(RG_ERR_SHAPE, "op %zu (%s): expected [N,%d,H,W] input", i, op.label.c_str(), op.in_c);
        const int64_t oh = out_size(sh[2], op.k, op.stride, op.pad), ow = out_size(sh[3], op.k, op.stride, op.pad);
        if (oh <= 0 || ow <= 0)
          return fail(RG_ERR_SHAPE, "op %zu (%s): kernel %d larger than padded input", i, op.label.c_str(), op.k);
        os.macs = (uint64_t)sh[0] * op.out_c * op.in_c * op.k * op.k * oh * ow;
        sh = {sh[0], op.out_c, oh, ow};
        break;
      }
      case RG_LAYER_MAXPOOL2D: {
        if (sh.size() != 4) return fail(RG_ERR_SHAPE, "op %zu (%s): expected a 4-D input", i, op.label.c_str());
        const int64_t oh = out_size(sh[2], op.k, op.stride, 0), ow = out_size(sh[3], op.k, op.stride, 0);
        if (oh <= 0 || ow <= 0)
          return fail(RG_ERR_SHAPE, "op %zu (%s): kernel %d larger than padded input", i, op.label.c_str(), op.k);
        sh = {sh[0], sh[1], oh, ow};
        break;
      }
      case RG_LAYER_FLATTEN: {
        int64_t rest = 1;
        for (size_t d = 1; d < sh.size(); ++d) rest *= sh[d];
        sh = {sh[0], rest};
        break;
      }
      case RG_LAYER_RESIDUAL_BEGIN:
        saved.push_back(sh);
        break;
      case RG_LAYER_RESIDUAL_END:
        if (saved.back() != sh)
          return fail(RG_ERR_SHAPE, "op %zu (%s): main path and shortcut shapes differ (%lld vs %lld elements)", i,
                      op.label.c_str(), (long long)numel(sh), (long long)numel(saved.back()));
        saved.pop_back();
        break;
      case RG_LAYER_ADAPTIVE_AVGPOOL2D:
        if (sh.size() != 4 || sh[2] <= 0 || sh[3] <= 0)
          return fail(RG_ERR_SHAPE, "op %zu (%s): expected a non-empty [N,C,H,W] input", i, op.label.c_str());
        sh = {sh[0], sh[1], op.k, op.stride};
        break;
      case RG_LAYER_EMBEDDING:
        if (sh.size() >= 8) return fail(RG_ERR_SHAPE, "op %zu (%s): input rank too high", i, op.label.c_str());
        sh.push_back(op.out_f);
        break;
      case RG_LAYER_RMSNORM:
      case RG_LAYER_SWIGLU:
        if (sh.back() != op.in_f)
          return fail(RG_ERR_SHAPE, "op %zu (%s): last dim %lld != %d", i, op.label.c_str(), (long long)sh.back(),
                      op.in_f);
        if (op.kind == RG_LAYER_SWIGLU) os.macs = 3ull * (uint64_t)(os.in_elems / op.in_f) * op.in_f * op.out_f;
        break;
      case RG_LAYER_CHANNEL_AFFINE:  // the f32 provider's elementwise affine over dim 1
        if (sh.size() < 2 || sh[1] != op.in_f)
          return fail(RG_ERR_SHAPE, "op %zu: ChannelAffine over %d channels needs dim 1 = %d", i, op.in_f, op.in_f);
        break;
      case RG_LAYER_ATTENTION:
        if (sh.size() != 3 || sh[2] != op.in_f)
          return fail(RG_ERR_SHAPE, "op %zu (%s): expected a [B, T, %d] input", i, op.label.c_str(), op.in_f);
        os.macs = 4ull * (uint64_t)sh[0] * sh[1] * op.in_f * op.in_f;  // the INT8 projections
        break;
      default:
        break;
    }
    os.out = sh;
    os.out_elems = numel(sh);
    out.push_back(std::move(os));
  }
  return RG_OK;
}

// Coverage of input rows/cols by a conv (a strided conv may skip pixels, which then
// do not enter the reference's im2col absmax).
static std::vector<uint8_t> coverage(int64_t in, int64_t k, int64_t stride, int64_t pad, int64_t out) {
  std::vector<uint8_t> cov((size_t)in, 0);
  for (int64_t o = 0; o < out; ++o)
    for (int64_t t = 0; t < k; ++t) {
      const int64_t i = o * stride + t - pad;
      if (i >= 0 && i < in) cov[(size_t)i] = 1;
    }
  return cov;
}

static bool all_covered(const std::vector<uint8_t>& v) {
  for (uint8_t c : v)
    if (!c) return false;
  return true;
}

struct RunPlan {
  std::vector<OpShape> shapes;
  // for every quantizing op: which earlier op writes its absmax (-1: a standalone pass)
  std::vector<int> amax_src;
  std::vector<int64_t> amax_slots;   // slots per op (1 or n images)
  std::vector<int64_t> amax_off;     // offset into the amax / scales buffers
  std::vector<std::vector<uint8_t>> rowcov, colcov;
  int64_t total_slots = 0;
  size_t cov_bytes = 0;
  std::vector<uint8_t> block_start;  // op i starts a fused Conv-Pool-Conv-Pool block
  std::vector<uint8_t> stem_start;   // op i is a 7x7 / 2 stem conv fused with the MaxPool(3, 2) after it
  // strided 1x1 / pad 0 shortcut convs: the op whose output is their block input (its
  // direct-3x3 producer can take their absmax into its epilogue), else -1; and the
  // reverse map, producer op -> shortcut op
  std::vector<int> amax2_src, amax2_for;
  // calibrated sessions: i8_out[j] = the consumer op whose i8 operand op j writes
  // directly (-1: none); i8_in[i]: op i's first Linear finds its operand written
  std::vector<int> i8_out;
  std::vector<uint8_t> i8_in;
};

// Ops that leave the main-path tensor as it is (reshape, saving a block input, a
// shortcut conv on the saved input).
static bool main_path_noop(int32_t kind) {
  return kind == RG_LAYER_FLATTEN || kind == RG_LAYER_RESIDUAL_BEGIN || kind == RG_LAYER_SHORTCUT_CONV2D;
}

// Activations f with max(f(a), f(b)) == f(max(a, b)) under round-to-nearest.
static bool non_decreasing(int32_t act, float p) {
  return act == RG_ACT_NONE || act == RG_ACT_RELU || (act == RG_ACT_LEAKY_RELU && p >= 0.0f);
}

// ops[i..i+3] = Conv(k3 s1 p1) MaxPool(2,2) Conv(k3 s1 p1) MaxPool(2,2) on a shape the
// fused kernel is instantiated for.
static bool block_at(const Session& s, const std::vector<OpShape>& shapes, size_t i) {
  if (i + 3 >= s.ops.size() || s.trace || (s.flags & RG_SESSION_NO_FUSION)) return false;
  const Op& c1 = s.ops[i];
  const Op& m1 = s.ops[i + 1];
  const Op& c2 = s.ops[i + 2];
  const Op& m2 = s.ops[i + 3];
  auto conv_ok = [](const Op& c) {
    return c.kind == RG_LAYER_CONV2D && c.k == 3 && c.stride == 1 && c.pad == 1 && c.w_scale_ch.empty() &&
           c.bias_finite && non_decreasing(c.act, c.param);
  };
  auto pool_ok = [](const Op& m) { return m.kind == RG_LAYER_MAXPOOL2D && m.k == 2 && m.stride == 2; };
  if (!conv_ok(c1) || !pool_ok(m1) || !conv_ok(c2) || !pool_ok(m2)) return false;
  const std::vector<int64_t>& in = shapes[i].in;
  return in.size() == 4 &&
         convblock_supported((int)in[1], c1.out_c, c2.out_c, (int)in[2], (int)in[3], c1.act, c2.act);
}

// ops[i..i+1] = Conv(k7 s2 p3, <= 4 -> 64 channels) MaxPool(3, 2): the fused stem.
static bool stem_at(const Session& s, const std::vector<OpShape>& shapes, size_t i) {
  if (i + 1 >= s.ops.size() || s.trace || (s.flags & RG_SESSION_NO_FUSION)) return false;
  const Op& c = s.ops[i];
  const Op& m = s.ops[i + 1];
  if (c.kind != RG_LAYER_CONV2D || !c.d_ws.p || m.kind != RG_LAYER_MAXPOOL2D) return false;
  const std::vector<int64_t>& in = shapes[i].in;
  return in.size() == 4 && stem_pool_shape_ok(in[0], (int32_t)in[1], (int32_t)in[2], (int32_t)in[3], c.k, c.stride,
                                               c.pad, c.out_c, m.k, m.stride);
}

static rg_status make_plan(const Session& s, const int64_t* shape, int32_t ndim, RunPlan& P) {
  RG_TRY(plan_shapes(s, shape, ndim, P.shapes));
  const size_t n = s.ops.size();
  P.amax_src.assign(n, -1);
  P.amax_slots.assign(n, 0);
  P.amax_off.assign(n, 0);
  P.rowcov.assign(n, {});
  P.colcov.assign(n, {});
  int64_t off = 0;
  for (size_t i = 0; i < n; ++i) {
    const Op& op = s.ops[i];
    const bool conv_like = op.kind == RG_LAYER_CONV2D || op.kind == RG_LAYER_SHORTCUT_CONV2D;
    const bool inner = op.kind == RG_LAYER_ATTENTION || op.kind == RG_LAYER_SWIGLU;  // two Linears in a row
    if (op.kind != RG_LAYER_LINEAR && !conv_like && !inner) continue;
    const OpShape& os = P.shapes[i];
    P.amax_slots[i] = op.kind == RG_LAYER_LINEAR ? 1 : inner ? 2 : os.in[0];
    P.amax_off[i] = off;
    off += std::max<int64_t>(P.amax_slots[i], 1);
    bool full = true;
    if (conv_like) {
      P.rowcov[i] = coverage(os.in[2], op.k, op.stride, op.pad, os.out[2]);
      P.colcov[i] = coverage(os.in[3], op.k, op.stride, op.pad, os.out[3]);
      full = all_covered(P.rowcov[i]) && all_covered(P.colcov[i]);
      if (!full) P.cov_bytes += P.rowcov[i].size() + P.colcov[i].size();
    }
    // a shortcut conv reads the saved block input: its own absmax pass
    if (op.kind == RG_LAYER_SHORTCUT_CONV2D || s.precision != RG_PREC_INT8) continue;
    // the producing op (Flatten only reshapes; a residual begin / shortcut leaves the main path)
    int j = (int)i - 1;
    while (j >= 0 && main_path_noop(s.ops[(size_t)j].kind)) --j;
    if (j < 0 || !full || (s.flags & RG_SESSION_NO_FUSION)) continue;
    const int pk = s.ops[(size_t)j].kind;
    if (pk == RG_LAYER_SOFTMAX && op.kind == RG_LAYER_CONV2D) continue;
    if (pk == RG_LAYER_LINEAR || pk == RG_LAYER_CONV2D || pk == RG_LAYER_MAXPOOL2D ||
        pk == RG_LAYER_ACTIVATION || pk == RG_LAYER_SOFTMAX || pk == RG_LAYER_RESIDUAL_END ||
        pk == RG_LAYER_ADAPTIVE_AVGPOOL2D || pk == RG_LAYER_EMBEDDING || pk == RG_LAYER_RMSNORM ||
        pk == RG_LAYER_ATTENTION || pk == RG_LAYER_SWIGLU)
      P.amax_src[i] = j;
  }
  P.total_slots = off;
  P.amax2_src.assign(n, -1);
  P.amax2_for.assign(n, -1);
  for (size_t i = 0; i < n; ++i) {
    const Op& op = s.ops[i];
    if (op.kind != RG_LAYER_SHORTCUT_CONV2D || op.k != 1 || op.pad != 0 || op.stride < 2 ||
        (s.flags & RG_SESSION_NO_FUSION) || s.precision != RG_PREC_INT8)
      continue;
    int depth = 0, b = -1;  // the residual begin that opens the shortcut's block
    for (int j = (int)i - 1; j >= 0 && b < 0; --j) {
      if (s.ops[(size_t)j].kind == RG_LAYER_RESIDUAL_END) ++depth;
      if (s.ops[(size_t)j].kind == RG_LAYER_RESIDUAL_BEGIN) {
        if (depth == 0) b = j;
        else --depth;
      }
    }
    int j = b - 1;
    while (j >= 0 && main_path_noop(s.ops[(size_t)j].kind)) --j;
    if (b < 0 || j < 0 || P.amax2_for[(size_t)j] >= 0) continue;
    P.amax2_src[i] = j;
    P.amax2_for[(size_t)j] = (int)i;
  }
  P.block_start.assign(n, 0);
  P.stem_start.assign(n, 0);
  for (size_t i = 0; i < n && s.precision == RG_PREC_INT8; ++i)
    if (block_at(s, P.shapes, i)) {
      P.block_start[i] = 1;
      i += 3;
    } else if (stem_at(s, P.shapes, i)) {
      P.stem_start[i] = 1;
      ++i;
    }
  P.i8_out.assign(n, -1);
  P.i8_in.assign(n, 0);
  if (s.calibrated) {
    for (size_t i = 0; i < n; ++i) {
      if (s.calib_off[i] < 0) continue;
      P.amax_src[i] = -1;  // frozen scale: the producer computes no absmax for it
      if (s.trace || (s.flags & RG_SESSION_NO_FUSION)) continue;
      int j = (int)i - 1;
      while (j >= 0 && main_path_noop(s.ops[(size_t)j].kind)) --j;
      if (j < 0) continue;
      const Op& c = s.ops[i];
      if (c.kind == RG_LAYER_LINEAR && j >= 3 && P.block_start[(size_t)j - 3] && c.kpad == c.in_f) {
        P.i8_out[(size_t)j - 3] = (int)i;  // the fused block writes the Linear's operand
        P.i8_in[i] = 1;
      } else if ((c.kind == RG_LAYER_ATTENTION || c.kind == RG_LAYER_SWIGLU) &&
                 s.ops[(size_t)j].kind == RG_LAYER_RMSNORM) {
        P.i8_out[(size_t)j] = (int)i;      // RMSNorm writes the block's projection operand
        P.i8_in[i] = 1;
      }
    }
  }
  return RG_OK;
}

static int find_consumer(const Session& s, size_t j) {
  if (s.ops[j].kind == RG_LAYER_SHORTCUT_CONV2D) return -1;  // its output feeds the residual add
  for (size_t i = j + 1; i < s.ops.size(); ++i) {
    if (main_path_noop(s.ops[i].kind)) continue;
    const int32_t k = s.ops[i].kind;
    if (k == RG_LAYER_LINEAR || k == RG_LAYER_CONV2D || k == RG_LAYER_ATTENTION || k == RG_LAYER_SWIGLU)
      return (int)i;
    return -1;
  }
  return -1;
}

template <class T>
static rg_status d2h_vec(std::vector<T>& v, const void* src, int64_t n, cudaStream_t st) {
  v.resize((size_t)std::max<int64_t>(n, 0));
  if (n > 0) RG_CUDA_TRY(cudaMemcpyAsync(v.data(), src, (size_t)n * sizeof(T), cudaMemcpyDeviceToHost, st));
  RG_CUDA_TRY(cudaStreamSynchronize(st));
  return RG_OK;
}

// Host input fed in chunks: when the program starts with a fused conv block (whose
// quantization is per image), the input copy is split along the batch on the copy
// stream and the block runs on each chunk as soon as it has landed, so the PCIe
// transfer overlaps the block; the ops after the block run once on the whole batch.
struct HostFeed {
  const float* x = nullptr;  // host input, nullptr: x_dev already holds the input
  int64_t chunk = 0;         // images per chunk
};
constexpr int64_t kFeedMinChunk = 2048;  // images; smaller chunks underfill the GPU
constexpr int kFeedMaxChunks = 8;

// Host output drained in chunks: when the program ends with a Linear on the tensor-core
// GEMM and the caller's output is page-locked host memory, the GEMM runs in row chunks
// and each chunk's device-to-host copy starts on the copy stream as soon as that chunk
// is written, so the PCIe transfer overlaps the rest of the GEMM.  Rows are independent
// in the GEMM, so the output is the same as one launch's.
struct HostDrain {
  float* y = nullptr;  // page-locked host output, nullptr: no drain
  bool done = false;   // the last op copied its output (drain_done marks the end)
};
constexpr int kDrainChunks = 8;
constexpr int64_t kDrainMinBytes = 64ll << 20;

static rg_status gemm_tc_drained(Session& s, const GemmArgs& g, HostDrain& d, cudaStream_t st, int32_t& launches) {
  const int64_t step = round_up((g.m + kDrainChunks - 1) / kDrainChunks, 128);
  int c = 0;
  for (int64_t r0 = 0; r0 < g.m; r0 += step, ++c) {
    GemmArgs gc = g;
    gc.m = std::min<int64_t>(step, g.m - r0);
    gc.a = g.a + r0 * g.lda;
    gc.out = g.out + r0 * g.n;
    if (!launch_gemm_tc(gc, s.num_sms, st)) {
      // copies of earlier chunks may still be writing the caller's buffer: let them end first
      cudaStreamSynchronize(s.copy_stream);
      return fail(RG_ERR_CUDA, "TMA descriptor encoding failed");
    }
    ++launches;
    RG_CUDA_TRY(cudaEventRecord(s.drain_events[(size_t)c], st));
    RG_CUDA_TRY(cudaStreamWaitEvent(s.copy_stream, s.drain_events[(size_t)c], 0));
    RG_CUDA_TRY(cudaMemcpyAsync(d.y + r0 * g.n, gc.out, (size_t)(gc.m * g.n) * 4, cudaMemcpyDeviceToHost,
                                s.copy_stream));
  }
  RG_CUDA_TRY(cudaEventRecord(s.drain_done, s.copy_stream));
  d.done = true;
  return RG_OK;
}

// Whether every row chunk of g would take the tensor-core GEMM.
static bool drain_eligible(const GemmArgs& g) {
  const int64_t step = round_up((g.m + kDrainChunks - 1) / kDrainChunks, 128);
  if (g.m < 2 * step || g.amax.ptr || g.acc) return false;
  GemmArgs first = g, tail = g;
  first.m = step;
  tail.m = g.m - (g.m - 1) / step * step;
  return gemm_tc_eligible(first) && gemm_tc_eligible(tail);
}

static bool feed_chunked(const Session& s, const RunPlan& P) {
  return !s.ops.empty() && P.block_start[0] && !s.trace && P.shapes[0].in[0] >= 2 * kFeedMinChunk;
}

// The GEMM of one INT8 Linear inside an extension op on its quantized operand q
// [rows, lin.kpad] with activation scale *a_scale; out is [rows, lin.out_f] f32, its
// absmax optionally sent to `sink`.
static rg_status run_gemm_q(Session& s, const Op& lin, const int8_t* q, int64_t rows, const float* a_scale, float* out,
                            AmaxSink sink, cudaStream_t st, int32_t& launches) {
  GemmArgs g;
  g.a = q; g.lda = lin.kpad;
  g.m = rows; g.n = lin.out_f; g.k = lin.kpad;
  g.w = lin.d_w.as<int8_t>(); g.ldb = lin.kpad;
  g.a_scale = a_scale;
  g.w_scale = lin.w_scale;
  g.w_scale_ch = lin.w_scale_ch.empty() ? nullptr : lin.d_wsc.as<float>();
  g.bias = lin.d_bias.as<float>();
  g.act = RG_ACT_NONE;
  g.out = out;
  g.amax = sink;
  g.err = s.errw.as<int>();
  g.wait_ns = g_tc_wait_ns.load();
  g.starve = g_tc_starve.load();
  const bool tc = gemm_tc_eligible(g);
  const bool narrow = !tc && gemm_narrow_eligible(g);
  if (tc) {
    if (!launch_gemm_tc(g, s.num_sms, st)) return fail(RG_ERR_CUDA, "%s: TMA descriptor encoding failed", lin.label.c_str());
    s.used_tc = true;
  } else if (narrow) {
    launch_gemm_narrow(g, st);
  } else {
    launch_gemm_simt(g, st);
  }
  ++launches;
  RG_LAUNCHED(tc ? "gemm_tc" : narrow ? "gemm_narrow" : "gemm_simt");
  return RG_OK;
}

// One INT8 Linear inside an extension op: the f32 input quantized with the per-tensor
// scale of absmax *am (first taken as the max over all ranks), then the GEMM.
static rg_status run_inner_linear(Session& s, const Op& lin, const float* src, int64_t rows, unsigned* am,
                                  float* sc, float* out, AmaxSink sink, cudaStream_t st, int32_t& launches) {
  if (s.comm && s.world > 1) RG_NCCL_TRY(ncclAllReduce(am, am, 1, ncclUint32, ncclMax, s.comm, st));
  int8_t* q = s.qbuf.as<int8_t>();
  launch_quantize_rows(src, rows, lin.in_f, lin.kpad, am, q, sc, st);
  ++launches;
  RG_LAUNCHED("quantize_rows");
  return run_gemm_q(s, lin, q, rows, sc, out, sink, st, launches);
}

// A program of exactly two INT8 Linears with dynamic per-tensor quantization runs as one
// cooperative kernel (launch_mlp2) when both are narrow; anything else op by op.
static bool mlp2_program(const Session& s, const RunPlan& P) {
  if (s.ops.size() != 2 || s.precision != RG_PREC_INT8 || s.trace || s.calibrated || (s.comm && s.world > 1) ||
      (s.flags & RG_SESSION_NO_FUSION))
    return false;
  const Op& a = s.ops[0];
  const Op& b = s.ops[1];
  return a.kind == RG_LAYER_LINEAR && b.kind == RG_LAYER_LINEAR && a.w_scale_ch.empty() && b.w_scale_ch.empty() &&
         b.in_f == a.out_f && P.amax_src[0] < 0;
}

// Runs the program on device buffers. x_dev is read only (with a HostFeed it is
// the staging buffer the feed fills); the output is left in y_dev or one of the
// session's activation buffers.
static rg_status execute(Session& s, const float* x_dev, const RunPlan& P, float* y_dev, cudaStream_t st,
                         bool record_events, const HostFeed& feed = HostFeed(), HostDrain* drain = nullptr) {
  const size_t n = s.ops.size();
  int64_t max_elems = 1, max_q = 16, max_ext0 = 0, max_ext1 = 0;
  for (size_t i = 0; i < n; ++i) {
    max_elems = std::max(max_elems, P.shapes[i].out_elems);
    const Op& op = s.ops[i];
    if (op.kind == RG_LAYER_LINEAR) max_q = std::max(max_q, P.shapes[i].in_elems / op.in_f * op.kpad);
    if (op.kind == RG_LAYER_CONV2D || op.kind == RG_LAYER_SHORTCUT_CONV2D) {
      const std::vector<int64_t>& in = P.shapes[i].in;  // NHWC with channels padded to cpad
      // (the fused stem's space-to-depth operand: 16 bytes per 2 x 2 pixels)
      max_q = std::max(max_q, in[0] * in[2] * in[3] * std::max<int64_t>(op.cpad, P.stem_start[i] ? 4 : 0));
      // the space-to-depth operand covers the image rounded up to even sizes
      if (op.dmode == DCONV_S2D) max_q = std::max(max_q, in[0] * ((in[2] + 1) / 2 * 2) * ((in[3] + 1) / 2 * 2) * op.cpad);
    }
    if (op.kind == RG_LAYER_ATTENTION || op.kind == RG_LAYER_SWIGLU) {
      const int64_t rows = P.shapes[i].in_elems / op.in_f;
      for (const Op& l : op.subs) max_q = std::max(max_q, rows * l.kpad);
      max_ext0 = std::max(max_ext0, rows * op.subs[0].out_f);
      max_ext1 = std::max(max_ext1, rows * op.subs[1].in_f);
    }
  }
  if (max_ext0) {
    RG_TRY(s.ext0.ensure((size_t)max_ext0 * 4));
    RG_TRY(s.ext1.ensure((size_t)max_ext1 * 4));
  }
  bool residual = false;
  for (size_t i = 0; i < n; ++i) residual = residual || s.ops[i].kind == RG_LAYER_RESIDUAL_BEGIN;
  RG_TRY(s.act0.ensure((size_t)max_elems * 4));
  RG_TRY(s.act1.ensure((size_t)max_elems * 4));
  if (residual) {  // saved block inputs (and shortcut outputs) stay live across main-path ops
    RG_TRY(s.act2.ensure((size_t)max_elems * 4));
    RG_TRY(s.act3.ensure((size_t)max_elems * 4));
  }
  float* pool[4] = {s.act0.as<float>(), s.act1.as<float>(), residual ? s.act2.as<float>() : nullptr,
                    residual ? s.act3.as<float>() : nullptr};
  std::vector<const float*> saved;  // residual block inputs, innermost last
  auto pick_dst = [&](const float* avoid) -> float* {
    for (float* b : pool) {
      if (!b || b == avoid) continue;
      bool busy = false;
      for (const float* v : saved) busy = busy || v == b;
      if (!busy) return b;
    }
    return nullptr;
  };
  RG_TRY(s.qbuf.ensure((size_t)round_up(max_q, 16) + 64));
  RG_TRY(s.amax.ensure((size_t)std::max<int64_t>(P.total_slots, 1) * 4));
  RG_TRY(s.scales.ensure((size_t)std::max<int64_t>(P.total_slots, 1) * 4));
  if (P.cov_bytes) RG_TRY(s.covbuf.ensure(P.cov_bytes));
  if (s.trace) {
    int64_t max_acc = 1;
    for (size_t i = 0; i < n; ++i)
      if (s.ops[i].kind == RG_LAYER_LINEAR || s.ops[i].kind == RG_LAYER_CONV2D)
        max_acc = std::max(max_acc, P.shapes[i].out_elems);
    RG_TRY(s.accbuf.ensure((size_t)max_acc * 4));
    s.traces.assign(n, TraceRec());
  }
  if (s.events.size() < n + 1) {
    for (cudaEvent_t e : s.events) cudaEventDestroy(e);
    s.events.assign(n + 1, nullptr);
    for (auto& e : s.events) RG_CUDA_TRY(cudaEventCreate(&e));
  }
  unsigned* amax = s.amax.as<unsigned>();
  float* scales = s.scales.as<float>();
  RG_CUDA_TRY(cudaMemsetAsync(amax, 0, (size_t)std::max<int64_t>(P.total_slots, 1) * 4, st));
  // coverage masks of strided convs
  std::vector<const uint8_t*> rc(n, nullptr), cc(n, nullptr);
  if (P.cov_bytes) {
    std::vector<uint8_t> host;
    for (size_t i = 0; i < n; ++i) {
      if (P.rowcov[i].empty() || (all_covered(P.rowcov[i]) && all_covered(P.colcov[i]))) continue;
      rc[i] = s.covbuf.as<uint8_t>() + host.size();
      host.insert(host.end(), P.rowcov[i].begin(), P.rowcov[i].end());
      cc[i] = s.covbuf.as<uint8_t>() + host.size();
      host.insert(host.end(), P.colcov[i].begin(), P.colcov[i].end());
    }
    RG_CUDA_TRY(cudaMemcpyAsync(s.covbuf.p, host.data(), host.size(), cudaMemcpyHostToDevice, st));
  }

  RG_PENDING("the first launch");
  bool fused_residual = false;
  int absorbed = 0;  // ops after a conv that ran inside it (an activation, a 2 x 2 max-pool)
  std::vector<uint8_t> amax2_done(n, 0);  // a shortcut's absmax came from its block input's producer
  const float* cur = x_dev;
  int32_t launches = 0;
  s.ev_of.assign(n + 1, 0);
  int next_ev = 1;
  // inside a graph capture an event record must be external to be timed afterwards
  auto record = [&](cudaEvent_t e) {
    return s.capturing ? cudaEventRecordWithFlags(e, st, cudaEventRecordExternal) : cudaEventRecord(e, st);
  };
  if (record_events) RG_CUDA_TRY(record(s.events[0]));
  for (size_t i = 0; i < n; ++i) {
    const Op& op = s.ops[i];
    const OpShape& os = P.shapes[i];
    const bool last = i + 1 == n;
    if (op.kind == RG_LAYER_RESIDUAL_BEGIN) {  // the block input stays where it is
      saved.push_back(cur);
      if (s.trace) RG_TRY(d2h_vec(s.traces[i].out, cur, os.out_elems, st));
      s.ev_of[i + 1] = s.ev_of[i];
      continue;
    }
    float* dst = pick_dst(op.kind == RG_LAYER_SHORTCUT_CONV2D ? saved.back() : cur);
    if (!dst) return fail(RG_ERR_UNSUPPORTED, "op %zu: residual blocks nested too deeply", i);
    if (last && y_dev) dst = y_dev;
    // absmax sink for the consumer of this op's output
    AmaxSink sink;
    const int cons = find_consumer(s, i);
    if (cons >= 0 && P.amax_src[(size_t)cons] == (int)i) {
      sink.ptr = amax + P.amax_off[(size_t)cons];
      const int64_t imgs = P.shapes[(size_t)cons].in[0];
      sink.elems_per_slot = (s.ops[(size_t)cons].kind == RG_LAYER_CONV2D && imgs > 0)
                                ? P.shapes[(size_t)cons].in_elems / imgs
                                : 0;
    }
    if (i == 0 && os.in_elems > 0 && mlp2_program(s, P)) {
      // both Linears in one kernel; its time is recorded on the first op
      const Op& l2 = s.ops[1];
      Mlp2Args ma;
      ma.x = cur; ma.m = os.in_elems / op.in_f;
      ma.k1 = op.in_f; ma.kpad1 = (int32_t)op.kpad; ma.n1 = op.out_f;
      ma.kpad2 = (int32_t)l2.kpad; ma.n2 = l2.out_f;
      ma.w1 = op.d_w.as<int8_t>(); ma.w2 = l2.d_w.as<int8_t>();
      ma.w1_scale = op.w_scale; ma.w2_scale = l2.w_scale;
      ma.b1 = op.d_bias.as<float>(); ma.b2 = l2.d_bias.as<float>();
      ma.act1 = op.act; ma.act2 = l2.act; ma.p1 = op.param; ma.p2 = l2.param;
      float* out = y_dev ? y_dev : dst;
      ma.y = out;
      // the absmaxes land in the ops' own slots, where a calibration run reads them
      ma.amax1 = amax + P.amax_off[0];
      ma.amax2 = amax + P.amax_off[1];
      ma.err = s.errw.as<int>();
      RG_TRY(s.mlpws.ensure(4 * sizeof(unsigned)));
      if (mlp2_eligible(ma) && launch_mlp2(ma, s.mlpws.as<unsigned>(), st)) {
        ++launches;
        RG_LAUNCHED("mlp2");
        RG_CUDA_TRY(cudaGetLastError());
        s.used_tc = true;  // (its error word is read after the run, as the tensor-core kernels')
        cur = out;
        if (record_events) RG_CUDA_TRY(record(s.events[(size_t)next_ev]));
        s.ev_of[1] = next_ev++;
        s.ev_of[2] = s.ev_of[1];
        break;
      }
      (void)cudaGetLastError();  // a refused cooperative launch leaves a (non-sticky) error: op by op instead
    }
    // The fused kernel bulk-copies images, so its input must start on a 16-byte
    // boundary; a caller's unaligned view takes the op-by-op path instead.
    if (P.block_start[i] && os.in_elems > 0 && (reinterpret_cast<uintptr_t>(cur) & 15) == 0) {
      // Conv-Pool-Conv-Pool in one kernel; its time is recorded on the first op.
      const Op& c2 = s.ops[i + 2];
      const OpShape& last_os = P.shapes[i + 3];
      ConvBlockArgs cb;
      cb.x = cur; cb.n = os.in[0]; cb.c0 = (int32_t)os.in[1]; cb.c1 = op.out_c; cb.c2 = c2.out_c;
      cb.h = (int32_t)os.in[2]; cb.w = (int32_t)os.in[3];
      cb.w1 = op.d_w.as<int8_t>(); cb.kpad1 = (int32_t)op.kpad; cb.w2 = c2.d_w.as<int8_t>(); cb.kpad2 = (int32_t)c2.kpad;
      cb.w1_scale = op.w_scale; cb.w2_scale = c2.w_scale; cb.b1 = op.d_bias.as<float>(); cb.b2 = c2.d_bias.as<float>();
      cb.act1 = op.act; cb.act2 = c2.act; cb.p1 = op.param; cb.p2 = c2.param;
      float* bdst = (i + 3 + 1 == n && y_dev) ? y_dev : dst;
      cb.out = bdst;
      cb.err = s.errw.as<int>();
      if (P.i8_out[i] >= 0) {  // calibrated: the block writes the next Linear's i8 operand
        cb.out_q = s.qbuf.as<int8_t>();
        cb.q_scale = s.d_calib.as<float>() + s.calib_off[(size_t)P.i8_out[i]];
      }
      const int bcons = find_consumer(s, i + 3);
      if (bcons >= 0 && P.amax_src[(size_t)bcons] == (int)(i + 3)) {
        cb.amax = amax + P.amax_off[(size_t)bcons];
        cb.amax_per_image = s.ops[(size_t)bcons].kind == RG_LAYER_CONV2D ? 1 : 0;
      }
      if (i == 0 && feed.x) {
        // chunked host input: copy chunk c on the copy stream, run the block on it
        const int64_t img_in = os.in_elems / cb.n, img_out = last_os.out_elems / cb.n;
        float* xs = const_cast<float*>(cur);
        int c = 0;
        for (int64_t off = 0; off < cb.n; off += feed.chunk, ++c) {
          const int64_t cnt = std::min<int64_t>(feed.chunk, cb.n - off);
          RG_CUDA_TRY(cudaMemcpyAsync(xs + off * img_in, feed.x + off * img_in, (size_t)(cnt * img_in) * 4,
                                      cudaMemcpyHostToDevice, s.copy_stream));
          RG_CUDA_TRY(cudaEventRecord(s.chunk_events[(size_t)c], s.copy_stream));
          RG_CUDA_TRY(cudaStreamWaitEvent(st, s.chunk_events[(size_t)c], 0));
          ConvBlockArgs cc = cb;
          cc.x = xs + off * img_in;
          cc.n = cnt;
          cc.out = bdst + off * img_out;
          if (cb.out_q) cc.out_q = cb.out_q + off * img_out;
          if (cb.amax && cb.amax_per_image) cc.amax = cb.amax + off;
          launch_convblock(cc, s.num_sms, st);
          ++launches;
          RG_LAUNCHED("convblock");
        }
      } else {
        launch_convblock(cb, s.num_sms, st);
        ++launches;
        RG_LAUNCHED("convblock");
      }
      s.used_tc = true;
      cur = bdst;
      (void)last_os;
      if (record_events) RG_CUDA_TRY(record(s.events[(size_t)next_ev]));
      s.ev_of[i + 1] = next_ev++;
      for (size_t j = i + 2; j <= i + 4; ++j) s.ev_of[j] = s.ev_of[i + 1];
      i += 3;
      continue;
    }
    if (P.stem_start[i] && os.in_elems > 0) {
      // Conv(7x7 / 2) + act + MaxPool(3, 2) in one kernel; its time is recorded on the conv.
      const Op& mp = s.ops[i + 1];
      unsigned* my_amax = amax + P.amax_off[i];
      float* my_scale = scales + P.amax_off[i];
      const int64_t N = os.in[0];
      const int32_t C = (int32_t)os.in[1], H = (int32_t)os.in[2], W = (int32_t)os.in[3];
      if (P.amax_src[i] < 0) {
        launch_image_absmax(cur, N, C, H, W, rc[i], cc[i], my_amax, st);
        ++launches;
        RG_LAUNCHED("image_absmax");
      }
      int8_t* q = s.qbuf.as<int8_t>();
      if (s.qbuf.bytes < (size_t)(N * H * W * 4))
        return fail(RG_ERR_UNSUPPORTED, "op %zu: the quantized-operand buffer is too small for the stem", i);
      launch_image_quantize_s2d(cur, N, C, H, W, my_amax, q, my_scale, st);
      ++launches;
      RG_LAUNCHED("image_quantize_s2d");
      StemPoolArgs sp;
      sp.q = q; sp.n = N; sp.h = H; sp.w = W;
      sp.wd = op.d_ws.as<int8_t>();
      sp.a_scale = my_scale; sp.w_scale = op.w_scale;
      sp.w_scale_ch = op.w_scale_ch.empty() ? nullptr : op.d_wsc.as<float>();
      sp.bias = op.d_bias.as<float>();
      sp.act = op.act; sp.act_param = op.param;
      sp.out = (i + 2 == n && y_dev) ? y_dev : dst;
      sp.err = s.errw.as<int>();
      const int pcons = find_consumer(s, i + 1);
      if (pcons >= 0 && P.amax_src[(size_t)pcons] == (int)(i + 1)) {
        sp.amax.ptr = amax + P.amax_off[(size_t)pcons];
        const int64_t imgs = P.shapes[(size_t)pcons].in[0];
        sp.amax.elems_per_slot = (s.ops[(size_t)pcons].kind == RG_LAYER_CONV2D && imgs > 0)
                                     ? P.shapes[(size_t)pcons].in_elems / imgs
                                     : 0;
      }
      if (!launch_stem_pool(sp, s.num_sms, st))
        return fail(RG_ERR_CUDA, "op %zu: the fused stem could not be launched", i);
      ++launches;
      RG_LAUNCHED("stem_pool");
      s.used_tc = true;
      cur = sp.out;
      (void)mp;
      if (record_events) RG_CUDA_TRY(record(s.events[(size_t)next_ev]));
      s.ev_of[i + 1] = next_ev++;
      s.ev_of[i + 2] = s.ev_of[i + 1];
      i += 1;
      continue;
    }
    if (os.in_elems == 0 || os.out_elems == 0) {  // empty batch: nothing to launch
      if (s.trace) s.traces[i] = TraceRec();
      if (op.kind == RG_LAYER_RESIDUAL_END) saved.pop_back();
      if (op.kind == RG_LAYER_SHORTCUT_CONV2D) {
        saved.back() = dst;
      } else if (op.kind != RG_LAYER_FLATTEN) {
        cur = dst;
      }
      s.ev_of[i + 1] = s.ev_of[i];
      continue;
    }
    switch (op.kind) {
      case RG_LAYER_LINEAR:
      case RG_LAYER_CONV2D:
      case RG_LAYER_SHORTCUT_CONV2D: {
        const bool shortcut = op.kind == RG_LAYER_SHORTCUT_CONV2D;
        fused_residual = false;
        if (s.precision != RG_PREC_INT8) {  // fp16_gemm_fused_into (npu.rs:431-445) or the f32 matmul
          Fp16Args f;
          f.f32 = s.precision == RG_PREC_F32 ? 1 : 0;
          f.x = shortcut ? saved.back() : cur;
          f.wt = op.d_wh.as<float>();
          f.bias = op.d_bias.as<float>();
          f.out = dst;
          f.act = op.act; f.act_param = op.param;
          f.exact = op.wh_exact ? 1 : 0;
          if (op.kind == RG_LAYER_LINEAR) {
            f.m = os.in_elems / op.in_f; f.n = op.out_f; f.k = op.in_f;
          } else {
            f.conv = 1;
            f.c = op.in_c; f.h = (int32_t)os.in[2]; f.w = (int32_t)os.in[3];
            f.ks = op.k; f.stride = op.stride; f.pad = op.pad;
            f.oh = (int32_t)os.out[2]; f.ow = (int32_t)os.out[3];
            f.m = os.in[0] * os.out[2] * os.out[3]; f.n = op.out_c; f.k = (int64_t)op.in_c * op.k * op.k;
          }
          // a conv followed by MaxPool2d(2, 2) (in the f32 provider with the standalone
          // activation between them) writes the pooled map directly
          int absorb = 0;
          if (op.kind == RG_LAYER_CONV2D && !s.trace && !(s.flags & RG_SESSION_NO_FUSION) && os.out[2] >= 2 &&
              os.out[3] >= 2) {
            size_t j = i + 1;
            int32_t pact = op.act;
            float pprm = op.param;
            if (f.f32 && j < n && s.ops[j].kind == RG_LAYER_ACTIVATION) {
              pact = s.ops[j].act;
              pprm = s.ops[j].param;
              ++j;
            }
            if (j < n && s.ops[j].kind == RG_LAYER_MAXPOOL2D && s.ops[j].k == 2 && s.ops[j].stride == 2) {
              f.pool = 1;
              f.act = pact; f.act_param = pprm;
              f.ph = (int32_t)(os.out[2] / 2);
              f.pw = (int32_t)(os.out[3] / 2);
              f.m = os.in[0] * f.ph * f.pw * 4;
              if (j + 1 == n && y_dev) f.out = dst = y_dev;
              absorb = (int)(j - i);
            }
          }
          if (!launch_fp16_gemm(f, st))
            return fail(RG_ERR_UNSUPPORTED, "op %zu: FP16 conv beyond the kernel's limits (C*k*k = %lld > 16384, "
                        "an image of 2^31 elements, or 2^31 output pixels in the batch)", i, (long long)f.k);
          ++launches;
          RG_LAUNCHED("fp16_gemm");
          if (shortcut) {
            saved.back() = dst;
            if (s.trace) RG_TRY(d2h_vec(s.traces[i].out, dst, os.out_elems, st));
          } else {
            cur = dst;
          }
          absorbed = absorb;
          break;
        }
        bool use3 = false;
        int dmode = -1;                  // direct-conv mode and its operand grid / channels
        int32_t d_h = 0, d_w = 0, d_cp = 0;
        const float* src = shortcut ? saved.back() : cur;
        unsigned* my_amax = amax + P.amax_off[i];
        float* my_scale = scales + P.amax_off[i];
        int8_t* q = s.qbuf.as<int8_t>();
        GemmArgs g;
        g.err = s.errw.as<int>();
        g.wait_ns = g_tc_wait_ns.load();
        g.starve = g_tc_starve.load();
        bool fused_q = false;
        // a calibrated Linear's frozen activation scale (device), else null
        const float* frozen = s.calibrated && s.calib_off[i] >= 0 ? s.d_calib.as<float>() + s.calib_off[i] : nullptr;
        if (op.kind == RG_LAYER_LINEAR && frozen) {
          const int64_t rows = os.in_elems / op.in_f;
          g.conv = false;
          g.m = rows; g.n = op.out_f; g.k = op.kpad;
          g.rows_per_scale = 0;
          g.out_l = 0;
          g.a = q; g.lda = op.kpad;
          if (!P.i8_in[i]) {  // (else its producer wrote the operand)
            // narrow layers quantize the f32 input with the frozen scale while loading it
            GemmArgs gf = g;
            gf.a = nullptr; gf.af = cur; gf.af_k = op.in_f; gf.af_scale = frozen;
            gf.w = op.d_w.as<int8_t>(); gf.ldb = op.kpad; gf.amax = sink;
            fused_q = !s.trace && gemm_narrow_eligible(gf);
            if (fused_q) {
              g.a = nullptr; g.af = cur; g.af_k = op.in_f; g.af_scale = frozen;
            } else {
              launch_quantize_rows_frozen(cur, rows, op.in_f, op.kpad, frozen, q, st);
              ++launches;
              RG_LAUNCHED("quantize_rows");
            }
          }
        } else if (op.kind == RG_LAYER_LINEAR) {
          const int64_t rows = os.in_elems / op.in_f;
          if (P.amax_src[i] < 0) { launch_absmax(cur, os.in_elems, my_amax, st); ++launches; RG_LAUNCHED("absmax"); }
          if (s.comm && s.world > 1)
            RG_NCCL_TRY(ncclAllReduce(my_amax, my_amax, 1, ncclUint32, ncclMax, s.comm, st));
          g.conv = false;
          g.m = rows; g.n = op.out_f; g.k = op.kpad;
          g.rows_per_scale = 0;
          g.out_l = 0;
          // Narrow layers read the f32 activation and quantize it while loading (one
          // launch, one pass); trace runs keep the separate quantizer (they record A_q).
          GemmArgs gf = g;
          gf.af = cur; gf.af_k = op.in_f; gf.af_amax = my_amax;
          gf.w = op.d_w.as<int8_t>(); gf.ldb = op.kpad; gf.amax = sink;
          fused_q = !s.trace && gemm_narrow_eligible(gf);
          if (fused_q) {
            g.af = cur; g.af_k = op.in_f; g.af_amax = my_amax;
          } else {
            launch_quantize_rows(cur, rows, op.in_f, op.kpad, my_amax, q, my_scale, st);
            ++launches;
            RG_LAUNCHED("quantize_rows");
            g.a = q; g.lda = op.kpad;
          }
        } else {
          const int64_t N = os.in[0];
          const int32_t C = op.in_c, H = (int32_t)os.in[2], W = (int32_t)os.in[3];
          if (P.amax_src[i] < 0 && !amax2_done[i]) {
            launch_image_absmax(src, N, C, H, W, rc[i], cc[i], my_amax, st);
            ++launches;
            RG_LAUNCHED("image_absmax");
          }
          const int32_t OH = (int32_t)os.out[2], OW = (int32_t)os.out[3];
          // The direct kernel reads 16-channel chunk planes of an operand whose grid is the
          // output grid: the image (3x3 / stride 1), its 2x2 pixel blocks (3x3 / stride 2,
          // even sizes), or the pixels a 1x1 conv reads.  Every other conv: NHWC, implicit GEMM.
          if (op.dmode >= 0 && op.d_w3.p && !s.trace && N <= 65535) {
            int32_t dh = OH, dw = OW, dcp = op.cpad;
            bool ok = true;
            if (op.dmode == DCONV_3X3) {
              ok = OH == H && OW == W;
            } else if (op.dmode == DCONV_S2D) {
              ok = OH == (H + 1) / 2 && OW == (W + 1) / 2 && rc[i] == nullptr;
              dcp = 4 * op.cpad;
            }
            if (ok && dconv_shape_ok(op.dmode, N, dh, dw, dcp, op.out_c)) {
              dmode = op.dmode;
              d_h = dh; d_w = dw; d_cp = dcp;
            }
          }
          use3 = dmode >= 0;
          // a strided 1x1 / pad 0 conv reads every s-th row and column: only those pixels
          // are quantized, into a compact operand, and the conv runs as a 1x1 / stride 1
          // conv over it
          const bool sub = op.k == 1 && op.pad == 0 && op.stride > 1 && !s.trace && (op.cpad & 15) == 0 &&
                           N <= 65535;
          const bool bounded = rc[i] == nullptr;  // the absmax covers every pixel quantized
          if (dmode == DCONV_S2D)
            launch_image_quantize_s2d_planar(src, N, C, H, W, op.cpad, my_amax, q, my_scale, st);
          else if (sub)
            launch_image_quantize_subsampled(src, N, C, H, W, op.stride, OH, OW, op.cpad, use3, my_amax, q, my_scale,
                                             st);
          else if (use3)
            launch_image_quantize_planar16(src, N, C, H, W, op.cpad, bounded, my_amax, q, my_scale, st);
          else
            launch_image_quantize_nhwc(src, N, C, H, W, op.cpad, bounded, my_amax, q, my_scale, st);
          ++launches;
          RG_LAUNCHED("image_quantize");
          g.a = q; g.conv = true;
          // padded channels hold zeros in both operands: the reduction runs over cpad per tap
          g.g.h = sub ? (int32_t)os.out[2] : H; g.g.w = sub ? (int32_t)os.out[3] : W;
          g.g.c = op.cpad; g.g.cpad = op.cpad; g.g.k = op.k; g.g.kxp = op.kxp;
          g.g.stride = sub ? 1 : op.stride;
          g.g.pad = op.pad;
          g.g.oh = (int32_t)os.out[2]; g.g.ow = (int32_t)os.out[3];
          const int64_t L = os.out[2] * os.out[3];
          g.m = N * L; g.n = op.out_c; g.k = op.kpad;
          g.rows_per_scale = L;
          g.out_l = L;
        }
        g.w = op.d_w.as<int8_t>(); g.ldb = op.kpad;
        g.a_scale = frozen ? frozen : my_scale;
        g.w_scale = op.w_scale;
        g.w_scale_ch = op.w_scale_ch.empty() ? nullptr : op.d_wsc.as<float>();
        g.bias = op.d_bias.as<float>();
        g.act = op.act; g.act_param = op.param;
        g.out = dst;
        g.acc = s.trace ? s.accbuf.as<int32_t>() : nullptr;
        g.amax = sink;
        // A main-path conv right before a residual block's end takes the add (and the
        // block's activation) into its epilogue; the add then launches nothing.
        // A shortcut conv right before the end does the same with the main path as its
        // residual (the f32 add commutes): its output becomes the main path.
        if ((op.kind == RG_LAYER_CONV2D || shortcut) && !s.trace && i + 1 < n &&
            s.ops[i + 1].kind == RG_LAYER_RESIDUAL_END && !saved.empty() &&
            P.shapes[i + 1].in_elems == os.out_elems &&
            (use3 ? dconv_eligible(g, dmode, d_h, d_w, d_cp) : conv_tc_eligible(g)) &&
            (s.ops[i + 1].act == RG_ACT_NONE || s.ops[i + 1].act == RG_ACT_RELU ||
             s.ops[i + 1].act == RG_ACT_LEAKY_RELU)) {
          const Op& re = s.ops[i + 1];
          g.residual = shortcut ? cur : saved.back();
          if (shortcut) {  // the output must not overwrite the main path it adds
            float* d2 = pick_dst(cur);
            if (!d2) return fail(RG_ERR_UNSUPPORTED, "op %zu: residual blocks nested too deeply", i);
            g.out = dst = d2;
          }
          g.res_act = re.act;
          g.res_param = re.param;
          if (i + 2 == n && y_dev) g.out = dst = y_dev;
          AmaxSink rsink;
          const int rcons = find_consumer(s, i + 1);
          if (rcons >= 0 && P.amax_src[(size_t)rcons] == (int)(i + 1)) {
            rsink.ptr = amax + P.amax_off[(size_t)rcons];
            const int64_t imgs = P.shapes[(size_t)rcons].in[0];
            rsink.elems_per_slot = (s.ops[(size_t)rcons].kind == RG_LAYER_CONV2D && imgs > 0)
                                       ? P.shapes[(size_t)rcons].in_elems / imgs
                                       : 0;
          }
          g.amax = rsink;
          fused_residual = true;
        }
        // the absmax of a later strided shortcut over this op's output (its block input)
        const int sc = use3 ? P.amax2_for[fused_residual ? i + 1 : i] : -1;
        if (sc >= 0 && !amax2_done[(size_t)sc] && P.shapes[(size_t)sc].in[2] == os.out[2] &&
            P.shapes[(size_t)sc].in[3] == os.out[3]) {
          g.amax2 = amax + P.amax_off[(size_t)sc];
          g.cov_s = s.ops[(size_t)sc].stride;
          g.cov_oh = (int32_t)P.shapes[(size_t)sc].out[2];
          g.cov_ow = (int32_t)P.shapes[(size_t)sc].out[3];
          amax2_done[(size_t)sc] = 1;
        }
        if (use3 && (!dconv_eligible(g, dmode, d_h, d_w, d_cp) ||
                     !launch_dconv(g, dmode, d_h, d_w, d_cp, op.d_w3.as<int8_t>(), s.num_sms, st)))
          return fail(RG_ERR_CUDA, "op %zu: the direct conv could not be launched", i);
        const bool conv3 = use3;
        const bool conv_tc = !conv3 && g.conv && conv_tc_eligible(g);
        const bool tc = !fused_q && !g.conv && gemm_tc_eligible(g);
        const bool narrow = fused_q || (!tc && !conv_tc && gemm_narrow_eligible(g));
        if (conv3) {
          s.used_tc = true;
        } else if (conv_tc) {
          if (!launch_conv_tc(g, s.num_sms, st)) return fail(RG_ERR_CUDA, "op %zu: TMA descriptor encoding failed", i);
          s.used_tc = true;
        } else if (tc && drain && drain->y && last && op.kind == RG_LAYER_LINEAR && g.out == y_dev && !s.trace &&
                   !s.capturing && drain_eligible(g)) {
          RG_TRY(gemm_tc_drained(s, g, *drain, st, launches));
          --launches;  // counted per chunk
          s.used_tc = true;
        } else if (tc) {
          if (!launch_gemm_tc(g, s.num_sms, st)) return fail(RG_ERR_CUDA, "op %zu: TMA descriptor encoding failed", i);
          s.used_tc = true;
        } else if (narrow) {
          launch_gemm_narrow(g, st);
        } else {
          launch_gemm_simt(g, st);
        }
        ++launches;
        RG_LAUNCHED(conv3 ? "conv3x3" : conv_tc ? "conv_tc" : tc ? "gemm_tc" : narrow ? "gemm_narrow" : "gemm_simt");
        if (s.trace) {
          TraceRec& t = s.traces[i];
          RG_TRY(d2h_vec(t.scales, frozen ? frozen : my_scale, P.amax_slots[i], st));
          RG_TRY(d2h_vec(t.acc, s.accbuf.p, os.out_elems, st));
          if (op.kind == RG_LAYER_LINEAR) {
            const int64_t rows = os.in_elems / op.in_f;
            std::vector<int8_t> tmp;
            RG_TRY(d2h_vec(tmp, q, rows * op.kpad, st));
            t.aq.resize((size_t)(rows * op.in_f));
            for (int64_t r = 0; r < rows; ++r)
              memcpy(&t.aq[(size_t)(r * op.in_f)], &tmp[(size_t)(r * op.kpad)], (size_t)op.in_f);
          } else {
            const int64_t N = os.in[0], C = os.in[1], HW = os.in[2] * os.in[3], CP = op.cpad;
            std::vector<int8_t> tmp;
            RG_TRY(d2h_vec(tmp, q, N * HW * CP, st));
            t.aq.resize((size_t)os.in_elems);
            for (int64_t b = 0; b < N; ++b)
              for (int64_t c = 0; c < C; ++c)
                for (int64_t p = 0; p < HW; ++p) t.aq[(size_t)((b * C + c) * HW + p)] = tmp[(size_t)((b * HW + p) * CP + c)];
          }
        }
        if (shortcut && !fused_residual) {
          saved.back() = dst;  // the shortcut replaces the saved block input
          if (s.trace) RG_TRY(d2h_vec(s.traces[i].out, dst, os.out_elems, st));
        } else {
          cur = dst;
        }
        break;
      }
      case RG_LAYER_RESIDUAL_END:
        launch_residual_add(cur, saved.back(), os.in_elems, op.act, op.param, dst, sink, st);
        ++launches;
        saved.pop_back();
        cur = dst;
        break;
      case RG_LAYER_CHANNEL_AFFINE: {  // f32 provider only (mod.rs:293-303)
        const int64_t c = op.in_f, inner = c > 0 && os.in[0] > 0 ? os.in_elems / (os.in[0] * c) : 0;
        launch_channel_affine(cur, os.in_elems, c, inner, op.d_wh.as<float>(), op.d_bias.as<float>(), dst, st);
        ++launches;
        RG_LAUNCHED("channel_affine");
        cur = dst;
        break;
      }
      case RG_LAYER_ADAPTIVE_AVGPOOL2D:
        launch_adaptive_avgpool(cur, os.in[0], (int32_t)os.in[1], (int32_t)os.in[2], (int32_t)os.in[3], op.k,
                                op.stride, dst, sink, st);
        ++launches;
        cur = dst;
        break;
      case RG_LAYER_MAXPOOL2D:
        launch_maxpool2d(cur, os.in[0], (int32_t)os.in[1], (int32_t)os.in[2], (int32_t)os.in[3], op.k,
                         op.stride, dst, sink, st);
        ++launches;
        cur = dst;
        break;
      case RG_LAYER_FLATTEN:
        if (last && y_dev) {
          RG_CUDA_TRY(cudaMemcpyAsync(y_dev, cur, (size_t)os.out_elems * 4, cudaMemcpyDeviceToDevice, st));
          cur = y_dev;
        }
        break;
      case RG_LAYER_ACTIVATION:
        launch_activation(cur, os.in_elems, op.act, op.param, dst, sink, st);
        ++launches;
        cur = dst;
        break;
      case RG_LAYER_SOFTMAX: {
        const int64_t lastd = os.in.back();
        launch_softmax(cur, lastd ? os.in_elems / lastd : 0, lastd, dst, sink, st);
        ++launches;
        cur = dst;
        break;
      }
      case RG_LAYER_EMBEDDING:
        launch_embedding(cur, os.in_elems, op.d_ext.as<float>(), op.in_f, op.out_f, dst, sink,
                         s.errw.as<int>() + 1, st);
        ++launches;
        RG_LAUNCHED("embedding");
        s.used_embed = true;
        cur = dst;
        break;
      case RG_LAYER_RMSNORM:
        // mean_dim multiplies the sum by 1/d (tensor/ops.rs:755-758)
        if (P.i8_out[i] >= 0) {  // calibrated: the consumer block's first projection operand
          const size_t c = (size_t)P.i8_out[i];
          RG_TRY(launch_rmsnorm(cur, os.in_elems / op.in_f, op.in_f, op.d_ext.as<float>(), op.param,
                                1.0f / (float)op.in_f, nullptr, AmaxSink(), st, s.qbuf.as<int8_t>(),
                                s.ops[c].subs[0].kpad, s.d_calib.as<float>() + s.calib_off[c]));
        } else {
          RG_TRY(launch_rmsnorm(cur, os.in_elems / op.in_f, op.in_f, op.d_ext.as<float>(), op.param,
                                1.0f / (float)op.in_f, dst, sink, st));
        }
        ++launches;
        RG_LAUNCHED("rmsnorm");
        cur = dst;
        break;
      case RG_LAYER_ATTENTION:
      case RG_LAYER_SWIGLU: {
        unsigned* am = amax + P.amax_off[i];  // [0]: the op's input, [1]: the inner activation
        float* sc = scales + P.amax_off[i];
        const int64_t rows = os.in_elems / op.in_f;
        // calibrated: frozen scales fz[0] (the input) and fz[1] (the inner activation)
        const float* fz = s.calibrated ? s.d_calib.as<float>() + s.calib_off[i] : nullptr;
        int8_t* q = s.qbuf.as<int8_t>();
        if (!fz && P.amax_src[i] < 0) { launch_absmax(cur, os.in_elems, am, st); ++launches; RG_LAUNCHED("absmax"); }
        AmaxSink inner;
        inner.ptr = fz ? nullptr : am + 1;
        float* e0 = s.ext0.as<float>();
        float* e1 = s.ext1.as<float>();
        if (fz) {
          if (!P.i8_in[i]) {
            launch_quantize_rows_frozen(cur, rows, op.in_f, op.subs[0].kpad, fz, q, st);
            ++launches;
            RG_LAUNCHED("quantize_rows");
          }
          RG_TRY(run_gemm_q(s, op.subs[0], q, rows, fz, e0, AmaxSink(), st, launches));
        } else {
          RG_TRY(run_inner_linear(s, op.subs[0], cur, rows, am, sc, e0, AmaxSink(), st, launches));
        }
        if (op.kind == RG_LAYER_ATTENTION) {
          const int32_t d = op.in_f, heads = op.out_f, dh = d / heads;
          const float scale = 1.0f / std::sqrt((float)dh);  // attention.rs: mul_scalar(1 / sqrt(dh))
          RG_TRY(launch_attention(e0, 3 * (int64_t)d, os.in[0], (int32_t)os.in[1], heads, dh, scale, e1, d, inner, st));
          ++launches;
          RG_LAUNCHED("attention");
          if (fz) {
            launch_quantize_rows_frozen(e1, rows, d, op.subs[1].kpad, fz + 1, q, st);
            ++launches;
            RG_LAUNCHED("quantize_rows");
          }
        } else if (fz) {  // the gate product written as the down projection's i8 operand
          launch_swiglu_mul(e0, rows, op.out_f, nullptr, AmaxSink(), st, q, op.subs[1].kpad, fz + 1);
          ++launches;
          RG_LAUNCHED("swiglu_mul");
        } else {
          launch_swiglu_mul(e0, rows, op.out_f, e1, inner, st);
          ++launches;
          RG_LAUNCHED("swiglu_mul");
        }
        if (fz) RG_TRY(run_gemm_q(s, op.subs[1], q, rows, fz + 1, dst, sink, st, launches));
        else RG_TRY(run_inner_linear(s, op.subs[1], e1, rows, am + 1, sc + 1, dst, sink, st, launches));
        cur = dst;
        break;
      }
      default:
        return fail(RG_ERR_UNSUPPORTED, "op %zu: unsupported kind %d", i, op.kind);
    }
    RG_CUDA_TRY(cudaGetLastError());
    if (s.trace && op.kind != RG_LAYER_SHORTCUT_CONV2D) RG_TRY(d2h_vec(s.traces[i].out, cur, os.out_elems, st));
    if (op.kind == RG_LAYER_FLATTEN) {
      s.ev_of[i + 1] = s.ev_of[i];  // a reshape: no kernel, no event
    } else {
      if (record_events) RG_CUDA_TRY(record(s.events[(size_t)next_ev]));
      s.ev_of[i + 1] = next_ev++;
    }
    if (fused_residual) {  // the residual end ran inside the conv: 0 ns on its record
      fused_residual = false;
      saved.pop_back();
      s.ev_of[i + 2] = s.ev_of[i + 1];
      ++i;
    }
    for (; absorbed > 0; --absorbed) {  // ops that ran inside the conv: 0 ns on their records
      s.ev_of[i + 2] = s.ev_of[i + 1];
      ++i;
    }
  }
  s.last.launches = launches;
  if (y_dev && cur != y_dev) {
    const int64_t elems = n ? P.shapes.back().out_elems : 0;
    if (elems) RG_CUDA_TRY(cudaMemcpyAsync(y_dev, cur, (size_t)elems * 4, cudaMemcpyDeviceToDevice, st));
  }
  return RG_OK;
}

static rg_status collect_profile(Session& s, const RunPlan& P, bool have_events, int64_t total_ns) {
  const size_t n = s.ops.size();
  s.last.valid = true;
  s.last.macs.assign(n, 0);
  s.last.ns.assign(n, 0);
  s.last.total_macs = 0;
  for (size_t i = 0; i < n; ++i) {
    s.last.macs[i] = P.shapes[i].macs;
    s.last.total_macs += P.shapes[i].macs;
    if (have_events) {
      float ms = 0.0f;
      const int e0 = s.ev_of[i], e1 = s.ev_of[i + 1];
      if (e1 != e0) RG_CUDA_TRY(cudaEventElapsedTime(&ms, s.events[(size_t)e0], s.events[(size_t)e1]));
      s.last.ns[i] = (int64_t)((double)ms * 1e6);
    }
  }
  s.last.total_ns = total_ns;
  return RG_OK;
}

static rg_status check_device(int dev) {
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0)
    return fail(RG_ERR_NO_DEVICE, "no CUDA device visible (%s); this provider has no CPU fallback",
                e == cudaSuccess ? "count 0" : cudaGetErrorString(e));
  if (dev < 0 || dev >= count) return fail(RG_ERR_INVALID_ARG, "device %d out of range (%d visible)", dev, count);
  cudaDeviceProp prop;
  RG_CUDA_TRY(cudaGetDeviceProperties(&prop, dev));
  if (prop.major != 10)
    return fail(RG_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a only", dev, prop.major,
                prop.minor);
  return RG_OK;
}

// ----------------------------------------------------------------------------
// RTIM reader (src/save.rs:227-279)
// ----------------------------------------------------------------------------
struct RtimLayers {
  std::vector<rg_layer_spec> specs;
  std::vector<std::vector<float>> store;
};

static rg_status read_rtim(const char* path, RtimLayers& out) {
  FILE* f = fopen(path, "rb");
  if (!f) return fail(RG_ERR_IO, "cannot open %s", path);
  std::unique_ptr<FILE, int (*)(FILE*)> guard(f, fclose);
  auto rd_u32 = [&](uint32_t& v) -> bool {
    unsigned char b[4];
    if (fread(b, 1, 4, f) != 4) return false;
    v = (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24);
    return true;
  };
  auto rd_f32 = [&](float& v) -> bool {
    uint32_t u;
    if (!rd_u32(u)) return false;
    memcpy(&v, &u, 4);
    return true;
  };
  auto rd_vec = [&](std::vector<float>& v) -> bool {
    uint32_t n;
    if (!rd_u32(n)) return false;
    v.resize(n);
    for (uint32_t i = 0; i < n; ++i)
      if (!rd_f32(v[i])) return false;
    return true;
  };
  char magic[4];
  if (fread(magic, 1, 4, f) != 4 || memcmp(magic, "RTIM", 4) != 0)
    return fail(RG_ERR_IO, "invalid RTIM model header");
  uint32_t count;
  if (!rd_u32(count)) return fail(RG_ERR_IO, "truncated RTIM file");
  out.store.reserve((size_t)count * 2);
  for (uint32_t i = 0; i < count; ++i) {
    uint32_t tag;
    if (!rd_u32(tag)) return fail(RG_ERR_IO, "truncated RTIM file");
    rg_layer_spec l;
    memset(&l, 0, sizeof l);
    l.kind = (int32_t)tag;
    uint32_t a = 0, b = 0, c = 0, d = 0, e = 0;
    bool ok = true;
    switch (tag) {
      case 1:
        ok = rd_u32(a) && rd_u32(b);
        l.in_features = (int32_t)a; l.out_features = (int32_t)b;
        break;
      case 2:
        ok = rd_u32(a) && rd_u32(b) && rd_u32(c) && rd_u32(d) && rd_u32(e);
        l.in_channels = (int32_t)a; l.out_channels = (int32_t)b; l.kernel = (int32_t)c;
        l.stride = (int32_t)d; l.padding = (int32_t)e;
        break;
      case 3: break;
      case 4:
        ok = rd_u32(a) && rd_u32(b);
        l.kernel = (int32_t)a; l.stride = (int32_t)b;
        break;
      case 5: break;
      case 6: {
        float p;
        ok = rd_u32(a) && rd_f32(p);
        if (ok && a > 5) return fail(RG_ERR_IO, "unknown activation tag %u", a);
        l.act = (int32_t)a;
        l.act_param = a == 5 ? p : 0.0f;
        break;
      }
      case 7: break;
      default:
        return fail(RG_ERR_IO, "unknown layer tag %u", tag);
    }
    if (ok && (tag == 1 || tag == 2 || tag == 3)) {
      out.store.emplace_back();
      std::vector<float>& w = out.store.back();
      ok = rd_vec(w);
      out.store.emplace_back();
      std::vector<float>& bb = out.store.back();
      ok = ok && rd_vec(bb);
    }
    if (!ok) return fail(RG_ERR_IO, "truncated RTIM file");
    out.specs.push_back(l);
  }
  // pointers into store (stable after all pushes)
  size_t si = 0;
  for (auto& l : out.specs) {
    if (l.kind == 1 || l.kind == 2 || l.kind == 3) {
      l.weight = out.store[si].data(); l.weight_len = (int64_t)out.store[si].size(); ++si;
      l.bias = out.store[si].data(); l.bias_len = (int64_t)out.store[si].size(); ++si;
    }
  }
  return RG_OK;
}

}  // namespace rg

// ============================================================================
// C ABI
// ============================================================================
using namespace rg;

struct rg_session {
  Session s;
};

// ---- error words of the kernel-level entry points ------------------------------
// A kernel-level call that runs a tensor-core kernel holds one word of this array for
// its duration, taken from a host-side free list per device: concurrent calls never
// share a word, and no call allocates device memory.  The last word is the sink of
// calls recorded in a stream capture (never read).
constexpr int kCallErrSlots = 64;
constexpr int kCallErrDevices = 64;
static __device__ int32_t g_call_err[kCallErrSlots];

struct CallErrPool {
  std::mutex mu;
  std::condition_variable cv;
  int32_t* base[kCallErrDevices] = {};
  uint64_t busy[kCallErrDevices] = {};
};
static CallErrPool g_err_pool;

struct CallErrSlot {
  int32_t* ptr = nullptr;
  int dev = -1, bit = -1;
  // the current device is `device` (its array's address is looked up with it current)
  rg_status acquire(int device, bool capture_sink) {
    if (device < 0 || device >= kCallErrDevices) return fail(RG_ERR_CUDA, "device %d out of range", device);
    std::unique_lock<std::mutex> lock(g_err_pool.mu);
    if (!g_err_pool.base[device]) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_call_err);
      if (e != cudaSuccess) return fail(RG_ERR_CUDA, "error-word array: %s", cudaGetErrorString(e));
      g_err_pool.base[device] = static_cast<int32_t*>(p);
    }
    dev = device;
    if (capture_sink) {
      ptr = g_err_pool.base[device] + (kCallErrSlots - 1);
      return RG_OK;
    }
    constexpr uint64_t kAll = (1ull << (kCallErrSlots - 1)) - 1;  // every word but the sink
    g_err_pool.cv.wait(lock, [&] { return (g_err_pool.busy[device] & kAll) != kAll; });
    bit = __builtin_ctzll(~g_err_pool.busy[device] & kAll);
    g_err_pool.busy[device] |= 1ull << bit;
    ptr = g_err_pool.base[device] + bit;
    return RG_OK;
  }
  ~CallErrSlot() {
    if (bit < 0) return;
    {
      std::lock_guard<std::mutex> lock(g_err_pool.mu);
      g_err_pool.busy[dev] &= ~(1ull << bit);
    }
    g_err_pool.cv.notify_one();
  }
};

extern "C" {

const char* rg_last_error(void) { return g_err.c_str(); }

const char* rg_version(void) { return "rustgears-b200 0.1.0 (sm_100a)"; }

int32_t rg_device_count(void) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  int ok = 0;
  for (int d = 0; d < count; ++d) {
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, d) == cudaSuccess && p.major == 10) ++ok;
  }
  return ok;
}

rg_status rg_session_create(const rg_layer_spec* layers, int32_t n_layers, const rg_session_options* opts,
                            rg_session** out) {
  if (!out || (n_layers > 0 && !layers) || n_layers < 0) return fail(RG_ERR_INVALID_ARG, "null argument");
  *out = nullptr;
  rg_session_options o = {0, RG_PREC_INT8, 0, 0};
  if (opts) o = *opts;
  if (o.precision != RG_PREC_INT8 && o.precision != RG_PREC_FP16 && o.precision != RG_PREC_F32)
    return fail(RG_ERR_INVALID_ARG, "precision %d: not an NpuPrecision or the f32 provider", o.precision);
  RG_TRY(check_device(o.device));
  RG_CUDA_TRY(cudaSetDevice(o.device));
  std::unique_ptr<rg_session> h(new rg_session());
  Session& s = h->s;
  s.device = o.device; s.precision = o.precision; s.weight_quant = o.weight_quant; s.flags = o.flags;
  RG_CUDA_TRY(cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, o.device));
  RG_CUDA_TRY(cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking));
  RG_CUDA_TRY(cudaStreamCreateWithFlags(&s.copy_stream, cudaStreamNonBlocking));
  s.chunk_events.assign(kFeedMaxChunks, nullptr);
  for (auto& e : s.chunk_events) RG_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  s.drain_events.assign(kDrainChunks, nullptr);
  for (auto& e : s.drain_events) RG_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  RG_CUDA_TRY(cudaEventCreateWithFlags(&s.drain_done, cudaEventDisableTiming));
  RG_TRY(s.errw.ensure(2 * sizeof(int)));
  RG_CUDA_TRY(cudaMemset(s.errw.p, 0, 2 * sizeof(int)));
  RG_TRY(compile(s, layers, n_layers));
  // calibration targets: one per Linear input (two per attention / SwiGLU block)
  s.calib_off.assign(s.ops.size(), -1);
  for (size_t i = 0; i < s.ops.size() && s.precision == RG_PREC_INT8; ++i) {
    const int32_t k = s.ops[i].kind;
    if (k != RG_LAYER_LINEAR && k != RG_LAYER_ATTENTION && k != RG_LAYER_SWIGLU) continue;
    s.calib_off[i] = s.calib_targets;
    s.calib_targets += k == RG_LAYER_LINEAR ? 1 : 2;
  }
  *out = h.release();
  return RG_OK;
}

rg_status rg_session_create_from_rtim(const char* path, const rg_session_options* opts, rg_session** out) {
  if (!path || !out) return fail(RG_ERR_INVALID_ARG, "null argument");
  RtimLayers L;
  RG_TRY(read_rtim(path, L));
  return rg_session_create(L.specs.data(), (int32_t)L.specs.size(), opts, out);
}

void rg_session_destroy(rg_session* h) {
  if (!h) return;
  Session& s = h->s;
  cudaSetDevice(s.device);
  if (s.stream) cudaStreamSynchronize(s.stream);
  if (s.copy_stream) cudaStreamSynchronize(s.copy_stream);
  // a captured program holds the communicator's all-reduce nodes: release it first
  if (s.graph.exec) cudaGraphExecDestroy(s.graph.exec);
  s.graph.exec = nullptr;
  if (s.comm) ncclCommDestroy(s.comm);
  for (cudaEvent_t e : s.events) cudaEventDestroy(e);
  for (cudaEvent_t e : s.chunk_events)
    if (e) cudaEventDestroy(e);
  for (cudaEvent_t e : s.drain_events)
    if (e) cudaEventDestroy(e);
  if (s.drain_done) cudaEventDestroy(s.drain_done);
  if (s.t0) cudaEventDestroy(s.t0);
  if (s.t1) cudaEventDestroy(s.t1);
  if (s.stream) cudaStreamDestroy(s.stream);
  if (s.copy_stream) cudaStreamDestroy(s.copy_stream);
  delete h;
}

rg_status rg_session_output_shape(rg_session* h, const int64_t* shape, int32_t ndim, int64_t* y_shape,
                                  int32_t* y_ndim) {
  if (!h || !shape || !y_shape || !y_ndim) return fail(RG_ERR_INVALID_ARG, "null argument");
  std::vector<OpShape> sh;
  RG_TRY(plan_shapes(h->s, shape, ndim, sh));
  const std::vector<int64_t> o = sh.empty() ? std::vector<int64_t>(shape, shape + ndim) : sh.back().out;
  for (size_t i = 0; i < o.size(); ++i) y_shape[i] = o[i];
  *y_ndim = (int32_t)o.size();
  return RG_OK;
}

// The program on device buffers through the session's CUDA graph, capturing it on
// the second identical run (the first sizes every buffer and sets every kernel
// attribute outside the capture).  Returns false when the run is not replayable
// and must go through execute() directly.
static rg_status run_graph(Session& s, const float* xd, const int64_t* shape, int32_t ndim, float* yd,
                           cudaStream_t st, bool events, std::shared_ptr<RunPlan>& P, bool& done) {
  done = false;
  Session::Graph& g = s.graph;
  const std::vector<int64_t> key(shape, shape + ndim);
  if (g.shape == key && g.x == xd && g.y == yd && g.events == events) {
    if (g.exec) {
      RG_CUDA_TRY(cudaGraphLaunch(g.exec, st));
      s.used_tc = s.used_tc || g.used_tc;
      s.used_embed = s.used_embed || g.used_embed;
      s.last.launches = g.launches;
      s.ev_of = g.ev_of;
      P = std::static_pointer_cast<RunPlan>(g.plan);
      done = true;
      return RG_OK;
    }
    if (g.off || ++g.seen < 2) return RG_OK;
  } else {
    if (g.exec) cudaGraphExecDestroy(g.exec);
    g = Session::Graph();
    g.shape = key; g.x = xd; g.y = yd; g.events = events; g.seen = 1;
    return RG_OK;
  }
  // second identical run: capture it
  P = std::make_shared<RunPlan>();
  RG_TRY(make_plan(s, shape, ndim, *P));
  if (P->cov_bytes) {  // (its host-to-device mask copy stays outside graphs)
    g.off = true;
    return RG_OK;
  }
  RG_CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
  s.capturing = true;
  const bool tc0 = s.used_tc, emb0 = s.used_embed;
  s.used_tc = s.used_embed = false;
  rg_status rs = execute(s, xd, *P, yd, st, events);
  s.capturing = false;
  cudaGraph_t graph = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(st, &graph);
  cudaError_t ie = cudaErrorUnknown;
  if (rs == RG_OK && ce == cudaSuccess) ie = cudaGraphInstantiate(&g.exec, graph, 0);
  if (graph) cudaGraphDestroy(graph);
  if (ie != cudaSuccess) {  // not capturable: this run and the next ones go through execute()
    g.exec = nullptr;
    g.off = true;
    s.used_tc = tc0;
    s.used_embed = emb0;
    cudaGetLastError();
    return RG_OK;
  }
  g.used_tc = s.used_tc;
  g.used_embed = s.used_embed;
  g.launches = s.last.launches;
  g.ev_of = s.ev_of;
  g.plan = P;
  s.used_tc = s.used_tc || tc0;
  s.used_embed = s.used_embed || emb0;
  RG_CUDA_TRY(cudaGraphLaunch(g.exec, st));
  done = true;
  return RG_OK;
}

static rg_status run_impl(rg_session* h, const float* x, bool x_host, const int64_t* shape, int32_t ndim, float* y,
                          bool y_host, int64_t y_cap, int64_t* y_shape, int32_t* y_ndim, cudaStream_t user_st,
                          bool async) {
  if (!h || !x || !shape || !y || !y_shape || !y_ndim) return fail(RG_ERR_INVALID_ARG, "null argument");
  Session& s = h->s;
  std::lock_guard<std::mutex> lock(s.mu);
  RG_CUDA_TRY(cudaSetDevice(s.device));
  std::shared_ptr<RunPlan> Pp;
  const bool same_as_graph = !x_host && !y_host && s.graph.exec && s.graph.x == x && s.graph.y == y &&
                             s.graph.shape == std::vector<int64_t>(shape, shape + ndim);
  if (same_as_graph) {
    Pp = std::static_pointer_cast<RunPlan>(s.graph.plan);
  } else {
    Pp = std::make_shared<RunPlan>();
    RG_TRY(make_plan(s, shape, ndim, *Pp));
  }
  const RunPlan& P = *Pp;
  int64_t in_elems = 1;
  for (int32_t i = 0; i < ndim; ++i) in_elems *= shape[i];
  const std::vector<int64_t> oshape = P.shapes.empty() ? std::vector<int64_t>(shape, shape + ndim) : P.shapes.back().out;
  int64_t out_elems = 1;
  for (int64_t d : oshape) out_elems *= d;
  if (out_elems > y_cap) return fail(RG_ERR_INVALID_ARG, "output needs %lld elements, capacity %lld",
                                     (long long)out_elems, (long long)y_cap);
  cudaStream_t st = user_st ? user_st : s.stream;
  const bool async_run = async && !x_host && !y_host && !s.trace;
  const bool events = !(s.flags & RG_SESSION_NO_PROFILE) && !async_run;
  if (events && !s.t0) {
    RG_CUDA_TRY(cudaEventCreate(&s.t0));
    RG_CUDA_TRY(cudaEventCreate(&s.t1));
  }
  if (events) RG_CUDA_TRY(cudaEventRecord(s.t0, st));
  const float* xd = x;
  HostFeed feed;
  if (x_host) {
    RG_TRY(s.xin.ensure((size_t)std::max<int64_t>(in_elems, 1) * 4));
    xd = s.xin.as<float>();
    if (feed_chunked(s, P)) {
      const int64_t batch = P.shapes[0].in[0];
      feed.x = x;
      feed.chunk = std::max<int64_t>(kFeedMinChunk, (batch + kFeedMaxChunks - 1) / kFeedMaxChunks);
      // the copy stream must not overwrite the staging buffer before earlier work on
      // this stream (a previous run's reads of it) is done
      cudaEvent_t ready = s.chunk_events[0];
      RG_CUDA_TRY(cudaEventRecord(ready, st));
      RG_CUDA_TRY(cudaStreamWaitEvent(s.copy_stream, ready, 0));
    } else {
      RG_CUDA_TRY(cudaMemcpyAsync(s.xin.p, x, (size_t)in_elems * 4, cudaMemcpyHostToDevice, st));
    }
  }
  float* yd = y;
  if (y_host) {
    RG_TRY(s.yout.ensure((size_t)std::max<int64_t>(out_elems, 1) * 4));
    yd = s.yout.as<float>();
  }
  rg_status rs = RG_OK;
  bool done = false;
  if (s.ops.empty()) {
    if (in_elems) RG_CUDA_TRY(cudaMemcpyAsync(yd, xd, (size_t)in_elems * 4, cudaMemcpyDeviceToDevice, st));
    done = true;
  } else if (!x_host && !y_host && !s.trace && !(s.flags & RG_SESSION_NO_GRAPH)) {
    // (with a communicator the capture holds the per-Linear max all-reduces too, so a
    // sharded step is one graph launch and host-side skew between ranks stays off it)
    std::shared_ptr<RunPlan> Pg;
    rs = run_graph(s, xd, shape, ndim, yd, st, events, Pg, done);
    if (rs == RG_OK && done && Pg) Pp = Pg;
  }
  HostDrain drain;
  if (y_host && !async_run && (int64_t)out_elems * 4 >= kDrainMinBytes) {
    cudaPointerAttributes pa;
    if (cudaPointerGetAttributes(&pa, y) == cudaSuccess && pa.type == cudaMemoryTypeHost) drain.y = y;
    else cudaGetLastError();  // (an unknown pointer only means: no drain)
  }
  if (rs == RG_OK && !done) rs = execute(s, xd, *Pp, yd, st, events, feed, &drain);
  if (rs != RG_OK) return rs;
  if (drain.done)
    RG_CUDA_TRY(cudaStreamWaitEvent(st, s.drain_done, 0));
  else if (y_host && out_elems)
    RG_CUDA_TRY(cudaMemcpyAsync(y, yd, (size_t)out_elems * 4, cudaMemcpyDeviceToHost, st));
  if (events) RG_CUDA_TRY(cudaEventRecord(s.t1, st));
  for (size_t i = 0; i < oshape.size(); ++i) y_shape[i] = oshape[i];
  *y_ndim = (int32_t)oshape.size();
  if (async_run) return RG_OK;
  RG_CUDA_TRY(cudaStreamSynchronize(st));
  if (s.used_tc || s.used_embed) {
    s.used_tc = s.used_embed = false;
    int32_t e[2] = {0, 0};
    RG_CUDA_TRY(cudaMemcpy(e, s.errw.p, sizeof e, cudaMemcpyDeviceToHost));
    if (e[0] || e[1]) RG_CUDA_TRY(cudaMemset(s.errw.p, 0, sizeof e));
    RG_TRY(rg_status_from_error_words(e));
  }
  int64_t total_ns = 0;
  if (events) {
    float ms = 0;
    RG_CUDA_TRY(cudaEventElapsedTime(&ms, s.t0, s.t1));
    total_ns = (int64_t)((double)ms * 1e6);
  }
  return collect_profile(s, *Pp, events && !s.ops.empty(), total_ns);
}

rg_status rg_session_run(rg_session* h, const float* x, const int64_t* shape, int32_t ndim, float* y, int64_t y_cap,
                         int64_t* y_shape, int32_t* y_ndim) {
  return run_impl(h, x, true, shape, ndim, y, true, y_cap, y_shape, y_ndim, nullptr, false);
}

rg_status rg_session_run_device(rg_session* h, const float* x_dev, const int64_t* shape, int32_t ndim, float* y_dev,
                                int64_t y_cap, int64_t* y_shape, int32_t* y_ndim, void* stream, int32_t flags) {
  return run_impl(h, x_dev, false, shape, ndim, y_dev, false, y_cap, y_shape, y_ndim, (cudaStream_t)stream,
                  (flags & RG_RUN_ASYNC) != 0);
}

rg_status rg_session_compilation_report(rg_session* h, char* buf, int64_t cap, int64_t* needed) {
  if (!h) return fail(RG_ERR_INVALID_ARG, "null session");
  const Session& s = h->s;
  const float ratio = s.npu_bytes == 0 ? 1.0f : (float)s.fp32_bytes / (float)s.npu_bytes;
  char head[512];
  if (s.precision == RG_PREC_F32) {  // CompiledProgram::Standard (mod.rs:200-206)
    snprintf(head, sizeof head, "InferenceSession [provider = CPU (FP32), device = cpu, ops = %zu (from %d raw layers)]",
             s.ops.size(), s.original_layers);
    const std::string r = head;
    if (needed) *needed = (int64_t)r.size() + 1;
    if (buf && cap > 0) {
      const size_t n = std::min<size_t>(r.size(), (size_t)cap - 1);
      memcpy(buf, r.data(), n);
      buf[n] = 0;
    }
    return RG_OK;
  }
  snprintf(head, sizeof head,
           "InferenceSession [provider = NPU (%s), layers: %d -> %zu fused ops, weights: %lld B -> %lld B (%.2fx compression)]\n  Pipeline: ",
           s.precision == RG_PREC_INT8 ? "INT8" : "FP16", s.original_layers, s.ops.size(), (long long)s.fp32_bytes,
           (long long)s.npu_bytes, (double)ratio);
  std::string r = head;
  for (size_t i = 0; i < s.ops.size(); ++i) {
    if (i) r += " -> ";
    r += s.ops[i].label;
  }
  if (needed) *needed = (int64_t)r.size() + 1;
  if (buf && cap > 0) {
    const size_t n = std::min<size_t>(r.size(), (size_t)cap - 1);
    memcpy(buf, r.data(), n);
    buf[n] = 0;
  }
  return RG_OK;
}

rg_status rg_session_last_profile(rg_session* h, rg_profile* prof, rg_op_record* records, int32_t cap) {
  if (!h || !prof) return fail(RG_ERR_INVALID_ARG, "null argument");
  Session& s = h->s;
  std::lock_guard<std::mutex> lock(s.mu);
  if (!s.last.valid) return fail(RG_ERR_NO_PROFILE, "no run yet");
  if (s.precision == RG_PREC_F32)  // last_npu_profile is None for the Cpu provider (mod.rs:193-195, 212-214)
    return fail(RG_ERR_NO_PROFILE, "the f32 provider records no NpuProfile");
  prof->precision = s.precision;
  prof->original_layers = s.original_layers;
  prof->fused_ops = (int32_t)s.ops.size();
  prof->n_records = (int32_t)s.ops.size();
  prof->fp32_weight_bytes = s.fp32_bytes;
  prof->npu_weight_bytes = s.npu_bytes;
  prof->total_macs = s.last.total_macs;
  prof->total_time_ns = s.last.total_ns;
  prof->kernel_launches = s.last.launches;
  prof->_reserved = 0;
  if (records)
    for (int32_t i = 0; i < std::min<int32_t>(cap, (int32_t)s.ops.size()); ++i) {
      memset(records[i].op, 0, sizeof records[i].op);
      strncpy(records[i].op, s.ops[(size_t)i].label.c_str(), sizeof(records[i].op) - 1);
      records[i].macs = s.last.macs[(size_t)i];
      records[i].duration_ns = s.last.ns[(size_t)i];
    }
  return RG_OK;
}

rg_status rg_session_num_ops(rg_session* h, int32_t* n_ops) {
  if (!h || !n_ops) return fail(RG_ERR_INVALID_ARG, "null argument");
  *n_ops = (int32_t)h->s.ops.size();
  return RG_OK;
}

rg_status rg_session_op_info(rg_session* h, int32_t i, rg_op_info* info) {
  if (!h || !info) return fail(RG_ERR_INVALID_ARG, "null argument");
  if (i < 0 || i >= (int32_t)h->s.ops.size()) return fail(RG_ERR_INVALID_ARG, "op %d out of range", i);
  const Op& op = h->s.ops[(size_t)i];
  memset(info, 0, sizeof *info);
  info->kind = op.kind; info->in_features = op.in_f; info->out_features = op.out_f;
  info->in_channels = op.in_c; info->out_channels = op.out_c; info->kernel = op.k;
  info->stride = op.stride; info->padding = op.pad; info->act = op.act; info->act_param = op.param;
  info->w_scale = op.w_scale; info->wq_len = (int64_t)op.wq.size(); info->bias_len = (int64_t)op.bias.size();
  strncpy(info->label, op.label.c_str(), sizeof(info->label) - 1);
  return RG_OK;
}

rg_status rg_session_op_weights(rg_session* h, int32_t i, int8_t* wq, int64_t cap, float* bias, int64_t bias_cap) {
  if (!h) return fail(RG_ERR_INVALID_ARG, "null session");
  if (i < 0 || i >= (int32_t)h->s.ops.size()) return fail(RG_ERR_INVALID_ARG, "op %d out of range", i);
  const Op& op = h->s.ops[(size_t)i];
  if (wq) {
    if (cap < (int64_t)op.wq.size()) return fail(RG_ERR_INVALID_ARG, "weight buffer too small");
    memcpy(wq, op.wq.data(), op.wq.size());
  }
  if (bias) {
    if (bias_cap < (int64_t)op.bias.size()) return fail(RG_ERR_INVALID_ARG, "bias buffer too small");
    memcpy(bias, op.bias.data(), op.bias.size() * 4);
  }
  return RG_OK;
}

rg_status rg_session_set_trace(rg_session* h, int32_t enable) {
  if (!h) return fail(RG_ERR_INVALID_ARG, "null session");
  std::lock_guard<std::mutex> lock(h->s.mu);
  h->s.trace = enable != 0;
  if (!h->s.trace) h->s.traces.clear();
  return RG_OK;
}

rg_status rg_session_trace_get(rg_session* h, int32_t op, int32_t item, void* buf, int64_t cap_bytes, int64_t* n_bytes) {
  if (!h || !n_bytes) return fail(RG_ERR_INVALID_ARG, "null argument");
  Session& s = h->s;
  std::lock_guard<std::mutex> lock(s.mu);
  if (op < 0 || op >= (int32_t)s.traces.size()) return fail(RG_ERR_INVALID_ARG, "no trace for op %d", op);
  const TraceRec& t = s.traces[(size_t)op];
  const void* src = nullptr;
  int64_t bytes = 0;
  switch (item) {
    case RG_TRACE_SCALES: src = t.scales.data(); bytes = (int64_t)t.scales.size() * 4; break;
    case RG_TRACE_AQ: src = t.aq.data(); bytes = (int64_t)t.aq.size(); break;
    case RG_TRACE_ACC: src = t.acc.data(); bytes = (int64_t)t.acc.size() * 4; break;
    case RG_TRACE_OUT: src = t.out.data(); bytes = (int64_t)t.out.size() * 4; break;
    default: return fail(RG_ERR_INVALID_ARG, "unknown trace item %d", item);
  }
  *n_bytes = bytes;
  if (buf) {
    if (cap_bytes < bytes) return fail(RG_ERR_INVALID_ARG, "trace buffer too small");
    if (bytes) memcpy(buf, src, (size_t)bytes);
  }
  return RG_OK;
}

// ---- static calibration (extension) ---------------------------------------------
// Installs (n > 0) or clears (n == 0) the frozen scales; the session's captured
// program no longer matches and is released.  Caller holds s.mu.
static rg_status set_calibration_locked(Session& s, const float* scales, int32_t n) {
  if (n != 0 && (!scales || n != s.calib_targets))
    return fail(RG_ERR_INVALID_ARG, "the session has %d calibration targets, got %d scales", s.calib_targets, n);
  for (int32_t j = 0; j < n; ++j)
    if (!(scales[j] > 0.0f) || !std::isfinite(scales[j]))
      return fail(RG_ERR_INVALID_ARG, "calibration scale %d is %g: scales must be finite and positive", j,
                  (double)scales[j]);
  RG_CUDA_TRY(cudaSetDevice(s.device));
  RG_CUDA_TRY(cudaStreamSynchronize(s.stream));
  if (s.graph.exec) cudaGraphExecDestroy(s.graph.exec);
  s.graph = Session::Graph();
  if (n == 0) {
    s.calibrated = false;
    s.calib.clear();
    return RG_OK;
  }
  s.calib.assign(scales, scales + n);
  RG_TRY(s.d_calib.ensure((size_t)n * sizeof(float)));
  RG_CUDA_TRY(cudaMemcpy(s.d_calib.p, scales, (size_t)n * sizeof(float), cudaMemcpyHostToDevice));
  s.calibrated = true;
  return RG_OK;
}

rg_status rg_session_calibration_targets(rg_session* h, int32_t* n) {
  if (!h || !n) return fail(RG_ERR_INVALID_ARG, "null argument");
  *n = h->s.calib_targets;
  return RG_OK;
}

rg_status rg_session_set_calibration(rg_session* h, const float* scales, int32_t n) {
  if (!h || n < 0) return fail(RG_ERR_INVALID_ARG, "null argument");
  Session& s = h->s;
  if (s.precision != RG_PREC_INT8) return fail(RG_ERR_UNSUPPORTED, "static calibration is for Npu(Int8) sessions");
  std::lock_guard<std::mutex> lock(s.mu);
  return set_calibration_locked(s, scales, n);
}

rg_status rg_session_get_calibration(rg_session* h, float* scales, int32_t cap) {
  if (!h || (!scales && cap > 0)) return fail(RG_ERR_INVALID_ARG, "null argument");
  Session& s = h->s;
  std::lock_guard<std::mutex> lock(s.mu);
  if (!s.calibrated) return fail(RG_ERR_INVALID_ARG, "the session is not calibrated");
  if (cap < s.calib_targets) return fail(RG_ERR_INVALID_ARG, "%d scales, capacity %d", s.calib_targets, cap);
  std::copy(s.calib.begin(), s.calib.end(), scales);
  return RG_OK;
}

rg_status rg_session_calibrate(rg_session* h, const float* x, const int64_t* shape, int32_t ndim) {
  if (!h || !x || !shape || ndim < 1 || ndim > 8) return fail(RG_ERR_INVALID_ARG, "bad calibration input");
  Session& s = h->s;
  if (s.precision != RG_PREC_INT8) return fail(RG_ERR_UNSUPPORTED, "static calibration is for Npu(Int8) sessions");
  {
    std::lock_guard<std::mutex> lock(s.mu);
    RG_TRY(set_calibration_locked(s, nullptr, 0));
  }
  // a run with the reference's dynamic scales leaves every Linear input's absmax (over
  // all ranks, when a communicator is attached) in its slot of the amax buffer
  int64_t ys[8];
  int32_t ynd = 0;
  RG_TRY(rg_session_output_shape(h, shape, ndim, ys, &ynd));
  int64_t out_elems = 1;
  for (int32_t i = 0; i < ynd; ++i) out_elems *= ys[i];
  std::vector<float> y((size_t)std::max<int64_t>(out_elems, 1));
  RG_TRY(run_impl(h, x, true, shape, ndim, y.data(), true, out_elems, ys, &ynd, nullptr, false));
  std::lock_guard<std::mutex> lock(s.mu);
  RunPlan P;
  RG_TRY(make_plan(s, shape, ndim, P));
  std::vector<uint32_t> bits((size_t)std::max<int64_t>(P.total_slots, 1), 0u);
  if (P.total_slots) RG_CUDA_TRY(cudaMemcpy(bits.data(), s.amax.p, (size_t)P.total_slots * 4, cudaMemcpyDeviceToHost));
  std::vector<float> sc((size_t)s.calib_targets);
  for (size_t i = 0; i < s.ops.size(); ++i) {
    if (s.calib_off[i] < 0) continue;
    const int parts = s.ops[i].kind == RG_LAYER_LINEAR ? 1 : 2;
    for (int j = 0; j < parts; ++j)  // QuantTensor::from_f32's scale (quantize.rs:19-20)
      sc[(size_t)(s.calib_off[i] + j)] = quant_scale<false>(u2f(bits[(size_t)(P.amax_off[i] + j)]));
  }
  return set_calibration_locked(s, sc.data(), s.calib_targets);
}

rg_status rg_nccl_unique_id(uint8_t id[128]) {
  if (!id) return fail(RG_ERR_INVALID_ARG, "null argument");
  ncclUniqueId u;
  RG_NCCL_TRY(ncclGetUniqueId(&u));
  static_assert(sizeof(u) == 128, "ncclUniqueId size");
  memcpy(id, &u, 128);
  return RG_OK;
}

rg_status rg_session_attach_comm(rg_session* h, const uint8_t id[128], int32_t rank, int32_t world) {
  if (!h || !id) return fail(RG_ERR_INVALID_ARG, "null argument");
  if (world < 1 || rank < 0 || rank >= world) return fail(RG_ERR_INVALID_ARG, "rank %d of %d", rank, world);
  Session& s = h->s;
  std::lock_guard<std::mutex> lock(s.mu);
  RG_CUDA_TRY(cudaSetDevice(s.device));
  // a program captured with the previous communicator (or none) is stale
  RG_CUDA_TRY(cudaStreamSynchronize(s.stream));
  if (s.graph.exec) cudaGraphExecDestroy(s.graph.exec);
  s.graph = Session::Graph();
  if (s.comm) {
    ncclCommDestroy(s.comm);
    s.comm = nullptr;
  }
  ncclUniqueId u;
  memcpy(&u, id, 128);
  RG_NCCL_TRY(ncclCommInitRank(&s.comm, world, u, rank));
  s.rank = rank;
  s.world = world;
  return RG_OK;
}

rg_status rg_session_allgather(rg_session* h, const float* send_dev, float* recv_dev, int64_t count, void* stream) {
  if (!h || !send_dev || !recv_dev) return fail(RG_ERR_INVALID_ARG, "null argument");
  Session& s = h->s;
  if (!s.comm) return fail(RG_ERR_INVALID_ARG, "no communicator attached");
  RG_CUDA_TRY(cudaSetDevice(s.device));
  cudaStream_t st = stream ? (cudaStream_t)stream : s.stream;
  RG_NCCL_TRY(ncclAllGather(send_dev, recv_dev, (size_t)count, ncclFloat32, s.comm, st));
  if (!stream) RG_CUDA_TRY(cudaStreamSynchronize(st));  // on a caller's stream it stays enqueued
  return RG_OK;
}

// ---- kernel-level entry points ---------------------------------------------------
rg_status rg_absmax_f32(const float* x, int64_t n, float* amax, void* stream) {
  if ((!x && n > 0) || !amax || n < 0) return fail(RG_ERR_INVALID_ARG, "null argument");
  cudaStream_t st = (cudaStream_t)stream;
  RG_CUDA_TRY(cudaMemsetAsync(amax, 0, 4, st));
  launch_absmax(x, n, reinterpret_cast<unsigned*>(amax), st);
  RG_CUDA_TRY(cudaGetLastError());
  return RG_OK;
}

rg_status rg_quantize_f32_i8(const float* x, int64_t rows, int64_t k, int64_t ldq, const float* amax, int8_t* q,
                             float* scale, void* stream) {
  if (!x || !amax || !q || rows < 0 || k <= 0 || ldq < k || (ldq & 15))
    return fail(RG_ERR_INVALID_ARG, "bad quantize arguments (ldq must be a multiple of 16 and >= k)");
  launch_quantize_rows(x, rows, k, ldq, reinterpret_cast<const unsigned*>(amax), q, scale, (cudaStream_t)stream);
  RG_CUDA_TRY(cudaGetLastError());
  return RG_OK;
}

static rg_status gemm_args_check(const int8_t* a, const int8_t* w, int64_t m, int64_t n, int64_t ld,
                                 const float* a_scale, const float* bias, float* out) {
  if (!a || !w || !a_scale || !bias || !out) return fail(RG_ERR_INVALID_ARG, "null argument");
  if (m < 0 || n <= 0 || ld <= 0 || (ld & 15)) return fail(RG_ERR_INVALID_ARG, "ld must be a positive multiple of 16");
  if ((reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(w) & 15))
    return fail(RG_ERR_INVALID_ARG, "operands must be 16-byte aligned");
  return RG_OK;
}

rg_status rg_gemm_i8_fused(const int8_t* a, const int8_t* w, int64_t m, int64_t n, int64_t ld, const float* a_scale,
                           float w_scale, const float* bias, int32_t act, float act_param, float* out, int32_t* acc,
                           float* out_amax, void* stream) {
  RG_TRY(gemm_args_check(a, w, m, n, ld, a_scale, bias, out));
  if (act < RG_ACT_NONE || act > RG_ACT_SILU) return fail(RG_ERR_INVALID_ARG, "unknown activation %d", act);
  GemmArgs g;
  g.a = a; g.lda = ld; g.w = w; g.ldb = ld; g.m = m; g.n = n; g.k = ld;
  g.a_scale = a_scale; g.w_scale = w_scale; g.bias = bias; g.act = act; g.act_param = act_param;
  g.out = out; g.acc = acc;
  g.amax.ptr = reinterpret_cast<unsigned*>(out_amax);
  int dev = 0, sms = 148;
  RG_CUDA_TRY(cudaGetDevice(&dev));
  RG_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  cudaStream_t st = (cudaStream_t)stream;
  if (!gemm_tc_eligible(g)) {  // CUDA-core kernels: no waits, enqueued and returned
    if (gemm_narrow_eligible(g)) launch_gemm_narrow(g, st);
    else launch_gemm_simt(g, st);
    RG_CUDA_TRY(cudaGetLastError());
    return RG_OK;
  }
  // The tensor-core kernel reports a bounded wait that gave up through an error word
  // of this call alone; the call waits for the kernel and turns the word into its
  // status.  Inside a stream capture nothing can be waited for: the captured kernel
  // writes a word no call reads (a timeout in a replay of that graph goes unreported).
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  RG_CUDA_TRY(cudaStreamIsCapturing(st, &cap));
  CallErrSlot slot;
  RG_TRY(slot.acquire(dev, cap != cudaStreamCaptureStatusNone));
  RG_CUDA_TRY(cudaMemsetAsync(slot.ptr, 0, sizeof(int32_t), st));
  g.err = slot.ptr;
  g.wait_ns = g_tc_wait_ns.load();
  g.starve = g_tc_starve.load();
  if (!launch_gemm_tc(g, sms, st)) return fail(RG_ERR_CUDA, "TMA descriptor encoding failed");
  RG_CUDA_TRY(cudaGetLastError());
  if (cap != cudaStreamCaptureStatusNone) return RG_OK;
  int32_t e[2] = {0, 0};
  RG_CUDA_TRY(cudaMemcpyAsync(e, slot.ptr, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
  RG_CUDA_TRY(cudaStreamSynchronize(st));
  return rg_status_from_error_words(e);
}

rg_status rg_status_from_error_words(const int32_t words[2]) {
  if (!words) return fail(RG_ERR_INVALID_ARG, "null argument");
  if (words[0]) return fail(RG_ERR_TIMEOUT, "a tensor-core kernel gave up on a bounded wait; results are invalid");
  if (words[1]) return fail(RG_ERR_INVALID_ARG, "Embedding: a token id is not below the vocabulary size");
  return RG_OK;
}

void rg_debug_set_tc_wait(uint64_t wait_ns, int32_t starve_loads) {
  g_tc_wait_ns.store(wait_ns);
  g_tc_starve.store(starve_loads ? 1 : 0);
}

int64_t rg_linear_i8_workspace_size(int64_t m, int64_t ld) { return round_up(m * ld, 256) + 256; }

rg_status rg_linear_i8(const float* x, int64_t m, int64_t k, const int8_t* w, int64_t n, int64_t ld, float w_scale,
                       const float* bias, int32_t act, float act_param, float* out, void* workspace, void* stream) {
  if (!x || !workspace || k <= 0 || ld < k) return fail(RG_ERR_INVALID_ARG, "bad linear arguments");
  cudaStream_t st = (cudaStream_t)stream;
  int8_t* q = reinterpret_cast<int8_t*>(workspace);
  unsigned* amax = reinterpret_cast<unsigned*>(reinterpret_cast<char*>(workspace) + round_up(m * ld, 256));
  float* scale = reinterpret_cast<float*>(amax + 1);
  RG_CUDA_TRY(cudaMemsetAsync(amax, 0, 4, st));
  launch_absmax(x, m * k, amax, st);
  RG_TRY(rg_quantize_f32_i8(x, m, k, ld, reinterpret_cast<float*>(amax), q, scale, stream));
  return rg_gemm_i8_fused(q, w, m, n, ld, scale, w_scale, bias, act, act_param, out, nullptr, nullptr, stream);
}

rg_status rg_maxpool2d_f32(const float* x, int64_t n, int32_t c, int32_t h, int32_t w, int32_t k, int32_t stride,
                           float* y, void* stream) {
  if (!x || !y || k <= 0 || stride <= 0 || h < k || w < k) return fail(RG_ERR_INVALID_ARG, "bad pool arguments");
  launch_maxpool2d(x, n, c, h, w, k, stride, y, AmaxSink(), (cudaStream_t)stream);
  RG_CUDA_TRY(cudaGetLastError());
  return RG_OK;
}

rg_status rg_softmax_f32(const float* x, int64_t outer, int64_t last, float* y, void* stream) {
  if (!x || !y) return fail(RG_ERR_INVALID_ARG, "null argument");
  launch_softmax(x, outer, last, y, AmaxSink(), (cudaStream_t)stream);
  RG_CUDA_TRY(cudaGetLastError());
  return RG_OK;
}

rg_status rg_activation_f32(const float* x, int64_t n, int32_t act, float act_param, float* y, void* stream) {
  if (!x || !y) return fail(RG_ERR_INVALID_ARG, "null argument");
  if (act < RG_ACT_NONE || act > RG_ACT_SILU) return fail(RG_ERR_INVALID_ARG, "unknown activation %d", act);
  launch_activation(x, n, act, act_param, y, AmaxSink(), (cudaStream_t)stream);
  RG_CUDA_TRY(cudaGetLastError());
  return RG_OK;
}

rg_status rg_attention_f32(const float* qkv, int64_t ld, int64_t batch, int32_t t, int32_t heads, int32_t head_dim,
                           float* out, int64_t ldo, void* stream) {
  if (!qkv || !out) return fail(RG_ERR_INVALID_ARG, "null argument");
  if (batch < 0 || t < 0 || heads <= 0 || head_dim <= 0 || ld < 3 * (int64_t)heads * head_dim ||
      ldo < (int64_t)heads * head_dim)
    return fail(RG_ERR_INVALID_ARG, "attention: inconsistent sizes");
  const float scale = 1.0f / std::sqrt((float)head_dim);  // attention.rs: mul_scalar(1 / sqrt(dh))
  RG_TRY(launch_attention(qkv, ld, batch, t, heads, head_dim, scale, out, ldo, AmaxSink(), (cudaStream_t)stream));
  RG_CUDA_TRY(cudaGetLastError());
  return RG_OK;
}

rg_status rg_selftest_fast_paths(uint64_t mismatches[6]) {
  if (!mismatches) return fail(RG_ERR_INVALID_ARG, "null argument");
  DevBuf counts;
  const rg_status st = counts.ensure(6 * sizeof(unsigned long long));
  if (st != RG_OK) return st;
  launch_selftest_fast_division(counts.as<unsigned long long>(), nullptr);
  RG_CUDA_TRY(cudaGetLastError());
  unsigned long long h[6];
  RG_CUDA_TRY(cudaMemcpy(h, counts.p, sizeof h, cudaMemcpyDeviceToHost));
  for (int i = 0; i < 6; ++i) mismatches[i] = h[i];
  return RG_OK;
}

}  // extern "C"
