// linear_noalloc.cu -- FusedLinear entry point that allocates no device memory.
//
// rg_linear_i8 needs a caller-provided workspace for the quantized activations
// and the activation scale.  Some callers cannot provide one: a host that has
// handed all device memory to its own pool and forbids other allocations, or a
// latency-critical loop that must not call cudaMalloc (which can block on the
// device and take driver locks).  rg_linear_i8_noalloc runs the same three
// kernels (absmax, quantize, fused GEMM) on a fixed scratch array that lives in
// this file as a static __device__ variable, so no call ever allocates.
//
// Limits and sharing:
//   * the scratch holds at most RG_LINEAR_NOALLOC_MAX_BYTES (16 MiB) of
//     quantized activations, i.e. m * ld <= 16 MiB; larger calls are rejected
//     with RG_ERR_INVALID_ARG before any device work;
//   * every GPU that loads this library holds its own copy of the array
//     (16 MiB + 256 B) until the process exits;
//   * all calls on a device share that one array and it keeps the last call's
//     contents: each call clears the absmax slot it accumulates into, and
//     rewrites everything else it reads.  Calls that overlap on the GPU (two
//     streams, or two host threads without ordering) race on the scratch.
//   * the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current) and caches it; make that
//     first call before any stream capture begins.  The cached address lives as
//     long as the process: after a cudaDeviceReset of a device it would be stale,
//     so a process that resets a device must not call this entry point on it again;
//   * like rg_linear_i8, a call whose GEMM runs on the tensor cores waits for it
//     and returns RG_ERR_TIMEOUT if one of its bounded waits gave up (the word
//     that reports it is a slot of a static device array held for this call).
#include <cuda_runtime.h>
#include <stdio.h>

#include <mutex>

#include "../../include/rg_npu.h"
#include "rg_kernels.h"

namespace {

// Layout (the one rg_linear_i8 expects of its workspace): the quantized rows
// [m, ld] from offset 0, then at the next 256-byte boundary the absmax slot
// (4 bytes, cleared by every call) and the activation scale (4 bytes).
constexpr size_t kHeaderBytes = 256;
constexpr size_t kMaxQuantBytes = RG_LINEAR_NOALLOC_MAX_BYTES;

// The scratch.  In host code `g_linear_scratch` names a host-side stand-in,
// not device memory: only the address from cudaGetSymbolAddress may be passed
// to a kernel.
static __device__ __align__(256) unsigned char g_linear_scratch[kHeaderBytes + kMaxQuantBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Set-up, once per device, with that device current.
cudaError_t scratch_for(int dev, void** out) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_linear_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" rg_status rg_linear_i8(const float* x, int64_t m, int64_t k, const int8_t* w, int64_t n, int64_t ld,
                                  float w_scale, const float* bias, int32_t act, float act_param, float* out,
                                  void* workspace, void* stream);

extern "C" rg_status rg_linear_i8_noalloc(const float* x, int64_t m, int64_t k, const int8_t* w, int64_t n,
                                          int64_t ld, float w_scale, const float* bias, int32_t act,
                                          float act_param, float* out, void* stream) {
  if (m < 0 || ld <= 0) return rg::set_last_error(RG_ERR_INVALID_ARG, "rg_linear_i8_noalloc: bad m or ld");
  // m * ld <= limit, tested by division so that no product can wrap
  if (m > (int64_t)kMaxQuantBytes / ld) {
    char msg[192];
    snprintf(msg, sizeof msg,
             "rg_linear_i8_noalloc: m = %lld rows of ld = %lld bytes exceeds the %zu-byte static scratch; "
             "use rg_linear_i8", (long long)m, (long long)ld, kMaxQuantBytes);
    return rg::set_last_error(RG_ERR_INVALID_ARG, msg);
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return rg::set_last_error(RG_ERR_CUDA, "rg_linear_i8_noalloc: no current device");
  void* scratch = nullptr;
  const cudaError_t e = scratch_for(dev, &scratch);
  if (e != cudaSuccess)
    return rg::set_last_error(RG_ERR_CUDA, cudaGetErrorString(e));
  return rg_linear_i8(x, m, k, w, n, ld, w_scale, bias, act, act_param, out, scratch, stream);
}
