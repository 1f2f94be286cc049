//! Raw declarations of librg_npu.so, one per entry point of `include/rg_npu.h`.
//!
//! The library replaces the CPU executor behind RustGears'
//! `ExecutionProvider::npu_int8()` (`src/inference/npu.rs`): a session is
//! `npu::compile` + `NpuProgram::execute` on a B200.  Every struct is
//! `#[repr(C)]` with the header's field order; `tests/test_rust_ffi.py` in the
//! repository checks names, argument counts, field orders and enum values
//! against the header.  This crate was written without a Rust toolchain at hand
//! (none exists on the machines it was built on): it is unverified by rustc.
#![allow(non_camel_case_types)]

use std::os::raw::{c_char, c_void};

/// `rg_status`: every entry point returns one (0 = success).
pub type rg_status = i32;
pub const RG_OK: rg_status = 0;
pub const RG_ERR_INVALID_ARG: rg_status = 1;
pub const RG_ERR_SHAPE: rg_status = 2;
pub const RG_ERR_CUDA: rg_status = 3;
pub const RG_ERR_NCCL: rg_status = 4;
pub const RG_ERR_TIMEOUT: rg_status = 5;
pub const RG_ERR_UNSUPPORTED: rg_status = 6;
pub const RG_ERR_IO: rg_status = 7;
pub const RG_ERR_OOM: rg_status = 8;
pub const RG_ERR_NO_DEVICE: rg_status = 9;
pub const RG_ERR_NO_PROFILE: rg_status = 10;

pub const RG_NPU_ABI_VERSION: i32 = 1;

/// `rg_layer_kind`: the `.rtim` tags (`src/save.rs:172-224`) and the extension kinds.
pub const RG_LAYER_LINEAR: i32 = 1;
pub const RG_LAYER_CONV2D: i32 = 2;
pub const RG_LAYER_CHANNEL_AFFINE: i32 = 3;
pub const RG_LAYER_MAXPOOL2D: i32 = 4;
pub const RG_LAYER_FLATTEN: i32 = 5;
pub const RG_LAYER_ACTIVATION: i32 = 6;
pub const RG_LAYER_SOFTMAX: i32 = 7;
pub const RG_LAYER_RESIDUAL_BEGIN: i32 = 8;
pub const RG_LAYER_RESIDUAL_END: i32 = 9;
pub const RG_LAYER_SHORTCUT_CONV2D: i32 = 10;
pub const RG_LAYER_ADAPTIVE_AVGPOOL2D: i32 = 11;
pub const RG_LAYER_EMBEDDING: i32 = 12;
pub const RG_LAYER_RMSNORM: i32 = 13;
pub const RG_LAYER_ATTENTION: i32 = 14;
pub const RG_LAYER_SWIGLU: i32 = 15;

/// `rg_activation`: the `.rtim` activation codes (`src/save.rs:206-214`) and SiLU.
pub const RG_ACT_NONE: i32 = 0;
pub const RG_ACT_RELU: i32 = 1;
pub const RG_ACT_SIGMOID: i32 = 2;
pub const RG_ACT_TANH: i32 = 3;
pub const RG_ACT_GELU: i32 = 4;
pub const RG_ACT_LEAKY_RELU: i32 = 5;
pub const RG_ACT_SILU: i32 = 6;

/// `rg_precision`: `NpuPrecision::Int8`, `NpuPrecision::Fp16`, and the f32 Cpu provider.
pub const RG_PREC_INT8: i32 = 0;
pub const RG_PREC_FP16: i32 = 1;
pub const RG_PREC_F32: i32 = 2;

pub const RG_SESSION_NO_PROFILE: i32 = 1;
pub const RG_SESSION_NO_FUSION: i32 = 2;
pub const RG_SESSION_NO_GRAPH: i32 = 4;
pub const RG_RUN_ASYNC: i32 = 1;

/// `rg_trace_item`.
pub const RG_TRACE_SCALES: i32 = 0;
pub const RG_TRACE_AQ: i32 = 1;
pub const RG_TRACE_ACC: i32 = 2;
pub const RG_TRACE_OUT: i32 = 3;

pub const RG_LINEAR_NOALLOC_MAX_BYTES: u32 = 16 << 20;

/// One reference `LayerSpec` (`src/inference/mod.rs:70-100`).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct rg_layer_spec {
    pub kind: i32,
    pub in_features: i32,
    pub out_features: i32,
    pub in_channels: i32,
    pub out_channels: i32,
    pub kernel: i32,
    pub stride: i32,
    pub padding: i32,
    pub weight: *const f32,
    pub weight_len: i64,
    pub bias: *const f32,
    pub bias_len: i64,
    pub act: i32,
    pub act_param: f32,
}

/// Opaque session handle (`InferenceSession` over the device program).
#[repr(C)]
pub struct rg_session {
    _private: [u8; 0],
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct rg_session_options {
    pub device: i32,
    pub precision: i32,
    pub weight_quant: i32,
    pub flags: i32,
}

/// `NpuProfile` (`src/inference/npu.rs:120-176`).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct rg_profile {
    pub precision: i32,
    pub original_layers: i32,
    pub fused_ops: i32,
    pub n_records: i32,
    pub fp32_weight_bytes: i64,
    pub npu_weight_bytes: i64,
    pub total_macs: u64,
    pub total_time_ns: i64,
    pub kernel_launches: i32,
    pub _reserved: i32,
}

/// `OpRecord` (`src/inference/npu.rs:109-116`).
#[repr(C)]
#[derive(Clone, Copy)]
pub struct rg_op_record {
    pub op: [c_char; 96],
    pub macs: u64,
    pub duration_ns: i64,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct rg_op_info {
    pub kind: i32,
    pub in_features: i32,
    pub out_features: i32,
    pub in_channels: i32,
    pub out_channels: i32,
    pub kernel: i32,
    pub stride: i32,
    pub padding: i32,
    pub act: i32,
    pub act_param: f32,
    pub w_scale: f32,
    pub wq_len: i64,
    pub bias_len: i64,
    pub label: [c_char; 96],
}

/// SplitMix64 state of the reference generator (`src/rng.rs:10-58`).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct rg_rng {
    pub state: u64,
}

#[link(name = "rg_npu")]
extern "C" {
    pub fn rg_last_error() -> *const c_char;
    pub fn rg_version() -> *const c_char;
    pub fn rg_device_count() -> i32;

    pub fn rg_session_create(layers: *const rg_layer_spec, n_layers: i32, opts: *const rg_session_options,
                             out: *mut *mut rg_session) -> rg_status;
    pub fn rg_session_create_from_rtim(path: *const c_char, opts: *const rg_session_options,
                                       out: *mut *mut rg_session) -> rg_status;
    pub fn rg_session_destroy(s: *mut rg_session);
    pub fn rg_session_output_shape(s: *mut rg_session, shape: *const i64, ndim: i32, y_shape: *mut i64,
                                   y_ndim: *mut i32) -> rg_status;
    pub fn rg_session_run(s: *mut rg_session, x: *const f32, shape: *const i64, ndim: i32, y: *mut f32,
                          y_cap: i64, y_shape: *mut i64, y_ndim: *mut i32) -> rg_status;
    pub fn rg_session_run_device(s: *mut rg_session, x_dev: *const f32, shape: *const i64, ndim: i32,
                                 y_dev: *mut f32, y_cap: i64, y_shape: *mut i64, y_ndim: *mut i32,
                                 stream: *mut c_void, flags: i32) -> rg_status;
    pub fn rg_session_compilation_report(s: *mut rg_session, buf: *mut c_char, cap: i64,
                                         needed: *mut i64) -> rg_status;
    pub fn rg_session_last_profile(s: *mut rg_session, prof: *mut rg_profile, records: *mut rg_op_record,
                                   cap: i32) -> rg_status;
    pub fn rg_session_num_ops(s: *mut rg_session, n_ops: *mut i32) -> rg_status;
    pub fn rg_session_op_info(s: *mut rg_session, op: i32, info: *mut rg_op_info) -> rg_status;
    pub fn rg_session_op_weights(s: *mut rg_session, op: i32, wq: *mut i8, cap: i64, bias: *mut f32,
                                 bias_cap: i64) -> rg_status;
    pub fn rg_session_calibration_targets(s: *mut rg_session, n: *mut i32) -> rg_status;
    pub fn rg_session_calibrate(s: *mut rg_session, x: *const f32, shape: *const i64, ndim: i32) -> rg_status;
    pub fn rg_session_set_calibration(s: *mut rg_session, scales: *const f32, n: i32) -> rg_status;
    pub fn rg_session_get_calibration(s: *mut rg_session, scales: *mut f32, cap: i32) -> rg_status;
    pub fn rg_session_set_trace(s: *mut rg_session, enable: i32) -> rg_status;
    pub fn rg_session_trace_get(s: *mut rg_session, op: i32, item: i32, buf: *mut c_void, cap_bytes: i64,
                                n_bytes: *mut i64) -> rg_status;

    pub fn rg_nccl_unique_id(id: *mut u8) -> rg_status;
    pub fn rg_session_attach_comm(s: *mut rg_session, id: *const u8, rank: i32, world: i32) -> rg_status;
    pub fn rg_session_allgather(s: *mut rg_session, send_dev: *const f32, recv_dev: *mut f32, count: i64,
                                stream: *mut c_void) -> rg_status;

    pub fn rg_absmax_f32(x: *const f32, n: i64, amax: *mut f32, stream: *mut c_void) -> rg_status;
    pub fn rg_quantize_f32_i8(x: *const f32, rows: i64, k: i64, ldq: i64, amax: *const f32, q: *mut i8,
                              scale: *mut f32, stream: *mut c_void) -> rg_status;
    pub fn rg_gemm_i8_fused(a: *const i8, w: *const i8, m: i64, n: i64, ld: i64, a_scale: *const f32,
                            w_scale: f32, bias: *const f32, act: i32, act_param: f32, out: *mut f32,
                            acc: *mut i32, out_amax: *mut f32, stream: *mut c_void) -> rg_status;
    pub fn rg_linear_i8_workspace_size(m: i64, ld: i64) -> i64;
    pub fn rg_linear_i8(x: *const f32, m: i64, k: i64, w: *const i8, n: i64, ld: i64, w_scale: f32,
                        bias: *const f32, act: i32, act_param: f32, out: *mut f32, workspace: *mut c_void,
                        stream: *mut c_void) -> rg_status;
    pub fn rg_linear_i8_noalloc(x: *const f32, m: i64, k: i64, w: *const i8, n: i64, ld: i64, w_scale: f32,
                                bias: *const f32, act: i32, act_param: f32, out: *mut f32,
                                stream: *mut c_void) -> rg_status;
    pub fn rg_status_from_error_words(words: *const i32) -> rg_status;
    pub fn rg_debug_set_tc_wait(wait_ns: u64, starve_loads: i32);
    pub fn rg_maxpool2d_f32(x: *const f32, n: i64, c: i32, h: i32, w: i32, k: i32, stride: i32, y: *mut f32,
                            stream: *mut c_void) -> rg_status;
    pub fn rg_softmax_f32(x: *const f32, outer: i64, last: i64, y: *mut f32, stream: *mut c_void) -> rg_status;
    pub fn rg_activation_f32(x: *const f32, n: i64, act: i32, act_param: f32, y: *mut f32,
                             stream: *mut c_void) -> rg_status;
    pub fn rg_attention_f32(qkv: *const f32, ld: i64, batch: i64, t: i32, heads: i32, head_dim: i32,
                            out: *mut f32, ldo: i64, stream: *mut c_void) -> rg_status;
    pub fn rg_selftest_fast_paths(mismatches: *mut u64) -> rg_status;

    pub fn rg_rng_seed(r: *mut rg_rng, seed: u64);
    pub fn rg_rng_next_u64(r: *mut rg_rng) -> u64;
    pub fn rg_rng_fill_uniform(r: *mut rg_rng, out: *mut f32, n: i64, lo: f32, hi: f32);
    pub fn rg_rng_fill_normal(r: *mut rg_rng, out: *mut f32, n: i64, std_scale: f32);
    pub fn rg_rng_fill_below(r: *mut rg_rng, out: *mut i64, n: i64, bound: u64);
    pub fn rg_kaiming_bound(fan_in: i64) -> f32;
    pub fn rg_bias_bound(fan_in: i64) -> f32;
}
