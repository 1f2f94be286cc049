//! `src/device/cuda.rs` for RustGears: the safe wrapper its `CompiledProgram::NpuCuda`
//! arm holds.  The dispatch change in `src/inference/mod.rs`: a variant
//! `NpuCuda(crate::device::cuda::Session)` built by `from_layers` for
//! `ExecutionProvider::Npu(p)`, whose `run` stores the returned profile in
//! `last_profile` and whose `compilation_report` is `Session::report`.
//!
//! It turns the reference IR (`LayerSpec`, `src/inference/mod.rs:70-100`) into the
//! C ABI's `rg_layer_spec` (kind = the `.rtim` tag, `src/save.rs:176-219`;
//! `ChannelAffine` carries `scale` / `shift` as `weight` / `bias`; activation codes as
//! `src/save.rs:206-214`), creates the device session, and maps `run` and the profile
//! back to `Tensor` and `NpuProfile` / `OpRecord` (`src/inference/npu.rs:107-176`).
//! Errors: creation returns `Err(message)`; `run` panics with the library's message,
//! as the reference's `run` panics on a shape mismatch.
//!
//! Written without a Rust toolchain (none exists on the machines this library was
//! built on): unverified by rustc.
use std::ffi::CStr;
use std::os::raw::c_char;
use std::time::Duration;

use rustgears_cuda_sys as sys;

use crate::inference::{Activation, LayerSpec, NpuPrecision, NpuProfile, OpRecord};
use crate::tensor::Tensor;

fn last_error() -> String {
    unsafe { CStr::from_ptr(sys::rg_last_error()).to_string_lossy().into_owned() }
}

fn check(st: sys::rg_status) -> Result<(), String> {
    if st == sys::RG_OK { Ok(()) } else { Err(format!("[rg_status {st}] {}", last_error())) }
}

fn act_code(a: &Activation) -> (i32, f32) {
    match a {
        Activation::None => (sys::RG_ACT_NONE, 0.0),
        Activation::Relu => (sys::RG_ACT_RELU, 0.0),
        Activation::Sigmoid => (sys::RG_ACT_SIGMOID, 0.0),
        Activation::Tanh => (sys::RG_ACT_TANH, 0.0),
        Activation::Gelu => (sys::RG_ACT_GELU, 0.0),
        Activation::LeakyRelu(s) => (sys::RG_ACT_LEAKY_RELU, *s),
    }
}

fn spec_of(l: &LayerSpec) -> sys::rg_layer_spec {
    let mut s = sys::rg_layer_spec {
        kind: 0, in_features: 0, out_features: 0, in_channels: 0, out_channels: 0, kernel: 0, stride: 0,
        padding: 0, weight: std::ptr::null(), weight_len: 0, bias: std::ptr::null(), bias_len: 0, act: 0,
        act_param: 0.0,
    };
    match l {
        LayerSpec::Linear { in_features, out_features, weight, bias } => {
            s.kind = sys::RG_LAYER_LINEAR;
            s.in_features = *in_features as i32;
            s.out_features = *out_features as i32;
            s.weight = weight.as_ptr();
            s.weight_len = weight.len() as i64;
            s.bias = bias.as_ptr();
            s.bias_len = bias.len() as i64;
        }
        LayerSpec::Conv2d { in_channels, out_channels, kernel, stride, padding, weight, bias } => {
            s.kind = sys::RG_LAYER_CONV2D;
            s.in_channels = *in_channels as i32;
            s.out_channels = *out_channels as i32;
            s.kernel = *kernel as i32;
            s.stride = *stride as i32;
            s.padding = *padding as i32;
            s.weight = weight.as_ptr();
            s.weight_len = weight.len() as i64;
            s.bias = bias.as_ptr();
            s.bias_len = bias.len() as i64;
        }
        LayerSpec::ChannelAffine { scale, shift } => {
            s.kind = sys::RG_LAYER_CHANNEL_AFFINE;
            s.weight = scale.as_ptr();
            s.weight_len = scale.len() as i64;
            s.bias = shift.as_ptr();
            s.bias_len = shift.len() as i64;
        }
        LayerSpec::MaxPool2d { kernel, stride } => {
            s.kind = sys::RG_LAYER_MAXPOOL2D;
            s.kernel = *kernel as i32;
            s.stride = *stride as i32;
        }
        LayerSpec::Flatten => s.kind = sys::RG_LAYER_FLATTEN,
        LayerSpec::Activation(a) => {
            s.kind = sys::RG_LAYER_ACTIVATION;
            let (code, p) = act_code(a);
            s.act = code;
            s.act_param = p;
        }
        LayerSpec::Softmax => s.kind = sys::RG_LAYER_SOFTMAX,
    }
    s
}

/// A compiled device program: `npu::compile` + uploaded weights on one GPU.
pub struct Session {
    h: *mut sys::rg_session,
    precision: NpuPrecision,
}

// The library serialises calls on one session internally (`run(&self)` may be
// called from several threads, as InferenceSession::run allows).
unsafe impl Send for Session {}
unsafe impl Sync for Session {}

impl Session {
    /// `from_layers(layers, ExecutionProvider::Npu(precision))` on CUDA device `device`.
    pub fn new(layers: &[LayerSpec], device: i32, precision: NpuPrecision) -> Result<Session, String> {
        let specs: Vec<sys::rg_layer_spec> = layers.iter().map(spec_of).collect();
        let opts = sys::rg_session_options {
            device,
            precision: match precision { NpuPrecision::Int8 => sys::RG_PREC_INT8, NpuPrecision::Fp16 => sys::RG_PREC_FP16 },
            weight_quant: 0,
            flags: 0,
        };
        let mut h: *mut sys::rg_session = std::ptr::null_mut();
        check(unsafe { sys::rg_session_create(specs.as_ptr(), specs.len() as i32, &opts, &mut h) })?;
        Ok(Session { h, precision })
    }

    /// `run` on host data (the copies to and from the device are part of the call),
    /// with the profile of that run.
    pub fn run(&self, input: &Tensor) -> (Tensor, NpuProfile) {
        let shape: Vec<i64> = input.shape().iter().map(|&d| d as i64).collect();
        let mut y_shape = [0i64; 8];
        let mut y_ndim = 0i32;
        let st = unsafe {
            sys::rg_session_output_shape(self.h, shape.as_ptr(), shape.len() as i32, y_shape.as_mut_ptr(), &mut y_ndim)
        };
        if let Err(e) = check(st) { panic!("InferenceSession::run: {e}"); }
        let out_dims: Vec<usize> = y_shape[..y_ndim as usize].iter().map(|&d| d as usize).collect();
        let n_out: usize = out_dims.iter().product();
        let mut y = vec![0.0f32; n_out];
        let x = input.to_vec();
        let st = unsafe {
            sys::rg_session_run(self.h, x.as_ptr(), shape.as_ptr(), shape.len() as i32, y.as_mut_ptr(), n_out as i64,
                                y_shape.as_mut_ptr(), &mut y_ndim)
        };
        if let Err(e) = check(st) { panic!("InferenceSession::run: {e}"); }
        (Tensor::from_vec(y, &out_dims), self.profile())
    }

    fn profile(&self) -> NpuProfile {
        let mut p = sys::rg_profile::default();
        let mut n = 0i32;
        unsafe { sys::rg_session_num_ops(self.h, &mut n) };
        let mut recs = vec![sys::rg_op_record { op: [0 as c_char; 96], macs: 0, duration_ns: 0 }; n.max(1) as usize];
        let st = unsafe { sys::rg_session_last_profile(self.h, &mut p, recs.as_mut_ptr(), n) };
        if let Err(e) = check(st) { panic!("last_npu_profile: {e}"); }
        let records = recs[..p.n_records.min(n).max(0) as usize]
            .iter()
            .map(|r| OpRecord {
                op: unsafe { CStr::from_ptr(r.op.as_ptr()).to_string_lossy().into_owned() },
                macs: r.macs,
                duration: Duration::from_nanos(r.duration_ns.max(0) as u64),
            })
            .collect();
        NpuProfile {
            precision: self.precision,
            original_layers: p.original_layers as usize,
            fused_ops: p.fused_ops as usize,
            fp32_weight_bytes: p.fp32_weight_bytes as usize,
            npu_weight_bytes: p.npu_weight_bytes as usize,
            total_macs: p.total_macs,
            total_time: Duration::from_nanos(p.total_time_ns.max(0) as u64),
            records,
        }
    }

    /// `compilation_report` (`NpuProgram::summary`, `src/inference/npu.rs:280-293`).
    pub fn report(&self) -> String {
        let mut need = 0i64;
        unsafe { sys::rg_session_compilation_report(self.h, std::ptr::null_mut(), 0, &mut need) };
        let mut buf = vec![0 as c_char; need.max(1) as usize];
        let st = unsafe { sys::rg_session_compilation_report(self.h, buf.as_mut_ptr(), need, &mut need) };
        if let Err(e) = check(st) { panic!("compilation_report: {e}"); }
        unsafe { CStr::from_ptr(buf.as_ptr()).to_string_lossy().into_owned() }
    }
}

impl Drop for Session {
    fn drop(&mut self) {
        unsafe { sys::rg_session_destroy(self.h) };
    }
}
