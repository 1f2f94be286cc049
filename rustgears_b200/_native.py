"""ctypes binding of librg_npu.so (the C ABI declared in include/rg_npu.h).

The library is the only compute path: importing this module fails loudly when
the shared object is missing, and every call returns the library's own error
when no sm_100 device is present.  There is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librg_npu.so")

RG_OK = 0
RG_ERR_INVALID_ARG, RG_ERR_SHAPE, RG_ERR_CUDA, RG_ERR_NCCL, RG_ERR_TIMEOUT = 1, 2, 3, 4, 5
RG_ERR_UNSUPPORTED, RG_ERR_IO, RG_ERR_OOM, RG_ERR_NO_DEVICE, RG_ERR_NO_PROFILE = 6, 7, 8, 9, 10
RG_TRACE_SCALES, RG_TRACE_AQ, RG_TRACE_ACC, RG_TRACE_OUT = 0, 1, 2, 3
RG_SESSION_NO_PROFILE, RG_SESSION_NO_FUSION, RG_SESSION_NO_GRAPH = 1, 2, 4
RG_RUN_ASYNC = 1


class RgError(RuntimeError):
    """A failed C-ABI call: ``status`` is the rg_status code."""

    def __init__(self, status: int, msg: str):
        super().__init__(f"[rg_status {status}] {msg}")
        self.status = status


class ShapeError(RgError):
    pass


class LayerSpecC(C.Structure):
    _fields_ = [
        ("kind", C.c_int32), ("in_features", C.c_int32), ("out_features", C.c_int32),
        ("in_channels", C.c_int32), ("out_channels", C.c_int32), ("kernel", C.c_int32),
        ("stride", C.c_int32), ("padding", C.c_int32),
        ("weight", C.POINTER(C.c_float)), ("weight_len", C.c_int64),
        ("bias", C.POINTER(C.c_float)), ("bias_len", C.c_int64),
        ("act", C.c_int32), ("act_param", C.c_float),
    ]


class SessionOptions(C.Structure):
    _fields_ = [("device", C.c_int32), ("precision", C.c_int32), ("weight_quant", C.c_int32),
                ("flags", C.c_int32)]


class ProfileC(C.Structure):
    _fields_ = [("precision", C.c_int32), ("original_layers", C.c_int32), ("fused_ops", C.c_int32),
                ("n_records", C.c_int32), ("fp32_weight_bytes", C.c_int64),
                ("npu_weight_bytes", C.c_int64), ("total_macs", C.c_uint64),
                ("total_time_ns", C.c_int64), ("kernel_launches", C.c_int32), ("_reserved", C.c_int32)]


class OpRecordC(C.Structure):
    _fields_ = [("op", C.c_char * 96), ("macs", C.c_uint64), ("duration_ns", C.c_int64)]


class OpInfoC(C.Structure):
    _fields_ = [("kind", C.c_int32), ("in_features", C.c_int32), ("out_features", C.c_int32),
                ("in_channels", C.c_int32), ("out_channels", C.c_int32), ("kernel", C.c_int32),
                ("stride", C.c_int32), ("padding", C.c_int32), ("act", C.c_int32),
                ("act_param", C.c_float), ("w_scale", C.c_float), ("wq_len", C.c_int64),
                ("bias_len", C.c_int64), ("label", C.c_char * 96)]


class RngC(C.Structure):
    _fields_ = [("state", C.c_uint64)]


# Every symbol include/rg_npu.h declares, with its ctypes signature.
_vp, _i32, _i64, _u64, _f32 = C.c_void_p, C.c_int32, C.c_int64, C.c_uint64, C.c_float
_f32p, _i64p, _i32p, _i8p = C.POINTER(C.c_float), C.POINTER(C.c_int64), C.POINTER(C.c_int32), C.POINTER(C.c_int8)
SIGNATURES = {
    "rg_last_error": ([], C.c_char_p),
    "rg_version": ([], C.c_char_p),
    "rg_device_count": ([], _i32),
    "rg_session_create": ([C.POINTER(LayerSpecC), _i32, C.POINTER(SessionOptions), C.POINTER(_vp)], _i32),
    "rg_session_create_from_rtim": ([C.c_char_p, C.POINTER(SessionOptions), C.POINTER(_vp)], _i32),
    "rg_session_destroy": ([_vp], None),
    "rg_session_output_shape": ([_vp, _i64p, _i32, _i64p, _i32p], _i32),
    "rg_session_run": ([_vp, _f32p, _i64p, _i32, _f32p, _i64, _i64p, _i32p], _i32),
    "rg_session_run_device": ([_vp, _vp, _i64p, _i32, _vp, _i64, _i64p, _i32p, _vp, _i32], _i32),
    "rg_session_compilation_report": ([_vp, C.c_char_p, _i64, _i64p], _i32),
    "rg_session_last_profile": ([_vp, C.POINTER(ProfileC), C.POINTER(OpRecordC), _i32], _i32),
    "rg_session_num_ops": ([_vp, _i32p], _i32),
    "rg_session_op_info": ([_vp, _i32, C.POINTER(OpInfoC)], _i32),
    "rg_session_op_weights": ([_vp, _i32, _i8p, _i64, _f32p, _i64], _i32),
    "rg_session_calibration_targets": ([_vp, _i32p], _i32),
    "rg_session_calibrate": ([_vp, _f32p, _i64p, _i32], _i32),
    "rg_session_set_calibration": ([_vp, _f32p, _i32], _i32),
    "rg_session_get_calibration": ([_vp, _f32p, _i32], _i32),
    "rg_session_set_trace": ([_vp, _i32], _i32),
    "rg_session_trace_get": ([_vp, _i32, _i32, _vp, _i64, _i64p], _i32),
    "rg_nccl_unique_id": ([C.POINTER(C.c_uint8)], _i32),
    "rg_session_attach_comm": ([_vp, C.POINTER(C.c_uint8), _i32, _i32], _i32),
    "rg_session_allgather": ([_vp, _vp, _vp, _i64, _vp], _i32),
    "rg_absmax_f32": ([_vp, _i64, _vp, _vp], _i32),
    "rg_quantize_f32_i8": ([_vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp], _i32),
    "rg_gemm_i8_fused": ([_vp, _vp, _i64, _i64, _i64, _vp, _f32, _vp, _i32, _f32, _vp, _vp, _vp, _vp], _i32),
    "rg_linear_i8_workspace_size": ([_i64, _i64], _i64),
    "rg_linear_i8": ([_vp, _i64, _i64, _vp, _i64, _i64, _f32, _vp, _i32, _f32, _vp, _vp, _vp], _i32),
    "rg_linear_i8_noalloc": ([_vp, _i64, _i64, _vp, _i64, _i64, _f32, _vp, _i32, _f32, _vp, _vp], _i32),
    "rg_status_from_error_words": ([_i32p], _i32),
    "rg_debug_set_tc_wait": ([_u64, _i32], None),
    "rg_maxpool2d_f32": ([_vp, _i64, _i32, _i32, _i32, _i32, _i32, _vp, _vp], _i32),
    "rg_softmax_f32": ([_vp, _i64, _i64, _vp, _vp], _i32),
    "rg_attention_f32": ([_vp, _i64, _i64, _i32, _i32, _i32, _vp, _i64, _vp], _i32),
    "rg_activation_f32": ([_vp, _i64, _i32, _f32, _vp, _vp], _i32),
    "rg_selftest_fast_paths": ([_vp], _i32),
    "rg_rng_seed": ([C.POINTER(RngC), _u64], None),
    "rg_rng_next_u64": ([C.POINTER(RngC)], _u64),
    "rg_rng_fill_uniform": ([C.POINTER(RngC), _f32p, _i64, _f32, _f32], None),
    "rg_rng_fill_normal": ([C.POINTER(RngC), _f32p, _i64, _f32], None),
    "rg_rng_fill_below": ([C.POINTER(RngC), _i64p, _i64, _u64], None),
    "rg_kaiming_bound": ([_i64], _f32),
    "rg_bias_bound": ([_i64], _f32),
}

_lib = None


def lib():
    """The loaded librg_npu.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m rustgears_b200.build` "
                              "(this provider has no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def last_error() -> str:
    return lib().rg_last_error().decode(errors="replace")


def check(status: int) -> None:
    if status != RG_OK:
        cls = ShapeError if status == RG_ERR_SHAPE else RgError
        raise cls(status, last_error())
