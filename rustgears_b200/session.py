"""``InferenceSession`` over ``ExecutionProvider::Npu(Int8 | Fp16)`` on the B200 library.

Mirrors the reference surface (src/inference/mod.rs:102-222, npu.rs:107-176):
``InferenceSession.from_module / from_layers / run / last_npu_profile /
compilation_report``, ``ExecutionProvider.npu / npu_int8 / npu_fp16``,
``NpuPrecision``, ``NpuProfile`` and ``OpRecord``.  Every call goes through
librg_npu.so; there is no CPU path.
"""
from __future__ import annotations

import ctypes as C
import datetime as _dt
import enum
from dataclasses import dataclass, field

import numpy as np

from . import _native
from .spec import (ACTIVATION, ADAPTIVE_AVGPOOL2D, ATTENTION, CHANNEL_AFFINE, CONV2D, EMBEDDING, LINEAR,
                   RESIDUAL_END, RMSNORM, SHORTCUT_CONV2D, SWIGLU, Activation, as_dict)

_MAX_RANK = 8


class NpuPrecision(enum.Enum):  # npu.rs:25-41
    Int8 = 0
    Fp16 = 1

    def __str__(self) -> str:
        return "INT8" if self is NpuPrecision.Int8 else "FP16"


class ExecutionProvider:
    """`ExecutionProvider` (mod.rs:102-138).  ``Npu(Int8)``, ``Npu(Fp16)`` and the f32
    ``Cpu`` provider (its arithmetic, on the B200) run here; ``Gpu(i)`` is the
    reference's wgpu runtime, which needs a graphics stack (unavailable on this box)."""

    __slots__ = ("kind", "index", "precision")

    def __init__(self, kind: str, index: int = 0, precision: NpuPrecision | None = None):
        self.kind, self.index, self.precision = kind, index, precision

    @classmethod
    def npu(cls) -> "ExecutionProvider":
        return cls("Npu", precision=NpuPrecision.Int8)

    @classmethod
    def npu_int8(cls) -> "ExecutionProvider":
        return cls("Npu", precision=NpuPrecision.Int8)

    @classmethod
    def npu_fp16(cls) -> "ExecutionProvider":
        return cls("Npu", precision=NpuPrecision.Fp16)

    @classmethod
    def Npu(cls, precision: NpuPrecision) -> "ExecutionProvider":
        return cls("Npu", precision=precision)

    @classmethod
    def cpu(cls) -> "ExecutionProvider":
        """`ExecutionProvider::Cpu`: run_standard's f32 arithmetic (mod.rs:260-331)."""
        return cls("Cpu")

    @classmethod
    def gpu(cls, index: int = 0) -> "ExecutionProvider":
        return cls("Gpu", index=index)

    def __eq__(self, o):
        return isinstance(o, ExecutionProvider) and (self.kind, self.index, self.precision) == (
            o.kind, o.index, o.precision)

    def __str__(self) -> str:
        if self.kind == "Npu":
            return f"NPU ({self.precision})"
        if self.kind == "Gpu":
            return f"GPU:{self.index} (FP32)"
        return "CPU (FP32)"


def _precision_code(provider: ExecutionProvider) -> int:
    """rg_session_options.precision: 0 Npu(Int8), 1 Npu(Fp16), 2 the f32 Cpu provider."""
    if provider.kind == "Npu":
        return provider.precision.value
    if provider.kind == "Cpu":
        return 2
    raise _native.RgError(_native.RG_ERR_UNSUPPORTED,
                          f"provider {provider}: the reference's wgpu runtime needs a graphics stack, "
                          "unavailable on this box")


def _fmt_duration(ns: int) -> str:
    """Rust `{:?}` of a `Duration` (e.g. 84.2µs, 1.5ms, 2.000001s)."""
    ns = int(ns)
    if ns >= 1_000_000_000:
        whole, frac, div, unit = ns // 1_000_000_000, ns % 1_000_000_000, 100_000_000, "s"
    elif ns >= 1_000_000:
        whole, frac, div, unit = ns // 1_000_000, ns % 1_000_000, 100_000, "ms"
    elif ns >= 1_000:
        whole, frac, div, unit = ns // 1_000, ns % 1_000, 100, "µs"
    else:
        return f"{ns}ns"
    digits = ""
    while frac > 0 and div > 0:
        digits += str(frac // div)
        frac %= div
        div //= 10
    return f"{whole}.{digits}{unit}" if digits else f"{whole}{unit}"


@dataclass
class OpRecord:  # npu.rs:107-116
    op: str
    macs: int
    duration_ns: int

    @property
    def duration(self) -> _dt.timedelta:
        return _dt.timedelta(microseconds=self.duration_ns / 1000.0)


@dataclass
class NpuProfile:  # npu.rs:118-176
    precision: NpuPrecision
    original_layers: int
    fused_ops: int
    fp32_weight_bytes: int
    npu_weight_bytes: int
    total_macs: int
    total_time_ns: int
    records: list = field(default_factory=list)
    kernel_launches: int = 0

    def compression_ratio(self) -> float:
        if self.npu_weight_bytes == 0:
            return 1.0
        return float(np.float32(self.fp32_weight_bytes) / np.float32(self.npu_weight_bytes))

    def gops(self) -> float:
        secs = max(self.total_time_ns / 1e9, 1e-9)
        return self.total_macs * 2.0 / secs / 1e9

    @property
    def total_time(self) -> _dt.timedelta:
        return _dt.timedelta(microseconds=self.total_time_ns / 1000.0)

    def __str__(self) -> str:
        s = (f"NPU Profile [{self.precision} | layers: {self.original_layers} -> {self.fused_ops} fused | "
             f"weights: {self.fp32_weight_bytes} B -> {self.npu_weight_bytes} B ({self.compression_ratio():.2f}x) | "
             f"MACs: {self.total_macs} | time: {_fmt_duration(self.total_time_ns)} ({self.gops():.2f} GOPS)]\n")
        for r in self.records:
            s += f"  - {r.op:<42} {r.macs:>10} MACs   {_fmt_duration(r.duration_ns)}\n"
        return s


def _layer_structs(layers):
    arr = (_native.LayerSpecC * max(1, len(layers)))()
    keep = []
    for i, l in enumerate(layers):
        s = arr[i]
        s.kind = l.kind
        if l.kind == LINEAR:
            s.in_features, s.out_features = l.in_features, l.out_features
            w, b = l.weight, l.bias
        elif l.kind in (CONV2D, SHORTCUT_CONV2D):
            s.in_channels, s.out_channels, s.kernel = l.in_channels, l.out_channels, l.kernel
            s.stride, s.padding = l.stride, l.padding
            w, b = l.weight, l.bias
        elif l.kind == CHANNEL_AFFINE:
            w, b = l.scale, l.shift
        elif l.kind in (EMBEDDING, RMSNORM, ATTENTION, SWIGLU):
            d = as_dict(l)
            s.in_features, s.out_features = d["in_features"], d.get("out_features", 0)
            s.act_param = d.get("act_param", 0.0)
            w, b = d["weight"], d.get("bias", np.zeros(0, np.float32))
        else:
            w = b = None
            if hasattr(l, "kernel"):
                s.kernel, s.stride = l.kernel, l.stride
            if l.kind == ADAPTIVE_AVGPOOL2D:
                s.kernel, s.stride = l.out_h, l.out_w
            if l.kind in (ACTIVATION, RESIDUAL_END):
                act = l.act if isinstance(l.act, Activation) else Activation(int(l.act))
                s.act, s.act_param = act.code, act.param
        if w is not None:
            w = np.ascontiguousarray(w, np.float32).reshape(-1)
            b = np.ascontiguousarray(b, np.float32).reshape(-1)
            keep += [w, b]
            s.weight, s.weight_len = w.ctypes.data_as(C.POINTER(C.c_float)), w.size
            s.bias, s.bias_len = b.ctypes.data_as(C.POINTER(C.c_float)), b.size
    return arr, keep


class InferenceSession:
    """A compiled Npu program (Int8 or Fp16 arm) resident on one B200."""

    def __init__(self, handle, provider: ExecutionProvider, raw_layers, device: int):
        self._h = handle
        self._provider = provider
        self._raw = list(raw_layers)
        self.device = device

    # -- construction ---------------------------------------------------------------
    @classmethod
    def from_module(cls, model, provider: ExecutionProvider, **kw) -> "InferenceSession":
        """`from_module` (mod.rs:155-159): ``model.eval()``, ``model.export()``, then from_layers."""
        model.eval()
        layers = model.export()
        return cls.from_layers(layers, provider, **kw)

    @classmethod
    def from_layers(cls, layers, provider: ExecutionProvider, device: int = 0,
                    weight_quant: str = "per_tensor", flags: int = 0) -> "InferenceSession":
        """`from_layers` (mod.rs:162-180) -> `npu::compile` on the device library."""
        opts = _native.SessionOptions(device, _precision_code(provider),
                                      {"per_tensor": 0, "per_channel": 1}[weight_quant], flags)
        arr, _keep = _layer_structs(layers)
        h = C.c_void_p()
        _native.check(_native.lib().rg_session_create(arr, len(layers), C.byref(opts), C.byref(h)))
        return cls(h, provider, layers, device)

    @classmethod
    def from_rtim(cls, path: str, provider: ExecutionProvider, device: int = 0,
                  weight_quant: str = "per_tensor", flags: int = 0) -> "InferenceSession":
        """`load_inference_layers(path)` + `from_layers`, parsed by the library itself."""
        from .rtim import load_inference_layers
        opts = _native.SessionOptions(device, _precision_code(provider),
                                      {"per_tensor": 0, "per_channel": 1}[weight_quant], flags)
        h = C.c_void_p()
        _native.check(_native.lib().rg_session_create_from_rtim(str(path).encode(), C.byref(opts), C.byref(h)))
        return cls(h, provider, load_inference_layers(path), device)

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            _native.lib().rg_session_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    # -- reference accessors ----------------------------------------------------------
    def provider(self) -> ExecutionProvider:
        return self._provider

    def raw_layers(self):
        return self._raw

    def compilation_report(self) -> str:
        need = C.c_int64(0)
        _native.check(_native.lib().rg_session_compilation_report(self._h, None, 0, C.byref(need)))
        buf = C.create_string_buffer(need.value)
        _native.check(_native.lib().rg_session_compilation_report(self._h, buf, need.value, C.byref(need)))
        return buf.value.decode()

    def last_npu_profile(self) -> NpuProfile | None:
        prof = _native.ProfileC()
        n = self.num_ops()
        recs = (_native.OpRecordC * max(1, n))()
        st = _native.lib().rg_session_last_profile(self._h, C.byref(prof), recs, n)
        if st == _native.RG_ERR_NO_PROFILE:
            return None
        _native.check(st)
        return NpuProfile(NpuPrecision(prof.precision), prof.original_layers, prof.fused_ops,
                          prof.fp32_weight_bytes, prof.npu_weight_bytes, prof.total_macs, prof.total_time_ns,
                          [OpRecord(recs[i].op.decode(), recs[i].macs, recs[i].duration_ns)
                           for i in range(prof.n_records)], prof.kernel_launches)

    # -- running --------------------------------------------------------------------
    def output_shape(self, shape) -> tuple:
        shape = np.asarray(shape, np.int64)
        ys = np.zeros(_MAX_RANK, np.int64)
        nd = C.c_int32(0)
        _native.check(_native.lib().rg_session_output_shape(
            self._h, shape.ctypes.data_as(C.POINTER(C.c_int64)), shape.size,
            ys.ctypes.data_as(C.POINTER(C.c_int64)), C.byref(nd)))
        return tuple(int(v) for v in ys[: nd.value])

    def run(self, x, out: np.ndarray | None = None) -> np.ndarray:
        """`run` (mod.rs:212-221) on a host array: H2D, the program, D2H."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        shape = np.asarray(x.shape, np.int64)
        oshape = self.output_shape(x.shape)
        if out is None:
            out = np.empty(oshape, np.float32)
        ys = np.zeros(_MAX_RANK, np.int64)
        nd = C.c_int32(0)
        _native.check(_native.lib().rg_session_run(
            self._h, x.ctypes.data_as(C.POINTER(C.c_float)), shape.ctypes.data_as(C.POINTER(C.c_int64)),
            x.ndim, out.ctypes.data_as(C.POINTER(C.c_float)), out.size,
            ys.ctypes.data_as(C.POINTER(C.c_int64)), C.byref(nd)))
        return out.reshape(oshape)

    def run_device(self, x, out=None, stream=None, asynchronous: bool = False):
        """Run on CUDA tensors (torch) of this session's device; returns ``out``."""
        import torch
        if not (x.is_cuda and x.dtype == torch.float32 and x.is_contiguous()):
            raise ValueError("run_device needs a contiguous float32 CUDA tensor")
        oshape = self.output_shape(tuple(x.shape))
        if out is None:
            out = torch.empty(oshape, dtype=torch.float32, device=x.device)
        shape = np.asarray(x.shape, np.int64)
        ys = np.zeros(_MAX_RANK, np.int64)
        nd = C.c_int32(0)
        st = stream if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
        _native.check(_native.lib().rg_session_run_device(
            self._h, C.c_void_p(x.data_ptr()), shape.ctypes.data_as(C.POINTER(C.c_int64)), x.ndim,
            C.c_void_p(out.data_ptr()), out.numel(), ys.ctypes.data_as(C.POINTER(C.c_int64)), C.byref(nd),
            C.c_void_p(st), _native.RG_RUN_ASYNC if asynchronous else 0))
        return out

    # -- introspection and tracing (tests) ----------------------------------------------
    def num_ops(self) -> int:
        n = C.c_int32(0)
        _native.check(_native.lib().rg_session_num_ops(self._h, C.byref(n)))
        return n.value

    def op_info(self, i: int) -> dict:
        info = _native.OpInfoC()
        _native.check(_native.lib().rg_session_op_info(self._h, i, C.byref(info)))
        d = {f: getattr(info, f) for f, _ in _native.OpInfoC._fields_}
        d["label"] = info.label.decode()
        return d

    def op_weights(self, i: int):
        info = self.op_info(i)
        wq = np.empty(info["wq_len"], np.int8)
        b = np.empty(info["bias_len"], np.float32)
        _native.check(_native.lib().rg_session_op_weights(
            self._h, i, wq.ctypes.data_as(C.POINTER(C.c_int8)), wq.size,
            b.ctypes.data_as(C.POINTER(C.c_float)), b.size))
        return wq, b

    # -- static calibration (extension; no counterpart in the reference) -------------
    def calibration_targets(self) -> int:
        """Frozen scales a calibration holds: one per Linear, two per attention / SwiGLU block."""
        n = C.c_int32(0)
        _native.check(_native.lib().rg_session_calibration_targets(self._h, C.byref(n)))
        return n.value

    def calibrate(self, x) -> np.ndarray:
        """Runs x with the reference's dynamic scales and freezes every Linear input's
        scale; later runs quantize with them (no absmax pass, no all-reduce; values
        beyond the calibrated range clamp).  Returns the frozen scales."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        shape = np.asarray(x.shape, np.int64)
        _native.check(_native.lib().rg_session_calibrate(self._h, x.ctypes.data_as(C.POINTER(C.c_float)),
                                                         shape.ctypes.data_as(C.POINTER(C.c_int64)), x.ndim))
        return self.calibration()

    def set_calibration(self, scales) -> None:
        """Install frozen scales, or ``None`` for the reference's dynamic scales."""
        if scales is None:
            _native.check(_native.lib().rg_session_set_calibration(self._h, None, 0))
            return
        sc = np.ascontiguousarray(scales, dtype=np.float32)
        _native.check(_native.lib().rg_session_set_calibration(self._h, sc.ctypes.data_as(C.POINTER(C.c_float)),
                                                               sc.size))

    def calibration(self):
        """The frozen scales, or ``None`` when the session uses dynamic scales."""
        n = self.calibration_targets()
        out = np.empty(max(n, 1), np.float32)
        st = _native.lib().rg_session_get_calibration(self._h, out.ctypes.data_as(C.POINTER(C.c_float)), out.size)
        if st == _native.RG_ERR_INVALID_ARG and "not calibrated" in _native.last_error():
            return None
        _native.check(st)
        return out[:n].copy()

    def set_trace(self, enable: bool) -> None:
        _native.check(_native.lib().rg_session_set_trace(self._h, int(enable)))

    def trace(self, op: int, item: int) -> np.ndarray:
        n = C.c_int64(0)
        _native.check(_native.lib().rg_session_trace_get(self._h, op, item, None, 0, C.byref(n)))
        dt = {_native.RG_TRACE_SCALES: np.float32, _native.RG_TRACE_AQ: np.int8,
              _native.RG_TRACE_ACC: np.int32, _native.RG_TRACE_OUT: np.float32}[item]
        buf = np.empty(n.value // np.dtype(dt).itemsize, dt)
        _native.check(_native.lib().rg_session_trace_get(self._h, op, item, buf.ctypes.data_as(C.c_void_p),
                                                         n.value, C.byref(n)))
        return buf
