"""TEST INFRASTRUCTURE ONLY: ctypes bindings to the C restatement of the
RustGears Npu(Int8) path (``oracle/npu_oracle.c``).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this module.  It is the parity checker and the timed
CPU baseline; the product library never calls it.

Layer specs are duck-typed: any object with the attributes of the reference's
``LayerSpec`` (``inference/mod.rs:70-100``) -- ``kind`` (RTIM tag 1..7),
``in_features``/``out_features``, ``in_channels``/``out_channels``/``kernel``/
``stride``/``padding``, ``weight``/``bias`` (f32 arrays; ``scale``/``shift``
for ChannelAffine), ``act``/``act_param`` -- or a dict with those keys.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

LINEAR, CONV2D, CHANNEL_AFFINE, MAXPOOL2D, FLATTEN, ACTIVATION, SOFTMAX = 1, 2, 3, 4, 5, 6, 7
# extensions (no reference LayerSpec): residual blocks, adaptive average pooling
RESIDUAL_BEGIN, RESIDUAL_END, SHORTCUT_CONV2D, ADAPTIVE_AVGPOOL2D = 8, 9, 10, 11
# extensions for the transformer configuration
EMBEDDING, RMSNORM, ATTENTION, SWIGLU = 12, 13, 14, 15
ACT_NONE, ACT_RELU, ACT_SIGMOID, ACT_TANH, ACT_GELU, ACT_LEAKY_RELU = 0, 1, 2, 3, 4, 5
ACT_SILU = 6  # extension: nn::Silu (nn/layers.rs:337-346)


class _Rng(C.Structure):
    _fields_ = [("state", C.c_uint64)]


class _Layer(C.Structure):
    _fields_ = [
        ("kind", C.c_int32), ("in_features", C.c_int32), ("out_features", C.c_int32),
        ("in_channels", C.c_int32), ("out_channels", C.c_int32), ("kernel", C.c_int32),
        ("stride", C.c_int32), ("padding", C.c_int32),
        ("weight", C.POINTER(C.c_float)), ("weight_len", C.c_int64),
        ("bias", C.POINTER(C.c_float)), ("bias_len", C.c_int64),
        ("act", C.c_int32), ("act_param", C.c_float),
    ]


class _Op(C.Structure):
    pass


_Op._fields_ = [
    ("kind", C.c_int32), ("in_features", C.c_int32), ("out_features", C.c_int32),
    ("in_channels", C.c_int32), ("out_channels", C.c_int32), ("kernel", C.c_int32),
    ("stride", C.c_int32), ("padding", C.c_int32),
    ("wq", C.POINTER(C.c_int8)), ("wq_len", C.c_int64), ("w_scale", C.c_float),
    ("bias", C.POINTER(C.c_float)), ("bias_len", C.c_int64),
    ("act", C.c_int32), ("act_param", C.c_float),
    ("sub", C.POINTER(_Op)), ("n_sub", C.c_int32), ("_pad2", C.c_int32),
    ("extra", C.POINTER(C.c_float)), ("extra_len", C.c_int64),
    ("wh", C.POINTER(C.c_float)), ("wh_len", C.c_int64),
    ("w_scale_ch", C.POINTER(C.c_float)),
    ("frozen", C.c_int32), ("frozen_scale", C.c_float), ("seen_scale", C.c_float), ("_pad3", C.c_int32),
]


class _Program(C.Structure):
    _fields_ = [
        ("precision", C.c_int32), ("original_layers", C.c_int32), ("n_ops", C.c_int32),
        ("_pad", C.c_int32), ("ops", C.POINTER(_Op)),
        ("fp32_bytes", C.c_int64), ("npu_bytes", C.c_int64),
    ]


def build():
    """Compile liboracle.so with oracle/Makefile (gcc)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        f32p, i8p, i32p, i64p = (C.POINTER(C.c_float), C.POINTER(C.c_int8),
                                 C.POINTER(C.c_int32), C.POINTER(C.c_int64))
        L.og_rng_seed.argtypes = [C.POINTER(_Rng), C.c_uint64]
        L.og_rng_next_u64.argtypes = [C.POINTER(_Rng)]
        L.og_rng_next_u64.restype = C.c_uint64
        L.og_rng_uniform.argtypes = [C.POINTER(_Rng)]
        L.og_rng_uniform.restype = C.c_float
        L.og_rng_normal.argtypes = [C.POINTER(_Rng)]
        L.og_rng_normal.restype = C.c_float
        L.og_fill_uniform_range.argtypes = [C.POINTER(_Rng), f32p, C.c_int64, C.c_float, C.c_float]
        L.og_fill_normal.argtypes = [C.POINTER(_Rng), f32p, C.c_int64]
        L.og_fill_normal_scaled.argtypes = [C.POINTER(_Rng), f32p, C.c_int64, C.c_float]
        L.og_fill_below.argtypes = [C.POINTER(_Rng), i64p, C.c_int64, C.c_uint64]
        L.og_kaiming_bound.argtypes = [C.c_int64]
        L.og_kaiming_bound.restype = C.c_float
        L.og_bias_bound.argtypes = [C.c_int64]
        L.og_bias_bound.restype = C.c_float
        L.og_act_apply.argtypes = [C.c_int32, C.c_float, C.c_float]
        L.og_act_apply.restype = C.c_float
        L.og_quantize_into.argtypes = [f32p, C.c_int64, i8p]
        L.og_quantize_into.restype = C.c_float
        L.og_round_fp16.argtypes = [C.c_float]
        L.og_round_fp16.restype = C.c_float
        L.og_compile.argtypes = [C.POINTER(_Layer), C.c_int32, C.c_int32]
        L.og_compile.restype = C.POINTER(_Program)
        L.og_compile_ex.argtypes = [C.POINTER(_Layer), C.c_int32, C.c_int32, C.c_int32]
        L.og_compile_ex.restype = C.POINTER(_Program)
        L.og_program_free.argtypes = [C.POINTER(_Program)]
        L.og_op_label.argtypes = [C.POINTER(_Op), C.c_char_p, C.c_int32]
        L.og_op_label.restype = C.c_int32
        L.og_program_summary.argtypes = [C.POINTER(_Program), C.c_int32, C.c_char_p, C.c_int32]
        L.og_program_summary.restype = C.c_int32
        L.og_op_linear.argtypes = [C.POINTER(_Op), f32p, C.c_int64, f32p, f32p, i8p, i32p, C.c_int32]
        L.og_op_linear_with_amax.argtypes = [C.POINTER(_Op), f32p, C.c_int64, C.c_float, f32p, C.c_int32]
        L.og_op_linear_rows.argtypes = [C.POINTER(_Op), f32p, C.c_int64, C.c_int64, C.c_int64,
                                        f32p, f32p, i32p, C.c_int32]
        L.og_op_conv2d.argtypes = [C.POINTER(_Op), f32p, C.c_int64, C.c_int32, C.c_int32, f32p,
                                   f32p, i8p, i32p, C.c_int32]
        L.og_maxpool2d.argtypes = [f32p, C.c_int64, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                   C.c_int32, f32p, C.c_int32]
        L.og_activation.argtypes = [f32p, C.c_int64, C.c_int32, C.c_float, f32p]
        L.og_softmax.argtypes = [f32p, C.c_int64, C.c_int64, f32p]
        L.og_adaptive_avgpool2d.argtypes = [f32p, C.c_int64, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                            C.c_int32, f32p]
        L.og_residual_add.argtypes = [f32p, f32p, C.c_int64, C.c_int32, C.c_float, f32p]
        L.og_embedding.argtypes = [C.POINTER(_Op), f32p, C.c_int64, f32p]
        L.og_embedding.restype = C.c_int32
        L.og_rmsnorm.argtypes = [C.POINTER(_Op), f32p, C.c_int64, f32p]
        L.og_attention.argtypes = [C.POINTER(_Op), f32p, C.c_int64, C.c_int64, f32p, C.c_int32]
        L.og_swiglu.argtypes = [C.POINTER(_Op), f32p, C.c_int64, f32p, C.c_int32]
        L.og_bmm_fma.argtypes = [f32p, f32p, C.c_int64, C.c_int64, C.c_int64, C.c_int64, f32p]
        L.og_out_size.argtypes = [C.c_int64] * 4
        L.og_out_size.restype = C.c_int64
        L.og_im2col.argtypes = [f32p] + [C.c_int32] * 8 + [f32p]
        L.og_execute.argtypes = [C.POINTER(_Program), f32p, i64p, C.c_int32, f32p, C.c_int64,
                                 i64p, i32p, C.c_int32, i64p, i64p]
        L.og_execute.restype = C.c_int32
        L.og_run_standard.argtypes = [C.POINTER(_Layer), C.c_int32, f32p, i64p, C.c_int32, f32p, C.c_int64,
                                      i64p, i32p]
        L.og_run_standard.restype = C.c_int32
        _lib = L
    return _lib


def _p(a, ct):
    return a.ctypes.data_as(C.POINTER(ct)) if a is not None else None


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# --------------------------------------------------------------------------
# RNG (src/rng.rs)
# --------------------------------------------------------------------------
class Rng:
    """SplitMix64 generator with the reference's f32 draws (rng.rs:10-58).

    ``Rng(42)`` is the state ``manual_seed(42)`` installs (rng.rs:71-73)."""

    def __init__(self, seed: int):
        self._s = _Rng()
        lib().og_rng_seed(C.byref(self._s), C.c_uint64(seed))

    def next_u64(self) -> int:
        return lib().og_rng_next_u64(C.byref(self._s))

    def uniform(self) -> float:
        return lib().og_rng_uniform(C.byref(self._s))

    def normal(self) -> float:
        return lib().og_rng_normal(C.byref(self._s))

    def uniform_tensor(self, shape, lo, hi) -> np.ndarray:  # Tensor::uniform (tensor/mod.rs:128-131)
        out = np.empty(int(np.prod(shape)), np.float32)
        lib().og_fill_uniform_range(C.byref(self._s), _p(out, C.c_float), out.size,
                                    C.c_float(lo), C.c_float(hi))
        return out.reshape(shape)

    def randn(self, shape) -> np.ndarray:  # Tensor::randn (tensor/mod.rs:116-119)
        out = np.empty(int(np.prod(shape)), np.float32)
        lib().og_fill_normal(C.byref(self._s), _p(out, C.c_float), out.size)
        return out.reshape(shape)

    def normal_init(self, shape, std) -> np.ndarray:  # init::normal (nn/init.rs:18-20)
        out = np.empty(int(np.prod(shape)), np.float32)
        lib().og_fill_normal_scaled(C.byref(self._s), _p(out, C.c_float), out.size, C.c_float(std))
        return out.reshape(shape)

    def below(self, shape, n) -> np.ndarray:  # Rng::below (rng.rs:47-49)
        out = np.empty(int(np.prod(shape)), np.int64)
        lib().og_fill_below(C.byref(self._s), _p(out, C.c_int64), out.size, C.c_uint64(n))
        return out.reshape(shape)

    def kaiming_uniform(self, shape, fan_in):  # nn/init.rs:6-9
        b = lib().og_kaiming_bound(fan_in)
        return self.uniform_tensor(shape, -b, b)

    def bias_uniform(self, shape, fan_in):  # nn/init.rs:23-26
        b = lib().og_bias_bound(fan_in)
        return self.uniform_tensor(shape, -b, b)


# --------------------------------------------------------------------------
# compile / program
# --------------------------------------------------------------------------
def _get(spec, name, default=None):
    if isinstance(spec, dict):
        return spec.get(name, default)
    return getattr(spec, name, default)


def _to_layers(specs):
    keep = []
    arr = (_Layer * max(1, len(specs)))()
    for i, s in enumerate(specs):
        L = arr[i]
        kind = int(_get(s, "kind"))
        L.kind = kind
        for f in ("in_features", "out_features", "in_channels", "out_channels", "kernel",
                  "stride", "padding"):
            setattr(L, f, int(_get(s, f, 0) or 0))
        if kind == CHANNEL_AFFINE:
            w, b = _get(s, "scale"), _get(s, "shift")
        else:
            w, b = _get(s, "weight"), _get(s, "bias")
        if w is not None:
            w = _f32(w).reshape(-1)
            keep.append(w)
            L.weight, L.weight_len = _p(w, C.c_float), w.size
        if b is not None:
            b = _f32(b).reshape(-1)
            keep.append(b)
            L.bias, L.bias_len = _p(b, C.c_float), b.size
        L.act = int(_get(s, "act", 0) or 0)
        L.act_param = float(_get(s, "act_param", 0.0) or 0.0)
    return arr, keep


class Op:
    """Read-only view of one compiled NpuOp (npu.rs:43-79)."""

    def __init__(self, raw: _Op):
        self.raw = raw
        for f, _ in _Op._fields_:
            if f not in ("wq", "bias", "sub", "extra", "wh", "w_scale_ch", "frozen", "frozen_scale", "seen_scale"):
                setattr(self, f, getattr(raw, f))
        self.sub = [Op(raw.sub[j]) for j in range(raw.n_sub)]
        self.wq = np.ctypeslib.as_array(raw.wq, shape=(raw.wq_len,)).copy() if raw.wq_len else None
        self.bias = np.ctypeslib.as_array(raw.bias, shape=(raw.bias_len,)).copy() if raw.bias_len else None
        self.wh = np.ctypeslib.as_array(raw.wh, shape=(raw.wh_len,)).copy() if raw.wh_len else None
        # per-output-channel weight scales (weight_quant=1), else None
        nsc = raw.out_features if raw.kind == LINEAR else raw.out_channels
        self.w_scale_ch = (np.ctypeslib.as_array(raw.w_scale_ch, shape=(nsc,)).copy()
                           if bool(raw.w_scale_ch) and nsc > 0 else None)

    def label(self) -> str:
        buf = C.create_string_buffer(256)
        lib().og_op_label(C.byref(self.raw), buf, 256)
        return buf.value.decode()


class Program:
    """``npu::compile`` output (npu.rs:188-276) plus per-op executors."""

    def __init__(self, specs, precision: int = 0, weight_quant: int = 0):
        """weight_quant 0: per-tensor weights (the reference, quantize.rs:18-24);
        1: per output channel (extension: the fused-Linear benchmark's "symmetric per-channel")."""
        arr, keep = _to_layers(list(specs))
        self._p = lib().og_compile_ex(arr, len(specs), precision, weight_quant)
        P = self._p.contents
        self.precision = P.precision
        self.original_layers = P.original_layers
        self.fp32_bytes = P.fp32_bytes
        self.npu_bytes = P.npu_bytes
        self.ops = [Op(P.ops[i]) for i in range(P.n_ops)]

    def __del__(self):
        try:
            lib().og_program_free(self._p)
        except Exception:
            pass

    # ---- static calibration (extension; no counterpart in the reference) ----------
    # One frozen per-tensor scale per Linear input: a Linear has one; an attention
    # block two (its input, shared by the q / k / v projections, and the attention
    # output that Wo reads); a SwiGLU block two (its input, shared by gate and up, and
    # the gated product that the down projection reads).
    def _calib_targets(self):
        out = []
        for i in range(len(self.ops)):
            raw = self._p.contents.ops[i]
            if raw.kind == LINEAR:
                out.append([raw])
            elif raw.kind == ATTENTION:
                out += [[raw.sub[0], raw.sub[1], raw.sub[2]], [raw.sub[3]]]
            elif raw.kind == SWIGLU:
                out += [[raw.sub[0], raw.sub[1]], [raw.sub[2]]]
        return out

    def calibrate(self, x, nthreads: int = 1) -> np.ndarray:
        """Runs x with the reference's dynamic scales and returns, per calibration
        target, the scale its Linear quantized with (the batch absmax / 127)."""
        self.set_calibration(None)
        self.execute(x, nthreads=nthreads)
        return self.seen_scales()

    def seen_scales(self) -> np.ndarray:
        """Per calibration target, the scale the last run (execute or run_sharded)
        quantized with: a sharded calibration reads them after run_sharded."""
        return np.array([t[0].seen_scale for t in self._calib_targets()], np.float32)

    def set_calibration(self, scales) -> None:
        """Freeze the Linear input scales (None: back to the reference's dynamic scales)."""
        targets = self._calib_targets()
        if scales is not None and len(scales) != len(targets):
            raise ValueError(f"{len(targets)} calibration scales expected, got {len(scales)}")
        for j, group in enumerate(targets):
            for raw in group:
                raw.frozen = 0 if scales is None else 1
                raw.frozen_scale = 0.0 if scales is None else float(np.float32(scales[j]))

    def summary(self, raw_count: int) -> str:
        buf = C.create_string_buffer(1 << 16)
        lib().og_program_summary(self._p, raw_count, buf, 1 << 16)
        return buf.value.decode()

    def compression_ratio(self) -> float:
        return 1.0 if self.npu_bytes == 0 else float(np.float32(self.fp32_bytes) / np.float32(self.npu_bytes))

    def execute(self, x, nthreads: int = 1):
        """Whole-program execute (npu.rs:296-421). Returns (y, per-op ns, per-op MACs)."""
        x = _f32(x)
        shape = np.array(x.shape, np.int64)
        cap = _out_capacity(self, x.shape)
        y = np.empty(cap, np.float32)
        ys = np.zeros(8, np.int64)
        nd = C.c_int32(0)
        ns = np.zeros(len(self.ops), np.int64)
        macs = np.zeros(len(self.ops), np.int64)
        rc = lib().og_execute(self._p, _p(x, C.c_float), _p(shape, C.c_int64), x.ndim,
                              _p(y, C.c_float), cap, _p(ys, C.c_int64), C.byref(nd), nthreads,
                              _p(ns, C.c_int64), _p(macs, C.c_int64))
        if rc != 0:
            raise RuntimeError(f"og_execute failed with {rc}")
        out_shape = tuple(int(v) for v in ys[: nd.value])
        return y[: int(np.prod(out_shape))].reshape(out_shape).copy(), ns, macs

    def run_sharded(self, x, allreduce_max, nthreads: int = 1):
        """Execute one batch shard; every Linear quantizes with
        ``allreduce_max(local_absmax)`` (the max over all shards)."""
        data = _f32(x)
        saved = []
        for i, op in enumerate(self.ops):
            if op.kind == LINEAR:
                rows = data.size // op.in_features
                a = np.abs(data.reshape(-1))
                local = np.float32(np.nanmax(a)) if a.size and not np.isnan(a).all() else np.float32(0)
                amax = np.float32(allreduce_max(max(local, np.float32(0))))
                y = np.empty((rows, op.out_features), np.float32)
                lib().og_op_linear_with_amax(C.byref(self._p.contents.ops[i]), _p(data, C.c_float), rows,
                                             C.c_float(amax), _p(y, C.c_float), nthreads)
                y = y.reshape(data.shape[:-1] + (op.out_features,))
            elif op.kind == CONV2D:
                n, c, h, w = data.shape
                oh = lib().og_out_size(h, op.kernel, op.stride, op.padding)
                ow = lib().og_out_size(w, op.kernel, op.stride, op.padding)
                y = np.empty((n, op.out_channels, oh, ow), np.float32)
                lib().og_op_conv2d(C.byref(self._p.contents.ops[i]), _p(data, C.c_float), n, h, w,
                                   _p(y, C.c_float), None, None, None, nthreads)
            elif op.kind == MAXPOOL2D:
                y = maxpool2d(data, op.kernel, op.stride, nthreads)
            elif op.kind == FLATTEN:
                y = data.reshape(data.shape[0], -1)
            elif op.kind == ACTIVATION:
                y = activation(data, op.act, op.act_param)
            elif op.kind == SOFTMAX:
                y = softmax(data)
            elif op.kind in (ATTENTION, SWIGLU):
                y = self._inner_sharded(i, op, data, allreduce_max, nthreads)
            else:
                y = self._extension_step(i, op, data, saved, nthreads)
            data = np.ascontiguousarray(y)
        return data

    def _inner_sharded(self, i, op, data, allreduce_max, nthreads):
        """Attention / SwiGLU on one batch shard: each inner Linear quantizes with the
        max over all shards of its input's absmax (og_attention / og_swiglu composed
        from the oracle's pieces with that scale)."""
        raw = self._p.contents.ops[i]

        def lin(j, v):
            v = np.ascontiguousarray(v, np.float32)
            sub = raw.sub[j]
            rows = v.size // sub.in_features
            a = np.abs(v.reshape(-1))
            local = np.float32(np.nanmax(a)) if a.size and not np.isnan(a).all() else np.float32(0)
            amax = np.float32(allreduce_max(max(local, np.float32(0))))
            y = np.empty((rows, sub.out_features), np.float32)
            lib().og_op_linear_with_amax(C.byref(sub), _p(v, C.c_float), rows, C.c_float(amax), _p(y, C.c_float),
                                         nthreads)
            return y
        d = op.in_features
        x2 = data.reshape(-1, d)
        if op.kind == SWIGLU:
            g, u = self._two(lin, x2)
            m = (g * act_apply(2, 0.0, g)).astype(np.float32)
            m = (m * u).astype(np.float32)
            return lin(2, m).reshape(data.shape)
        b, t, _ = data.shape
        h = op.out_features
        dh = d // h
        q, k, v = (lin(j, x2).reshape(b, t, h, dh).transpose(0, 2, 1, 3).reshape(b * h, t, dh).copy()
                   for j in range(3))
        kt = np.ascontiguousarray(k.transpose(0, 2, 1))
        sc = np.empty((b * h, t, t), np.float32)
        lib().og_bmm_fma(_p(q, C.c_float), _p(kt, C.c_float), b * h, t, dh, t, _p(sc, C.c_float))
        sc = (sc * (np.float32(1.0) / np.sqrt(np.float32(dh))).astype(np.float32)).astype(np.float32)
        pm = np.ascontiguousarray(softmax(sc))
        o = np.empty((b * h, t, dh), np.float32)
        lib().og_bmm_fma(_p(pm, C.c_float), _p(v, C.c_float), b * h, t, t, dh, _p(o, C.c_float))
        merged = o.reshape(b, h, t, dh).transpose(0, 2, 1, 3).reshape(b * t, d)
        return lin(3, merged).reshape(data.shape)

    @staticmethod
    def _two(lin, x2):
        return lin(0, x2), lin(1, x2)

    def _conv_on(self, i, op, data, nthreads):
        n, c, h, w = data.shape
        oh = lib().og_out_size(h, op.kernel, op.stride, op.padding)
        ow = lib().og_out_size(w, op.kernel, op.stride, op.padding)
        y = np.empty((n, op.out_channels, oh, ow), np.float32)
        lib().og_op_conv2d(C.byref(self._p.contents.ops[i]), _p(data, C.c_float), n, h, w,
                           _p(y, C.c_float), None, None, None, nthreads)
        return y

    def _extension_step(self, i, op, data, saved, nthreads):
        """Residual blocks and adaptive pooling (extension kinds): returns the new main tensor."""
        if op.kind == RESIDUAL_BEGIN:
            saved.append(np.ascontiguousarray(data).copy())
            return data
        if op.kind == SHORTCUT_CONV2D:
            saved[-1] = self._conv_on(i, op, saved[-1], nthreads)
            return data
        if op.kind == RESIDUAL_END:
            return residual_add(data, saved.pop(), op.act, op.act_param)
        if op.kind == ADAPTIVE_AVGPOOL2D:
            return adaptive_avgpool2d(data, op.kernel, op.stride)
        raw = C.byref(self._p.contents.ops[i])
        data = _f32(data)
        if op.kind == EMBEDDING:
            y = np.empty(data.shape + (op.out_features,), np.float32)
            if lib().og_embedding(raw, _p(data, C.c_float), data.size, _p(y, C.c_float)) != 0:
                raise IndexError("Embedding: index out of range")
            return y
        y = np.empty_like(data)
        if op.kind == RMSNORM:
            lib().og_rmsnorm(raw, _p(data, C.c_float), data.size // op.in_features, _p(y, C.c_float))
        elif op.kind == ATTENTION:
            b, t, _ = data.shape
            lib().og_attention(raw, _p(data, C.c_float), b, t, _p(y, C.c_float), nthreads)
        elif op.kind == SWIGLU:
            lib().og_swiglu(raw, _p(data, C.c_float), data.size // op.in_features, _p(y, C.c_float), nthreads)
        else:
            raise ValueError(op.kind)
        return y

    def run_traced(self, x, nthreads: int = 1):
        """Execute op by op and record every intermediate (for golden vectors):
        a list of dicts with the op label, input, a_scale(s), i8 activations,
        i32 accumulators and the f32 output."""
        trace = []
        data = _f32(x)
        saved = []
        for i, op in enumerate(self.ops):
            rec = {"label": op.label(), "kind": op.kind}
            if op.kind == LINEAR:
                rows = data.size // op.in_features
                y = np.empty((rows, op.out_features), np.float32)
                aq = np.empty((rows, op.in_features), np.int8)
                acc = np.empty((rows, op.out_features), np.int32)
                sa = C.c_float(0)
                lib().og_op_linear(C.byref(self._p.contents.ops[i]), _p(data, C.c_float), rows,
                                   _p(y, C.c_float), C.byref(sa), _p(aq, C.c_int8), _p(acc, C.c_int32),
                                   nthreads)
                rec.update(a_scale=np.float32(sa.value), aq=aq, acc=acc)
                y = y.reshape(data.shape[:-1] + (op.out_features,))
            elif op.kind == CONV2D:
                n, c, h, w = data.shape
                oh = lib().og_out_size(h, op.kernel, op.stride, op.padding)
                ow = lib().og_out_size(w, op.kernel, op.stride, op.padding)
                y = np.empty((n, op.out_channels, oh, ow), np.float32)
                sc = np.empty(n, np.float32)
                aq = np.empty((n, c, h, w), np.int8)
                acc = np.empty((n, op.out_channels, oh, ow), np.int32)
                lib().og_op_conv2d(C.byref(self._p.contents.ops[i]), _p(data, C.c_float), n, h, w,
                                   _p(y, C.c_float), _p(sc, C.c_float), _p(aq, C.c_int8),
                                   _p(acc, C.c_int32), nthreads)
                rec.update(a_scales=sc, aq=aq, acc=acc)
            elif op.kind == MAXPOOL2D:
                y = maxpool2d(data, op.kernel, op.stride, nthreads)
            elif op.kind == FLATTEN:
                y = data.reshape(data.shape[0], -1)
            elif op.kind == ACTIVATION:
                y = activation(data, op.act, op.act_param)
            elif op.kind == SOFTMAX:
                y = softmax(data)
            else:
                y = self._extension_step(i, op, data, saved, nthreads)
            # a shortcut conv's output is the new saved block input; the main path goes on
            rec["y"] = saved[-1] if op.kind == SHORTCUT_CONV2D else y
            trace.append(rec)
            data = np.ascontiguousarray(y)
        return data, trace


def _out_capacity(prog: Program, in_shape) -> int:
    """Upper bound on every intermediate's element count (shape walk of execute)."""
    shape = list(in_shape)
    best = int(np.prod(shape))
    for op in prog.ops:
        if op.kind == LINEAR:
            shape[-1] = op.out_features
        elif op.kind == CONV2D:
            n, _, h, w = shape
            shape = [n, op.out_channels, int(lib().og_out_size(h, op.kernel, op.stride, op.padding)),
                     int(lib().og_out_size(w, op.kernel, op.stride, op.padding))]
        elif op.kind == MAXPOOL2D:
            n, c, h, w = shape
            shape = [n, c, int(lib().og_out_size(h, op.kernel, op.stride, 0)),
                     int(lib().og_out_size(w, op.kernel, op.stride, 0))]
        elif op.kind == FLATTEN:
            shape = [shape[0], int(np.prod(shape[1:]))]
        elif op.kind == ADAPTIVE_AVGPOOL2D:
            shape = [shape[0], shape[1], op.kernel, op.stride]
        elif op.kind == EMBEDDING:
            shape = shape + [op.out_features]
        elif op.kind == SWIGLU:
            best = max(best, int(np.prod(shape[:-1])) * op.out_features)
        best = max(best, int(np.prod(shape)))
    return max(best, 1)


# --------------------------------------------------------------------------
# single kernels
# --------------------------------------------------------------------------
def quantize(x):
    """QuantTensor::from_f32 (quantize.rs:18-24) -> (i8 array, scale)."""
    x = _f32(x)
    q = np.empty(x.shape, np.int8)
    s = lib().og_quantize_into(_p(x, C.c_float), x.size, _p(q, C.c_int8))
    return q, np.float32(s)


def act_apply(act: int, param: float, x):
    x = _f32(x)
    y = np.empty_like(x)
    lib().og_activation(_p(x, C.c_float), x.size, act, C.c_float(param), _p(y, C.c_float))
    return y


def activation(x, act: int, param: float = 0.0):
    return act_apply(act, param, x)


def maxpool2d(x, k: int, stride: int, nthreads: int = 1):
    x = _f32(x)
    n, c, h, w = x.shape
    oh = lib().og_out_size(h, k, stride, 0)
    ow = lib().og_out_size(w, k, stride, 0)
    y = np.empty((n, c, oh, ow), np.float32)
    lib().og_maxpool2d(_p(x, C.c_float), n, c, h, w, k, stride, _p(y, C.c_float), nthreads)
    return y


def softmax(x):
    x = _f32(x)
    last = x.shape[-1]
    y = np.empty_like(x)
    lib().og_softmax(_p(x, C.c_float), x.size // last if last else 0, last, _p(y, C.c_float))
    return y


def adaptive_avgpool2d(x, oh: int, ow: int):
    x = _f32(x)
    n, c, h, w = x.shape
    y = np.empty((n, c, oh, ow), np.float32)
    lib().og_adaptive_avgpool2d(_p(x, C.c_float), n, c, h, w, oh, ow, _p(y, C.c_float))
    return y


def residual_add(x, s, act: int, param: float = 0.0):
    x, s = _f32(x), _f32(s)
    assert x.shape == s.shape
    y = np.empty_like(x)
    lib().og_residual_add(_p(x, C.c_float), _p(s, C.c_float), x.size, act, C.c_float(param), _p(y, C.c_float))
    return y


def attention_core(qkv, b: int, t: int, heads: int, dh: int):
    """The f32 core of og_attention on projected q, k, v: qkv [b*t, 3d] -> [b*t, d]
    (heads split, bmm with k^T in the CPU matmul's FMA order, * 1/sqrt(dh), softmax,
    bmm with v, heads merged; nn/attention.rs:178-196)."""
    d = heads * dh
    qkv = _f32(qkv).reshape(b, t, 3, heads, dh)
    q, k, v = (np.ascontiguousarray(qkv[:, :, j].transpose(0, 2, 1, 3).reshape(b * heads, t, dh)) for j in range(3))
    kt = np.ascontiguousarray(k.transpose(0, 2, 1))
    sc = np.empty((b * heads, t, t), np.float32)
    lib().og_bmm_fma(_p(q, C.c_float), _p(kt, C.c_float), b * heads, t, dh, t, _p(sc, C.c_float))
    sc = (sc * (np.float32(1.0) / np.sqrt(np.float32(dh))).astype(np.float32)).astype(np.float32)
    pm = np.ascontiguousarray(softmax(sc))
    o = np.empty((b * heads, t, dh), np.float32)
    lib().og_bmm_fma(_p(pm, C.c_float), _p(v, C.c_float), b * heads, t, t, dh, _p(o, C.c_float))
    return o.reshape(b, heads, t, dh).transpose(0, 2, 1, 3).reshape(b * t, d)


def linear_rows(op: Op, prog: Program, op_index: int, x, r0: int, r1: int, nthreads: int = 1):
    """FusedLinear on rows [r0, r1) with the activation scale over the whole x
    (row sampling for shapes too large for the CPU)."""
    x = _f32(x)
    rows = x.size // op.in_features
    y = np.empty((r1 - r0, op.out_features), np.float32)
    acc = np.empty((r1 - r0, op.out_features), np.int32)
    sa = C.c_float(0)
    lib().og_op_linear_rows(C.byref(prog._p.contents.ops[op_index]), _p(x, C.c_float), rows, r0, r1,
                            _p(y, C.c_float), C.byref(sa), _p(acc, C.c_int32), nthreads)
    return y, acc, np.float32(sa.value)


def linear_given_amax(prog: Program, op_index: int, x, amax: float, nthreads: int = 1):
    """FusedLinear (npu.rs:307-318) on the rows of x, quantized with the scale of the
    given absmax instead of x's own: the absmax of a larger tensor these rows were
    sampled from (or of every shard of a sharded batch)."""
    x = _f32(x)
    op = prog._p.contents.ops[op_index]
    rows = x.size // op.in_features
    y = np.empty((rows, op.out_features), np.float32)
    lib().og_op_linear_with_amax(C.byref(op), _p(x, C.c_float), rows, C.c_float(amax), _p(y, C.c_float), nthreads)
    return y


def run_standard(specs, x):
    """The f32 ExecutionProvider::Cpu arm: fold_batch_norm + run_standard (mod.rs:162-166,
    260-331), the matmuls in the reference CPU matmul's FMA order (og_bmm_fma)."""
    arr, keep = _to_layers(list(specs))
    x = _f32(x)
    shape = np.array(x.shape, np.int64)
    cap = max(1, _out_capacity(Program(specs), x.shape))  # shapes are those of the Int8 program
    y = np.empty(cap, np.float32)
    ys = np.zeros(8, np.int64)
    nd = C.c_int32(0)
    rc = lib().og_run_standard(arr, len(specs), _p(x, C.c_float), _p(shape, C.c_int64), x.ndim, _p(y, C.c_float), cap,
                               _p(ys, C.c_int64), C.byref(nd))
    if rc != 0:
        raise RuntimeError(f"og_run_standard failed with {rc}")
    out_shape = tuple(int(v) for v in ys[: nd.value])
    return y[: int(np.prod(out_shape))].reshape(out_shape).copy()
