"""TEST INFRASTRUCTURE ONLY: a second restatement of the reference's Npu(Int8) path,
in numpy, written from the Rust sources independently of oracle/npu_oracle.c.

It exists to pin the C oracle: tests/test_npu_numpy.py runs both on every golden
case of the reference's layer kinds and requires the same i8 activations, i32
accumulators, activation scales, f32 outputs, labels, byte counts and summary.
Nothing in the product imports it.

What it follows (paths in the reference project):
* fold_batch_norm          src/inference/mod.rs:225-257
* npu::compile             src/inference/npu.rs:188-276 (labels 83-104, summary 280-293)
* NpuProgram::execute      src/inference/npu.rs:296-421 (Int8 arm)
* QuantTensor::from_f32 / quantize_into, byte_size, int8_gemm_fused(_serial)
                           src/inference/quantize.rs:18-45, 93-144
* Activation::apply        src/inference/mod.rs:38-53 -> UnaryOp::apply src/device/backend.rs:61-78
* im2col_into, out_size, max_pool2d
                           src/kernels.rs:10-96, 165-213
* transpose2d              src/tensor/shape.rs:98-123
* softmax_raw              src/tensor/ops.rs:1058-1076

f32 arithmetic is numpy float32 (IEEE single, one rounding per operation, no
contraction); integer sums are exact.  The transcendentals are the ones the
reference calls: Rust's f32::exp / f32::tanh are glibc's expf / tanhf, called
here through ctypes on the host's libm.
"""
from __future__ import annotations

import ctypes
import ctypes.util

import numpy as np

LINEAR, CONV2D, CHANNEL_AFFINE, MAXPOOL2D, FLATTEN, ACTIVATION, SOFTMAX = 1, 2, 3, 4, 5, 6, 7
A_NONE, A_RELU, A_SIGMOID, A_TANH, A_GELU, A_LEAKY = 0, 1, 2, 3, 4, 5

_libm = ctypes.CDLL(ctypes.util.find_library("m"))
_libm.expf.argtypes = [ctypes.c_float]
_libm.expf.restype = ctypes.c_float
_libm.tanhf.argtypes = [ctypes.c_float]
_libm.tanhf.restype = ctypes.c_float
F = np.float32


def _map(fn, x):
    """A libm float function over every element of a float32 array."""
    x = np.asarray(x, F)
    return np.array([fn(float(v)) for v in x.ravel()], F).reshape(x.shape)


def expf(x):
    return _map(_libm.expf, x)


def tanhf(x):
    return _map(_libm.tanhf, x)


# ---- Activation::apply ---------------------------------------------------------------
def act_apply(act: int, param: float, x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, F)
    if act == A_NONE:
        return x
    if act == A_RELU:            # x.max(0.0): f32::max returns the non-NaN operand
        return np.where(np.isnan(x), F(0), np.maximum(x, F(0))).astype(F)
    if act == A_SIGMOID:         # 1.0 / (1.0 + (-x).exp())
        return (F(1) / (F(1) + expf(-x))).astype(F)
    if act == A_TANH:
        return tanhf(x)
    if act == A_GELU:            # 0.5 * x * (1.0 + (GELU_C * (x + 0.044715 * x * x * x)).tanh())
        inner = ((F(0.044715) * x) * x) * x
        t = tanhf(F(0.7978846) * (x + inner))
        return ((F(0.5) * x) * (F(1) + t)).astype(F)
    if act == A_LEAKY:           # if x > 0.0 { x } else { s * x }
        return np.where(x > 0, x, F(param) * x).astype(F)
    raise ValueError(act)


def act_name(act: int, param: float) -> str:
    if act == A_LEAKY:           # Rust `{}` of an f32: shortest round-trip, no exponent
        s = np.format_float_positional(F(param), trim="-")
        return f"LeakyReLU({s})"
    return {A_NONE: "none", A_RELU: "ReLU", A_SIGMOID: "Sigmoid", A_TANH: "Tanh", A_GELU: "GELU"}[act]


# ---- QuantTensor ---------------------------------------------------------------------
def quantize(values: np.ndarray):
    """QuantTensor::from_f32: (i8 data, scale).  max_abs = fold(0, max(|v|)) ignores NaN
    (f32::max); scale = max_abs < 1e-12 ? 1 : max_abs / 127; q = (v * inv).round()
    (half away from zero) .clamp(-127, 127) as i8 (NaN -> 0)."""
    v = np.asarray(values, F).ravel()
    a = np.abs(v)
    a = a[~np.isnan(a)]
    max_abs = F(a.max()) if a.size else F(0)
    scale = F(1) if max_abs < F(1e-12) else F(max_abs / F(127))
    inv = F(F(1) / scale)
    with np.errstate(invalid="ignore", over="ignore"):   # inf * inv, NaN: as the reference
        t = (v * inv).astype(F).astype(np.float64)
    r = np.where(t >= 0, np.floor(t + 0.5), np.ceil(t - 0.5))
    r = np.clip(r, -127, 127)
    r = np.where(np.isnan(r), 0, r)
    return r.astype(np.int8), scale


def quantize_with(values: np.ndarray, scale) -> np.ndarray:
    """The same rounding with a scale taken elsewhere (the image's, for a conv trace)."""
    inv = F(F(1) / F(scale))
    t = (np.asarray(values, F) * inv).astype(F).astype(np.float64)
    r = np.clip(np.where(t >= 0, np.floor(t + 0.5), np.ceil(t - 0.5)), -127, 127)
    return np.where(np.isnan(r), 0, r).astype(np.int8)


def gemm_fused(aq, a_scale, op):
    """int8_gemm_fused: acc = sum_k a*w (exact i32); out = act((acc as f32) * (sa * sw) + bias[c])."""
    n = op["bias"].size
    acc = aq.astype(np.int64) @ op["wq"].reshape(n, -1).astype(np.int64).T
    assert np.abs(acc).max(initial=0) < 2 ** 31
    acc = acc.astype(np.int32)
    cs = F(F(a_scale) * op["ws"])
    with np.errstate(invalid="ignore", over="ignore"):
        val = (acc.astype(F) * cs).astype(F) + op["bias"]
    return act_apply(op["act"][0], op["act"][1], val.astype(F)), acc


# ---- kernels.rs -------------------------------------------------------------------------
def out_size(inp: int, k: int, stride: int, pad: int) -> int:
    padded = inp + 2 * pad
    assert k > 0 and stride > 0 and padded >= k
    return (padded - k) // stride + 1


def im2col(img: np.ndarray, k: int, stride: int, pad: int, oh: int, ow: int) -> np.ndarray:
    """[C, H, W] -> [C*k*k, OH*OW], row (ch*k + ki)*k + kj, zeros outside the image."""
    c, h, w = img.shape
    p = np.zeros((c, h + 2 * pad, w + 2 * pad), F)
    p[:, pad:pad + h, pad:pad + w] = img
    cols = np.empty((c, k, k, oh, ow), F)
    for ki in range(k):
        for kj in range(k):
            cols[:, ki, kj] = p[:, ki:ki + stride * (oh - 1) + 1:stride, kj:kj + stride * (ow - 1) + 1:stride]
    return cols.reshape(c * k * k, oh * ow)


def max_pool2d(x: np.ndarray, k: int, stride: int) -> np.ndarray:
    """Window max in row-major order: best = v when v > best or v is NaN (pad 0)."""
    n, c, h, w = x.shape
    oh, ow = out_size(h, k, stride, 0), out_size(w, k, stride, 0)
    best = np.full((n, c, oh, ow), -np.inf, F)
    for ki in range(k):
        for kj in range(k):
            v = x[:, :, ki:ki + stride * (oh - 1) + 1:stride, kj:kj + stride * (ow - 1) + 1:stride]
            best = np.where((v > best) | np.isnan(v), v, best)
    return best.astype(F)


def softmax(x: np.ndarray) -> np.ndarray:
    """softmax_raw over the last dim: max by fold(-inf, f32::max), exp(x - max), serial f32 sum, divide."""
    shape = x.shape
    x2 = np.asarray(x, F).reshape(-1, shape[-1])
    finite = np.where(np.isnan(x2), -np.inf, x2)
    mx = finite.max(axis=1, initial=-np.inf).astype(F)
    e = expf((x2 - mx[:, None]).astype(F))
    s = np.zeros(x2.shape[0], F)
    for j in range(x2.shape[1]):
        s = (s + e[:, j]).astype(F)
    return (e / s[:, None]).astype(F).reshape(shape)


# ---- compile ----------------------------------------------------------------------------
def fold_batch_norm(layers):
    """A ChannelAffine whose channel count equals the previous Linear / Conv2d's outputs is
    folded into it: w[.., c] *= scale[c], b[c] = b[c] * scale[c] + shift[c]."""
    out = []
    for l in layers:
        l = dict(l)
        if l["kind"] == CHANNEL_AFFINE and out:
            prev = out[-1]
            sc = np.asarray(l["scale"] if "scale" in l else l["weight"], F).ravel()
            sh = np.asarray(l["shift"] if "shift" in l else l["bias"], F).ravel()
            if prev["kind"] == LINEAR and prev["out_features"] == sc.size:
                w = np.asarray(prev["weight"], F).reshape(prev["in_features"], prev["out_features"]).copy()
                prev["weight"] = (w * sc[None, :]).astype(F).ravel()
                prev["bias"] = (np.asarray(prev["bias"], F) * sc + sh).astype(F)
                continue
            if prev["kind"] == CONV2D and prev["out_channels"] == sc.size:
                w = np.asarray(prev["weight"], F).reshape(prev["out_channels"], -1).copy()
                prev["weight"] = (w * sc[:, None]).astype(F).ravel()
                prev["bias"] = (np.asarray(prev["bias"], F) * sc + sh).astype(F)
                continue
        out.append(l)
    return out


def compile_program(layers):
    f = fold_batch_norm(layers)
    ops, fp32_bytes, npu_bytes, i = [], 0, 0, 0
    while i < len(f):
        l = f[i]
        nxt = f[i + 1] if i + 1 < len(f) and f[i + 1]["kind"] == ACTIVATION else None
        act = (nxt["act"], float(nxt.get("act_param", 0.0))) if nxt else (A_NONE, 0.0)
        k = l["kind"]
        if k == LINEAR:
            fin, fout = l["in_features"], l["out_features"]
            w = np.asarray(l["weight"], F).reshape(fin, fout)
            wq, ws = quantize(w.T)              # transpose2d -> [out, in], per tensor
            b = np.asarray(l["bias"], F)
            fp32_bytes += (w.size + b.size) * 4
            npu_bytes += (wq.size + 4) + b.size * 4
            ops.append(dict(kind=LINEAR, fin=fin, fout=fout, wq=wq, ws=ws, bias=b, act=act))
            i += 2 if nxt else 1
        elif k == CONV2D:
            w = np.asarray(l["weight"], F).reshape(l["out_channels"], -1)
            wq, ws = quantize(w)
            b = np.asarray(l["bias"], F)
            fp32_bytes += (w.size + b.size) * 4
            npu_bytes += (wq.size + 4) + b.size * 4
            ops.append(dict(kind=CONV2D, cin=l["in_channels"], cout=l["out_channels"], k=l["kernel"],
                            stride=l["stride"], pad=l["padding"], wq=wq, ws=ws, bias=b, act=act))
            i += 2 if nxt else 1
        elif k == CHANNEL_AFFINE:          # standalone: a diagonal Linear, no byte accounting
            sc = np.asarray(l["scale"] if "scale" in l else l["weight"], F).ravel()
            sh = np.asarray(l["shift"] if "shift" in l else l["bias"], F).ravel()
            c = sc.size
            wq, ws = quantize(np.diag(sc).astype(F))
            ops.append(dict(kind=LINEAR, fin=c, fout=c, wq=wq, ws=ws, bias=sh, act=(A_NONE, 0.0)))
            i += 1
        elif k == MAXPOOL2D:
            ops.append(dict(kind=MAXPOOL2D, k=l["kernel"], stride=l["stride"]))
            i += 1
        elif k in (FLATTEN, SOFTMAX):
            ops.append(dict(kind=k))
            i += 1
        elif k == ACTIVATION:
            ops.append(dict(kind=ACTIVATION, act=(l["act"], float(l.get("act_param", 0.0)))))
            i += 1
        else:
            raise ValueError(f"layer kind {k} is not one of the reference's")
    return dict(ops=ops, fp32_bytes=fp32_bytes, npu_bytes=npu_bytes, raw=len(layers))


def label(op) -> str:
    k = op["kind"]
    if k == LINEAR:
        a = op["act"]
        return (f"NPU::Gemm({op['fin']}->{op['fout']})" if a[0] == A_NONE
                else f"NPU::FusedGemmAct({op['fin']}->{op['fout']}, {act_name(*a)})")
    if k == CONV2D:
        a = op["act"]
        return (f"NPU::Conv2d({op['cin']}->{op['cout']}, k={op['k']})" if a[0] == A_NONE
                else f"NPU::FusedConv2dAct({op['cin']}->{op['cout']}, k={op['k']}, {act_name(*a)})")
    if k == MAXPOOL2D:
        return f"NPU::MaxPool2d(k={op['k']})"
    if k == FLATTEN:
        return "NPU::Flatten"
    if k == ACTIVATION:
        return f"NPU::Act({act_name(*op['act'])})"
    return "NPU::Softmax"


def summary(prog) -> str:
    ratio = 1.0 if prog["npu_bytes"] == 0 else float(F(prog["fp32_bytes"]) / F(prog["npu_bytes"]))
    names = " -> ".join(label(o) for o in prog["ops"])
    return (f"InferenceSession [provider = NPU (INT8), layers: {prog['raw']} -> {len(prog['ops'])} fused ops, "
            f"weights: {prog['fp32_bytes']} B -> {prog['npu_bytes']} B ({ratio:.2f}x compression)]\n"
            f"  Pipeline: {names}")


# ---- execute ----------------------------------------------------------------------------
def execute_traced(prog, x, frozen=None):
    """NpuProgram::execute on the Int8 arm; returns (y, [per-op dict(label, y, and for
    Linear / Conv2d: scales, aq, acc)]).  `frozen` (the static-calibration extension):
    one scale per Linear, in op order, used instead of the batch absmax's."""
    data = np.asarray(x, F)
    trace = []
    li = 0
    for op in prog["ops"]:
        rec = {"label": label(op)}
        k = op["kind"]
        if k == LINEAR:
            rows = data.size // op["fin"]
            a2 = data.reshape(rows, op["fin"])
            if frozen is None:
                aq, sa = quantize(a2)             # per tensor over the whole batch
            else:
                sa = F(frozen[li])
                aq = quantize_with(a2, sa)        # the same rounding and clamp, a fixed scale
            li += 1
            aq = aq.reshape(rows, op["fin"])
            y, acc = gemm_fused(aq, sa, op)
            rec.update(scales=np.array([sa], F), aq=aq, acc=acc)
            data = y.reshape(data.shape[:-1] + (op["fout"],))
        elif k == CONV2D:
            n, c, h, w = data.shape
            oh, ow = out_size(h, op["k"], op["stride"], op["pad"]), out_size(w, op["k"], op["stride"], op["pad"])
            out = np.empty((n, op["cout"], oh, ow), F)
            acc_all = np.empty((n, op["cout"], oh, ow), np.int32)
            scales = np.empty(n, F)
            aq_img = np.empty((n, c, h, w), np.int8)
            for b in range(n):
                cols_t = im2col(data[b], op["k"], op["stride"], op["pad"], oh, ow).T   # [L, ckk]
                q, sa = quantize(cols_t)          # per image, over its im2col matrix
                y, acc = gemm_fused(q.reshape(cols_t.shape), sa, op)
                out[b] = y.T.reshape(op["cout"], oh, ow)
                acc_all[b] = acc.T.reshape(op["cout"], oh, ow)
                scales[b] = sa
                aq_img[b] = quantize_with(data[b], sa)
            rec.update(scales=scales, aq=aq_img, acc=acc_all)
            data = out
        elif k == MAXPOOL2D:
            data = max_pool2d(data, op["k"], op["stride"])
        elif k == FLATTEN:
            data = data.reshape(data.shape[0], -1)
        elif k == ACTIVATION:
            data = act_apply(op["act"][0], op["act"][1], data)
        else:
            data = softmax(data)
        rec["y"] = data
        trace.append(rec)
    return data, trace
