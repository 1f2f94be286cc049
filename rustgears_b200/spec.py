"""The portable layer IR: ``LayerSpec`` and ``Activation``
(src/inference/mod.rs:24-100), with the reference's Display strings."""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

LINEAR, CONV2D, CHANNEL_AFFINE, MAXPOOL2D, FLATTEN, ACTIVATION, SOFTMAX = 1, 2, 3, 4, 5, 6, 7
# extensions (no reference LayerSpec): residual blocks, adaptive average pooling
RESIDUAL_BEGIN, RESIDUAL_END, SHORTCUT_CONV2D, ADAPTIVE_AVGPOOL2D = 8, 9, 10, 11
# extensions for transformer encoders: token embedding, RMSNorm, multi-head attention, SwiGLU
EMBEDDING, RMSNORM, ATTENTION, SWIGLU = 12, 13, 14, 15


def _fmt_f32(v: float) -> str:
    """Rust `{}` of an f32: the shortest decimal that round-trips, no exponent."""
    f = np.float32(v)
    for prec in range(0, 61):
        s = f"{float(f):.{prec}f}"
        if np.float32(float(s)) == f:
            return s
    return repr(float(f))


class Activation:
    """`Activation` enum (mod.rs:24-33); codes are the .rtim tags (save.rs:206-214).
    Code 6, SiLU (the reference's nn::Silu, layers.rs:337-346), is an extension with
    no .rtim tag."""

    NONE_CODE, RELU_CODE, SIGMOID_CODE, TANH_CODE, GELU_CODE, LEAKY_RELU_CODE, SILU_CODE = range(7)
    _NAMES = {0: "none", 1: "ReLU", 2: "Sigmoid", 3: "Tanh", 4: "GELU", 6: "SiLU"}

    __slots__ = ("code", "param")

    def __init__(self, code: int, param: float = 0.0):
        if code not in range(7):
            raise ValueError(f"unknown activation tag {code}")
        self.code = int(code)
        self.param = float(np.float32(param)) if code == 5 else 0.0

    @classmethod
    def leaky_relu(cls, slope: float) -> "Activation":
        return cls(5, slope)

    def __eq__(self, other):
        return isinstance(other, Activation) and (self.code, self.param) == (other.code, other.param)

    def __hash__(self):
        return hash((self.code, self.param))

    def __str__(self) -> str:  # impl Display (mod.rs:56-67)
        if self.code == 5:
            return f"LeakyReLU({_fmt_f32(self.param)})"
        return self._NAMES[self.code]

    def __repr__(self) -> str:
        return f"Activation.{str(self)}"


Activation.NONE = Activation(0)
Activation.RELU = Activation(1)
Activation.SIGMOID = Activation(2)
Activation.TANH = Activation(3)
Activation.GELU = Activation(4)
Activation.SILU = Activation(6)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32).reshape(-1))


@dataclass
class Linear:
    in_features: int
    out_features: int
    weight: np.ndarray  # [in, out] row-major
    bias: np.ndarray
    kind: int = field(default=LINEAR, init=False)

    def __post_init__(self):
        self.weight, self.bias = _f32(self.weight), _f32(self.bias)


@dataclass
class Conv2d:
    in_channels: int
    out_channels: int
    kernel: int
    stride: int
    padding: int
    weight: np.ndarray  # [O, C, k, k]
    bias: np.ndarray
    kind: int = field(default=CONV2D, init=False)

    def __post_init__(self):
        self.weight, self.bias = _f32(self.weight), _f32(self.bias)


@dataclass
class ChannelAffine:
    scale: np.ndarray
    shift: np.ndarray
    kind: int = field(default=CHANNEL_AFFINE, init=False)

    def __post_init__(self):
        self.scale, self.shift = _f32(self.scale), _f32(self.shift)


@dataclass
class MaxPool2d:
    kernel: int
    stride: int
    kind: int = field(default=MAXPOOL2D, init=False)


@dataclass
class Flatten:
    kind: int = field(default=FLATTEN, init=False)


@dataclass
class ActivationLayer:
    act: Activation
    kind: int = field(default=ACTIVATION, init=False)


@dataclass
class Softmax:
    kind: int = field(default=SOFTMAX, init=False)


# --- extensions: ResNet-style residual blocks and adaptive average pooling ---------
@dataclass
class ResidualBegin:
    """Saves the current activation as the input of a residual block."""
    kind: int = field(default=RESIDUAL_BEGIN, init=False)


@dataclass
class ShortcutConv2d:
    """A Conv2d (same fields and INT8 semantics) applied to the saved block input."""
    in_channels: int
    out_channels: int
    kernel: int
    stride: int
    padding: int
    weight: np.ndarray  # [O, C, k, k]
    bias: np.ndarray
    kind: int = field(default=SHORTCUT_CONV2D, init=False)

    def __post_init__(self):
        self.weight, self.bias = _f32(self.weight), _f32(self.bias)


@dataclass
class ResidualEnd:
    """y = act(x + saved): closes the block (f32 add, then the activation)."""
    act: Activation = field(default_factory=lambda: Activation(0))
    kind: int = field(default=RESIDUAL_END, init=False)


@dataclass
class AdaptiveAvgPool2d:
    out_h: int
    out_w: int
    kind: int = field(default=ADAPTIVE_AVGPOOL2D, init=False)


# --- extensions: transformer encoder ops (f32 outside the INT8 Linears) -----------
@dataclass
class Embedding:
    """Embedding::forward (nn/layers.rs:438-446): token ids (f32 values) -> table rows."""
    vocab: int
    dim: int
    table: np.ndarray  # [vocab, dim]
    kind: int = field(default=EMBEDDING, init=False)

    def __post_init__(self):
        self.table = _f32(self.table)


@dataclass
class RMSNorm:
    """RMSNorm::forward (nn/norm.rs:413-417): x / sqrt(mean(x^2) + eps) * weight."""
    dim: int
    weight: np.ndarray
    eps: float = 1e-6
    kind: int = field(default=RMSNORM, init=False)

    def __post_init__(self):
        self.weight = _f32(self.weight)
        self.eps = float(np.float32(self.eps))


@dataclass
class Attention:
    """Non-causal multi-head attention (nn/attention.rs:162-196) whose q, k, v and o
    projections (each Linear::new, weight [d, d], bias [d]) run on the INT8 path."""
    dim: int
    heads: int
    wq: np.ndarray
    bq: np.ndarray
    wk: np.ndarray
    bk: np.ndarray
    wv: np.ndarray
    bv: np.ndarray
    wo: np.ndarray
    bo: np.ndarray
    kind: int = field(default=ATTENTION, init=False)

    def __post_init__(self):
        for n in ("wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo"):
            setattr(self, n, _f32(getattr(self, n)))

    @property
    def weight(self) -> np.ndarray:
        return np.concatenate([self.wq, self.wk, self.wv, self.wo])

    @property
    def bias(self) -> np.ndarray:
        return np.concatenate([self.bq, self.bk, self.bv, self.bo])


@dataclass
class SwiGLU:
    """SwiGLU (nn/layers.rs:507-513): down((g * sigmoid(g)) * u) with bias-free INT8
    Linears gate, up [dim, hidden] and down [hidden, dim]."""
    dim: int
    hidden: int
    w_gate: np.ndarray
    w_up: np.ndarray
    w_down: np.ndarray
    kind: int = field(default=SWIGLU, init=False)

    def __post_init__(self):
        self.w_gate, self.w_up, self.w_down = _f32(self.w_gate), _f32(self.w_up), _f32(self.w_down)

    @property
    def weight(self) -> np.ndarray:
        return np.concatenate([self.w_gate, self.w_up, self.w_down])


class LayerSpec:
    """Namespace mirroring the Rust enum: ``LayerSpec.Linear(...)`` etc."""

    Linear = Linear
    Conv2d = Conv2d
    ChannelAffine = ChannelAffine
    MaxPool2d = MaxPool2d
    Flatten = Flatten
    Activation = ActivationLayer
    Softmax = Softmax
    # extensions
    ResidualBegin = ResidualBegin
    ShortcutConv2d = ShortcutConv2d
    ResidualEnd = ResidualEnd
    AdaptiveAvgPool2d = AdaptiveAvgPool2d
    Embedding = Embedding
    RMSNorm = RMSNorm
    Attention = Attention
    SwiGLU = SwiGLU


def as_dict(spec) -> dict:
    """Flat view (the oracle and the C ABI take these field names)."""
    d = {"kind": spec.kind}
    if spec.kind == LINEAR:
        d.update(in_features=spec.in_features, out_features=spec.out_features, weight=spec.weight, bias=spec.bias)
    elif spec.kind == CONV2D:
        d.update(in_channels=spec.in_channels, out_channels=spec.out_channels, kernel=spec.kernel,
                 stride=spec.stride, padding=spec.padding, weight=spec.weight, bias=spec.bias)
    elif spec.kind == CHANNEL_AFFINE:
        d.update(scale=spec.scale, shift=spec.shift)
    elif spec.kind == MAXPOOL2D:
        d.update(kernel=spec.kernel, stride=spec.stride)
    elif spec.kind == ACTIVATION:
        d.update(act=spec.act.code, act_param=spec.act.param)
    elif spec.kind == SHORTCUT_CONV2D:
        d.update(in_channels=spec.in_channels, out_channels=spec.out_channels, kernel=spec.kernel,
                 stride=spec.stride, padding=spec.padding, weight=spec.weight, bias=spec.bias)
    elif spec.kind == RESIDUAL_END:
        d.update(act=spec.act.code, act_param=spec.act.param)
    elif spec.kind == ADAPTIVE_AVGPOOL2D:
        d.update(kernel=spec.out_h, stride=spec.out_w)
    elif spec.kind == EMBEDDING:
        d.update(in_features=spec.vocab, out_features=spec.dim, weight=spec.table)
    elif spec.kind == RMSNORM:
        d.update(in_features=spec.dim, weight=spec.weight, act_param=spec.eps)
    elif spec.kind == ATTENTION:
        d.update(in_features=spec.dim, out_features=spec.heads, weight=spec.weight, bias=spec.bias)
    elif spec.kind == SWIGLU:
        d.update(in_features=spec.dim, out_features=spec.hidden, weight=spec.weight)
    return d
