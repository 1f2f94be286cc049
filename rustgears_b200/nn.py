"""Model-side builders whose ``export()`` yields the reference's ``LayerSpec``s.

Construction draws weights from the global generator in the reference's
order (``Linear::new`` weight then bias, nn/layers.rs:27-34; ``Conv2d::new``,
108-119; kaiming/bias bounds, nn/init.rs:6-26), so ``manual_seed(s)`` followed
by the same ``Sequential`` gives bit-identical parameters.  Only inference
export lives here: forward/backward training code is the reference's.
"""
from __future__ import annotations

import numpy as np

from . import rng
from .spec import Activation, ActivationLayer, ChannelAffine, Conv2d as Conv2dSpec, Flatten as FlattenSpec
from .spec import Linear as LinearSpec, MaxPool2d as MaxPool2dSpec, Softmax as SoftmaxSpec
from .spec import AdaptiveAvgPool2d as AdaptiveAvgPool2dSpec, ResidualBegin, ResidualEnd, ShortcutConv2d
from .spec import Attention as AttentionSpec, Embedding as EmbeddingSpec, RMSNorm as RMSNormSpec
from .spec import SwiGLU as SwiGLUSpec


class Module:
    """`Module` trait subset used by `InferenceSession::from_module` (nn/mod.rs:26-68)."""

    training = True

    def name(self) -> str:
        return type(self).__name__

    def set_training(self, t: bool) -> None:
        self.training = t

    def eval(self) -> None:
        self.set_training(False)

    def train(self) -> None:
        self.set_training(True)

    def export(self):
        raise NotImplementedError(f"layer '{self.name()}' does not support export")


class Sequential(Module):
    def __init__(self, *layers):
        self.layers = list(layers)

    def add(self, layer: Module) -> "Sequential":
        self.layers.append(layer)
        return self

    def set_training(self, t: bool) -> None:
        for l in self.layers:
            l.set_training(t)

    def export(self):  # nn/mod.rs:204-210
        out = []
        for l in self.layers:
            out.extend(l.export())
        return out


class Linear(Module):
    """Weight [in, out] (kaiming uniform), bias [out] (bias uniform)."""

    def __init__(self, in_features: int, out_features: int, weight=None, bias=None):
        self.in_features, self.out_features = in_features, out_features
        self.weight = (np.asarray(weight, np.float32).reshape(in_features, out_features) if weight is not None
                       else rng.kaiming_uniform((in_features, out_features), in_features))
        if bias is not None:
            self.bias = np.asarray(bias, np.float32).reshape(out_features)
        elif weight is None:
            self.bias = rng.bias_uniform((out_features,), in_features)
        else:
            self.bias = None

    @classmethod
    def no_bias(cls, in_features: int, out_features: int) -> "Linear":
        l = cls(in_features, out_features)
        l.bias = None
        return l

    def name(self) -> str:
        return f"Linear({self.in_features}, {self.out_features})"

    def export(self):  # nn/layers.rs:74-81
        b = self.bias if self.bias is not None else np.zeros(self.out_features, np.float32)
        return [LinearSpec(self.in_features, self.out_features, self.weight, b)]


class Conv2d(Module):
    def __init__(self, in_channels: int, out_channels: int, kernel_size: int, weight=None, bias=None):
        fan_in = in_channels * kernel_size * kernel_size
        self.in_channels, self.out_channels, self.kernel_size = in_channels, out_channels, kernel_size
        self.stride_, self.padding_ = 1, 0
        self.weight = (np.asarray(weight, np.float32).reshape(out_channels, in_channels, kernel_size, kernel_size)
                       if weight is not None else
                       rng.kaiming_uniform((out_channels, in_channels, kernel_size, kernel_size), fan_in))
        self.bias = (np.asarray(bias, np.float32).reshape(out_channels) if bias is not None
                     else rng.bias_uniform((out_channels,), fan_in))

    def stride(self, s: int) -> "Conv2d":
        self.stride_ = s
        return self

    def padding(self, p: int) -> "Conv2d":
        self.padding_ = p
        return self

    def export(self):  # nn/layers.rs:151-161
        return [Conv2dSpec(self.in_channels, self.out_channels, self.kernel_size, self.stride_, self.padding_,
                           self.weight, self.bias)]


class BatchNorm(Module):
    """Exported as ``ChannelAffine`` (nn/norm.rs:335-343): scale = g / sqrt(rv + eps)."""

    def __init__(self, num_features: int, spatial: bool = False):
        self.num_features = num_features
        self.spatial = spatial
        self.gamma = np.ones(num_features, np.float32)
        self.beta = np.zeros(num_features, np.float32)
        self.running_mean = np.zeros(num_features, np.float32)
        self.running_var = np.ones(num_features, np.float32)
        self.eps = np.float32(1e-5)

    def name(self) -> str:
        return f"BatchNorm{'2d' if self.spatial else '1d'}({self.num_features})"

    def export(self):
        scale = (self.gamma / np.sqrt((self.running_var + self.eps).astype(np.float32))).astype(np.float32)
        shift = (self.beta - (self.running_mean * scale).astype(np.float32)).astype(np.float32)
        return [ChannelAffine(scale, shift)]


def BatchNorm1d(num_features: int) -> BatchNorm:
    return BatchNorm(num_features, False)


def BatchNorm2d(num_features: int) -> BatchNorm:
    return BatchNorm(num_features, True)


class MaxPool2d(Module):
    def __init__(self, kernel: int, stride: int | None = None):
        self.kernel, self.stride = kernel, kernel if stride is None else stride

    def export(self):
        return [MaxPool2dSpec(self.kernel, self.stride)]


class Flatten(Module):
    def export(self):
        return [FlattenSpec()]


class Identity(Module):
    def export(self):
        return []


class Dropout(Module):
    def __init__(self, p: float):
        self.p = p

    def export(self):  # inference is the identity (nn/layers.rs:411-413)
        return []


class _Act(Module):
    ACT = Activation.NONE

    def export(self):
        return [ActivationLayer(self.ACT)]


class Relu(_Act):
    ACT = Activation.RELU


class Sigmoid(_Act):
    ACT = Activation.SIGMOID


class Tanh(_Act):
    ACT = Activation.TANH


class Gelu(_Act):
    ACT = Activation.GELU


class Silu(_Act):
    """nn::Silu (layers.rs:337-346): x * sigmoid(x).  Extension export: the reference
    has the layer but no Activation variant for it."""
    ACT = Activation.SILU


class LeakyRelu(Module):
    def __init__(self, slope: float):
        self.slope = slope

    def export(self):
        return [ActivationLayer(Activation.leaky_relu(self.slope))]


class Softmax(Module):
    def export(self):
        return [SoftmaxSpec()]


class AdaptiveAvgPool2d(Module):
    """Extension export (the reference has the op, tensor/ops.rs:994-1014, but no LayerSpec)."""

    def __init__(self, out_h: int, out_w: int | None = None):
        self.out_h, self.out_w = out_h, out_h if out_w is None else out_w

    def export(self):
        return [AdaptiveAvgPool2dSpec(self.out_h, self.out_w)]


class BasicBlock(Module):
    """ResNet basic block (extension export): y = relu(bn2(conv2(relu(bn1(conv1(x))))) + shortcut(x)),
    shortcut = identity, or bn(conv1x1/stride(x)) when the stride or width changes.
    Construction draws conv1, bn1, conv2, bn2, then the projection conv, in that order."""

    def __init__(self, in_ch: int, out_ch: int, stride: int = 1):
        self.conv1 = Conv2d(in_ch, out_ch, 3).stride(stride).padding(1)
        self.bn1 = BatchNorm2d(out_ch)
        self.conv2 = Conv2d(out_ch, out_ch, 3).padding(1)
        self.bn2 = BatchNorm2d(out_ch)
        self.proj = None
        if stride != 1 or in_ch != out_ch:
            self.proj = Conv2d(in_ch, out_ch, 1).stride(stride)
            self.proj_bn = BatchNorm2d(out_ch)

    def batchnorms(self):
        return [self.bn1, self.bn2] + ([self.proj_bn] if self.proj is not None else [])

    def export(self):
        out = [ResidualBegin()]
        out += self.conv1.export() + self.bn1.export() + [ActivationLayer(Activation.RELU)]
        out += self.conv2.export() + self.bn2.export()
        if self.proj is not None:
            c = self.proj
            out += [ShortcutConv2d(c.in_channels, c.out_channels, c.kernel_size, c.stride_, c.padding_, c.weight,
                                   c.bias)] + self.proj_bn.export()
        out += [ResidualEnd(Activation.RELU)]
        return out


class Embedding(Module):
    """Embedding::new (nn/layers.rs:430-433) draws the table ~ std * N(0,1) (std 0.1;
    configurations may pass their own std or table)."""

    def __init__(self, num_embeddings: int, dim: int, weight=None, std: float = 0.1):
        self.num_embeddings, self.dim = num_embeddings, dim
        self.weight = (np.asarray(weight, np.float32).reshape(num_embeddings, dim) if weight is not None
                       else rng.normal_init((num_embeddings, dim), std))

    def export(self):
        return [EmbeddingSpec(self.num_embeddings, self.dim, self.weight)]


class RMSNorm(Module):
    """RMSNorm::new (nn/norm.rs:396-403): weight ones, eps 1e-6 (no draws)."""

    def __init__(self, dim: int, eps: float = 1e-6):
        self.dim, self.eps = dim, eps
        self.weight = np.ones(dim, np.float32)

    def export(self):
        return [RMSNormSpec(self.dim, self.weight, self.eps)]


class MultiHeadAttention(Module):
    """MultiHeadAttention::new (nn/attention.rs:130-143), non-causal, no RoPE:
    Linear::new for wq, wk, wv, wo in that order."""

    def __init__(self, d_model: int, heads: int):
        if d_model <= 0 or heads <= 0 or d_model % heads:
            raise ValueError("d_model must be a positive multiple of heads")
        self.d_model, self.heads = d_model, heads
        self.wq, self.wk = Linear(d_model, d_model), Linear(d_model, d_model)
        self.wv, self.wo = Linear(d_model, d_model), Linear(d_model, d_model)

    def export(self):
        return [AttentionSpec(self.d_model, self.heads, self.wq.weight, self.wq.bias, self.wk.weight, self.wk.bias,
                              self.wv.weight, self.wv.bias, self.wo.weight, self.wo.bias)]


class SwiGLU(Module):
    """SwiGLU::new (nn/layers.rs:492-497): Linear::no_bias gate, up, down (each still
    draws its dropped bias)."""

    def __init__(self, in_features: int, hidden_features: int, out_features: int | None = None):
        out_features = in_features if out_features is None else out_features
        if out_features != in_features:
            raise ValueError("the SwiGLU op keeps the model width (out_features == in_features)")
        self.in_features, self.hidden_features = in_features, hidden_features
        self.gate = Linear.no_bias(in_features, hidden_features)
        self.up = Linear.no_bias(in_features, hidden_features)
        self.down = Linear.no_bias(hidden_features, in_features)

    def export(self):
        return [SwiGLUSpec(self.in_features, self.hidden_features, self.gate.weight, self.up.weight,
                           self.down.weight)]


class PreNormEncoderLayer(Module):
    """x += Attention(RMSNorm(x)); x += SwiGLU(RMSNorm(x)) (extension export; built in
    the order norm1, attention, norm2, SwiGLU)."""

    def __init__(self, d_model: int, heads: int, hidden: int):
        self.norm1 = RMSNorm(d_model)
        self.attn = MultiHeadAttention(d_model, heads)
        self.norm2 = RMSNorm(d_model)
        self.ffn = SwiGLU(d_model, hidden)

    def export(self):
        return ([ResidualBegin()] + self.norm1.export() + self.attn.export() + [ResidualEnd(Activation.NONE)] +
                [ResidualBegin()] + self.norm2.export() + self.ffn.export() + [ResidualEnd(Activation.NONE)])


def draw_bn_stats(model: Module, mean_range=(-0.1, 0.1), var_range=(0.5, 1.5)) -> None:
    """Seeded BatchNorm running statistics (benchmark configurations): for each
    BatchNorm in order, running_mean ~ U(mean_range) then running_var ~ U(var_range)."""
    layers = model.layers if isinstance(model, Sequential) else [model]
    for l in layers:
        for bn in (l.batchnorms() if isinstance(l, BasicBlock) else [l]):
            if isinstance(bn, BatchNorm):
                bn.running_mean = rng.uniform((bn.num_features,), *mean_range)
                bn.running_var = rng.uniform((bn.num_features,), *var_range)
