"""TEST INFRASTRUCTURE ONLY: the benchmark configurations built with the
oracle's restatement of the reference RNG and initialisers.

Draw order (the reference's global RNG after ``manual_seed(seed)``):
module construction order -- every ``Linear::new`` / ``Conv2d::new`` draws its
weight and then its bias (nn/layers.rs:27-34, 108-119) -- then each BatchNorm's
running statistics (mean ~ U(-0.1, 0.1), then var ~ U(0.5, 1.5)), then the
input.  BatchNorm gamma = 1 and beta = 0 (nn/norm.rs:56-59); its export is
``scale = g / sqrt(rv + eps)``, ``shift = b - rm * scale`` with eps = 1e-5
(nn/norm.rs:335-343).
"""
from __future__ import annotations

import numpy as np

from .oracle import (ACT_GELU, ACT_RELU, ACTIVATION, ADAPTIVE_AVGPOOL2D, ATTENTION, CHANNEL_AFFINE, CONV2D,
                     EMBEDDING, FLATTEN, LINEAR, MAXPOOL2D, RESIDUAL_BEGIN, RESIDUAL_END, RMSNORM, SHORTCUT_CONV2D,
                     SWIGLU, Rng)


def linear(rng: Rng, fin: int, fout: int) -> dict:  # Linear::new (nn/layers.rs:27-34)
    w = rng.kaiming_uniform((fin, fout), fin)
    b = rng.bias_uniform((fout,), fin)
    return dict(kind=LINEAR, in_features=fin, out_features=fout, weight=w, bias=b)


def conv2d(rng: Rng, cin: int, cout: int, k: int, stride: int = 1, padding: int = 0) -> dict:
    fan_in = cin * k * k  # Conv2d::new (nn/layers.rs:108-119)
    w = rng.kaiming_uniform((cout, cin, k, k), fan_in)
    b = rng.bias_uniform((cout,), fan_in)
    return dict(kind=CONV2D, in_channels=cin, out_channels=cout, kernel=k, stride=stride,
                padding=padding, weight=w, bias=b)


def batchnorm(c: int) -> dict:
    """Placeholder until the stats are drawn; filled by ``draw_bn_stats``."""
    return dict(kind=CHANNEL_AFFINE, _bn=c)


def draw_bn_stats(rng: Rng, layers: list) -> list:
    out = []
    for l in layers:
        if l.get("_bn"):
            c = l["_bn"]
            rm = rng.uniform_tensor((c,), -0.1, 0.1)
            rv = rng.uniform_tensor((c,), 0.5, 1.5)
            g = np.ones(c, np.float32)
            b = np.zeros(c, np.float32)
            eps = np.float32(1e-5)
            scale = (g / np.sqrt(rv + eps)).astype(np.float32)
            shift = (b - rm * scale).astype(np.float32)
            out.append(dict(kind=CHANNEL_AFFINE, scale=scale, shift=shift))
        else:
            out.append(l)
    return out


def act(a: int, p: float = 0.0) -> dict:
    return dict(kind=ACTIVATION, act=a, act_param=p)


def c1_mlp(batch: int = 64, seed: int = 42):
    """README MLP: Linear(4,32)+BN1d(32)+ReLU+Linear(32,3); x [batch,4] ~ N(0,1)."""
    rng = Rng(seed)
    layers = [linear(rng, 4, 32), batchnorm(32), act(ACT_RELU), linear(rng, 32, 3)]
    layers = draw_bn_stats(rng, layers)
    x = rng.randn((batch, 4))
    return layers, x


def c2_cnn(batch: int = 256, seed: int = 42):
    """Small CNN: x [B,1,28,28] ~ U(0,1)."""
    rng = Rng(seed)
    layers = [conv2d(rng, 1, 16, 3, 1, 1), batchnorm(16), act(ACT_RELU), dict(kind=MAXPOOL2D, kernel=2, stride=2),
              conv2d(rng, 16, 32, 3, 1, 1), batchnorm(32), act(ACT_RELU), dict(kind=MAXPOOL2D, kernel=2, stride=2),
              dict(kind=FLATTEN), linear(rng, 1568, 128), act(ACT_RELU), linear(rng, 128, 10)]
    layers = draw_bn_stats(rng, layers)
    x = rng.uniform_tensor((batch, 1, 28, 28), 0.0, 1.0)
    return layers, x


def c3_linear(m: int, k: int, n: int, seed: int = 42, rows: int | None = None):
    """Single fused INT8 Linear + GELU: W [K,N] ~ 0.02 N(0,1), bias ~ 0.01 N(0,1),
    A [M,K] ~ N(0,1).  ``rows`` draws only the first rows of A (same values)."""
    rng = Rng(seed)
    w = rng.normal_init((k, n), 0.02)
    b = rng.normal_init((n,), 0.01)
    x = rng.randn((rows if rows is not None else m, k))
    layers = [dict(kind=LINEAR, in_features=k, out_features=n, weight=w, bias=b), act(ACT_GELU)]
    return layers, x


def integration_model(seed: int = 2026):
    """Structure of tests/integration.rs:128-164 (BN stats seeded instead of warmed
    by a training forward, which is outside this path); x [8,1,8,8]."""
    rng = Rng(seed)
    layers = [conv2d(rng, 1, 4, 3, 1, 1), batchnorm(4), act(ACT_RELU), dict(kind=MAXPOOL2D, kernel=2, stride=2),
              dict(kind=FLATTEN), linear(rng, 64, 16), batchnorm(16), act(ACT_RELU), linear(rng, 16, 4)]
    layers = draw_bn_stats(rng, layers)
    x = rng.randn((8, 1, 8, 8))
    return layers, x


def usage_doc_model(seed: int = 42):
    """docs/USAGE.md:360-380 example: Linear(16,64)+BN1d(64)+ReLU+Linear(64,4), x [32,16]."""
    rng = Rng(seed)
    layers = [linear(rng, 16, 64), batchnorm(64), act(ACT_RELU), linear(rng, 64, 4)]
    layers = draw_bn_stats(rng, layers)
    x = rng.randn((32, 16))
    return layers, x


def acts_mlp(batch: int = 16, seed: int = 7):
    """Every activation the IR has, fused and standalone, plus a final Softmax."""
    from .oracle import ACT_LEAKY_RELU, ACT_SIGMOID, ACT_TANH, SOFTMAX
    rng = Rng(seed)
    layers = [linear(rng, 5, 7), act(ACT_SIGMOID), linear(rng, 7, 6), act(ACT_TANH),
              linear(rng, 6, 9), act(ACT_GELU), act(ACT_LEAKY_RELU, 0.2), linear(rng, 9, 4),
              act(ACT_LEAKY_RELU, 0.01), linear(rng, 4, 3), dict(kind=SOFTMAX)]
    x = rng.randn((batch, 5))
    return layers, x


def strided_cnn(batch: int = 3, seed: int = 11):
    """Strided/padded convs, incl. a 1x1 stride-2 conv that skips pixels, an odd
    maxpool and a Linear on the flattened map."""
    rng = Rng(seed)
    layers = [conv2d(rng, 3, 8, 3, 2, 1), batchnorm(8), act(ACT_RELU),
              conv2d(rng, 8, 12, 1, 2, 0),
              dict(kind=MAXPOOL2D, kernel=3, stride=2),
              conv2d(rng, 12, 16, 2, 1, 0), act(ACT_GELU),
              dict(kind=FLATTEN), linear(rng, 16, 5)]
    layers = draw_bn_stats(rng, layers)
    x = rng.randn((batch, 3, 19, 17))
    return layers, x


def affine_first(batch: int = 6, seed: int = 5):
    """A leading BatchNorm (no Linear/Conv to fold into: runs as a diagonal
    FusedLinear, npu.rs:254-270) and a standalone activation."""
    rng = Rng(seed)
    layers = [batchnorm(10), act(ACT_RELU), linear(rng, 10, 6), batchnorm(6), linear(rng, 6, 4)]
    layers = draw_bn_stats(rng, layers)
    x = rng.randn((batch, 10))
    return layers, x


def basic_block(rng: Rng, cin: int, cout: int, stride: int) -> list:
    """ResNet basic block (extension kinds): conv3x3/stride + BN + ReLU, conv3x3 + BN,
    projection conv1x1/stride + BN when the shape changes, add, ReLU.  Weights are
    drawn conv1, conv2, projection (construction order)."""
    layers = [dict(kind=RESIDUAL_BEGIN), conv2d(rng, cin, cout, 3, stride, 1), batchnorm(cout), act(ACT_RELU),
              conv2d(rng, cout, cout, 3, 1, 1), batchnorm(cout)]
    if stride != 1 or cin != cout:
        sc = conv2d(rng, cin, cout, 1, stride, 0)
        sc["kind"] = SHORTCUT_CONV2D
        layers += [sc, batchnorm(cout)]
    return layers + [dict(kind=RESIDUAL_END, act=ACT_RELU, act_param=0.0)]


def resnet(batch: int, image: int, widths, classes: int, seed: int = 42, stem_k: int = 7):
    """ResNet-18 layout (the ResNet benchmark configuration): conv7x7/2 p3 + BN + ReLU, MaxPool 3x3/2
    (pad 0, the reference's max_pool2d), 4 stages of 2 basic blocks (first block of
    stages 2-4 stride 2 with a projection), AdaptiveAvgPool2d(1), Flatten, Linear.
    x ~ N(0,1) [batch, 3, image, image].  Conv and Linear weights are drawn in module
    order, then the BatchNorm statistics, then the input."""
    rng = Rng(seed)
    layers = [conv2d(rng, 3, widths[0], stem_k, 2, stem_k // 2), batchnorm(widths[0]), act(ACT_RELU),
              dict(kind=MAXPOOL2D, kernel=3, stride=2)]
    cin = widths[0]
    for si, w in enumerate(widths):
        for bi in range(2):
            layers += basic_block(rng, cin, w, 2 if (si > 0 and bi == 0) else 1)
            cin = w
    layers += [dict(kind=ADAPTIVE_AVGPOOL2D, kernel=1, stride=1), dict(kind=FLATTEN), linear(rng, cin, classes)]
    layers = draw_bn_stats(rng, layers)
    x = rng.randn((batch, 3, image, image))
    return layers, x


def resnet18(batch: int = 2, image: int = 224, seed: int = 42):
    return resnet(batch, image, (64, 128, 256, 512), 1000, seed)


def resnet_mini(batch: int = 3, seed: int = 9):
    """Two-stage residual net on 24x24 inputs (identity and projection blocks)."""
    return resnet(batch, 24, (8, 16), 10, seed, stem_k=3)


def transformer(batch: int, seq: int, d: int, heads: int, hidden: int, n_layers: int, vocab: int,
                seed: int = 42):
    """Pre-norm transformer encoder (extension kinds): Embedding (table ~ 0.02 N(0,1)),
    then per layer x += Attention(RMSNorm(x)) and x += SwiGLU(RMSNorm(x)); attention
    Linears with bias (MultiHeadAttention::new, nn/attention.rs:130-143), SwiGLU Linears
    bias-free (SwiGLU::new, nn/layers.rs:492-497), RMSNorm weight ones, eps 1e-6.
    Draw order: the table, then per layer Wq, bq, Wk, bk, Wv, bv, Wo, bo, then Wgate,
    Wup, Wdown each followed by its dropped bias; then the token ids ~ U[0, vocab)
    [batch, seq] as f32."""
    rng = Rng(seed)
    table = rng.normal_init((vocab, d), 0.02)
    layers = [dict(kind=EMBEDDING, in_features=vocab, out_features=d, weight=table)]
    for _ in range(n_layers):
        w, b = [], []
        for _ in range(4):
            w.append(rng.kaiming_uniform((d, d), d))
            b.append(rng.bias_uniform((d,), d))
        # Linear::no_bias builds Linear::new and drops the bias (nn/layers.rs:37-41): the
        # bias is still drawn
        g = rng.kaiming_uniform((d, hidden), d); rng.bias_uniform((hidden,), d)
        u = rng.kaiming_uniform((d, hidden), d); rng.bias_uniform((hidden,), d)
        dn = rng.kaiming_uniform((hidden, d), hidden); rng.bias_uniform((d,), hidden)
        norm = lambda: dict(kind=RMSNORM, in_features=d, weight=np.ones(d, np.float32), act_param=1e-6)
        layers += [dict(kind=RESIDUAL_BEGIN), norm(),
                   dict(kind=ATTENTION, in_features=d, out_features=heads, weight=np.concatenate([x.ravel() for x in w]),
                        bias=np.concatenate(b)),
                   dict(kind=RESIDUAL_END, act=0, act_param=0.0),
                   dict(kind=RESIDUAL_BEGIN), norm(),
                   dict(kind=SWIGLU, in_features=d, out_features=hidden,
                        weight=np.concatenate([g.ravel(), u.ravel(), dn.ravel()])),
                   dict(kind=RESIDUAL_END, act=0, act_param=0.0)]
    ids = rng.below((batch, seq), vocab).astype(np.float32)
    return layers, ids


def transformer_c5(batch: int = 64, seq: int = 512, n_layers: int = 12, seed: int = 42):
    """The transformer benchmark configuration: 12 layers, d_model 1024, 16 heads, SwiGLU
    hidden 2816, vocabulary 32000, sequence 512."""
    return transformer(batch, seq, 1024, 16, 2816, n_layers, 32000, seed)


def transformer_mini(batch: int = 2, seq: int = 12, seed: int = 13):
    return transformer(batch, seq, 64, 4, 96, 2, 500, seed)


# name -> builder of (layers, x) used by the golden fixtures and the parity tests
CASES = {
    "usage_doc": usage_doc_model,
    "integration": integration_model,
    "c1_mlp_64": lambda: c1_mlp(64),
    "c2_cnn_4": lambda: c2_cnn(4),
    "c3_linear_small": lambda: c3_linear(32, 64, 48),
    "acts_mlp": acts_mlp,
    "strided_cnn": strided_cnn,
    "affine_first": affine_first,
    "resnet_mini": resnet_mini,
    "transformer_mini": transformer_mini,
}
