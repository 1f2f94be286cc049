"""The benchmark configurations, built with the reference's generator.

Draw order after ``manual_seed(seed)``: module construction (each Linear /
Conv2d draws weight then bias), then each BatchNorm's running statistics
(mean ~ U(-0.1, 0.1), then var ~ U(0.5, 1.5)), then the input.  The inputs
are synthetic with the shapes and distributions the configurations name.
"""
from __future__ import annotations

import numpy as np

from . import nn, rng


def c1_mlp(batch: int = 64, seed: int = 42, row_offset: int = 0):
    """README MLP: Linear(4,32)+BatchNorm1d(32)+ReLU+Linear(32,3); x [batch,4] ~ N(0,1).
    ``row_offset`` draws rows [row_offset, row_offset + batch) of a larger batch."""
    rng.manual_seed(seed)
    model = nn.Sequential(nn.Linear(4, 32), nn.BatchNorm1d(32), nn.Relu(), nn.Linear(32, 3))
    nn.draw_bn_stats(model)
    rng.advance(2 * 4 * row_offset)
    return model, rng.randn((batch, 4))


def c2_cnn(batch: int = 256, seed: int = 42, row_offset: int = 0):
    """Small CNN on x [B,1,28,28] ~ U(0,1) (images [row_offset, row_offset + batch))."""
    rng.manual_seed(seed)
    model = nn.Sequential(
        nn.Conv2d(1, 16, 3).padding(1), nn.BatchNorm2d(16), nn.Relu(), nn.MaxPool2d(2),
        nn.Conv2d(16, 32, 3).padding(1), nn.BatchNorm2d(32), nn.Relu(), nn.MaxPool2d(2),
        nn.Flatten(), nn.Linear(1568, 128), nn.Relu(), nn.Linear(128, 10))
    nn.draw_bn_stats(model)
    rng.advance(28 * 28 * row_offset)
    return model, rng.rand((batch, 1, 28, 28))


C3_SHAPES = [(4096, 4096, 4096), (16384, 8192, 8192), (65536, 4096, 14336)]


def c3_linear(m: int, k: int, n: int, seed: int = 42, rows: int | None = None, row_offset: int = 0):
    """Fused INT8 Linear + GELU: W [K,N] ~ 0.02 N(0,1), bias ~ 0.01 N(0,1), A [M,K] ~ N(0,1).
    ``rows`` draws only the first rows of A (identical values)."""
    rng.manual_seed(seed)
    w = rng.normal_init((k, n), 0.02)
    b = rng.normal_init((n,), 0.01)
    model = nn.Sequential(nn.Linear(k, n, weight=w, bias=b), nn.Gelu())
    rng.advance(2 * k * row_offset)
    x = rng.randn((rows if rows is not None else m, k))
    return model, x


def resnet(batch: int, image: int, widths, classes: int, seed: int = 42, stem_k: int = 7, row_offset: int = 0):
    """ResNet-18 layout (extension kinds): conv stem k x k / 2 + BN + ReLU, MaxPool 3x3/2
    (pad 0, the reference's max_pool2d), 4 stages of 2 basic blocks (first block of
    stages 2+ stride 2 with a projection), AdaptiveAvgPool2d(1), Flatten, Linear.
    x ~ N(0,1) [batch, 3, image, image] (images [row_offset, row_offset + batch))."""
    rng.manual_seed(seed)
    layers = [nn.Conv2d(3, widths[0], stem_k).stride(2).padding(stem_k // 2), nn.BatchNorm2d(widths[0]), nn.Relu(),
              nn.MaxPool2d(3, 2)]
    cin = widths[0]
    for si, w in enumerate(widths):
        for bi in range(2):
            layers.append(nn.BasicBlock(cin, w, 2 if (si > 0 and bi == 0) else 1))
            cin = w
    layers += [nn.AdaptiveAvgPool2d(1), nn.Flatten(), nn.Linear(cin, classes)]
    model = nn.Sequential(*layers)
    nn.draw_bn_stats(model)
    rng.advance(2 * 3 * image * image * row_offset)
    return model, rng.randn((batch, 3, image, image))


def c4_resnet18(batch: int = 128, seed: int = 42, row_offset: int = 0, image: int = 224):
    """The ResNet-18-shaped INT8 CNN benchmark: x [B,3,224,224] ~ N(0,1), 1000 classes."""
    return resnet(batch, image, (64, 128, 256, 512), 1000, seed, 7, row_offset)


def transformer(batch: int, seq: int, d: int, heads: int, hidden: int, n_layers: int, vocab: int,
                seed: int = 42, row_offset: int = 0):
    """Pre-norm transformer encoder (extension kinds): Embedding(vocab, d) with the table
    ~ 0.02 N(0,1), then n_layers x PreNormEncoderLayer(d, heads, hidden); token ids
    ~ U[0, vocab) [batch, seq] as f32 (sequences [row_offset, row_offset + batch))."""
    rng.manual_seed(seed)
    model = nn.Sequential(nn.Embedding(vocab, d, std=0.02),
                          *[nn.PreNormEncoderLayer(d, heads, hidden) for _ in range(n_layers)])
    rng.advance(seq * row_offset)
    return model, rng.below((batch, seq), vocab).astype(np.float32)


def c5_transformer(batch: int = 64, seed: int = 42, row_offset: int = 0, seq: int = 512, n_layers: int = 12):
    """The transformer configuration: 12 layers, d_model 1024, 16 heads, SwiGLU hidden
    2816, vocabulary 32000, sequence 512, batch 64."""
    return transformer(batch, seq, 1024, 16, 2816, n_layers, 32000, seed, row_offset)


def input_only(config: str, batch: int, seed: int = 42) -> np.ndarray:
    return {"c1": c1_mlp, "c2": c2_cnn}[config](batch, seed)[1]
