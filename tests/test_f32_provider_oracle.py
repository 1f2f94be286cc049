"""The oracle's f32 ExecutionProvider::Cpu arm (fold_batch_norm + run_standard,
src/inference/mod.rs:162-166, 260-331) against an independent numpy restatement.

run_standard multiplies through the reference CPU matmul (src/device/cpu.rs:43-64,
233-395): every output is an FMA chain in k order from 0, except the columns past the
last full 8-wide block, which accumulate unfused.  numpy has no f32 FMA, so the FMA is
evaluated in exact rational arithmetic and rounded once to f32 (the helper of the
transformer extension's matmul-order test)."""
import numpy as np

from oracle import configs, oracle
from oracle.oracle import ACT_RELU
from tests.test_transformer_ext import _fma_exact as _fma32


def matmul_ref(a, b):
    m, k = a.shape
    n = b.shape[1]
    nv = n // 8 * 8
    out = np.zeros((m, n), np.float32)
    for i in range(m):
        for j in range(n):
            acc = np.float32(0.0)
            for p in range(k):
                if j < nv:
                    acc = _fma32(a[i, p], b[p, j], acc)
                else:
                    acc = np.float32(acc + np.float32(a[i, p] * b[p, j]))
            out[i, j] = acc
    return out


def test_linear_matches_restatement(oracle_lib):
    rng = np.random.default_rng(8)
    k, n, m = 13, 11, 5   # 11 columns: 8 in an FMA block, 3 unfused
    w = rng.standard_normal((k, n)).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    x = rng.standard_normal((m, k)).astype(np.float32)
    layers = [dict(kind=configs.LINEAR, in_features=k, out_features=n, weight=w, bias=b), configs.act(ACT_RELU)]
    y = oracle.run_standard(layers, x)
    want = np.maximum(matmul_ref(x, w) + b, np.float32(0))
    assert np.array_equal(y, want.astype(np.float32))


def test_conv_matches_restatement(oracle_lib):
    rng = np.random.default_rng(9)
    cin, cout, kk, st, pad, h, wd = 2, 3, 3, 1, 1, 4, 5   # L = 20: pixels 16..19 unfused
    w = rng.standard_normal((cout, cin, kk, kk)).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    x = rng.standard_normal((2, cin, h, wd)).astype(np.float32)
    layers = [dict(kind=configs.CONV2D, in_channels=cin, out_channels=cout, kernel=kk, stride=st, padding=pad,
                   weight=w.ravel(), bias=b)]
    y = oracle.run_standard(layers, x)
    xp = np.zeros((2, cin, h + 2, wd + 2), np.float32)
    xp[:, :, 1:1 + h, 1:1 + wd] = x
    for im in range(2):
        cols = np.stack([xp[im, :, oy:oy + 3, ox:ox + 3].ravel() for oy in range(h) for ox in range(wd)], axis=1)
        want = matmul_ref(w.reshape(cout, -1), cols) + b[:, None]
        assert np.array_equal(y[im].reshape(cout, -1), want.astype(np.float32))


def test_folds_and_keeps_standalone_affine(oracle_lib):
    layers, x = configs.usage_doc_model()
    y = oracle.run_standard(layers, x)
    assert y.shape == (32, 4) and np.all(np.isfinite(y))
    scale = np.array([2.0, -0.5, 3.0], np.float32)
    shift = np.array([0.25, 1.0, -2.0], np.float32)
    xa = np.arange(12, dtype=np.float32).reshape(2, 3, 2) * np.float32(0.3)
    ya = oracle.run_standard([dict(kind=oracle.CHANNEL_AFFINE, scale=scale, shift=shift)], xa)
    assert np.array_equal(ya, xa * scale[None, :, None] + shift[None, :, None])
