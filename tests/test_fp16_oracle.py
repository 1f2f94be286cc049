"""The oracle's FP16 arm (NpuPrecision::Fp16) against independent numpy restatements.

The reference emulates an FP16 MAC array on the CPU (src/inference/npu.rs:425-445):
activations and weights are rounded by `round_fp16` (src/inference/quantize.rs:50-64),
the products are summed in f32 in k order, and the sum plus bias is rounded again
before the activation.  Nothing in the reference pins these values (its tests only
exercise the Int8 arm), so the oracle is checked here against a second restatement
written from the same lines.
"""
import numpy as np
import pytest

from oracle import configs, oracle
from oracle.oracle import ACT_GELU, ACT_RELU


def round_fp16_np(x):
    """quantize.rs:50-64 on f32 bit patterns."""
    b = np.asarray(x, np.float32).view(np.uint32)
    e = ((b >> 23) & 0xFF).astype(np.int64) - 127
    r = ((b + np.uint32(1 << 12)) & np.uint32(~0x1FFF & 0xFFFFFFFF)).astype(np.uint32)
    r = np.where(e > 15, (b & np.uint32(0x80000000)) | np.uint32(0x477FE000), r)
    r = np.where(e < -14, np.uint32(0), r)
    return r.astype(np.uint32).view(np.float32)


def fp16_gemm_np(a, w_t, bias, act, oracle_lib):
    """fp16_gemm_fused_into (npu.rs:431-445): serial f32 sums, no FMA."""
    m, k = a.shape
    n = w_t.shape[0]
    ar = round_fp16_np(a)
    out = np.empty((m, n), np.float32)
    for r in range(m):
        for c in range(n):
            acc = np.float32(0.0)
            for i in range(k):
                acc = np.float32(acc + np.float32(ar[r, i] * w_t[c, i]))
            v = round_fp16_np(np.float32(acc + bias[c]))
            out[r, c] = oracle_lib.lib().og_act_apply(act, 0.0, float(v))
    return out


def test_round_fp16_edges(oracle_lib):
    vals = np.array([0.0, -0.0, 1.0, -1.0, 65504.0, 65519.0, 65520.0, -65520.0, 65535.0, 70000.0,
                     np.inf, -np.inf, np.nan, 2.0 ** -14, -(2.0 ** -14), 2.0 ** -15, 6.1e-5, 1e-8,
                     1.0 + 2.0 ** -11, 1.0 + 2.0 ** -12, 1.0 + 3 * 2.0 ** -12, 3.14159265], np.float32)
    rng = np.random.default_rng(1)
    bits = rng.integers(0, 2 ** 32, 200000, dtype=np.uint64).astype(np.uint32)
    allv = np.concatenate([vals, bits.view(np.float32)])
    got = np.array([oracle_lib.lib().og_round_fp16(float(v)) for v in allv], np.float32)
    want = round_fp16_np(allv)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # the reference's own quirks: subnormal-range values flush to +0 (sign dropped),
    # inf and NaN clamp to +-65504, the carry of the mantissa can reach 65536
    assert round_fp16_np(np.float32(-1e-6)).view(np.uint32) == 0
    assert round_fp16_np(np.float32(np.nan)) in (np.float32(65504), np.float32(-65504))
    assert round_fp16_np(np.float32(65520.0)) == np.float32(65536.0)


def test_fp16_linear_matches_restatement(oracle_lib):
    rng = np.random.default_rng(3)
    k, n, m = 37, 11, 9
    w = (rng.standard_normal((k, n)) * 0.3).astype(np.float32)
    b = (rng.standard_normal(n) * 0.1).astype(np.float32)
    layers = [dict(kind=configs.LINEAR, in_features=k, out_features=n, weight=w, bias=b), configs.act(ACT_GELU)]
    p = oracle.Program(layers, precision=1)
    assert np.array_equal(p.ops[0].wh.reshape(n, k), round_fp16_np(w.T))
    x = (rng.standard_normal((m, k)) * 2).astype(np.float32)
    x[0, 0], x[1, 1], x[2, 2] = np.nan, np.inf, 1e-7
    y, _, macs = p.execute(x)
    want = fp16_gemm_np(x, round_fp16_np(w.T), b, ACT_GELU, oracle_lib)
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32))
    assert macs.tolist() == [m * k * n]


def test_fp16_conv_matches_restatement(oracle_lib):
    rng = np.random.default_rng(4)
    cin, cout, kk, st, pad, h, wd, nb = 3, 5, 3, 2, 1, 7, 6, 2
    w = (rng.standard_normal((cout, cin, kk, kk)) * 0.2).astype(np.float32)
    b = (rng.standard_normal(cout) * 0.1).astype(np.float32)
    layers = [dict(kind=configs.CONV2D, in_channels=cin, out_channels=cout, kernel=kk, stride=st, padding=pad,
                   weight=w.ravel(), bias=b), configs.act(ACT_RELU)]
    p = oracle.Program(layers, precision=1)
    x = rng.standard_normal((nb, cin, h, wd)).astype(np.float32)
    y, _, _ = p.execute(x)
    oh, ow = (h + 2 * pad - kk) // st + 1, (wd + 2 * pad - kk) // st + 1
    xp = np.zeros((nb, cin, h + 2 * pad, wd + 2 * pad), np.float32)
    xp[:, :, pad:pad + h, pad:pad + wd] = x
    for im in range(nb):
        cols = np.empty((oh * ow, cin * kk * kk), np.float32)  # im2col row (c, ky, kx), transposed
        for oy in range(oh):
            for ox in range(ow):
                cols[oy * ow + ox] = xp[im, :, oy * st:oy * st + kk, ox * st:ox * st + kk].ravel()
        want = fp16_gemm_np(cols, round_fp16_np(w.reshape(cout, -1)), b, ACT_RELU, oracle_lib)
        assert np.array_equal(y[im].reshape(cout, -1), want.T), im


def test_fp16_program_report(oracle_lib):
    layers, x = configs.usage_doc_model()
    p = oracle.Program(layers, precision=1)
    # npu.rs:212-215: FP16 weight bytes are 2 per weight and bias value
    assert p.npu_bytes == (16 * 64 + 64 + 64 * 4 + 4) * 2
    assert p.summary(len(layers)).startswith("InferenceSession [provider = NPU (FP16), layers: 4 -> 2 fused ops")
    y, _, _ = p.execute(x)
    assert y.shape == (32, 4) and np.all(np.isfinite(y))


def test_fp16_standalone_affine_keeps_unrounded_diagonal(oracle_lib):
    scale = np.array([1.0 + 2.0 ** -13, -0.3, 7.0e-6], np.float32)
    shift = np.array([0.5, 0.25, -1.0], np.float32)
    layers = [dict(kind=oracle.CHANNEL_AFFINE, scale=scale, shift=shift)]
    p = oracle.Program(layers, precision=1)
    assert np.array_equal(p.ops[0].wh.reshape(3, 3), np.diag(scale))
    x = np.array([[1.0, 2.0, 3.0], [-4.0, 1e-3, 65530.0]], np.float32)
    y, _, _ = p.execute(x)
    want = fp16_gemm_np(x, np.diag(scale).astype(np.float32), shift, 0, oracle_lib)
    assert np.array_equal(y, want)


def test_fp16_rejects_extension_blocks(oracle_lib):
    layers, x = configs.transformer_mini(1, 4)
    with pytest.raises(RuntimeError):
        oracle.Program(layers, precision=1).execute(x)
