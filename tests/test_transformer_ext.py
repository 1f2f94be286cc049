"""Transformer extension kinds (embedding, RMSNorm, attention, SwiGLU): the oracle's
new f32 pieces against independent restatements of their definitions, and the
product-side builder against the oracle's configuration.  CPU only."""
import ctypes as C
from fractions import Fraction

import numpy as np
import pytest

from oracle import configs, oracle
from rustgears_b200 import configs as pc
from rustgears_b200 import spec as S
from tests.helpers import assert_same


def _p(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _fma_exact(a, b, c):
    """fmaf: a*b + c rounded once to f32 (exact rational arithmetic, then one rounding)."""
    v = Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c))
    return _round_f32(v)


def _round_f32(v: Fraction) -> np.float32:
    if v == 0:
        return np.float32(0.0)
    # nearest f32 by bisection on the two f32 neighbours of the f64 nearest value
    f = np.float32(float(v))
    lo = f if Fraction(float(f)) <= v else np.nextafter(f, np.float32(-np.inf))
    hi = np.nextafter(lo, np.float32(np.inf))
    dlo, dhi = v - Fraction(float(lo)), Fraction(float(hi)) - v
    if dlo < dhi:
        return lo
    if dhi < dlo:
        return hi
    return lo if (lo.view(np.uint32) & 1) == 0 else hi  # ties to even


@pytest.mark.parametrize("m,k,n", [(3, 5, 11), (2, 9, 16), (4, 3, 7)])
def test_bmm_fma_order(oracle_lib, m, k, n):
    """cpu_matmul (device/cpu.rs:234-395): every output an FMA chain over k from 0 for
    columns in full 8-wide blocks; columns past them accumulate c += a * b unfused."""
    rng = np.random.default_rng(m * 100 + n)
    a = rng.standard_normal((2, m, k)).astype(np.float32)
    b = rng.standard_normal((2, k, n)).astype(np.float32)
    c = np.empty((2, m, n), np.float32)
    oracle.lib().og_bmm_fma(_p(a), _p(b), 2, m, k, n, _p(c))
    ref = np.empty_like(c)
    nv = n // 8 * 8
    for g in range(2):
        for i in range(m):
            for j in range(n):
                acc = np.float32(0.0)
                for p in range(k):
                    if j < nv:
                        acc = _fma_exact(a[g, i, p], b[g, p, j], acc)
                    else:
                        acc = np.float32(acc + np.float32(a[g, i, p] * b[g, p, j]))
                ref[g, i, j] = acc
    assert_same(c, ref, "bmm")


def _rmsnorm_def(x, w, eps):
    d = x.shape[-1]
    inv_d = np.float32(np.float32(1.0) / np.float32(d))
    y = np.empty_like(x)
    for r in range(x.shape[0]):
        s = np.float32(0.0)
        for v in x[r]:
            s = np.float32(s + np.float32(v * v))
        rms = np.float32(np.sqrt(np.float32(np.float32(s * inv_d) + np.float32(eps))))
        y[r] = (x[r] / rms).astype(np.float32) * w
    return y


def test_rmsnorm_definition(oracle_lib):
    layers, _ = configs.transformer(1, 4, 24, 2, 16, 1, 10, seed=2)
    prog = oracle.Program(layers)
    i = next(k for k, op in enumerate(prog.ops) if op.kind == oracle.RMSNORM)
    x = np.random.default_rng(1).standard_normal((5, 24)).astype(np.float32) * np.float32(7.0)
    y = np.empty_like(x)
    oracle.lib().og_rmsnorm(C.byref(prog._p.contents.ops[i]), _p(x), 5, _p(y))
    w = np.asarray(layers[2]["weight"], np.float32)
    assert_same(y, _rmsnorm_def(x, w, np.float32(1e-6)), "rmsnorm")


def test_embedding_ids(oracle_lib):
    layers, _ = configs.transformer(1, 4, 8, 2, 8, 1, 6, seed=2)
    prog = oracle.Program(layers[:1])
    table = np.asarray(layers[0]["weight"], np.float32).reshape(6, 8)
    ids = np.array([[0.0, 5.9, np.nan, -3.0, 2.5]], np.float32)
    y, _, _ = prog.execute(ids)
    assert_same(y[0], table[[0, 5, 0, 0, 2]], "ids as usize")
    for bad in (6.0, 1e20, np.inf):
        with pytest.raises(RuntimeError):
            prog.execute(np.array([[bad]], np.float32))


def test_attention_composition(oracle_lib):
    """og_attention = the q/k/v Linears, head split, bmm with k^T, scale, softmax, bmm
    with v, merge, o Linear — composed here from the oracle's separate pieces."""
    b, t, d, h = 2, 11, 24, 3
    dh = d // h
    layers, _ = configs.transformer(b, t, d, h, 16, 1, 10, seed=4)
    prog = oracle.Program(layers)
    ai = next(k for k, op in enumerate(prog.ops) if op.kind == oracle.ATTENTION)
    raw = prog._p.contents.ops[ai]
    x = np.random.default_rng(3).standard_normal((b, t, d)).astype(np.float32)
    y = np.empty_like(x)
    oracle.lib().og_attention(C.byref(raw), _p(x), b, t, _p(y), 1)

    def lin(j, v):
        out = np.empty((v.shape[0], d), np.float32)
        oracle.lib().og_op_linear(C.byref(raw.sub[j]), _p(np.ascontiguousarray(v)), v.shape[0], _p(out), None,
                                  None, None, 1)
        return out
    xs = x.reshape(b * t, d)
    q, k, v = (lin(j, xs).reshape(b, t, h, dh).transpose(0, 2, 1, 3).reshape(b * h, t, dh).copy() for j in range(3))
    kt = np.ascontiguousarray(k.transpose(0, 2, 1))
    sc = np.empty((b * h, t, t), np.float32)
    oracle.lib().og_bmm_fma(_p(q), _p(kt), b * h, t, dh, t, _p(sc))
    sc = (sc * np.float32(np.float32(1.0) / np.float32(np.sqrt(np.float32(dh))))).astype(np.float32)
    p = oracle.softmax(sc)
    o = np.empty((b * h, t, dh), np.float32)
    oracle.lib().og_bmm_fma(_p(np.ascontiguousarray(p)), _p(v), b * h, t, t, dh, _p(o))
    merged = o.reshape(b, h, t, dh).transpose(0, 2, 1, 3).reshape(b * t, d).copy()
    assert_same(y.reshape(b * t, d), lin(3, merged), "attention")
    # the core the device entry rg_attention_f32 is checked against
    qkv = np.concatenate([lin(j, xs) for j in range(3)], axis=1)
    assert_same(oracle.attention_core(qkv, b, t, h, dh), merged, "attention core")


def test_swiglu_composition(oracle_lib):
    layers, _ = configs.transformer(1, 3, 16, 2, 24, 1, 10, seed=6)
    prog = oracle.Program(layers)
    si = next(k for k, op in enumerate(prog.ops) if op.kind == oracle.SWIGLU)
    raw = prog._p.contents.ops[si]
    x = np.random.default_rng(5).standard_normal((7, 16)).astype(np.float32)
    y = np.empty_like(x)
    oracle.lib().og_swiglu(C.byref(raw), _p(x), 7, _p(y), 1)

    def lin(j, v, n):
        out = np.empty((v.shape[0], n), np.float32)
        oracle.lib().og_op_linear(C.byref(raw.sub[j]), _p(np.ascontiguousarray(v)), v.shape[0], _p(out), None,
                                  None, None, 1)
        return out
    g, u = lin(0, x, 24), lin(1, x, 24)
    sig = oracle.act_apply(2, 0.0, g)
    m = ((g * sig).astype(np.float32) * u).astype(np.float32)
    assert_same(y, lin(2, m, 16), "swiglu")


@pytest.mark.parametrize("kw", [dict(batch=2, seq=10, d=32, heads=2, hidden=48, n_layers=2, vocab=90, seed=1),
                                dict(batch=1, seq=5, d=64, heads=4, hidden=24, n_layers=1, vocab=7, seed=8)])
def test_builder_matches_oracle_config(kw):
    model, x = pc.transformer(**kw)
    layers, xo = configs.transformer(**kw)
    assert_same(x, xo, "ids")
    exported = [S.as_dict(l) for l in model.export()]
    assert len(exported) == len(layers)
    for e, o in zip(exported, layers):
        assert e["kind"] == o["kind"]
        for k in ("in_features", "out_features", "act"):
            if k in o:
                assert e.get(k, 0) == o[k], (k, e["kind"])
        if "act_param" in o:
            assert np.float32(e.get("act_param", 0.0)) == np.float32(o["act_param"])
        for k in ("weight", "bias"):
            if k in o:
                assert_same(np.asarray(e[k]).reshape(-1), np.asarray(o[k], np.float32).reshape(-1), k)


def test_row_offset_draws_the_same_sequences():
    _, x = pc.transformer(3, 6, 16, 2, 8, 1, 50, seed=4)
    _, x1 = pc.transformer(2, 6, 16, 2, 8, 1, 50, seed=4, row_offset=1)
    assert_same(x1, x[1:], "row offset")


def test_c5_work_per_sample(oracle_lib):
    """INT8 MACs of one 512-token sequence at the benchmark's widths: 12 layers x 512 x
    (4 d^2 + 3 d h) = 78.92e9 (157.84 INT8 GOPs per sample)."""
    d, h, t = 1024, 2816, 512
    assert 12 * t * (4 * d * d + 3 * d * h) == 78_920_024_064
