"""Transformer extension ops on the device vs the oracle, through the C ABI:
embedding, RMSNorm, multi-head attention (both attention kernels: the general one
and the head-size-64 tiled one), SwiGLU, residual adds, at small and full widths.
Bar: bit-exact f32 outputs (every f32 step follows the reference order)."""
import numpy as np
import pytest

from oracle import configs, oracle
from rustgears_b200 import ExecutionProvider, InferenceSession, _native
from rustgears_b200 import configs as pc
from tests.helpers import assert_same, session_for

pytestmark = pytest.mark.gpu


def _run_both(layers, x, nthreads=16):
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=nthreads)
    return session_for(layers).run(x), ref


@pytest.mark.parametrize("b,t,d,heads,hidden", [
    (2, 136, 128, 2, 160),   # head size 64, t % 128 != 0: partial key chunks and query blocks
    (1, 512, 128, 2, 96),    # the benchmark's sequence length and head size
    (3, 64, 192, 3, 64),     # one query block, one key chunk
    (2, 520, 64, 1, 32),     # t above the tiled kernel's limit: general kernel, head size 64
    (2, 13, 64, 4, 40),      # odd t: score columns past the last 8-block unfused
    (1, 24, 60, 5, 24),      # head size 12: P.V columns past the last 8-block unfused
])
def test_transformer_shapes(gpu, oracle_lib, b, t, d, heads, hidden):
    layers, x = configs.transformer(b, t, d, heads, hidden, 2, 1000, seed=b * 1000 + t)
    y, ref = _run_both(layers, x)
    assert_same(y, ref, f"b{b} t{t} d{d} h{heads}")


def test_transformer_full_width_layers(gpu, oracle_lib):
    """Two layers at the benchmark's widths (d_model 1024, 16 heads, hidden 2816,
    vocabulary 32000), one sequence of 512 tokens: the tensor-core projections with
    per-column scales and the tiled attention kernel at full size."""
    layers, x = configs.transformer(1, 512, 1024, 16, 2816, 2, 32000, seed=42)
    y, ref = _run_both(layers, x, nthreads=32)
    assert_same(y, ref, "full width")


def test_product_builder_matches_oracle(gpu, oracle_lib):
    model, x = pc.transformer(2, 40, 128, 2, 96, 2, 700, seed=5)
    layers, xo = configs.transformer(2, 40, 128, 2, 96, 2, 700, seed=5)
    assert_same(x, xo, "ids")
    sess = InferenceSession.from_module(model, ExecutionProvider.npu_int8())
    ref, _, macs = oracle.Program(layers).execute(x)
    assert_same(sess.run(x), ref, "from_module")
    prof = sess.last_npu_profile()
    assert [r.macs for r in prof.records] == macs.tolist()


def test_token_ids_edge_values(gpu, oracle_lib):
    layers, x = configs.transformer(2, 16, 64, 2, 32, 1, 50, seed=3)
    x = x.copy()
    x[0, 0], x[0, 1], x[0, 2], x[1, 3] = np.nan, -5.0, 0.999, 49.9  # -> ids 0, 0, 0, 49
    y, ref = _run_both(layers, x)
    assert_same(y, ref, "edge ids")
    for bad in (50.0, 1e30, np.inf):
        xb = x.copy()
        xb[1, 7] = bad
        with pytest.raises(RuntimeError):  # og_execute: -6, an id out of range
            oracle.Program(layers).execute(xb)
        sess = session_for(layers)
        with pytest.raises(_native.RgError):
            sess.run(xb)
        assert_same(sess.run(x), ref, "session usable after the error")


def test_large_activations(gpu, oracle_lib):
    """Saturating softmax rows (scores far apart) and large residual values."""
    layers, x = configs.transformer(1, 64, 128, 2, 64, 1, 30, seed=8)
    for l in layers:
        if l["kind"] == oracle.EMBEDDING:
            l["weight"] = (l["weight"] * np.float32(3e3)).astype(np.float32)
    y, ref = _run_both(layers, x)
    assert_same(y, ref, "large")


def test_empty_batch_and_shape_errors(gpu, oracle_lib):
    layers, x = configs.transformer(1, 8, 64, 2, 32, 1, 20, seed=1)
    sess = session_for(layers)
    assert sess.run(x[:0]).shape == (0, 8, 64)
    with pytest.raises(_native.RgError):  # attention needs [B, T, d]
        sess.run(np.zeros((8,), np.float32))
