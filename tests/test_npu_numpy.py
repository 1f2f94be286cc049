"""Pins the C oracle (oracle/npu_oracle.c) with a second, independent restatement of
the reference's Npu(Int8) path (tests/npu_numpy.py, numpy, written from the Rust
sources): on every golden case made of the reference's own layer kinds, the two
must agree on every op's label, activation scale(s), i8 activations, i32
accumulators and f32 output, on the weight byte counts and on the summary string.
A drift in either restatement fails this test."""
import os

import numpy as np
import pytest

from oracle import configs
from tests import npu_numpy as npn
from tests.helpers import assert_same

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
REFERENCE_KINDS = {1, 2, 3, 4, 5, 6, 7}
CASES = [c for c in sorted(configs.CASES)
         if all(l["kind"] in REFERENCE_KINDS for l in configs.CASES[c]()[0])]


def test_cases_cover_the_reference_kinds():
    assert {"usage_doc", "integration", "c1_mlp_64", "c2_cnn_4", "c3_linear_small", "acts_mlp", "strided_cnn",
            "affine_first"} <= set(CASES)


@pytest.mark.parametrize("name", CASES)
def test_numpy_restatement_matches_the_c_oracle(name):
    g = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    layers, x = configs.CASES[name]()
    assert_same(x, g["x"], "input")
    prog = npn.compile_program(layers)
    assert npn.summary(prog) == str(g["summary"])
    assert (prog["fp32_bytes"], prog["npu_bytes"]) == (int(g["fp32_bytes"]), int(g["npu_bytes"]))
    y, trace = npn.execute_traced(prog, x)
    assert len(trace) == int(g["n_ops"])
    for i, t in enumerate(trace):
        assert t["label"] == str(g[f"op{i}_label"])
        assert_same(t["y"].reshape(g[f"op{i}_y"].shape), g[f"op{i}_y"], f"{name} op{i} out")
        if f"op{i}_aq" in g:
            assert_same(t["scales"], g[f"op{i}_scales"], f"{name} op{i} scales")
            assert_same(t["aq"].reshape(g[f"op{i}_aq"].shape), g[f"op{i}_aq"], f"{name} op{i} aq")
            assert_same(t["acc"].reshape(g[f"op{i}_acc"].shape), g[f"op{i}_acc"], f"{name} op{i} acc")
    assert_same(y, g["y"], f"{name} output")


@pytest.mark.parametrize("what", ["nan", "inf", "zeros", "tiny", "huge"])
def test_special_values_agree(oracle_lib, what):
    """NaN, inf, all-zero (scale 1), tiny and huge inputs through both restatements."""
    from oracle import oracle
    layers, x = configs.acts_mlp()
    x = x.copy()
    if what == "nan":
        x[1, 2] = np.nan
    elif what == "inf":
        x[0, 0] = np.inf
        x[3, 1] = -np.inf
    elif what == "zeros":
        x[:] = 0
    elif what == "tiny":
        x *= np.float32(1e-30)
    else:
        x *= np.float32(1e30)
    ref, _, _ = oracle.Program(layers).execute(x)
    y, _ = npn.execute_traced(npn.compile_program(layers), x)
    assert_same(y, ref, what)


@pytest.mark.parametrize("name", ["c1_mlp_64", "c2_cnn_4", "acts_mlp", "affine_first", "integration"])
def test_static_calibration_restatements_agree(oracle_lib, name):
    """The calibration extension: the oracle's calibration scales equal the numpy
    restatement's dynamic Linear scales on the calibration batch, and both run another
    batch (twice the range, so values clamp) with those scales frozen, bit for bit."""
    from oracle import oracle
    layers, x = configs.CASES[name]()
    prog = oracle.Program(layers)
    scales = prog.calibrate(x)
    npp = npn.compile_program(layers)
    _, trace = npn.execute_traced(npp, x)
    dyn = np.array([t["scales"][0] for t, op in zip(trace, npp["ops"]) if op["kind"] == npn.LINEAR], np.float32)
    assert_same(scales, dyn, "calibration scales")
    x2 = (x * np.float32(2.0)).astype(np.float32)
    prog.set_calibration(scales)
    y_c, _, _ = prog.execute(x2)
    y_n, tr2 = npn.execute_traced(npp, x2, frozen=scales)
    assert_same(y_c, y_n, f"{name} frozen")
    assert any(np.abs(t["aq"]).max() == 127 for t in tr2 if "aq" in t)
    prog.set_calibration(None)
    assert_same(prog.execute(x2)[0], npn.execute_traced(npp, x2)[0], f"{name} dynamic again")
