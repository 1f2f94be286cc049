"""The oracle re-run against the committed golden fixtures (tests/golden/*.npz)."""
import os

import numpy as np
import pytest

from oracle import configs, oracle
from tests.helpers import assert_same

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("name", sorted(configs.CASES))
def test_oracle_matches_golden(oracle_lib, name):
    g = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    layers, x = configs.CASES[name]()
    assert_same(x, g["x"], "input")
    p = oracle.Program(layers)
    assert p.summary(len(layers)) == str(g["summary"])
    assert (p.fp32_bytes, p.npu_bytes) == (int(g["fp32_bytes"]), int(g["npu_bytes"]))
    y, trace = p.run_traced(x)
    assert len(trace) == int(g["n_ops"])
    for i, t in enumerate(trace):
        assert t["label"] == str(g[f"op{i}_label"])
        assert_same(t["y"], g[f"op{i}_y"], f"op{i} y")
        if "aq" in t:
            sc = np.atleast_1d(np.asarray(t.get("a_scale", t.get("a_scales")), np.float32))
            assert_same(sc, g[f"op{i}_scales"], f"op{i} scales")
            assert_same(t["aq"], g[f"op{i}_aq"], f"op{i} aq")
            assert_same(t["acc"], g[f"op{i}_acc"], f"op{i} acc")
    assert_same(y, g["y"], "output")
