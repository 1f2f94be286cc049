"""SiLU activation extension: the reference's nn::Silu (src/nn/layers.rs:337-346)
computes x.mul(x.sigmoid()) but has no Activation variant or .rtim tag, so code 6 is
an IR extension.  The oracle's SiLU must be the reference's two steps: the sigmoid of
UnaryOp::apply (device/backend.rs:72) rounded to f32, then one f32 multiply."""
import numpy as np
import pytest

from oracle import oracle
from oracle.oracle import ACT_SIGMOID, ACT_SILU
from rustgears_b200 import nn, rtim
from rustgears_b200.spec import Activation


def test_oracle_silu_is_x_times_sigmoid(oracle_lib):
    L = oracle_lib.lib()
    rng = np.random.default_rng(6)
    xs = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 8,
                         np.array([0.0, -0.0, 88.8, -88.8, 1e-30, -1e-30, np.inf, -np.inf], np.float32)])
    for x in xs:
        sg = np.float32(L.og_act_apply(ACT_SIGMOID, 0.0, float(x)))
        with np.errstate(invalid="ignore"):
            want = np.float32(np.float32(x) * sg)
        got = np.float32(L.og_act_apply(ACT_SILU, 0.0, float(x)))
        assert got.view(np.uint32) == want.view(np.uint32) or (np.isnan(got) and np.isnan(want)), x


def test_silu_label_and_export(oracle_lib):
    layers = [dict(kind=oracle.LINEAR, in_features=3, out_features=2, weight=np.ones((3, 2), np.float32),
                   bias=np.zeros(2, np.float32)), dict(kind=oracle.ACTIVATION, act=ACT_SILU)]
    p = oracle.Program(layers)
    assert p.ops[0].label() == "NPU::FusedGemmAct(3->2, SiLU)"
    assert str(Activation.SILU) == "SiLU"
    assert [type(l).__name__ for l in nn.Silu().export()] == ["ActivationLayer"]


def test_silu_has_no_rtim_tag(tmp_path):
    from rustgears_b200.spec import ActivationLayer
    with pytest.raises(rtim.RtimError):
        rtim.encode_layers([ActivationLayer(Activation.SILU)])
