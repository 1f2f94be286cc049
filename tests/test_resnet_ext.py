"""Residual blocks and adaptive pooling (extension kinds for the ResNet-18 config):
the product-side builder against the oracle's configuration, the oracle's new ops
against their definitions, and IR validation.  CPU only."""
import numpy as np
import pytest

from oracle import configs, oracle
from rustgears_b200 import configs as pc
from rustgears_b200 import spec as S
from tests.helpers import assert_same


def _flat(spec_obj):
    d = S.as_dict(spec_obj)
    return {k: (np.asarray(v, np.float32) if isinstance(v, np.ndarray) else v) for k, v in d.items()}


@pytest.mark.parametrize("kw", [dict(batch=2, image=24, widths=(8, 16), classes=10, seed=9, stem_k=3),
                                dict(batch=1, image=64, widths=(16, 32, 64), classes=7, seed=3)])
def test_builder_matches_oracle_config(kw):
    model, x = pc.resnet(**kw)
    layers, xo = configs.resnet(kw["batch"], kw["image"], kw["widths"], kw["classes"], kw["seed"],
                                stem_k=kw.get("stem_k", 7))
    assert_same(x, xo, "input")
    exported = [_flat(l) for l in model.export()]
    assert len(exported) == len(layers)
    for e, o in zip(exported, layers):
        assert e["kind"] == o["kind"]
        for k in ("in_channels", "out_channels", "kernel", "stride", "padding", "in_features", "out_features",
                  "act", "act_param"):
            if k in o:
                assert e.get(k, 0) == o[k], (k, e, o)
        for k in ("weight", "bias", "scale", "shift"):
            if k in o:
                assert_same(np.asarray(e[k]).reshape(-1), np.asarray(o[k], np.float32).reshape(-1), k)


def test_row_offset_draws_the_same_images():
    _, x = pc.resnet(3, 16, (8,), 5, seed=4, stem_k=3)
    _, x1 = pc.resnet(2, 16, (8,), 5, seed=4, stem_k=3, row_offset=1)
    assert_same(x1, x[1:], "row offset")


def test_adaptive_avgpool_definition(oracle_lib):
    x = np.random.default_rng(0).standard_normal((2, 3, 7, 5)).astype(np.float32)
    for oh, ow in [(1, 1), (3, 2), (7, 5), (4, 4)]:
        y = oracle.adaptive_avgpool2d(x, oh, ow)
        ref = np.empty((2, 3, oh, ow), np.float32)
        for i in range(oh):
            for j in range(ow):
                y0, y1 = i * 7 // oh, -(-(i + 1) * 7 // oh)
                x0, x1 = j * 5 // ow, -(-(j + 1) * 5 // ow)
                for p in range(6):
                    s = np.float32(0)
                    for yy in range(y0, y1):
                        for xx in range(x0, x1):
                            s = np.float32(s + x.reshape(6, 7, 5)[p, yy, xx])
                    ref.reshape(6, oh, ow)[p, i, j] = np.float32(s / np.float32((y1 - y0) * (x1 - x0)))
        assert_same(y, ref, f"{oh}x{ow}")


def test_residual_add_definition(oracle_lib):
    r = np.random.default_rng(1)
    a, b = r.standard_normal(100).astype(np.float32), r.standard_normal(100).astype(np.float32)
    assert_same(oracle.residual_add(a, b, oracle.ACT_RELU), np.maximum(a + b, np.float32(0)), "relu(a+b)")
    assert_same(oracle.residual_add(a, b, oracle.ACT_NONE), a + b, "a+b")


def test_identity_block_with_zero_weights_is_relu_of_input(oracle_lib):
    """A block whose convs have zero weights and biases adds nothing: y = relu(x)."""
    z = lambda *s: np.zeros(s, np.float32)
    layers = [dict(kind=oracle.RESIDUAL_BEGIN),
              dict(kind=oracle.CONV2D, in_channels=4, out_channels=4, kernel=3, stride=1, padding=1,
                   weight=z(4, 4, 3, 3), bias=z(4)),
              dict(kind=oracle.ACTIVATION, act=oracle.ACT_RELU, act_param=0.0),
              dict(kind=oracle.CONV2D, in_channels=4, out_channels=4, kernel=3, stride=1, padding=1,
                   weight=z(4, 4, 3, 3), bias=z(4)),
              dict(kind=oracle.RESIDUAL_END, act=oracle.ACT_RELU, act_param=0.0)]
    x = np.random.default_rng(2).standard_normal((2, 4, 6, 6)).astype(np.float32)
    y, _, _ = oracle.Program(layers).execute(x)
    assert_same(y, np.maximum(x, np.float32(0)), "relu(x)")


def test_resnet18_shape_and_work(oracle_lib):
    layers, _ = configs.resnet18(1)
    p = oracle.Program(layers)
    labels = [op.label() for op in p.ops]
    assert labels[0] == "NPU::FusedConv2dAct(3->64, k=7, ReLU)"
    assert labels.count("NPU::ResidualBegin") == 8 and labels.count("NPU::ShortcutConv2d(64->128, k=1)") == 1
    assert labels[-3:] == ["NPU::AdaptiveAvgPool2d(1x1)", "NPU::Flatten", "NPU::Gemm(512->1000)"]
