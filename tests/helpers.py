"""Shared helpers for the tests."""
import numpy as np


def assert_same(a, b, what=""):
    """Bit-exact equality of values: NaN matches NaN, -0.0 matches +0.0."""
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape, f"{what}: shape {a.shape} != {b.shape}"
    if a.dtype.kind == "f":
        ok = (a == b) | (np.isnan(a) & np.isnan(b))
    else:
        ok = a == b
    if not ok.all():
        idx = np.argwhere(~ok)[:5]
        raise AssertionError(f"{what}: {int((~ok).sum())} of {a.size} differ; first {idx.tolist()}: "
                             f"{[a[tuple(i)] for i in idx]} vs {[b[tuple(i)] for i in idx]}")


def spec_from_dict(d):
    """Oracle-style layer dict -> product LayerSpec object."""
    from rustgears_b200 import spec as S
    k = d["kind"]
    if k == S.LINEAR:
        return S.Linear(d["in_features"], d["out_features"], d["weight"], d["bias"])
    if k == S.CONV2D:
        return S.Conv2d(d["in_channels"], d["out_channels"], d["kernel"], d["stride"], d["padding"],
                        d["weight"], d["bias"])
    if k == S.CHANNEL_AFFINE:
        return S.ChannelAffine(d["scale"], d["shift"])
    if k == S.MAXPOOL2D:
        return S.MaxPool2d(d["kernel"], d["stride"])
    if k == S.FLATTEN:
        return S.Flatten()
    if k == S.ACTIVATION:
        return S.ActivationLayer(S.Activation(d["act"], d.get("act_param", 0.0)))
    if k == S.SOFTMAX:
        return S.Softmax()
    if k == S.RESIDUAL_BEGIN:
        return S.ResidualBegin()
    if k == S.SHORTCUT_CONV2D:
        return S.ShortcutConv2d(d["in_channels"], d["out_channels"], d["kernel"], d["stride"], d["padding"],
                                d["weight"], d["bias"])
    if k == S.RESIDUAL_END:
        return S.ResidualEnd(S.Activation(d.get("act", 0), d.get("act_param", 0.0)))
    if k == S.ADAPTIVE_AVGPOOL2D:
        return S.AdaptiveAvgPool2d(d["kernel"], d["stride"])
    if k == S.EMBEDDING:
        return S.Embedding(d["in_features"], d["out_features"], d["weight"])
    if k == S.RMSNORM:
        return S.RMSNorm(d["in_features"], d["weight"], d.get("act_param", 1e-6))
    if k == S.ATTENTION:
        dm = d["in_features"]
        w = np.asarray(d["weight"], np.float32).reshape(4, dm * dm)
        b = np.asarray(d["bias"], np.float32).reshape(4, dm)
        return S.Attention(dm, d["out_features"], w[0], b[0], w[1], b[1], w[2], b[2], w[3], b[3])
    if k == S.SWIGLU:
        dm, h = d["in_features"], d["out_features"]
        w = np.asarray(d["weight"], np.float32).ravel()
        return S.SwiGLU(dm, h, w[:dm * h], w[dm * h:2 * dm * h], w[2 * dm * h:])
    raise ValueError(k)


def session_for(layers, **kw):
    from rustgears_b200 import ExecutionProvider, InferenceSession
    return InferenceSession.from_layers([spec_from_dict(l) for l in layers], ExecutionProvider.npu_int8(), **kw)
