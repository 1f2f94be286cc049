"""The FP16 arm (ExecutionProvider::npu_fp16(), NpuPrecision::Fp16) on the device vs the oracle.

Reference: fp16_gemm_fused_into (src/inference/npu.rs:431-445) with round_fp16
(src/inference/quantize.rs:50-64).  Bar: bit-exact f32 outputs -- the products of two
fp16 values are exact in f32, so a k-ordered FMA chain reproduces the reference's
serial sum exactly (no tolerance needed).
"""
import os

import numpy as np
import pytest

from oracle import configs, oracle
from rustgears_b200 import ExecutionProvider, InferenceSession, _native
from tests.helpers import assert_same, spec_from_dict

pytestmark = pytest.mark.gpu
FP16 = 1


def fp16_session(layers, **kw):
    return InferenceSession.from_layers([spec_from_dict(l) for l in layers], ExecutionProvider.npu_fp16(), **kw)


def ref_fp16(layers, x):
    y, _, macs = oracle.Program(layers, precision=FP16).execute(x, nthreads=os.cpu_count() or 1)
    return y, macs


@pytest.mark.parametrize("name", sorted(n for n in configs.CASES if n != "transformer_mini"))
def test_cases_match_oracle(gpu, oracle_lib, name):
    layers, x = configs.CASES[name]()
    sess = fp16_session(layers)
    y = sess.run(x)
    ref, macs = ref_fp16(layers, x)
    assert_same(y, ref, name)
    prog = oracle.Program(layers, precision=FP16)
    assert sess.compilation_report() == prog.summary(len(layers))
    prof = sess.last_npu_profile()
    assert str(prof.precision) == "FP16"
    assert (prof.fp32_weight_bytes, prof.npu_weight_bytes) == (prog.fp32_bytes, prog.npu_bytes)
    assert [r.macs for r in prof.records] == macs.tolist()


@pytest.mark.parametrize("case,batch", [("c1", 4096), ("c2", 256), ("c2", 3), ("c2", 1)])
def test_configs_at_batch(gpu, oracle_lib, case, batch):
    layers, x = {"c1": configs.c1_mlp, "c2": configs.c2_cnn}[case](batch)
    ref, _ = ref_fp16(layers, x)
    assert_same(fp16_session(layers).run(x), ref, f"{case} batch {batch}")


@pytest.mark.parametrize("mkn", [(1, 16, 16), (77, 100, 33), (130, 1568, 128), (64, 4, 3), (300, 7, 65)])
def test_linear_shapes(gpu, oracle_lib, mkn):
    m, k, n = mkn
    layers, x = configs.c3_linear(m, k, n, seed=m + k + n)
    ref, _ = ref_fp16(layers, x)
    assert_same(fp16_session(layers).run(x), ref, f"fp16 linear {mkn}")


@pytest.mark.parametrize("cin,cout,k,st,pad,h,w", [(3, 8, 3, 1, 1, 9, 7), (5, 70, 3, 2, 1, 11, 10),
                                                  (16, 32, 1, 2, 0, 8, 8), (2, 4, 7, 2, 3, 15, 13),
                                                  (1, 16, 3, 1, 0, 6, 6)])
def test_conv_shapes(gpu, oracle_lib, cin, cout, k, st, pad, h, w):
    from oracle.oracle import ACT_RELU
    rng = np.random.default_rng(cin * 100 + cout)
    wt = (rng.standard_normal((cout, cin, k, k)) * 0.3).astype(np.float32)
    b = (rng.standard_normal(cout) * 0.1).astype(np.float32)
    layers = [dict(kind=configs.CONV2D, in_channels=cin, out_channels=cout, kernel=k, stride=st, padding=pad,
                   weight=wt.ravel(), bias=b), configs.act(ACT_RELU)]
    x = rng.standard_normal((3, cin, h, w)).astype(np.float32)
    ref, _ = ref_fp16(layers, x)
    assert_same(fp16_session(layers).run(x), ref, "fp16 conv")


def test_special_values(gpu, oracle_lib):
    layers, x = configs.c1_mlp(64)
    sess = fp16_session(layers)
    cases = {"zeros": np.zeros_like(x), "nan": x.copy(), "inf": x.copy(), "tiny": x * np.float32(1e-30),
             "huge": x * np.float32(1e30), "fp16_edges": x * np.float32(65519.0)}
    cases["nan"][3, 1] = np.nan
    cases["inf"][5, 2] = np.inf
    for what, xx in cases.items():
        ref, _ = ref_fp16(layers, xx)
        assert_same(sess.run(xx), ref, what)


def test_device_buffers_and_graph_replay(gpu, oracle_lib):
    torch = gpu
    layers, x = configs.c2_cnn(64)
    ref, _ = ref_fp16(layers, x)
    sess = fp16_session(layers)
    xd = torch.from_numpy(x).cuda()
    for _ in range(3):  # the third identical run replays a CUDA graph
        yd = sess.run_device(xd)
        assert_same(yd.cpu().numpy(), ref, "device run")


def test_extension_blocks_are_int8_only(gpu):
    layers, _ = configs.transformer_mini(1, 4)
    with pytest.raises(_native.RgError) as e:
        fp16_session(layers)
    assert e.value.status == _native.RG_ERR_UNSUPPORTED


@pytest.mark.parametrize("cin,cout,k,st,pad,h,w,act", [(1, 16, 3, 1, 1, 28, 28, 1), (3, 8, 3, 1, 1, 15, 13, 5),
                                                       (5, 70, 3, 2, 1, 11, 10, 0), (2, 4, 5, 1, 2, 9, 9, 4)])
def test_conv_with_fused_max_pool(gpu, oracle_lib, cin, cout, k, st, pad, h, w, act):
    """An FP16 conv followed by MaxPool2d(2, 2) writes the pooled map in the same kernel
    (odd maps drop the last row / column as the pool does); special values in the input
    (a NaN that must propagate through the pool, an inf); against the oracle and the
    unfused session, bit for bit, with one launch fewer."""
    rng = np.random.default_rng(cin * 100 + cout + h)
    wt = (rng.standard_normal((cout, cin, k, k)) * 0.3).astype(np.float32)
    b = (rng.standard_normal(cout) * 0.1).astype(np.float32)
    layers = [dict(kind=configs.CONV2D, in_channels=cin, out_channels=cout, kernel=k, stride=st, padding=pad,
                   weight=wt.ravel(), bias=b), configs.act(act, 0.1),
              dict(kind=configs.MAXPOOL2D, kernel=2, stride=2)]
    x = rng.standard_normal((5, cin, h, w)).astype(np.float32)
    x[1, 0, h // 2, w // 2] = np.nan
    x[2, 0, 1, 1] = np.inf
    ref, _ = ref_fp16(layers, x)
    fused = fp16_session(layers)
    assert_same(fused.run(x), ref, "fused conv + pool")
    n_fused = fused.last_npu_profile().kernel_launches
    unfused = fp16_session(layers, flags=_native.RG_SESSION_NO_FUSION)
    assert_same(unfused.run(x), ref, "conv, then pool")
    assert n_fused == unfused.last_npu_profile().kernel_launches - 1
