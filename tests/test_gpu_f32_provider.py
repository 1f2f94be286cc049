"""The f32 ExecutionProvider::Cpu arm on the device vs the oracle's run_standard.

Reference: from_layers folds BatchNorm for the Cpu provider (src/inference/mod.rs:
162-166) and run_standard (mod.rs:260-331) walks the folded layers one by one, its
matmuls through the CPU matmul (src/device/cpu.rs:233-395: FMA chains in k order,
unfused tails past the last full 8-wide column block).  Bar: bit-exact f32 outputs.
"""
import numpy as np
import pytest

from oracle import configs, oracle
from oracle.oracle import ACT_GELU, ACT_RELU
from rustgears_b200 import ExecutionProvider, InferenceSession, _native
from tests.helpers import assert_same, spec_from_dict

pytestmark = pytest.mark.gpu
REFERENCE_KINDS = {"usage_doc", "integration", "c1_mlp_64", "c2_cnn_4", "c3_linear_small", "acts_mlp",
                   "strided_cnn", "affine_first"}


def cpu_session(layers):
    return InferenceSession.from_layers([spec_from_dict(l) for l in layers], ExecutionProvider.cpu())


@pytest.mark.parametrize("name", sorted(REFERENCE_KINDS))
def test_cases_match_oracle(gpu, oracle_lib, name):
    layers, x = configs.CASES[name]()
    sess = cpu_session(layers)
    assert_same(sess.run(x), oracle.run_standard(layers, x), name)
    # CompiledProgram::Standard: report format (mod.rs:200-206), no NpuProfile
    nfold = oracle_lib.Program(layers).original_layers
    assert sess.compilation_report().startswith("InferenceSession [provider = CPU (FP32), device = cpu, ops = ")
    assert sess.compilation_report().endswith(f"(from {nfold} raw layers)]")
    assert sess.last_npu_profile() is None


@pytest.mark.parametrize("mkn", [(1, 16, 16), (77, 100, 33), (130, 1568, 128), (64, 4, 3), (300, 7, 13)])
def test_linear_shapes(gpu, oracle_lib, mkn):
    m, k, n = mkn
    layers, x = configs.c3_linear(m, k, n, seed=m + k + n)
    assert_same(cpu_session(layers).run(x), oracle.run_standard(layers, x), f"f32 linear {mkn}")


@pytest.mark.parametrize("cin,cout,k,st,pad,h,w", [(3, 8, 3, 1, 1, 5, 5), (5, 70, 3, 2, 1, 11, 10),
                                                  (16, 32, 1, 2, 0, 8, 8), (1, 16, 3, 1, 1, 28, 28)])
def test_conv_shapes(gpu, oracle_lib, cin, cout, k, st, pad, h, w):
    rng = np.random.default_rng(cin * 100 + cout + h)
    wt = rng.standard_normal((cout, cin, k, k)).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    layers = [dict(kind=configs.CONV2D, in_channels=cin, out_channels=cout, kernel=k, stride=st, padding=pad,
                   weight=wt.ravel(), bias=b), configs.act(ACT_GELU)]
    x = rng.standard_normal((3, cin, h, w)).astype(np.float32)
    assert_same(cpu_session(layers).run(x), oracle.run_standard(layers, x), "f32 conv")


def test_special_values_and_device_runs(gpu, oracle_lib):
    torch = gpu
    layers, x = configs.c1_mlp(64)
    sess = cpu_session(layers)
    xx = x.copy()
    xx[3, 1], xx[5, 2], xx[7, 0] = np.nan, np.inf, -np.inf
    assert_same(sess.run(xx), oracle.run_standard(layers, xx), "specials")
    layers, x = configs.c2_cnn(32)
    sess = cpu_session(layers)
    ref = oracle.run_standard(layers, x)
    xd = torch.from_numpy(x).cuda()
    for _ in range(3):  # the third identical run replays a CUDA graph
        assert_same(sess.run_device(xd).cpu().numpy(), ref, "device run")


def test_extension_kinds_and_gpu_provider_rejected(gpu):
    layers, _ = configs.resnet_mini()
    with pytest.raises(_native.RgError) as e:
        cpu_session(layers)
    assert e.value.status == _native.RG_ERR_UNSUPPORTED
    layers, _ = configs.c1_mlp(4)
    with pytest.raises(_native.RgError) as e:
        InferenceSession.from_layers([spec_from_dict(l) for l in layers], ExecutionProvider.gpu(0))
    assert e.value.status == _native.RG_ERR_UNSUPPORTED


@pytest.mark.parametrize("cin,cout,k,st,pad,h,w,act", [(1, 16, 3, 1, 1, 10, 10, ACT_RELU), (3, 8, 3, 1, 1, 15, 13, ACT_GELU),
                                                       (5, 70, 3, 2, 1, 11, 10, None), (2, 4, 5, 1, 2, 9, 9, ACT_RELU)])
def test_conv_activation_pool_in_one_kernel(gpu, oracle_lib, cin, cout, k, st, pad, h, w, act):
    """Conv2d, its activation layer and MaxPool2d(2, 2) in one kernel: each pixel's sum
    (FMA chain, or unfused past the matmul's last full 8-wide block of pixels: the 10 x
    10 case puts such pixels inside pool windows), its activation, then the pool's
    NaN-propagating max; a NaN and an inf in the input; bit-exact against run_standard."""
    rng = np.random.default_rng(cin * 100 + cout + h)
    wt = rng.standard_normal((cout, cin, k, k)).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    layers = [dict(kind=configs.CONV2D, in_channels=cin, out_channels=cout, kernel=k, stride=st, padding=pad,
                   weight=wt.ravel(), bias=b)]
    if act is not None:
        layers.append(configs.act(act))
    layers.append(dict(kind=configs.MAXPOOL2D, kernel=2, stride=2))
    x = rng.standard_normal((4, cin, h, w)).astype(np.float32)
    x[1, 0, h // 2, w // 2] = np.nan
    x[2, 0, 1, 1] = np.inf
    ref = oracle.run_standard(layers, x)
    assert_same(cpu_session(layers).run(x), ref, "f32 conv + act + pool")
