"""Every benchmark configuration at the size it is stated at, against the oracle,
through the C ABI (InferenceSession -> librg_npu.so):

* C2 small CNN at B = 32768 (the whole batch compared), host and device buffers;
* C3 65536 x 4096 x 14336 + GELU: every row computed on the device, rows sampled
  across the batch compared (the oracle quantizes them with the absmax of the
  whole 1 GiB input, as the reference's serial pass over the batch does,
  src/inference/npu.rs:312);
* C4 ResNet-18 at B = 128 (the whole batch; the final Linear's scale is the
  absmax over all 128 images' pooled features);
* C5 transformer: 12 layers, d_model 1024, 16 heads, SwiGLU 2816, one sequence
  of 512 tokens;
* C3 with per-output-channel i8 weights (the configuration's "symmetric per-channel";
  an extension of the reference's per-tensor QuantTensor, restated in the
  oracle as og_compile_ex(weight_quant = 1)).

Bar: bit-exact f32 outputs (the north star allows 1e-5 relative on f32; every
f32 step is restated operation by operation, so equality is asserted).
"""
import os

import numpy as np
import pytest

from oracle import configs, oracle
from tests.helpers import assert_same, session_for

pytestmark = pytest.mark.gpu
NT = os.cpu_count() or 1


def _absmax(x):
    """fold(0, max(|v|)) over the tensor (no NaN in these inputs)."""
    return float(np.max(np.abs(x))) if x.size else 0.0


def test_c2_full_batch_32768(gpu, oracle_lib):
    torch = gpu
    layers, x = configs.c2_cnn(32768)
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=NT)
    sess = session_for(layers)
    assert_same(sess.run(x), ref, "C2 B=32768, host buffers")
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty(ref.shape, dtype=torch.float32, device="cuda")
    for _ in range(3):  # the third identical run replays the captured graph
        yd.fill_(float("nan"))
        sess.run_device(xd, yd)
        torch.cuda.synchronize()
        assert_same(yd.cpu().numpy(), ref, "C2 B=32768, device buffers")


def _sampled_rows(m, n_random, seed):
    return np.unique(np.concatenate([[0, 1, m // 2, m - 1],
                                     np.random.default_rng(seed).integers(0, m, n_random)])).astype(np.int64)


@pytest.mark.parametrize("weight_quant", [0, 1])
def test_c3c_full_size_sampled_rows(gpu, oracle_lib, weight_quant):
    torch = gpu
    m, k, n = 65536, 4096, 14336
    layers, x = configs.c3_linear(m, k, n)
    prog = oracle.Program(layers, weight_quant=weight_quant)
    sess = session_for(layers, weight_quant=("per_tensor", "per_channel")[weight_quant])
    xd = torch.from_numpy(x).cuda()
    yd = sess.run_device(xd)
    torch.cuda.synchronize()
    rows = _sampled_rows(m, 20, 3 + weight_quant)
    got = yd[torch.from_numpy(rows).cuda()].cpu().numpy()
    del yd, xd
    ref = oracle.linear_given_amax(prog, 0, x[rows], _absmax(x), nthreads=NT)
    assert_same(got, ref, f"C3c sampled rows (weight_quant {weight_quant})")
    wq, _ = sess.op_weights(0)
    assert np.array_equal(wq, prog.ops[0].wq)


def test_c3a_per_channel_full_size(gpu, oracle_lib):
    torch = gpu
    m = k = n = 4096
    layers, x = configs.c3_linear(m, k, n)
    prog = oracle.Program(layers, weight_quant=1)
    sess = session_for(layers, weight_quant="per_channel")
    xd = torch.from_numpy(x).cuda()
    yd = sess.run_device(xd)
    torch.cuda.synchronize()
    rows = _sampled_rows(m, 60, 11)
    ref = oracle.linear_given_amax(prog, 0, x[rows], _absmax(x), nthreads=NT)
    assert_same(yd[torch.from_numpy(rows).cuda()].cpu().numpy(), ref, "C3a per-channel")
    assert sess.compilation_report() == prog.summary(len(layers))


def test_c4_resnet18_batch_128(gpu, oracle_lib):
    layers, x = configs.resnet18(128)
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=NT)
    assert_same(session_for(layers).run(x), ref, "C4 ResNet-18 B=128")


def test_c5_twelve_layers_512_tokens(gpu, oracle_lib):
    layers, ids = configs.transformer_c5(batch=1)
    ref, _, _ = oracle.Program(layers).execute(ids, nthreads=NT)
    sess = session_for(layers)
    assert_same(sess.run(ids), ref, "C5 12 layers x 512 tokens")
    assert sess.last_npu_profile().original_layers == len(layers)


@pytest.mark.parametrize("case", ["c1_mlp_64", "c2_cnn_4", "strided_cnn", "affine_first", "resnet_mini",
                                  "c3_linear_small"])
def test_per_channel_weights_match_oracle(gpu, oracle_lib, case):
    """Per-output-channel weights through every op kind that quantizes weights
    (Linear, Conv2d incl. the direct and stem kernels' fallbacks, a standalone
    ChannelAffine's diagonal Linear, shortcut convs): same i8 weights, same
    byte accounting and bit-exact outputs against og_compile_ex(weight_quant=1)."""
    layers, x = configs.CASES[case]()
    prog = oracle.Program(layers, weight_quant=1)
    sess = session_for(layers, weight_quant="per_channel")
    ref, _, _ = prog.execute(x, nthreads=NT)
    assert_same(sess.run(x), ref, f"{case} per-channel")
    for i, op in enumerate(prog.ops):
        if op.wq is not None and op.kind in (oracle.LINEAR, oracle.CONV2D):
            wq, b = sess.op_weights(i)
            assert np.array_equal(wq, op.wq), (case, i)
    assert sess.last_npu_profile().npu_weight_bytes == prog.npu_bytes
    assert sess.compilation_report() == prog.summary(len(layers))


@pytest.mark.parametrize("mkn", [(256, 512, 384), (300, 64, 10), (77, 100, 48), (4100, 1568, 128), (33, 4, 3)])
def test_per_channel_linear_paths(gpu, oracle_lib, mkn):
    """Per-channel scales in the tcgen05, narrow (N <= 32) and SIMT GEMM epilogues."""
    m, k, n = mkn
    layers, x = configs.c3_linear(m, k, n, seed=m + n)
    prog = oracle.Program(layers, weight_quant=1)
    ref, _, _ = prog.execute(x, nthreads=NT)
    assert_same(session_for(layers, weight_quant="per_channel").run(x), ref, f"per-channel {mkn}")
