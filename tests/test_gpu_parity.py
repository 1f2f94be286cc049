"""Device path vs the oracle and the golden fixtures, through the C ABI.

Bar: bit-exact for the i8 activations, i32 accumulators and activation
scales, and for the f32 outputs too (every f32 step is restated operation by
operation; the f32 tolerance the path allows, 1e-5 relative, is not needed).
"""
import os
import threading

import numpy as np
import pytest

from oracle import configs, oracle
from rustgears_b200 import ExecutionProvider, InferenceSession, _native, rtim
from tests.helpers import assert_same, session_for, spec_from_dict

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
pytestmark = pytest.mark.gpu


def _compare_trace(sess, g, nops):
    for i in range(nops):
        assert sess.op_info(i)["label"] == str(g[f"op{i}_label"])
        assert_same(sess.trace(i, _native.RG_TRACE_OUT).reshape(g[f"op{i}_y"].shape), g[f"op{i}_y"], f"op{i} out")
        if f"op{i}_aq" in g:
            assert_same(sess.trace(i, _native.RG_TRACE_SCALES), g[f"op{i}_scales"], f"op{i} scales")
            assert_same(sess.trace(i, _native.RG_TRACE_AQ).reshape(g[f"op{i}_aq"].shape), g[f"op{i}_aq"], f"op{i} aq")
            assert_same(sess.trace(i, _native.RG_TRACE_ACC).reshape(g[f"op{i}_acc"].shape), g[f"op{i}_acc"],
                        f"op{i} acc")


@pytest.mark.parametrize("name", sorted(configs.CASES))
def test_session_matches_golden(gpu, oracle_lib, name):
    g = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    layers, x = configs.CASES[name]()
    sess = session_for(layers)
    assert sess.compilation_report() == str(g["summary"])
    sess.set_trace(True)
    y = sess.run(x)
    assert_same(y, g["y"], "output")
    _compare_trace(sess, g, int(g["n_ops"]))
    prof = sess.last_npu_profile()
    assert prof.original_layers == len(layers) and prof.fused_ops == int(g["n_ops"])
    assert (prof.fp32_weight_bytes, prof.npu_weight_bytes) == (int(g["fp32_bytes"]), int(g["npu_bytes"]))
    _, _, macs = oracle.Program(layers).execute(x)
    assert [r.macs for r in prof.records] == macs.tolist() and prof.total_macs == int(macs.sum())
    assert [r.op for r in prof.records] == [str(g[f"op{i}_label"]) for i in range(int(g["n_ops"]))]


def test_quantized_weights_match_oracle(gpu, oracle_lib):
    for name in sorted(configs.CASES):
        layers, _ = configs.CASES[name]()
        prog = oracle.Program(layers)
        sess = session_for(layers)
        for i, op in enumerate(prog.ops):
            info = sess.op_info(i)
            if op.wq is not None:
                wq, b = sess.op_weights(i)
                assert np.array_equal(wq, op.wq), (name, i)
                assert np.array_equal(b, op.bias), (name, i)
                assert np.float32(info["w_scale"]) == np.float32(op.w_scale), (name, i)


@pytest.mark.parametrize("case,batch", [("c1", 65536), ("c1", 1), ("c2", 256), ("c2", 1), ("c2", 3)])
def test_configs_at_batch(gpu, oracle_lib, case, batch):
    layers, x = {"c1": configs.c1_mlp, "c2": configs.c2_cnn}[case](batch)
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=os.cpu_count() or 1)
    assert_same(session_for(layers).run(x), ref, f"{case} batch {batch}")


@pytest.mark.parametrize("mkn", [(1, 16, 16), (77, 100, 33), (256, 512, 384), (130, 1568, 128), (64, 4, 3),
                                 (300, 7, 1), (129, 33, 5), (1000, 100, 17), (70, 3, 32)])
def test_linear_shapes(gpu, oracle_lib, mkn):
    m, k, n = mkn
    layers, x = configs.c3_linear(m, k, n, seed=m + k + n)
    prog = oracle.Program(layers)
    ref, trace = prog.run_traced(x)
    sess = session_for(layers)
    sess.set_trace(True)
    assert_same(sess.run(x), ref, f"linear {mkn}")
    assert_same(sess.trace(0, _native.RG_TRACE_ACC).reshape(m, n), trace[0]["acc"], "acc")
    # without tracing, narrow layers quantize their f32 input while loading it
    assert_same(session_for(layers).run(x), ref, f"linear {mkn}, untraced")


def test_empty_batch(gpu, oracle_lib):
    layers, _ = configs.c2_cnn(1)
    y = session_for(layers).run(np.zeros((0, 1, 28, 28), np.float32))
    assert y.shape == (0, 10)
    layers, _ = configs.c1_mlp(1)
    assert session_for(layers).run(np.zeros((0, 4), np.float32)).shape == (0, 3)


def test_special_values(gpu, oracle_lib):
    layers, x = configs.c1_mlp(64)
    prog = oracle.Program(layers)
    sess = session_for(layers)
    cases = {"zeros": np.zeros_like(x), "nan": x.copy(), "inf": x.copy(), "tiny": x * np.float32(1e-30),
             "huge": x * np.float32(1e30)}
    cases["nan"][3, 1] = np.nan
    cases["inf"][5, 2] = np.inf
    for what, xx in cases.items():
        ref, _, _ = prog.execute(xx)
        assert_same(sess.run(xx), ref, what)


def test_rtim_drop_in(gpu, oracle_lib, tmp_path):
    layers, x = configs.c2_cnn(5)
    specs = [spec_from_dict(l) for l in layers]
    p = tmp_path / "c2.rtim"
    rtim.save_layers(specs, p)
    a = InferenceSession.from_rtim(str(p), ExecutionProvider.npu_int8())
    b = InferenceSession.from_layers(rtim.load_inference_layers(p), ExecutionProvider.npu_int8())
    ref, _, _ = oracle.Program(layers).execute(x)
    assert_same(a.run(x), ref, "from_rtim")
    assert_same(b.run(x), ref, "load_inference_layers + from_layers")
    assert a.compilation_report() == b.compilation_report()


def test_run_device_and_concurrency(gpu, oracle_lib):
    torch = gpu
    layers, x = configs.c2_cnn(64)
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=8)
    sess = session_for(layers)
    xd = torch.from_numpy(x).cuda()
    yd = sess.run_device(xd)
    torch.cuda.synchronize()
    assert_same(yd.cpu().numpy(), ref, "run_device")
    results = [None] * 4

    def worker(i):
        results[i] = sess.run(x)

    ts = [threading.Thread(target=worker, args=(i,)) for i in range(4)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    for r in results:
        assert_same(r, ref, "concurrent run")


@pytest.mark.parametrize("case", ["c2_cnn_4", "transformer_mini", "resnet_mini", "c1_mlp_64"])
def test_repeated_device_runs_replay_a_graph(gpu, oracle_lib, case):
    """Identical device-buffer runs replay a captured CUDA graph from the second one on:
    same results (also after the input changes in place), per-op profile records
    still timed; a session with RG_SESSION_NO_GRAPH agrees."""
    torch = gpu
    layers, x = configs.CASES[case]()
    ref, _, macs = oracle.Program(layers).execute(x, nthreads=8)
    for flags in (0, _native.RG_SESSION_NO_GRAPH):
        sess = session_for(layers, flags=flags)
        xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
        yd = torch.empty(ref.shape, dtype=torch.float32, device="cuda")
        for _ in range(4):
            yd.fill_(np.nan)
            sess.run_device(xd, yd)
            torch.cuda.synchronize()
            assert_same(yd.cpu().numpy(), ref, f"run {flags}")
            prof = sess.last_npu_profile()
            assert [r.macs for r in prof.records] == macs.tolist()
            assert prof.total_time_ns > 0
        x2 = (x * np.float32(0.5)).astype(np.float32)
        xd.copy_(torch.from_numpy(x2))
        sess.run_device(xd, yd)
        torch.cuda.synchronize()
        ref2, _, _ = oracle.Program(layers).execute(x2, nthreads=8)
        assert_same(yd.cpu().numpy(), ref2, f"new input {flags}")


def test_shape_errors(gpu):
    layers, _ = configs.c2_cnn(1)
    sess = session_for(layers)
    with pytest.raises(_native.ShapeError):
        sess.run(np.zeros((2, 3, 28, 28), np.float32))
    with pytest.raises(_native.ShapeError):
        sess.run(np.zeros((2, 28, 28), np.float32))
    layers, _ = configs.c1_mlp(1)
    with pytest.raises(_native.ShapeError):
        session_for(layers).run(np.zeros((4, 5), np.float32))


@pytest.mark.parametrize("shape", [(4096, 4096, 4096), (16384, 8192, 8192)])
def test_c3_full_size_sampled_rows(gpu, oracle_lib, shape):
    """Full-size C3: the device runs every row; rows sampled across the batch are
    checked against the oracle, whose scale is the absmax over the whole input."""
    torch = gpu
    from rustgears_b200 import configs as pconfigs
    m, k, n = shape
    model, x = pconfigs.c3_linear(m, k, n)
    layers = model.export()
    sess = InferenceSession.from_layers(layers, ExecutionProvider.npu_int8())
    xd = torch.from_numpy(x).cuda()
    yd = sess.run_device(xd)
    torch.cuda.synchronize()
    from rustgears_b200.spec import as_dict
    prog = oracle.Program([as_dict(l) for l in layers])
    rows = np.unique(np.concatenate([[0, m - 1], np.random.default_rng(1).integers(0, m, 30)]))
    for r in rows:
        yr, _, _ = oracle.linear_rows(prog.ops[0], prog, 0, x, int(r), int(r) + 1, nthreads=8)
        assert_same(yd[int(r)].cpu().numpy(), yr[0], f"row {r}")


@pytest.mark.parametrize("special", ["plain", "zero_nan_huge", "inf", "leaky"])
def test_fused_cnn_block_matches_unfused_and_oracle(gpu, oracle_lib, special):
    """The Conv-Pool-Conv-Pool kernel (pools on the i32 accumulators, exact because the
    epilogue is monotone) against the op-by-op path and the oracle; an image holding
    inf takes the kernel's reference-order fallback."""
    layers, x = configs.c2_cnn(12)
    x = x.copy()
    if special == "zero_nan_huge":
        x[1] = 0.0
        x[3, 0, 5, 5] = np.nan
        x[4] *= np.float32(1e30)
        x[5] *= -1.0
    elif special == "inf":
        x[2, 0, 3, 4] = np.inf
    elif special == "leaky":
        layers = [dict(l, act=5, act_param=0.1) if l["kind"] == 6 else l for l in layers]
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=8)
    fused = session_for(layers)
    unfused = session_for(layers, flags=_native.RG_SESSION_NO_FUSION)
    assert_same(fused.run(x), ref, "fused")
    assert_same(unfused.run(x), ref, "unfused")
    prof = fused.last_npu_profile()
    assert prof.kernel_launches < unfused.last_npu_profile().kernel_launches


def test_fused_cnn_block_pipeline_depth(gpu, oracle_lib):
    """1500 images: every CTA of the persistent block kernel runs ~10 images through its
    rings (input slots, double-buffered operands and TMEM), with special images spread
    over the batch so the per-image fallback runs mid-pipeline."""
    layers, x = configs.c2_cnn(1500)
    x = x.copy()
    x[7] = 0.0
    x[300, 0, 1, 2] = np.nan
    x[301] *= np.float32(1e30)
    x[777, 0, 9, 9] = np.inf
    x[1499, 0, 27, 27] = -np.inf
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=8)
    assert_same(session_for(layers).run(x), ref, "fused, 1500 images")


def test_fused_cnn_block_unaligned_input_view(gpu, oracle_lib):
    """The block kernel bulk-copies images and needs 16-byte aligned input; an input view
    4 bytes into its allocation takes the op-by-op path with the same results."""
    torch = gpu
    layers, x = configs.c2_cnn(5)
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=8)
    sess = session_for(layers)
    flat = torch.empty(x.size + 1, dtype=torch.float32, device="cuda")
    view = flat[1:].view(x.shape)
    view.copy_(torch.from_numpy(x))
    assert view.data_ptr() % 16 == 4
    y = sess.run_device(view)
    torch.cuda.synchronize()
    assert_same(y.cpu().numpy(), ref, "unaligned view")


def test_host_input_fed_in_chunks(gpu, oracle_lib):
    """A host-buffer run of a program that starts with the fused CNN block copies the
    input in chunks on a second stream and runs the block per chunk (6000 images: three
    chunks); results equal the oracle, special images on both sides of a chunk edge."""
    layers, x = configs.c2_cnn(6000)
    x = x.copy()
    x[2047, 0, 0, 0] = np.inf
    x[2048] = 0.0
    x[4095, 0, 13, 13] = np.nan
    x[5999] *= np.float32(-3.0)
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=8)
    sess = session_for(layers)
    assert_same(sess.run(x), ref, "chunked host input")
    assert_same(sess.run(x), ref, "chunked host input, second run")


def test_resnet18_full_size_matches_oracle(gpu, oracle_lib):
    """The ResNet-18 benchmark layout at 224 x 224 (batch 2): residual blocks, projection
    shortcuts, stride-2 convs with their covered-pixel absmax, adaptive pooling."""
    layers, x = configs.resnet18(2)
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=16)
    assert_same(session_for(layers).run(x), ref, "resnet18")


@pytest.mark.parametrize("special", ["plain", "zero_nan_inf"])
def test_resnet_mini_special_images(gpu, oracle_lib, special):
    layers, x = configs.resnet_mini(batch=5)
    x = x.copy()
    if special == "zero_nan_inf":
        x[0] = 0.0
        x[1, 2, 3, 4] = np.nan
        x[3, 0, 0, 0] = np.inf
        x[4] *= np.float32(1e20)
    ref, _, _ = oracle.Program(layers).execute(x)
    assert_same(session_for(layers).run(x), ref, special)
    assert session_for(layers).run(x[:0]).shape == (0, 10)


def test_residual_ir_errors(gpu):
    from rustgears_b200 import spec as S
    conv = lambda c: S.Conv2d(c, c, 3, 1, 1, np.zeros((c, c, 3, 3), np.float32), np.zeros(c, np.float32))
    bad = [
        [S.ResidualBegin(), conv(4)],                                   # not closed
        [conv(4), S.ResidualEnd()],                                     # end without begin
        [S.ShortcutConv2d(4, 4, 1, 1, 0, np.zeros((4, 4, 1, 1), np.float32), np.zeros(4, np.float32))],
    ]
    for layers in bad:
        with pytest.raises(_native.RgError):
            InferenceSession.from_layers(layers, ExecutionProvider.npu_int8())
    # main path and shortcut disagree in shape: a shape error at run time
    sess = InferenceSession.from_layers(
        [S.ResidualBegin(), S.Conv2d(4, 8, 3, 1, 1, np.zeros((8, 4, 3, 3), np.float32), np.zeros(8, np.float32)),
         S.ResidualEnd()], ExecutionProvider.npu_int8())
    with pytest.raises(_native.RgError):
        sess.run(np.zeros((1, 4, 5, 5), np.float32))


@pytest.mark.parametrize("b,c,n,h,w,act", [(2, 64, 64, 56, 56, 1), (3, 128, 80, 13, 9, 0), (1, 64, 256, 7, 7, 4),
                                           (2, 192, 64, 5, 31, 1), (4, 64, 128, 1, 1, 0), (1, 64, 64, 3, 120, 5),
                                           (2, 64, 64, 14, 14, 6)])
def test_direct_3x3_conv(gpu, oracle_lib, b, c, n, h, w, act):
    """3x3 / stride 1 / pad 1 convs with channels padded to a multiple of 64 run on the
    direct kernel (zero-padded TMA tiles, shifted A operands): every shape class against
    the oracle, with and without a residual block around it."""
    rng = np.random.default_rng(b * 1000 + c + n + h * w)
    wgt = (rng.standard_normal((n, c, 3, 3)) * 0.05).astype(np.float32)
    bias = (rng.standard_normal(n) * 0.1).astype(np.float32)
    x = rng.standard_normal((b, c, h, w)).astype(np.float32)
    conv = dict(kind=oracle.CONV2D, in_channels=c, out_channels=n, kernel=3, stride=1, padding=1, weight=wgt, bias=bias)
    layers = [conv] + ([dict(kind=oracle.ACTIVATION, act=act, act_param=0.1)] if act else [])
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=8)
    assert_same(session_for(layers).run(x), ref, f"conv {c}->{n} {h}x{w}")
    if n == c:  # a residual block around it: the add fused into the conv's epilogue
        blk = [dict(kind=oracle.RESIDUAL_BEGIN), conv, dict(kind=oracle.RESIDUAL_END, act=1, act_param=0.0)]
        ref2, _, _ = oracle.Program(blk).execute(x, nthreads=8)
        assert_same(session_for(blk).run(x), ref2, "residual")


@pytest.mark.parametrize("b,c,h,w,act", [(2, 3, 224, 224, 1), (3, 1, 32, 46, 0), (1, 4, 20, 224, 5), (5, 2, 8, 8, 4),
                                         (2, 3, 64, 30, 2), (1, 3, 14, 230, 1), (2, 3, 64, 64, 6)])
def test_fused_stem(gpu, oracle_lib, b, c, h, w, act):
    """Conv(k7 s2 p3 -> 64) + activation + MaxPool(3, 2), the ResNet stem: one kernel over
    the space-to-depth operand with the pool folded into the conv's epilogue, against the
    oracle (and against the session's own unfused path)."""
    from rustgears_b200 import _native
    rng = np.random.default_rng(b * 100 + c + h + w)
    wgt = (rng.standard_normal((64, c, 7, 7)) * 0.05).astype(np.float32)
    bias = (rng.standard_normal(64) * 0.1).astype(np.float32)
    x = rng.standard_normal((b, c, h, w)).astype(np.float32)
    layers = [dict(kind=oracle.CONV2D, in_channels=c, out_channels=64, kernel=7, stride=2, padding=3, weight=wgt,
                   bias=bias)]
    if act:
        layers.append(dict(kind=oracle.ACTIVATION, act=act, act_param=0.1))
    layers.append(dict(kind=oracle.MAXPOOL2D, kernel=3, stride=2))
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=8)
    sess = session_for(layers)
    assert_same(sess.run(x), ref, f"stem {c}ch {h}x{w}")
    if w // 2 <= 112:  # rows up to 112 conv columns wide: absmax, s2d quantizer, fused stem
        assert sess.last_npu_profile().kernel_launches == 3
    plain = session_for(layers, flags=_native.RG_SESSION_NO_FUSION)
    assert_same(plain.run(x), ref, "unfused")
    assert plain.last_npu_profile().kernel_launches > 3


@pytest.mark.parametrize("batch,image", [(3, 96), (2, 112), (2, 130)])
def test_resnet_two_stage_paths(gpu, oracle_lib, batch, image):
    """ResNet-18 widths (64, 128) at small images: the fused stem, direct 3x3 convs with
    the block's residual add, the stage-2 projection shortcut (its covered-pixel absmax
    taken in the epilogue of the conv that writes its block input, its compact
    every-other-pixel operand), against the oracle; one image holds an inf."""
    layers, x = configs.resnet(batch, image, (64, 128), 10, seed=image)
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=16)
    assert_same(session_for(layers).run(x), ref, f"resnet {image}")
    x = x.copy()
    x[batch - 1, 1, 5, 7] = np.inf
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=16)
    assert_same(session_for(layers).run(x), ref, f"resnet {image} with inf")


@pytest.mark.parametrize("b,c,n,h,w,k,st,pad,act", [
    (2, 64, 128, 55, 55, 3, 2, 1, 1),   # odd size: the space-to-depth operand's last row / column is padding
    (2, 64, 128, 28, 28, 3, 2, 1, 6),   # SiLU (activation extension)
    (3, 64, 64, 28, 28, 3, 2, 1, 0),
    (2, 128, 256, 14, 14, 3, 2, 1, 1),
    (1, 192, 80, 9, 13, 3, 2, 1, 5),
    (2, 64, 128, 55, 55, 1, 2, 0, 0),   # strided 1x1: compact operand
    (2, 128, 64, 20, 20, 1, 1, 0, 1),
    (1, 256, 512, 7, 7, 1, 1, 0, 0),
])
def test_direct_conv_modes(gpu, oracle_lib, b, c, n, h, w, k, st, pad, act):
    """The direct conv kernel's other tap sets: 3x3 / stride 2 / pad 1 as 2x2 taps over
    the space-to-depth operand, 1x1 over the image or over the pixels a strided 1x1
    conv reads; against the oracle."""
    rng = np.random.default_rng(b * 1000 + c + n + h * w + k * st)
    wgt = (rng.standard_normal((n, c, k, k)) * 0.05).astype(np.float32)
    bias = (rng.standard_normal(n) * 0.1).astype(np.float32)
    x = rng.standard_normal((b, c, h, w)).astype(np.float32)
    layers = [dict(kind=oracle.CONV2D, in_channels=c, out_channels=n, kernel=k, stride=st, padding=pad, weight=wgt,
                   bias=bias)]
    if act:
        layers.append(dict(kind=oracle.ACTIVATION, act=act, act_param=0.1))
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=8)
    assert_same(session_for(layers).run(x), ref, f"conv k{k} s{st} {c}->{n} {h}x{w}")


@pytest.mark.parametrize("mkn", [(512, 1568, 128), (300, 64, 10), (77, 100, 48), (4100, 4096, 260)])
def test_silu_linear(gpu, oracle_lib, mkn):
    """The SiLU activation extension (nn::Silu, src/nn/layers.rs:337-346) fused into the
    Linear epilogues: tensor-core, narrow and SIMT GEMMs, bit-exact against the oracle."""
    from oracle.oracle import ACT_SILU
    m, k, n = mkn
    rng = np.random.default_rng(m + k + n)
    w = (rng.standard_normal((k, n)) * 0.05).astype(np.float32)
    b = (rng.standard_normal(n) * 0.1).astype(np.float32)
    layers = [dict(kind=oracle.LINEAR, in_features=k, out_features=n, weight=w, bias=b),
              dict(kind=oracle.ACTIVATION, act=ACT_SILU)]
    x = rng.standard_normal((m, k)).astype(np.float32)
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=8)
    sess = session_for(layers)
    assert sess.op_info(0)["label"].endswith(", SiLU)")
    assert_same(sess.run(x), ref, f"silu linear {mkn}")


def test_silu_conv_implicit_gemm(gpu, oracle_lib):
    """A 5x5 conv (implicit-GEMM tensor-core path) with the SiLU extension; a CNN block
    with SiLU (not monotone, so the pooled fused block does not apply) runs op by op."""
    from oracle.oracle import ACT_SILU
    rng = np.random.default_rng(55)
    w = (rng.standard_normal((32, 16, 5, 5)) * 0.05).astype(np.float32)
    b = (rng.standard_normal(32) * 0.1).astype(np.float32)
    layers = [dict(kind=oracle.CONV2D, in_channels=16, out_channels=32, kernel=5, stride=1, padding=2, weight=w,
                   bias=b), dict(kind=oracle.ACTIVATION, act=ACT_SILU)]
    x = rng.standard_normal((3, 16, 20, 18)).astype(np.float32)
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=8)
    assert_same(session_for(layers).run(x), ref, "silu conv 5x5")
    layers, x = configs.c2_cnn(64)
    for l in layers:
        if l["kind"] == oracle.ACTIVATION:
            l["act"] = ACT_SILU
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=8)
    assert_same(session_for(layers).run(x), ref, "c2 with SiLU")


@pytest.mark.parametrize("scale", [1.0, 8.0, 1e3, 1e-30])
def test_gelu_epilogue_outside_the_common_range(gpu, oracle_lib, scale):
    """The tensor-core GEMM's GELU epilogue takes a short tanh path for arguments in
    [2^-25, 7.5) and recomputes the others with the general one: pre-activations scaled
    so that few, most or all values leave that range (and inf / NaN rows), bit-exact
    against the oracle."""
    layers, x = configs.c3_linear(512, 512, 384, seed=21)
    layers = [dict(l, weight=np.asarray(l["weight"]) * np.float32(scale)) if l["kind"] == oracle.LINEAR else l
              for l in layers]
    x = x.copy()
    x[7, 3] = np.inf
    x[9, 0] = np.nan
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=8)
    assert_same(session_for(layers).run(x), ref, f"gelu scale {scale}")
    x[7, 3] = 0.0
    x[9, 0] = 0.0
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=8)
    assert_same(session_for(layers).run(x), ref, f"gelu scale {scale}, finite")


@pytest.mark.parametrize("mkn", [(256, 512, 512), (200, 512, 264)])
@pytest.mark.parametrize("act", [None, 1, 2, 3, 4, 5, 6])
def test_tensor_core_gemm_every_activation(gpu, oracle_lib, act, mkn):
    """Every activation through the tcgen05 GEMM's two instance families: whole tiles
    (M a multiple of 128, N of 256, per-tensor scale, no absmax or accumulator dump:
    the branch-free instance) and ragged tiles, bit-exact against the oracle."""
    m, k, n = mkn
    rng = np.random.default_rng(m + n + (act or 0))
    w = (rng.standard_normal((k, n)) * 0.05).astype(np.float32)
    b = (rng.standard_normal(n) * 0.1).astype(np.float32)
    layers = [dict(kind=oracle.LINEAR, in_features=k, out_features=n, weight=w, bias=b)]
    if act is not None:
        layers.append(dict(kind=oracle.ACTIVATION, act=act, act_param=0.1))
    x = (rng.standard_normal((m, k)) * 2.0).astype(np.float32)
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=8)
    assert_same(session_for(layers).run(x), ref, f"act {act} linear {mkn}")


@pytest.mark.parametrize("mkn", [(8192, 1024, 2048), (10001, 512, 1700)])
def test_host_output_drained_in_chunks(gpu, oracle_lib, mkn):
    """A program ending in a tensor-core Linear whose host output is page-locked and at
    least 64 MiB: the GEMM runs in row chunks, each copied to the host as soon as it
    is written (whole chunks, and a ragged last chunk and row tile).  Same result as the
    single-launch path (pageable output) and the oracle, twice in a row on one session."""
    torch = gpu
    layers, x = configs.c3_linear(*mkn, seed=11)
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=8)
    sess = session_for(layers)
    plain = sess.run(x)
    assert_same(plain, ref, "pageable output")
    pinned = torch.empty(ref.shape, dtype=torch.float32, pin_memory=True)
    for i in range(2):
        pinned.fill_(float("nan"))
        y = sess.run(x, out=pinned.numpy())
        assert_same(y, ref, f"page-locked output, run {i}")
    drained = sess.last_npu_profile().kernel_launches
    sess.run(x)
    assert drained > sess.last_npu_profile().kernel_launches  # one GEMM launch per chunk


@pytest.mark.parametrize("mkn", [(1, 4, 32, 3), (64, 4, 32, 3), (65536, 4, 32, 3), (5000, 33, 17, 10),
                                 (3000, 64, 32, 32), (999, 16, 1, 1), (160000, 4, 32, 3)])
def test_two_narrow_linears_in_one_launch(gpu, oracle_lib, mkn):
    """A program of two narrow Linears runs as one cooperative kernel (input absmax, first
    Linear with the hidden row in registers, hidden absmax, second Linear; the last shape
    has more rows than resident threads and takes the op-by-op path): bit-exact against
    the oracle and the unfused session, with one kernel launch per run where it fits."""
    m, k, n1, n2 = mkn
    rng = np.random.default_rng(m + k + n1 + n2)
    w1 = (rng.standard_normal((k, n1)) * 0.3).astype(np.float32)
    b1 = (rng.standard_normal(n1) * 0.1).astype(np.float32)
    w2 = (rng.standard_normal((n1, n2)) * 0.3).astype(np.float32)
    b2 = (rng.standard_normal(n2) * 0.1).astype(np.float32)
    act = {(5000, 33, 17, 10): 4, (999, 16, 1, 1): 5, (3000, 64, 32, 32): 2}.get(mkn, 1)  # GELU, leaky, sigmoid
    layers = [dict(kind=oracle.LINEAR, in_features=k, out_features=n1, weight=w1, bias=b1),
              dict(kind=oracle.ACTIVATION, act=act, act_param=0.1),
              dict(kind=oracle.LINEAR, in_features=n1, out_features=n2, weight=w2, bias=b2)]
    x = rng.standard_normal((m, k)).astype(np.float32)
    ref, _, _ = oracle.Program(layers).execute(x, nthreads=8)
    sess = session_for(layers)
    assert_same(sess.run(x), ref, f"mlp {mkn}")
    assert_same(session_for(layers, flags=_native.RG_SESSION_NO_FUSION).run(x), ref, f"mlp {mkn} unfused")
    if m <= 148 * 4 * 256:
        assert sess.last_npu_profile().kernel_launches == 1
