"""Static calibration (extension): the device path against the oracle's restatement
(oracle.Program.calibrate / set_calibration, pinned by tests/test_npu_numpy.py).

A session calibrated on one batch freezes every Linear input's scale (two per
attention / SwiGLU block); later runs quantize with them, clamping values beyond the
calibrated range, and the producers that can write the Linear's i8 operand directly
(the fused CNN block, RMSNorm, the SwiGLU gate product).  Bar: the frozen scales,
the outputs (host and device buffers, captured-graph replays) and traced i8
activations / i32 accumulators equal the oracle's bit for bit."""
import numpy as np
import pytest

from oracle import configs, oracle
from rustgears_b200 import _native
from tests.helpers import assert_same, session_for

pytestmark = pytest.mark.gpu


def _batches(name):
    """(layers, calibration batch, run batch): the run batch has twice the range."""
    if name == "c2_256":
        layers, x = configs.c2_cnn(512)
        return layers, x[:256], (x[256:] * np.float32(2.0)).astype(np.float32)
    if name == "c2_6000":   # host input fed to the fused block in chunks
        layers, x = configs.c2_cnn(6000)
        return layers, x[:1000], (x * np.float32(1.5)).astype(np.float32)
    if name == "transformer_mini":
        layers, x = configs.transformer_mini(batch=4)
        return layers, x[:2], x[2:]
    layers, x = configs.CASES[name]()
    return layers, x, (x * np.float32(2.0)).astype(np.float32)


@pytest.mark.parametrize("name", ["c2_256", "c2_6000", "transformer_mini", "c1_mlp_64", "c3_linear_small", "acts_mlp",
                                  "resnet_mini", "affine_first", "integration"])
def test_calibrated_session_matches_oracle(gpu, oracle_lib, name):
    torch = gpu
    layers, xc, xr = _batches(name)
    prog = oracle.Program(layers)
    ref_scales = prog.calibrate(xc, nthreads=8)
    sess = session_for(layers)
    assert sess.calibration() is None and sess.calibration_targets() == ref_scales.size
    assert_same(sess.calibrate(xc), ref_scales, f"{name} scales")
    prog.set_calibration(ref_scales)
    ref, _, _ = prog.execute(xr, nthreads=8)
    assert_same(sess.run(xr), ref, f"{name} host run")
    xd = torch.from_numpy(np.ascontiguousarray(xr)).cuda()
    yd = torch.empty(ref.shape, dtype=torch.float32, device="cuda")
    for _ in range(3):  # direct run, graph capture, graph replay
        yd.fill_(float("nan"))
        sess.run_device(xd, yd)
        torch.cuda.synchronize()
        assert_same(yd.cpu().numpy(), ref, f"{name} device run")
    # back to the reference's dynamic scales
    sess.set_calibration(None)
    prog.set_calibration(None)
    ref_dyn, _, _ = prog.execute(xr, nthreads=8)
    assert_same(sess.run(xr), ref_dyn, f"{name} dynamic again")


def test_calibrated_trace_matches_oracle(gpu, oracle_lib):
    """Traced calibrated run: each Linear's scale is the frozen one and its i8 operand
    and i32 accumulators equal the oracle's."""
    layers, xc, xr = _batches("c1_mlp_64")
    prog = oracle.Program(layers)
    scales = prog.calibrate(xc)
    prog.set_calibration(scales)
    _, trace = prog.run_traced(xr)
    sess = session_for(layers)
    sess.set_calibration(scales)
    sess.set_trace(True)
    sess.run(xr)
    for i, t in enumerate(trace):
        if "aq" not in t:
            continue
        assert_same(sess.trace(i, _native.RG_TRACE_SCALES)[:1], np.atleast_1d(np.float32(t["a_scale"])), f"op{i}")
        assert_same(sess.trace(i, _native.RG_TRACE_AQ).reshape(t["aq"].shape), t["aq"], f"op{i} aq")
        assert_same(sess.trace(i, _native.RG_TRACE_ACC).reshape(t["acc"].shape), t["acc"], f"op{i} acc")


def test_calibrated_c2_launches_fewer_kernels(gpu, oracle_lib):
    """The fused block writes the Linear's i8 operand: no absmax and no quantize pass."""
    layers, x = configs.c2_cnn(4096)
    sess = session_for(layers)
    sess.run(x)
    dynamic = sess.last_npu_profile().kernel_launches
    sess.calibrate(x[:512])
    sess.run(x)
    assert sess.last_npu_profile().kernel_launches < dynamic


def test_calibration_errors(gpu):
    layers, x = configs.c1_mlp(8)
    sess = session_for(layers)
    n = sess.calibration_targets()
    assert n == 2
    with pytest.raises(_native.RgError):
        sess.set_calibration(np.ones(n + 1, np.float32))
    with pytest.raises(_native.RgError):
        sess.set_calibration(np.array([1.0, 0.0], np.float32))
    with pytest.raises(_native.RgError):
        sess.set_calibration(np.array([1.0, np.inf], np.float32))
    assert sess.calibration() is None
    from rustgears_b200 import ExecutionProvider, InferenceSession
    from tests.helpers import spec_from_dict
    fp16 = InferenceSession.from_layers([spec_from_dict(l) for l in layers], ExecutionProvider.npu_fp16())
    with pytest.raises(_native.RgError) as e:
        fp16.calibrate(x)
    assert e.value.status == _native.RG_ERR_UNSUPPORTED
