"""Kernel-level C-ABI entry points on device buffers vs the oracle."""
import ctypes as C

import numpy as np
import pytest

from oracle import configs, oracle
from rustgears_b200 import _native
from tests.helpers import assert_same

pytestmark = pytest.mark.gpu


def ptr(t):
    return C.c_void_p(t.data_ptr())


def test_absmax_and_quantize(gpu, oracle_lib):
    torch = gpu
    L = _native.lib()
    rng = np.random.default_rng(0)
    for rows, k in [(1, 1), (3, 5), (1000, 4096), (777, 130)]:
        x = (rng.standard_normal((rows, k)) * 3).astype(np.float32)
        x.reshape(-1)[rng.integers(0, x.size)] = np.nan
        xd = torch.from_numpy(x).cuda()
        amax = torch.zeros(1, dtype=torch.float32, device="cuda")
        _native.check(L.rg_absmax_f32(ptr(xd), x.size, ptr(amax), None))
        ld = (k + 15) // 16 * 16
        q = torch.full((rows, ld), 99, dtype=torch.int8, device="cuda")
        sc = torch.zeros(1, dtype=torch.float32, device="cuda")
        _native.check(L.rg_quantize_f32_i8(ptr(xd), rows, k, ld, ptr(amax), ptr(q), ptr(sc), None))
        torch.cuda.synchronize()
        qref, sref = oracle.quantize(x)
        assert sc.item() == float(sref)
        qq = q.cpu().numpy()
        assert_same(qq[:, :k], qref, "q")
        assert (qq[:, k:] == 0).all()


def test_gemm_fused_with_acc(gpu, oracle_lib):
    torch = gpu
    L = _native.lib()
    layers, x = configs.c3_linear(200, 300, 90, seed=3)
    prog = oracle.Program(layers)
    ref, tr = prog.run_traced(x)
    op = prog.ops[0]
    m, k, n, ld = 200, 300, 90, 304
    a = np.zeros((m, ld), np.int8); a[:, :k] = tr[0]["aq"]
    w = np.zeros((n, ld), np.int8); w[:, :k] = op.wq.reshape(n, k)
    ad, wd = torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda()
    sa = torch.tensor([float(tr[0]["a_scale"])], dtype=torch.float32, device="cuda")
    bias = torch.from_numpy(op.bias).cuda()
    out = torch.empty((m, n), dtype=torch.float32, device="cuda")
    acc = torch.empty((m, n), dtype=torch.int32, device="cuda")
    amax = torch.zeros(1, dtype=torch.float32, device="cuda")
    _native.check(L.rg_gemm_i8_fused(ptr(ad), ptr(wd), m, n, ld, ptr(sa), C.c_float(op.w_scale), ptr(bias),
                                     op.act, C.c_float(op.act_param), ptr(out), ptr(acc), ptr(amax), None))
    torch.cuda.synchronize()
    assert_same(acc.cpu().numpy(), tr[0]["acc"], "acc")
    assert_same(out.cpu().numpy(), ref, "out")
    assert amax.item() == float(np.max(np.abs(ref)))
    # the one-call FusedLinear entry point with a caller-owned workspace
    xd = torch.from_numpy(x).cuda()
    ws = torch.empty(L.rg_linear_i8_workspace_size(m, ld), dtype=torch.uint8, device="cuda")
    out2 = torch.empty((m, n), dtype=torch.float32, device="cuda")
    _native.check(L.rg_linear_i8(ptr(xd), m, k, ptr(wd), n, ld, C.c_float(op.w_scale), ptr(bias), op.act,
                                 C.c_float(op.act_param), ptr(out2), ptr(ws), None))
    torch.cuda.synchronize()
    assert_same(out2.cpu().numpy(), ref, "linear_i8")


def test_maxpool_softmax_activation(gpu, oracle_lib):
    torch = gpu
    L = _native.lib()
    rng = np.random.default_rng(5)
    x = rng.standard_normal((3, 5, 11, 9)).astype(np.float32)
    x[0, 1, 2, 3] = np.nan
    x[1, 2, :4, :4] = -np.inf
    for k, s in [(2, 2), (3, 2), (3, 1), (11, 1)]:
        if k > 9:
            continue
        ref = oracle.maxpool2d(x, k, s)
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty(ref.shape, dtype=torch.float32, device="cuda")
        _native.check(L.rg_maxpool2d_f32(ptr(xd), 3, 5, 11, 9, k, s, ptr(yd), None))
        torch.cuda.synchronize()
        assert_same(yd.cpu().numpy(), ref, f"maxpool k{k}s{s}")
    z = (rng.standard_normal((37, 19)) * 5).astype(np.float32)
    zd = torch.from_numpy(z).cuda()
    yd = torch.empty_like(zd)
    _native.check(L.rg_softmax_f32(ptr(zd), 37, 19, ptr(yd), None))
    torch.cuda.synchronize()
    assert_same(yd.cpu().numpy(), oracle.softmax(z), "softmax")
    for act, p in [(0, 0.0), (1, 0.0), (2, 0.0), (3, 0.0), (4, 0.0), (5, 0.01), (5, 0.2)]:
        _native.check(L.rg_activation_f32(ptr(zd), z.size, act, C.c_float(p), ptr(yd), None))
        torch.cuda.synchronize()
        assert_same(yd.cpu().numpy(), oracle.activation(z, act, p), f"act {act}")


@pytest.mark.parametrize("b,t,heads,dh", [(2, 512, 2, 64), (1, 136, 3, 64), (2, 13, 4, 12), (1, 520, 1, 64),
                                          (3, 8, 2, 64)])
def test_attention_core(gpu, oracle_lib, b, t, heads, dh):
    """rg_attention_f32 against the oracle's attention core (both attention kernels)."""
    torch = gpu
    L = _native.lib()
    d = heads * dh
    qkv = (np.random.default_rng(t + dh).standard_normal((b * t, 3 * d)) * 2).astype(np.float32)
    ref = oracle.attention_core(qkv, b, t, heads, dh)
    xd = torch.from_numpy(qkv).cuda()
    yd = torch.empty((b * t, d), dtype=torch.float32, device="cuda")
    _native.check(L.rg_attention_f32(ptr(xd), 3 * d, b, t, heads, dh, ptr(yd), d, None))
    torch.cuda.synchronize()
    assert_same(yd.cpu().numpy(), ref, f"attention b{b} t{t} h{heads} dh{dh}")
