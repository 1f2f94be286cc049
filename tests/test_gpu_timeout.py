"""A tensor-core kernel whose bounded wait runs out reports RG_ERR_TIMEOUT to the call
it belongs to, and the context stays usable.

The wait is made to run out by the library's test hook rg_debug_set_tc_wait: the
GEMM's producer issues no operand loads, so the barrier the MMA issuer waits on is
one that nothing arrives on, and every wait is bounded by 1 ms.  No fault, trap or
endless loop is involved: the kernel's roles leave their loops, drain, free TMEM,
set the call's error word and return.  After the hook is cleared the same calls are
bit-exact against the oracle again.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import configs, oracle
from rustgears_b200 import _native
from tests.helpers import assert_same, session_for

pytestmark = pytest.mark.gpu
WAIT_NS = 1_000_000


def _p(t):
    return C.c_void_p(t.data_ptr())


@pytest.fixture
def starve():
    L = _native.lib()
    yield lambda on: L.rg_debug_set_tc_wait(WAIT_NS if on else 0, 1 if on else 0)
    L.rg_debug_set_tc_wait(0, 0)


def _operands(torch, m, k, n, seed):
    layers, x = configs.c3_linear(m, k, n, seed=seed)
    prog = oracle.Program(layers)
    ref, trace = prog.run_traced(x)
    ld = (k + 15) // 16 * 16
    a = np.zeros((m, ld), np.int8)
    a[:, :k] = np.asarray(trace[0]["aq"]).reshape(m, k)
    w = np.zeros((n, ld), np.int8)
    w[:, :k] = prog.ops[0].wq.reshape(n, k)
    sa = np.array([trace[0]["a_scale"]], np.float32)
    dev = lambda v: torch.from_numpy(np.ascontiguousarray(v)).cuda()
    return dict(a=dev(a), w=dev(w), sa=dev(sa), bias=dev(prog.ops[0].bias), ws=prog.ops[0].w_scale,
                act=prog.ops[0].act, ld=ld, m=m, n=n, ref=ref, layers=layers, x=x)


def _gemm(torch, o):
    out = torch.full((o["m"], o["n"]), float("nan"), dtype=torch.float32, device="cuda")
    st = _native.lib().rg_gemm_i8_fused(_p(o["a"]), _p(o["w"]), o["m"], o["n"], o["ld"], _p(o["sa"]),
                                       C.c_float(o["ws"]), _p(o["bias"]), o["act"], C.c_float(0.0), _p(out),
                                       None, None, None)
    return st, out


def test_gemm_timeout_is_reported_then_recovers(gpu, starve):
    torch = gpu
    o = _operands(torch, 256, 512, 384, 5)    # m*n*k >= 2^22: the tcgen05 kernel
    st, out = _gemm(torch, o)
    assert st == _native.RG_OK
    assert_same(out.cpu().numpy(), o["ref"], "before")
    starve(True)
    st, _ = _gemm(torch, o)
    assert st == _native.RG_ERR_TIMEOUT, _native.last_error()
    assert "bounded wait" in _native.last_error()
    starve(False)
    st, out = _gemm(torch, o)
    assert st == _native.RG_OK, _native.last_error()
    assert_same(out.cpu().numpy(), o["ref"], "after")


def test_session_timeout_is_its_own(gpu, starve):
    """The run that timed out reports it; another session's run does not inherit it,
    and the session's next run (its error word cleared) is bit-exact."""
    layers, x = configs.c3_linear(300, 512, 384, seed=9)
    ref, _, _ = oracle.Program(layers).execute(x)
    a = session_for(layers, flags=_native.RG_SESSION_NO_GRAPH)
    b = session_for(layers, flags=_native.RG_SESSION_NO_GRAPH)
    assert_same(b.run(x), ref, "b before")
    starve(True)
    with pytest.raises(_native.RgError) as e:
        a.run(x)
    assert e.value.status == _native.RG_ERR_TIMEOUT
    starve(False)
    assert_same(b.run(x), ref, "b after a's timeout")
    assert_same(a.run(x), ref, "a after its timeout")


def test_noalloc_timeout_is_reported(gpu, starve):
    torch = gpu
    layers, x = configs.c3_linear(256, 512, 384, seed=6)
    prog = oracle.Program(layers)
    ref, _, _ = prog.execute(x)
    op = prog.ops[0]
    ld = 512
    w = torch.from_numpy(op.wq.reshape(384, 512).copy()).cuda()
    b = torch.from_numpy(op.bias).cuda()
    xd = torch.from_numpy(x).cuda()
    out = torch.empty((256, 384), dtype=torch.float32, device="cuda")
    L = _native.lib()
    call = lambda: L.rg_linear_i8_noalloc(_p(xd), 256, 512, _p(w), 384, ld, C.c_float(op.w_scale), _p(b), op.act,
                                          C.c_float(0.0), _p(out), None)
    starve(True)
    assert call() == _native.RG_ERR_TIMEOUT
    starve(False)
    assert call() == _native.RG_OK
    torch.cuda.synchronize()
    assert_same(out.cpu().numpy(), ref, "noalloc after timeout")
