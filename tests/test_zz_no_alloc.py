"""rg_linear_i8_noalloc: the FusedLinear entry point that allocates no device
memory, for callers that cannot call cudaMalloc (a host whose own pool owns
all device memory, or a hot loop that must not block in the allocator).

It runs on a static scratch array inside the library.  Its results must equal
the oracle's FusedLinear (src/inference/npu.rs:307-318, the activation scale
over the whole input) and the workspace-taking rg_linear_i8 exactly, on calls
in a row that reuse that scratch, through every GEMM the library dispatches to
(tcgen05, narrow N <= 32, SIMT), and at the size limit itself.  This file is
collected last so that a failure here does not stop the other tests.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import configs, oracle
from rustgears_b200 import _native
from tests.helpers import assert_same

pytestmark = pytest.mark.gpu
LIMIT = 16 << 20   # RG_LINEAR_NOALLOC_MAX_BYTES


def _p(t):
    return C.c_void_p(t.data_ptr())


def _case(torch, m, k, n, seed):
    layers, x = configs.c3_linear(m, k, n, seed=seed)
    prog = oracle.Program(layers)
    ref, _, _ = prog.execute(x, nthreads=8)
    op = prog.ops[0]
    ld = (k + 15) // 16 * 16
    w = np.zeros((n, ld), np.int8)
    w[:, :k] = op.wq.reshape(n, k)
    return (torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), torch.from_numpy(op.bias).cuda(),
            op.w_scale, op.act, ld, ref)


def _both(torch, m, k, n, seed):
    """(noalloc output, rg_linear_i8 output, oracle output) for one case."""
    L = _native.lib()
    x, w, b, ws_scale, act, ld, ref = _case(torch, m, k, n, seed)
    ws = torch.empty(L.rg_linear_i8_workspace_size(m, ld), dtype=torch.uint8, device="cuda")
    with_ws = torch.empty((m, n), dtype=torch.float32, device="cuda")
    _native.check(L.rg_linear_i8(_p(x), m, k, _p(w), n, ld, C.c_float(ws_scale), _p(b), act, C.c_float(0.0),
                                 _p(with_ws), _p(ws), None))
    out = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    _native.check(L.rg_linear_i8_noalloc(_p(x), m, k, _p(w), n, ld, C.c_float(ws_scale), _p(b), act,
                                         C.c_float(0.0), _p(out), None))
    torch.cuda.synchronize()
    return out.cpu().numpy(), with_ws.cpu().numpy(), ref


@pytest.mark.parametrize("mkn", [(300, 200, 90),      # tcgen05 GEMM
                                 (300, 64, 10),       # narrow (N <= 32)
                                 (77, 100, 48)])      # SIMT (m * n * k < 2^22)
def test_noalloc_matches_oracle_and_workspace_entry_point(gpu, mkn):
    torch = gpu
    m, k, n = mkn
    # two calls in a row on different inputs: the second must not see the first's scratch
    for seed in (1, 2):
        out, with_ws, ref = _both(torch, m, k, n, seed)
        assert_same(out, ref, f"noalloc vs oracle {mkn} seed {seed}")
        assert_same(out, with_ws, f"noalloc vs rg_linear_i8 {mkn} seed {seed}")


def test_noalloc_at_the_size_limit(gpu):
    """m * ld exactly RG_LINEAR_NOALLOC_MAX_BYTES: the absmax and scale sit in the
    array's last 256 bytes."""
    torch = gpu
    m, k, n = LIMIT // 256, 256, 64
    for seed in (3, 4):
        out, with_ws, ref = _both(torch, m, k, n, seed)
        assert_same(out, ref, f"noalloc at the limit, seed {seed}")
        assert_same(out, with_ws, f"noalloc vs rg_linear_i8 at the limit, seed {seed}")


def test_noalloc_rejects_oversized_calls(gpu):
    L = _native.lib()
    st = L.rg_linear_i8_noalloc(None, LIMIT // 64 + 1, 64, None, 8, 64, C.c_float(1.0), None, 0, C.c_float(0.0),
                                None, None)
    assert st == _native.RG_ERR_INVALID_ARG
    assert "exceeds" in _native.last_error()
    # a product m * ld that would wrap a signed 64-bit integer is rejected, not wrapped
    st = L.rg_linear_i8_noalloc(None, 1 << 62, 64, None, 8, 64, C.c_float(1.0), None, 0, C.c_float(0.0),
                                None, None)
    assert st == _native.RG_ERR_INVALID_ARG
    assert "exceeds" in _native.last_error()
