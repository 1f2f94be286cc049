"""rg_linear_i8_noalloc: the FusedLinear entry point that allocates no device
memory, for callers that cannot call cudaMalloc (a host whose own pool owns
all device memory, or a hot loop that must not block in the allocator).

It runs on a static scratch array inside the library, so its results must
equal the workspace-taking rg_linear_i8 exactly (the bit-exact bar every
parity test here uses), on consecutive calls that reuse that scratch.  This
file is collected last so that a failure here does not stop the other tests.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import configs, oracle
from rustgears_b200 import _native

pytestmark = pytest.mark.gpu


def _p(t):
    return C.c_void_p(t.data_ptr())


def _case(torch, m, k, n, seed):
    layers, x = configs.c3_linear(m, k, n, seed=seed)
    op = oracle.Program(layers).ops[0]
    ld = (k + 15) // 16 * 16
    w = np.zeros((n, ld), np.int8)
    w[:, :k] = op.wq.reshape(n, k)
    return (torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), torch.from_numpy(op.bias).cuda(),
            op.w_scale, op.act, ld)


def test_noalloc_matches_workspace_entry_point(gpu):
    torch = gpu
    L = _native.lib()
    m, k, n = 300, 200, 90
    # two calls in a row on different inputs: the second must not see the first's scratch
    for seed in (1, 2):
        x, w, b, ws_scale, act, ld = _case(torch, m, k, n, seed)
        ws = torch.empty(L.rg_linear_i8_workspace_size(m, ld), dtype=torch.uint8, device="cuda")
        ref = torch.empty((m, n), dtype=torch.float32, device="cuda")
        _native.check(L.rg_linear_i8(_p(x), m, k, _p(w), n, ld, C.c_float(ws_scale), _p(b), act, C.c_float(0.0),
                                     _p(ref), _p(ws), None))
        out = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        _native.check(L.rg_linear_i8_noalloc(_p(x), m, k, _p(w), n, ld, C.c_float(ws_scale), _p(b), act,
                                             C.c_float(0.0), _p(out), None))
        torch.cuda.synchronize()
        assert torch.equal(out, ref), f"call with seed {seed} differs"


def test_noalloc_rejects_oversized_calls(gpu):
    L = _native.lib()
    limit = 16 << 20
    st = L.rg_linear_i8_noalloc(None, limit // 64 + 1, 64, None, 8, 64, C.c_float(1.0), None, 0, C.c_float(0.0),
                                None, None)
    assert st == _native.RG_ERR_INVALID_ARG
    assert "exceeds" in _native.last_error()
