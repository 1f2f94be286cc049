"""Device GELU / Sigmoid / Tanh against glibc (the reference's libm) on a
strided sweep of all 2^32 float bit patterns plus edge values: bit-exact."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle
from rustgears_b200 import _native
from tests.helpers import assert_same

pytestmark = pytest.mark.gpu


def sweep(stride=251):
    bits = np.arange(0, 2**32, stride, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    edge = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-38, -1e-38, 1.0, -1.0, 22.0, -22.0,
                     0.5493061, 88.72, -88.72, 3.4e38, -3.4e38], np.float32)
    return np.concatenate([x, edge])


@pytest.mark.parametrize("act,param", [(4, 0.0), (2, 0.0), (3, 0.0), (5, 0.01), (6, 0.0)])
def test_activation_sweep(gpu, oracle_lib, act, param):
    torch = gpu
    x = sweep()
    ref = oracle.activation(x, act, param)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty_like(xd)
    _native.check(_native.lib().rg_activation_f32(C.c_void_p(xd.data_ptr()), x.size, act, C.c_float(param),
                                                  C.c_void_p(yd.data_ptr()), None))
    torch.cuda.synchronize()
    assert_same(yd.cpu().numpy(), ref, f"act {act}")


def test_fast_paths_are_exact_on_every_input(gpu):
    """tanh, GELU, the quantization scale and its reciprocal divide with Markstein's
    reciprocal-and-correction sequence and quantization rounds by a biased add and
    truncation; the device self-test compares each with the IEEE division / roundf
    on all 2^32 f32 inputs; and the GEMM epilogue's common-range tanh (and GELU
    through it) equals the general restatement on every input it is used for."""
    counts = (C.c_uint64 * 6)()
    _native.check(_native.lib().rg_selftest_fast_paths(counts))
    assert list(counts) == [0, 0, 0, 0, 0, 0]
