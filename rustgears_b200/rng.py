"""The reference's global generator (src/rng.rs): SplitMix64 with f32 draws,
``manual_seed`` and the tensor initialisers, run by librg_npu's C++ code so
that weights and inputs are bit-identical to the reference's."""
from __future__ import annotations

import ctypes as C
import threading

import numpy as np

from . import _native


class Rng:
    """One SplitMix64 stream (rng.rs:10-58)."""

    def __init__(self, seed: int):
        self._s = _native.RngC()
        _native.lib().rg_rng_seed(C.byref(self._s), C.c_uint64(seed & (2**64 - 1)))

    def next_u64(self) -> int:
        return _native.lib().rg_rng_next_u64(C.byref(self._s))

    def uniform_tensor(self, shape, lo: float, hi: float) -> np.ndarray:
        out = np.empty(int(np.prod(shape)), np.float32)
        _native.lib().rg_rng_fill_uniform(C.byref(self._s), out.ctypes.data_as(C.POINTER(C.c_float)),
                                          out.size, C.c_float(lo), C.c_float(hi))
        return out.reshape(shape)

    def randn(self, shape, std: float = 1.0) -> np.ndarray:
        out = np.empty(int(np.prod(shape)), np.float32)
        _native.lib().rg_rng_fill_normal(C.byref(self._s), out.ctypes.data_as(C.POINTER(C.c_float)),
                                         out.size, C.c_float(std))
        return out.reshape(shape)

    def advance(self, draws: int) -> None:
        """Skip ``draws`` 64-bit draws (SplitMix64 is a counter: state += draws * G)."""
        self._s.state = (self._s.state + draws * 0x9E3779B97F4A7C15) % 2**64

    def below(self, shape, n: int) -> np.ndarray:
        out = np.empty(int(np.prod(shape)), np.int64)
        _native.lib().rg_rng_fill_below(C.byref(self._s), out.ctypes.data_as(C.POINTER(C.c_int64)),
                                        out.size, C.c_uint64(n))
        return out.reshape(shape)


_lock = threading.Lock()
_global = None


def _g() -> Rng:
    global _global
    if _global is None:
        _global = Rng(0x5EED)  # default seed (rng.rs:66)
    return _global


def manual_seed(seed: int) -> None:  # rng.rs:71-73
    global _global
    with _lock:
        _global = Rng(seed)


def randn(shape) -> np.ndarray:  # Tensor::randn (tensor/mod.rs:116-119)
    with _lock:
        return _g().randn(shape)


def rand(shape) -> np.ndarray:  # Tensor::rand (tensor/mod.rs:122-125)
    with _lock:
        return _g().uniform_tensor(shape, 0.0, 1.0)


def uniform(shape, lo: float, hi: float) -> np.ndarray:  # Tensor::uniform (tensor/mod.rs:128-131)
    with _lock:
        return _g().uniform_tensor(shape, lo, hi)


def normal_init(shape, std: float) -> np.ndarray:  # init::normal (nn/init.rs:18-20)
    with _lock:
        return _g().randn(shape, std)


def kaiming_uniform(shape, fan_in: int) -> np.ndarray:  # nn/init.rs:6-9
    b = _native.lib().rg_kaiming_bound(fan_in)
    return uniform(shape, -b, b)


def bias_uniform(shape, fan_in: int) -> np.ndarray:  # nn/init.rs:23-26
    b = _native.lib().rg_bias_bound(fan_in)
    return uniform(shape, -b, b)


def advance(draws: int) -> None:
    """Skip ``draws`` draws of the global generator (a batch shard starts mid-stream)."""
    with _lock:
        _g().advance(draws)


def below(shape, n: int) -> np.ndarray:  # Rng::below (rng.rs:47-49)
    with _lock:
        return _g().below(shape, n)
