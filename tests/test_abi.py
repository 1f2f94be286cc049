"""The C ABI: every symbol include/rg_npu.h declares is exported; no CPU fallback."""
import ctypes as C
import os
import re

import numpy as np

from rustgears_b200 import _native

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "rg_npu.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\**\s*(rg_[a-z_0-9]+)\s*\(", src, flags=re.M))
    return names


def test_header_declares_entry_points():
    names = declared_functions()
    assert {"rg_session_create", "rg_session_run", "rg_session_last_profile",
            "rg_session_compilation_report", "rg_gemm_i8_fused", "rg_last_error"} <= names
    assert len(names) >= 30


def test_library_exports_every_declared_symbol():
    L = _native.lib()
    for name in sorted(declared_functions()):
        assert hasattr(L, name), f"{name} declared in rg_npu.h but not exported"


def test_bindings_cover_header():
    assert declared_functions() == set(_native.SIGNATURES)


def test_version_and_errors():
    L = _native.lib()
    assert L.rg_version().decode().startswith("rustgears-b200")
    # invalid arguments are rejected before any device work
    assert L.rg_session_create(None, 1, None, None) == _native.RG_ERR_INVALID_ARG
    assert "null" in _native.last_error()


def test_no_cpu_fallback_without_gpu():
    L = _native.lib()
    if L.rg_device_count() > 0:
        return  # on a GPU box the session tests cover the device path
    spec = (_native.LayerSpecC * 1)()
    spec[0].kind = 5  # Flatten
    h = C.c_void_p()
    st = L.rg_session_create(spec, 1, None, C.byref(h))
    assert st == _native.RG_ERR_NO_DEVICE
    assert "no CPU fallback" in _native.last_error()


def test_rng_abi_values():
    L = _native.lib()
    r = _native.RngC()
    L.rg_rng_seed(C.byref(r), 0x9E3779B97F4A7C15)
    assert L.rg_rng_next_u64(C.byref(r)) == 0xE220A8397B1DCDAF
    assert np.float32(L.rg_kaiming_bound(4)) == np.sqrt(np.float32(6.0) / np.float32(4.0))


def test_error_words_map_to_statuses():
    """The mapping every run and kernel-level call applies to its device error words,
    driven from the host with forced words (no device needed)."""
    L = _native.lib()
    words = (C.c_int32 * 2)
    assert L.rg_status_from_error_words(words(0, 0)) == _native.RG_OK
    assert L.rg_status_from_error_words(words(1, 0)) == _native.RG_ERR_TIMEOUT
    assert "bounded wait" in _native.last_error()
    assert L.rg_status_from_error_words(words(1, 1)) == _native.RG_ERR_TIMEOUT
    assert L.rg_status_from_error_words(words(0, 1)) == _native.RG_ERR_INVALID_ARG
    assert "vocabulary" in _native.last_error()
    assert L.rg_status_from_error_words(None) == _native.RG_ERR_INVALID_ARG
