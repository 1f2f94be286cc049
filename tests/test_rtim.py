""".rtim format (src/save.rs:165-279): Python writer/reader and the library's own reader."""
import ctypes as C
import os
import struct

import numpy as np
import pytest

from rustgears_b200 import _native, configs, nn, rtim
from rustgears_b200.spec import Activation, ActivationLayer, Flatten, Softmax


def test_roundtrip(tmp_path):
    model, _ = configs.c2_cnn(2)
    layers = model.export() + [ActivationLayer(Activation.leaky_relu(0.125)), Softmax()]
    p = tmp_path / "m.rtim"
    rtim.save_layers(layers, p)
    back = rtim.load_inference_layers(p)
    assert len(back) == len(layers)
    for a, b in zip(layers, back):
        assert a.kind == b.kind
        for f in ("weight", "bias", "scale", "shift"):
            if hasattr(a, f):
                assert np.array_equal(getattr(a, f), getattr(b, f))
        for f in ("in_features", "out_features", "in_channels", "out_channels", "kernel", "stride", "padding"):
            if hasattr(a, f):
                assert getattr(a, f) == getattr(b, f)
        if hasattr(a, "act"):
            assert a.act == b.act


def test_layout_bytes(tmp_path):
    layers = [Flatten(), ActivationLayer(Activation.RELU)]
    data = rtim.encode_layers(layers)
    assert data == b"RTIM" + struct.pack("<IIIIf", 2, 5, 6, 1, 0.0)


def test_errors(tmp_path):
    p = tmp_path / "bad.rtim"
    p.write_bytes(b"XXXX" + struct.pack("<I", 0))
    with pytest.raises(IOError, match="invalid RTIM model header"):
        rtim.load_inference_layers(p)
    p.write_bytes(b"RTIM" + struct.pack("<II", 1, 9))
    with pytest.raises(IOError, match="unknown layer tag 9"):
        rtim.load_inference_layers(p)
    p.write_bytes(b"RTIM" + struct.pack("<III", 1, 6, 8) + struct.pack("<f", 0))
    with pytest.raises(IOError, match="unknown activation tag 8"):
        rtim.load_inference_layers(p)


def test_native_reader_errors(tmp_path):
    # The library parses .rtim itself before touching a device.
    L = _native.lib()
    opts = _native.SessionOptions(0, 0, 0, 0)
    h = C.c_void_p()
    p = tmp_path / "bad.rtim"
    p.write_bytes(b"NOPE")
    assert L.rg_session_create_from_rtim(str(p).encode(), C.byref(opts), C.byref(h)) == _native.RG_ERR_IO
    assert "invalid RTIM model header" in _native.last_error()
    p.write_bytes(b"RTIM" + struct.pack("<II", 1, 42))
    assert L.rg_session_create_from_rtim(str(p).encode(), C.byref(opts), C.byref(h)) == _native.RG_ERR_IO
    assert "unknown layer tag 42" in _native.last_error()
    p.write_bytes(b"RTIM" + struct.pack("<IIII", 1, 1, 4, 3))
    assert L.rg_session_create_from_rtim(str(p).encode(), C.byref(opts), C.byref(h)) == _native.RG_ERR_IO
    assert "truncated" in _native.last_error()


def test_atomic_write_keeps_original_on_failure(tmp_path, monkeypatch):
    # save.rs:285-302: an injected write failure leaves the old file intact and no temp file.
    p = tmp_path / "m.rtim"
    p.write_bytes(b"original")

    def boom(*a, **k):
        raise OSError("injected write failure")

    monkeypatch.setattr(os, "fsync", boom)
    with pytest.raises(OSError, match="injected"):
        rtim.save_layers([Flatten()], p)
    assert p.read_bytes() == b"original"
    assert os.listdir(tmp_path) == ["m.rtim"]
    monkeypatch.undo()
    rtim.save_layers([Flatten()], p)
    assert rtim.load_inference_layers(p)[0].kind == 5
