""".rtim portable inference format (src/save.rs:165-279).

Little-endian: magic ``RTIM``, u32 layer count, then per layer a u32 tag
(1 Linear, 2 Conv2d, 3 ChannelAffine, 4 MaxPool2d, 5 Flatten, 6 Activation,
7 Softmax) followed by its u32 fields and u32-length-prefixed f32 vectors.
Writes are atomic (temporary file + rename, as ``write_atomic``, save.rs:21-32).
"""
from __future__ import annotations

import os
import struct
import tempfile

import numpy as np

from .spec import (ACTIVATION, CHANNEL_AFFINE, CONV2D, FLATTEN, LINEAR, MAXPOOL2D, SOFTMAX, Activation,
                   ActivationLayer, ChannelAffine, Conv2d, Flatten, Linear, MaxPool2d, Softmax)

MAGIC = b"RTIM"


def _vec(v) -> bytes:
    a = np.ascontiguousarray(v, dtype="<f4").reshape(-1)
    return struct.pack("<I", a.size) + a.tobytes()


def encode_layers(layers) -> bytes:
    out = [MAGIC, struct.pack("<I", len(layers))]
    for l in layers:
        k = l.kind
        if k == LINEAR:
            out += [struct.pack("<III", 1, l.in_features, l.out_features), _vec(l.weight), _vec(l.bias)]
        elif k == CONV2D:
            out += [struct.pack("<IIIIII", 2, l.in_channels, l.out_channels, l.kernel, l.stride, l.padding),
                    _vec(l.weight), _vec(l.bias)]
        elif k == CHANNEL_AFFINE:
            out += [struct.pack("<I", 3), _vec(l.scale), _vec(l.shift)]
        elif k == MAXPOOL2D:
            out += [struct.pack("<III", 4, l.kernel, l.stride)]
        elif k == FLATTEN:
            out += [struct.pack("<I", 5)]
        elif k == ACTIVATION:
            if l.act.code > 5:
                raise RtimError(f"activation {l.act} has no .rtim tag (save.rs:206-214)")
            out += [struct.pack("<II", 6, l.act.code), struct.pack("<f", l.act.param)]
        elif k == SOFTMAX:
            out += [struct.pack("<I", 7)]
        else:
            raise ValueError(f"unknown layer kind {k}")
    return b"".join(out)


def write_atomic(path, data: bytes) -> None:
    path = os.fspath(path)
    d = os.path.dirname(os.path.abspath(path))
    fd, tmp = tempfile.mkstemp(dir=d, prefix=".rtim-")
    try:
        with os.fdopen(fd, "wb") as f:
            f.write(data)
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, path)
    except BaseException:
        try:
            os.unlink(tmp)
        except OSError:
            pass
        raise


def save_layers(layers, path) -> None:  # save.rs:172-224
    write_atomic(path, encode_layers(layers))


def save_inference_model(module, path) -> None:  # save.rs:165-169
    module.eval()
    save_layers(module.export(), path)


class RtimError(IOError):
    pass


def decode_layers(buf: bytes):
    pos = 0

    def take(n):
        nonlocal pos
        if pos + n > len(buf):
            raise RtimError("truncated RTIM file")
        b = buf[pos:pos + n]
        pos += n
        return b

    def u32():
        return struct.unpack("<I", take(4))[0]

    def f32():
        return struct.unpack("<f", take(4))[0]

    def vec():
        n = u32()
        return np.frombuffer(take(4 * n), dtype="<f4").astype(np.float32)

    if take(4) != MAGIC:
        raise RtimError("invalid RTIM model header")
    count = u32()
    out = []
    for _ in range(count):
        tag = u32()
        if tag == 1:
            i, o = u32(), u32()
            out.append(Linear(i, o, vec(), vec()))
        elif tag == 2:
            ic, oc, k, s, p = u32(), u32(), u32(), u32(), u32()
            out.append(Conv2d(ic, oc, k, s, p, vec(), vec()))
        elif tag == 3:
            out.append(ChannelAffine(vec(), vec()))
        elif tag == 4:
            out.append(MaxPool2d(u32(), u32()))
        elif tag == 5:
            out.append(Flatten())
        elif tag == 6:
            code, p = u32(), f32()
            if code > 5:
                raise RtimError(f"unknown activation tag {code}")
            out.append(ActivationLayer(Activation(code, p)))
        elif tag == 7:
            out.append(Softmax())
        else:
            raise RtimError(f"unknown layer tag {tag}")
    return out


def load_inference_layers(path):  # save.rs:227-279
    with open(path, "rb") as f:
        return decode_layers(f.read())
