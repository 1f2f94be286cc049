"""Batch sharding across the GPUs of one node (one process per GPU).

Each rank holds a full copy of the quantized weights and runs a contiguous
slice of the batch.  Conv2d/pool/activation are per sample; every Linear
quantizes with the absmax of the WHOLE batch (src/inference/npu.rs:312), so
the library max-all-reduces that one f32 over NCCL before quantizing, which
keeps every rank's result bit-identical to a single device's.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native


def shard_range(batch: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous split of ``batch`` rows; the first ``batch % world`` ranks take one extra."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    base, rem = divmod(batch, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def new_unique_id() -> bytes:
    buf = (C.c_uint8 * 128)()
    _native.check(_native.lib().rg_nccl_unique_id(buf))
    return bytes(buf)


def exchange_unique_id(rank: int, make_id=new_unique_id, group=None) -> bytes:
    """Rank 0 creates the communicator id; every rank receives it through the
    already-initialised torch.distributed process group (gloo or nccl)."""
    import torch.distributed as dist
    obj = [make_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    uid = obj[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != 128:
        raise RuntimeError("bad communicator id received")
    return bytes(uid)


def attach(session, rank: int, world: int, uid: bytes) -> None:
    """Join ``session`` to the NCCL communicator ``uid`` as ``rank`` of ``world``."""
    buf = (C.c_uint8 * 128).from_buffer_copy(uid)
    _native.check(_native.lib().rg_session_attach_comm(session.handle, buf, rank, world))


def allgather(session, send, recv) -> None:
    """All-gather equal-sized float32 CUDA tensors over the session's communicator."""
    import torch
    st = torch.cuda.current_stream(send.device).cuda_stream
    _native.check(_native.lib().rg_session_allgather(session.handle, C.c_void_p(send.data_ptr()),
                                                     C.c_void_p(recv.data_ptr()), send.numel(),
                                                     C.c_void_p(st)))


def gather_rows(parts) -> np.ndarray:
    """Host-side concatenation of per-rank outputs in rank order."""
    return np.concatenate([np.asarray(p) for p in parts], axis=0)
