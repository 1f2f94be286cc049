"""Batch sharding over 2 GPUs (one process per GPU, NCCL): every Linear's absmax (each
inner projection of attention and SwiGLU included) is max-all-reduced, so the
gathered output equals one device's output bit for bit.
Skipped when fewer than 2 GPUs are visible."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, case, out_dir):
    import datetime

    import torch
    import torch.distributed as tdist

    from oracle import configs
    from rustgears_b200 import dist
    from tests.helpers import session_for

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    tdist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        layers, x = configs.CASES[case]()
        sess = session_for(layers, device=rank)
        uid = dist.exchange_unique_id(rank)
        dist.attach(sess, rank, world, uid)
        a, b = dist.shard_range(x.shape[0], rank, world)
        xd = torch.from_numpy(np.ascontiguousarray(x[a:b])).cuda(rank)
        y = sess.run_device(xd)
        torch.cuda.synchronize(rank)
        first = y.cpu().numpy()
        # the second identical run captures the program (all-reduces included) in a CUDA
        # graph, the third replays it: same bits every time
        for _ in range(2):
            y.fill_(float("nan"))
            sess.run_device(xd, y)
            torch.cuda.synchronize(rank)
            again = y.cpu().numpy()
            assert np.array_equal(again, first) or np.array_equal(np.isnan(again), np.isnan(first)) and \
                np.array_equal(np.nan_to_num(again), np.nan_to_num(first))
        np.save(os.path.join(out_dir, f"y{rank}.npy"), first)
        # all-gather of equal shards through the session's communicator
        send = torch.full((8,), float(rank + 1), device=f"cuda:{rank}")
        recv = torch.empty((8 * world,), device=f"cuda:{rank}")
        dist.allgather(sess, send, recv)
        torch.cuda.synchronize(rank)
        assert recv.cpu().tolist() == [float(r + 1) for r in range(world) for _ in range(8)]
        del sess
    finally:
        tdist.destroy_process_group()


@pytest.mark.parametrize("case", ["c2_cnn_4", "c1_mlp_64", "integration", "transformer_mini", "resnet_mini"])
def test_two_gpu_sharding_is_bit_exact(gpu, oracle_lib, tmp_path, case):
    torch = gpu
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from oracle import configs, oracle
    from rustgears_b200 import dist
    world = 2
    mp.start_processes(_rank, args=(world, _port(), case, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    y = dist.gather_rows([np.load(tmp_path / f"y{r}.npy") for r in range(world)])
    layers, x = configs.CASES[case]()
    ref, _, _ = oracle.Program(layers).execute(x)
    assert np.array_equal(y, ref)
