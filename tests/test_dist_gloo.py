"""Multi-rank host logic on CPU (gloo, world size 2): batch sharding with one
absmax max-all-reduce per Linear reproduces the single-device result bit for
bit, and the communicator id reaches every rank."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from rustgears_b200 import dist


def test_shard_range():
    for batch in (0, 1, 7, 64, 65537):
        for world in (1, 2, 3, 8):
            parts = [dist.shard_range(batch, r, world) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == batch
            assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
            sizes = [b - a for a, b in parts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        dist.shard_range(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, case, out_dir):
    import torch
    import torch.distributed as tdist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    tdist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import configs, oracle
        layers, x = configs.CASES[case]()
        prog = oracle.Program(layers)
        s0, s1 = dist.shard_range(x.shape[0], rank, world)

        def allreduce_max(v):
            t = torch.tensor([float(v)], dtype=torch.float32)
            tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
            return t.item()

        y = prog.run_sharded(x[s0:s1], allreduce_max)
        np.save(os.path.join(out_dir, f"y{rank}.npy"), y)
        uid = dist.exchange_unique_id(rank, make_id=lambda: bytes(range(128)))
        assert uid == bytes(range(128))
    finally:
        tdist.destroy_process_group()


@pytest.mark.parametrize("case", ["c2_cnn_4", "c1_mlp_64", "integration", "affine_first", "transformer_mini"])
def test_sharded_equals_single(oracle_lib, tmp_path, case):
    from oracle import configs, oracle
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), case, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    y = dist.gather_rows([np.load(tmp_path / f"y{r}.npy") for r in range(world)])
    layers, x = configs.CASES[case]()
    ref, _, _ = oracle.Program(layers).execute(x)
    assert np.array_equal(y, ref)
    # the per-shard scale would NOT give the same answer when a Linear sees the batch
    if any(l["kind"] in (1, 14, 15) for l in layers):
        prog = oracle.Program(layers)
        local = [prog.run_sharded(x[a:b], lambda v: v) for a, b in
                 (dist.shard_range(x.shape[0], r, world) for r in range(world))]
        assert not np.array_equal(np.concatenate(local), ref)


def _other_batch(case, x):
    """A batch to run with scales calibrated on x: twice the range (values clamp), or
    for token ids the sequences in reverse order."""
    if case.startswith("transformer"):
        return np.ascontiguousarray(x[::-1])
    return (x * np.float32(2.0)).astype(np.float32)


def _worker_calibrated(rank, world, port, case, out_dir):
    import torch
    import torch.distributed as tdist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    tdist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import configs, oracle
        layers, x = configs.CASES[case]()
        prog = oracle.Program(layers)
        s0, s1 = dist.shard_range(x.shape[0], rank, world)

        def allreduce_max(v):
            t = torch.tensor([float(v)], dtype=torch.float32)
            tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
            return t.item()

        # calibration over the sharded batch: every Linear's absmax all-reduced
        prog.run_sharded(x[s0:s1], allreduce_max)
        scales = prog.seen_scales()
        np.save(os.path.join(out_dir, f"s{rank}.npy"), scales)
        # a calibrated run needs no collective: each rank runs its shard alone
        prog.set_calibration(scales)
        x2 = _other_batch(case, x)
        y, _, _ = prog.execute(x2[s0:s1])
        np.save(os.path.join(out_dir, f"y{rank}.npy"), y)
    finally:
        tdist.destroy_process_group()


@pytest.mark.parametrize("case", ["c2_cnn_4", "c1_mlp_64", "transformer_mini"])
def test_sharded_calibration_equals_single(oracle_lib, tmp_path, case):
    """Static calibration across ranks: the scales a sharded calibration run freezes are
    the single-device ones, and a calibrated sharded run (no collective at all) gathers
    to the single-device calibrated output bit for bit."""
    from oracle import configs, oracle
    world = 2
    mp.start_processes(_worker_calibrated, args=(world, _free_port(), case, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    layers, x = configs.CASES[case]()
    prog = oracle.Program(layers)
    scales = prog.calibrate(x)
    for r in range(world):
        assert np.array_equal(np.load(tmp_path / f"s{r}.npy"), scales)
    prog.set_calibration(scales)
    ref, _, _ = prog.execute(_other_batch(case, x))
    y = dist.gather_rows([np.load(tmp_path / f"y{r}.npy") for r in range(world)])
    assert np.array_equal(y, ref)
