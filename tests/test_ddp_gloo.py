"""Data-parallel host logic on CPU ranks (gloo, world size 2 and 4).

The reference splits the global batch evenly over ranks and DDP averages the
dense gradients (src/train/common.py:186-199, 256-263).  Here each rank runs
the oracle backward on its shard, the flat GradientBuffer is allreduce-averaged,
and the result must equal (full-batch gradient) / world within fp32
summation-order tolerance.  A rank that dies before the collective must make
the others fail with a timeout, not hang."""

import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup(rank, world, port, timeout_s=60):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from stockfish_trainer_b200 import ddp

    rt = ddp.init_from_env("gloo", timeout_s=timeout_s)
    assert rt.rank == rank and rt.world_size == world
    return rt


def _worker_allreduce(rank, world, port, out_dir):
    _setup(rank, world, port)
    import oracle
    from stockfish_trainer_b200 import ddp, positions

    B, C = 256, 24
    fs = "HalfKAv2_hm^"
    T = positions.feature_set_info(fs)[1]
    first, n = ddp.shard(B, rank, world)
    white, black, _ = positions.synthetic_batch(n, fs, seed=3, first=first)
    rng = np.random.default_rng(10)
    g_all = rng.standard_normal((2, B, C), dtype=np.float32)
    g0, g1 = g_all[0, first:first + n], g_all[1, first:first + n]
    dW, dB = oracle.ft_backward_pair(white, black, g0, g1, T)
    buf = ddp.GradientBuffer(T, C, torch.device("cpu"))
    buf.weight.copy_(torch.from_numpy(dW))
    buf.bias.copy_(torch.from_numpy(dB))
    buf.allreduce_mean(world, chunks=3 if rank >= 0 else 1)
    np.save(os.path.join(out_dir, f"w{rank}.npy"), buf.weight.numpy())
    np.save(os.path.join(out_dir, f"b{rank}.npy"), buf.bias.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_backward_allreduce_matches_full_batch(tmp_path, world):
    import oracle
    from stockfish_trainer_b200 import positions

    port = _free_port()
    mp.start_processes(_worker_allreduce, args=(world, port, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    B, C = 256, 24
    fs = "HalfKAv2_hm^"
    T = positions.feature_set_info(fs)[1]
    white, black, _ = positions.synthetic_batch(B, fs, seed=3)
    g_all = np.random.default_rng(10).standard_normal((2, B, C), dtype=np.float32)
    rW, rB = oracle.ft_backward_pair(white, black, g_all[0], g_all[1], T)
    w0 = np.load(tmp_path / "w0.npy")
    for r in range(world):  # every rank holds the same averaged gradient
        np.testing.assert_array_equal(np.load(tmp_path / f"w{r}.npy"), w0)
        np.testing.assert_array_equal(np.load(tmp_path / f"b{r}.npy"), np.load(tmp_path / "b0.npy"))
    np.testing.assert_allclose(w0, rW / world, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(np.load(tmp_path / "b0.npy"), rB / world, rtol=1e-5, atol=1e-5)


def test_shard_rejects_uneven_batch():
    sys.path.insert(0, ROOT)
    from stockfish_trainer_b200 import ddp

    assert ddp.shard(65536, 3, 8) == (3 * 8192, 8192)
    with pytest.raises(ValueError):
        ddp.shard(100, 0, 3)


def _worker_dead_rank(rank, world, port, out_dir):
    _setup(rank, world, port, timeout_s=5)
    from stockfish_trainer_b200 import ddp

    buf = ddp.GradientBuffer(8, 4, torch.device("cpu"))
    buf.flat.fill_(1.0)
    if rank == 1:
        os._exit(0)  # leaves between steps, before its collective
    try:
        buf.allreduce_mean(world)
        result = "completed"
    except Exception as e:  # gloo reports the missing peer
        result = "error: " + type(e).__name__
    with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as f:
        f.write(result)
    os._exit(0)


def test_dead_rank_is_detected_not_hung(tmp_path):
    port = _free_port()
    ctx = mp.start_processes(_worker_dead_rank, args=(2, port, str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=90)
    alive = [p for p in ctx.processes if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung waiting for a dead peer"
    assert (tmp_path / "r0.txt").read_text().startswith("error")
