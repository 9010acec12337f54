"""Row-sharded Ranger22 training step (stockfish_trainer_b200/sharded.py) with
the native kernels, against the unsharded path: the averaged dense gradient,
then ``optim.Ranger22FT`` over the whole table on every rank.  Six training
steps (forward with the index phase, backward, update; the lookahead merges at
step 5), parameters compared bit for bit after every step.

* one GPU, a one-rank NCCL group: the row blocks, per-block updates of the
  packed state and stream ordering against one update over the whole table;
* two GPUs (skipped with fewer): each rank's shard of the batch, the
  reduce-scatter / per-rank update / all-gather against allreduce + the whole
  update on every rank ((a + b) / 2 is one rounding in any order)."""

import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

pytestmark = pytest.mark.gpu

FS = "Full_Threats+HalfKAv2_hm^"
B, C, STEPS, LR = 4096, 264, 6, 8.75e-4


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _batch(rank, world, dev):
    from stockfish_trainer_b200 import ddp, positions

    first, n = ddp.shard(B, rank, world)
    white, black, _ = positions.synthetic_batch(n, FS, seed=31, first=first)
    return torch.from_numpy(white).to(dev), torch.from_numpy(black).to(dev), n


def _grads(step, rank, world, dev):
    from stockfish_trainer_b200 import ddp

    first, n = ddp.shard(B, rank, world)
    gen = torch.Generator(device=dev).manual_seed(500 + step)
    g = torch.randn(2, B, C, device=dev, generator=gen)
    return g[0, first:first + n].contiguous(), g[1, first:first + n].contiguous()


def _params(dev):
    from stockfish_trainer_b200 import positions

    T = positions.feature_set_info(FS)[1]
    gen = torch.Generator(device=dev).manual_seed(9)
    return torch.randn(T, C, device=dev, generator=gen) * 0.01, torch.randn(C, device=dev, generator=gen) * 0.01


def _train(rank, world, dev, sharded_opt: bool, n_blocks=4):
    """Returns the parameters after each step."""
    import torch.distributed as dist

    from stockfish_trainer_b200 import ddp, optim, sharded
    from stockfish_trainer_b200.feature_transformer import ops

    i0, i1, n = _batch(rank, world, dev)
    K = i0.shape[1]
    W, bias = _params(dev)
    T = W.shape[0]
    ws = ops.alloc_workspace(n, K, T, C, 2, dev)
    o0, o1 = torch.empty(n, C, device=dev), torch.empty(n, C, device=dev)
    if sharded_opt:
        opt = sharded.ShardedRanger22FT(W, bias, LR, n_blocks=n_blocks)
    else:
        Wp, bp = torch.nn.Parameter(W), torch.nn.Parameter(bias)
        opt = optim.Ranger22FT([Wp, bp], lr=LR)
        buf = ddp.GradientBuffer(T, C, dev)
    history = []
    for step in range(STEPS):
        g0, g1 = _grads(step, rank, world, dev)
        ops.forward_pair_prepare(i0, i1, W, bias, o0, o1, ws)
        if sharded_opt:
            opt.backward_step(g0, g1, n, K, ws)
        else:
            ops.backward_apply(g0, g1, n, K, buf.weight, buf.bias, False, ws)
            if world > 1:
                dist.all_reduce(buf.flat, op=dist.ReduceOp.AVG)
            Wp.grad, bp.grad = buf.weight, buf.bias
            opt.step()
        history.append((W.cpu().numpy().copy(), bias.cpu().numpy().copy()))
    return history


def test_sharded_one_rank_group_matches_whole_update(cuda):
    import torch.distributed as dist

    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{_free_port()}", rank=0, world_size=1,
                            device_id=cuda)
    try:
        got = _train(0, 1, cuda, True, n_blocks=5)
        want = _train(0, 1, cuda, False)
    finally:
        dist.destroy_process_group()
    for step, ((gw, gb), (ww, wb)) in enumerate(zip(got, want)):
        np.testing.assert_array_equal(gw, ww, err_msg=f"table after step {step + 1}")
        np.testing.assert_array_equal(gb, wb, err_msg=f"bias after step {step + 1}")


def _worker(rank, world, port, out_dir):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from stockfish_trainer_b200 import ddp

    rt = ddp.init_from_env("nccl", timeout_s=60)
    dev = torch.device("cuda", rt.local_rank)
    torch.cuda.set_device(dev)
    got = _train(rank, world, dev, True)
    want = _train(rank, world, dev, False)
    for step, ((gw, gb), (ww, wb)) in enumerate(zip(got, want)):
        np.save(os.path.join(out_dir, f"r{rank}_s{step}_eq.npy"),
                np.array([np.array_equal(gw, ww), np.array_equal(gb, wb)]))
    np.save(os.path.join(out_dir, f"w{rank}.npy"), got[-1][0])
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_sharded_matches_allreduce_and_whole_update(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    for r in range(world):
        for step in range(STEPS):
            eq = np.load(tmp_path / f"r{r}_s{step}_eq.npy")
            assert eq.all(), f"rank {r} step {step + 1}: sharded parameters differ from the unsharded path"
    np.testing.assert_array_equal(np.load(tmp_path / "w0.npy"), np.load(tmp_path / "w1.npy"))
