"""Row-sharded Ranger22 step (stockfish_trainer_b200/sharded.py) on CPU ranks
(gloo, world size 2 and 4), the native kernels replaced by the oracle: each
rank's "backward" hands out a seeded partial gradient, the update is the numpy
restatement of the reference's Ranger22 update (oracle/ranger22.py).

Over six steps (the lookahead merges at step 5) every rank must end with the
table and bias of the unsharded path: the gradient averaged over ranks, then
Ranger22 over the whole table.  Two ranks: bit for bit ((a + b) / 2 is one
rounding in any order).  Four ranks: within fp32 summation-order tolerance
(gloo's allreduce order depends on the buffer it is given)."""

import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

T, C, STEPS, LR = 96, 40, 6, 8.75e-4


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _partial(rank, step):
    rng = np.random.default_rng(1000 * step + rank)
    return (rng.standard_normal((T, C)) * 1e-2).astype(np.float32), (rng.standard_normal(C) * 1e-2).astype(
        np.float32)


def _initial():
    rng = np.random.default_rng(7)
    return (rng.standard_normal((T, C)) * 0.05).astype(np.float32), (rng.standard_normal(C) * 0.05).astype(np.float32)


class _OracleKernels:
    def __init__(self, rank):
        self.rank = rank
        self.step = 0

    def block_gradient(self, grad0, grad1, batch, max_active, weight_grad, bias_grad, workspace, row_begin, row_end,
                       with_bias):
        w, b = _partial(self.rank, self.step)
        weight_grad[row_begin:row_end] = torch.from_numpy(w[row_begin:row_end])
        if with_bias:
            bias_grad.copy_(torch.from_numpy(b))

    def update(self, p, grad, variance_ma, gma_cur, gma_prev, scalars, lookahead, merge, alpha):
        from oracle import ranger22 as oracle_r22

        oracle_r22.update(p.numpy(), grad.numpy(), variance_ma.numpy(), gma_cur.numpy(), gma_prev.numpy(),
                          np.array(scalars, np.float32), lookahead.numpy(), merge, alpha)


def _worker(rank, world, port, out_dir, n_blocks):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from stockfish_trainer_b200 import ddp, sharded

    ddp.init_from_env("gloo", timeout_s=60)
    w0, b0 = _initial()
    W, bias = torch.from_numpy(w0.copy()), torch.from_numpy(b0.copy())
    kern = _OracleKernels(rank)
    opt = sharded.ShardedRanger22FT(W, bias, LR, n_blocks=n_blocks, kernels=kern)
    assert opt.variance_ma.shape == (T // world, C)  # only this rank's rows carry state
    for step in range(STEPS):
        kern.step = step
        opt.backward_step(None, None, 0, 0, None)
    np.save(os.path.join(out_dir, f"w{rank}.npy"), W.numpy())
    np.save(os.path.join(out_dir, f"b{rank}.npy"), bias.numpy())
    dist.barrier()
    dist.destroy_process_group()


def _unsharded(world):
    """Average of the ranks' gradients, then the update over the whole table."""
    sys.path.insert(0, ROOT)
    from oracle import ranger22 as oracle_r22

    W, bias = _initial()
    state = {k: (np.zeros_like(W), np.zeros_like(bias)) for k in ("v", "m", "mn")}
    la_w, la_b = W.copy(), bias.copy()
    for step in range(STEPS):
        gw = sum(_partial(r, step)[0] for r in range(world)) / np.float32(world)
        gb = sum(_partial(r, step)[1] for r in range(world)) / np.float32(world)
        n = step + 1
        sc = oracle_r22.scalars(LR, n)
        merge = n % 5 == 0
        for j, (p, g, la) in enumerate(((W, gw.astype(np.float32), la_w), (bias, gb.astype(np.float32), la_b))):
            m_cur, m_prev = (state["m"][j], state["mn"][j]) if n % 2 == 1 else (state["mn"][j], state["m"][j])
            oracle_r22.update(p, g, state["v"][j], m_cur, m_prev, sc, la, merge, 0.5)
    return W, bias


@pytest.mark.parametrize("world,n_blocks", [(2, 3), (4, 4)])
def test_sharded_step_matches_unsharded(tmp_path, world, n_blocks):
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), n_blocks), nprocs=world, join=True,
                       start_method="spawn")
    rW, rB = _unsharded(world)
    w0 = np.load(tmp_path / "w0.npy")
    for r in range(world):  # every rank ends with the same parameters
        np.testing.assert_array_equal(np.load(tmp_path / f"w{r}.npy"), w0)
        np.testing.assert_array_equal(np.load(tmp_path / f"b{r}.npy"), np.load(tmp_path / "b0.npy"))
    if world == 2:
        np.testing.assert_array_equal(w0, rW)
        np.testing.assert_array_equal(np.load(tmp_path / "b0.npy"), rB)
    else:
        np.testing.assert_allclose(w0, rW, rtol=1e-6, atol=1e-8)
        np.testing.assert_allclose(np.load(tmp_path / "b0.npy"), rB, rtol=1e-6, atol=1e-8)


def test_row_block_bounds():
    sys.path.insert(0, ROOT)
    from stockfish_trainer_b200 import sharded

    b = sharded.row_block_bounds(85296, 4, 8)
    assert b[0] == 0 and b[-1] == 85296 and len(b) == 5
    assert all((b[i + 1] - b[i]) % 8 == 0 and b[i + 1] > b[i] for i in range(4))
    assert sharded.row_block_bounds(16, 100, 8) == [0, 8, 16]
    with pytest.raises(ValueError):
        sharded.row_block_bounds(85297, 4, 8)
