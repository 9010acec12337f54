"""Column-sharded FT step (stockfish_trainer_b200/colsharded.py) on CPU ranks
(gloo, world size 2, 3 and 4), the native kernels replaced by the C oracle.

Each rank passes its own positions' index rows and output gradients; it must
get back its positions' full output rows and its columns of the averaged
weight and bias gradients.  Against the oracle over the whole batch on one
process: outputs bit for bit; gradients bit for bit against the full-batch
backward of the 1/N-scaled output gradients (the sharded step sums in the
one-GPU order), and -- N a power of two -- against the full-batch gradient
times 1/N."""

import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

T, C, K, B = 97, 72, 9, 24


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    rng = np.random.default_rng(11)
    W = (rng.standard_normal((T, C)) * 0.1).astype(np.float32)
    bias = (rng.standard_normal(C) * 0.1).astype(np.float32)
    idx = rng.integers(0, T, size=(2, B, K)).astype(np.int32)
    idx[rng.random((2, B, K)) < 0.25] = -1  # holes anywhere in the row
    idx[:, :, 3] = 5  # a hot row, and repeats within a row
    idx[:, 0, 4] = 5
    g = rng.standard_normal((2, B, C)).astype(np.float32)
    return W, bias, idx, g


class _OracleKernels:
    """colsharded._CudaKernels' signatures over the C oracle."""

    @staticmethod
    def alloc_workspace(batch, max_active, num_inputs, width, device):
        return {"T": num_inputs}

    @staticmethod
    def forward_prepare(idx0, idx1, weight, bias, out0, out1, workspace):
        import oracle

        workspace["idx"] = (idx0.numpy().copy(), idx1.numpy().copy())
        out0.copy_(torch.from_numpy(oracle.ft_forward(idx0.numpy(), weight.numpy(), bias.numpy())))
        out1.copy_(torch.from_numpy(oracle.ft_forward(idx1.numpy(), weight.numpy(), bias.numpy())))

    @staticmethod
    def backward_apply(grad0, grad1, batch, max_active, weight_grad, bias_grad, workspace):
        import oracle

        i0, i1 = workspace["idx"]
        dW, dB = oracle.ft_backward_pair(i0, i1, grad0.numpy(), grad1.numpy(), workspace["T"])
        weight_grad.copy_(torch.from_numpy(dW))
        bias_grad.copy_(torch.from_numpy(dB))


def _worker(rank, world, port, out_dir):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from stockfish_trainer_b200 import colsharded, ddp

    ddp.init_from_env("gloo", timeout_s=60)
    W, bias, idx, g = _inputs()
    sh = colsharded.ColumnShardedFT(T, C, B, K, device="cpu", kernels=_OracleKernels())
    b = B // world
    lo = rank * b
    Wc = sh.shard_columns(torch.from_numpy(W))
    bc = sh.shard_columns(torch.from_numpy(bias))
    assert Wc.shape == (T, sh.width) and Wc.is_contiguous()
    Wp, bp = Wc.clone().requires_grad_(), bc.clone().requires_grad_()
    i0 = torch.from_numpy(idx[0, lo:lo + b].copy())
    i1 = torch.from_numpy(idx[1, lo:lo + b].copy())
    o0, o1 = colsharded.SparseLinearPairColumnSharded.apply(i0, i1, Wp, bp, sh)
    torch.autograd.backward([o0, o1], [torch.from_numpy(g[0, lo:lo + b].copy()),
                                       torch.from_numpy(g[1, lo:lo + b].copy())])
    full = sh.gather_columns(Wp.grad)  # every rank's columns, joined
    np.savez(os.path.join(out_dir, f"r{rank}.npz"), o0=o0.detach().numpy(), o1=o1.detach().numpy(),
             dW=Wp.grad.numpy(), dB=bp.grad.numpy(), c0=sh.c0, c1=sh.c1, full=full.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3, 4])
def test_column_sharded_step_matches_one_process(tmp_path, world):
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    sys.path.insert(0, ROOT)
    import oracle

    W, bias, idx, g = _inputs()
    out0 = oracle.ft_forward(idx[0], W, bias)
    out1 = oracle.ft_forward(idx[1], W, bias)
    scale = np.float32(1.0 / world)
    dW_s, dB_s = oracle.ft_backward_pair(idx[0], idx[1], g[0] * scale, g[1] * scale, T)
    dW_full, dB_full = oracle.ft_backward_pair(idx[0], idx[1], g[0], g[1], T)
    b = B // world
    cols = []
    for r in range(world):
        z = np.load(tmp_path / f"r{r}.npz")
        c0, c1 = int(z["c0"]), int(z["c1"])
        cols.append((c0, c1))
        np.testing.assert_array_equal(z["o0"], out0[r * b:(r + 1) * b])
        np.testing.assert_array_equal(z["o1"], out1[r * b:(r + 1) * b])
        np.testing.assert_array_equal(z["dW"], dW_s[:, c0:c1])
        np.testing.assert_array_equal(z["dB"], dB_s[c0:c1])
        np.testing.assert_array_equal(z["full"], dW_s)
        if world & (world - 1) == 0:
            np.testing.assert_array_equal(z["dW"], dW_full[:, c0:c1] * scale)
    assert cols[0][0] == 0 and cols[-1][1] == C
    assert all(cols[i][1] == cols[i + 1][0] for i in range(world - 1))


def test_column_slices():
    sys.path.insert(0, ROOT)
    from stockfish_trainer_b200 import colsharded

    assert [(b - a) // 4 for a, b in colsharded.column_slices(1048, 8)] == [34, 34, 34, 32, 32, 32, 32, 32]
    assert [(b - a) // 4 for a, b in colsharded.column_slices(1048, 4)] == [66, 66, 66, 64]
    assert [(b - a) // 4 for a, b in colsharded.column_slices(1048, 2)] == [131, 131]
    for C_ in (1048, 1040, 264, 1024, 520, 72, 16):
        for n in range(1, 9):
            if C_ // 4 < n:
                with pytest.raises(ValueError):
                    colsharded.column_slices(C_, n)
                continue
            s = colsharded.column_slices(C_, n)
            assert len(s) == n and s[0][0] == 0 and s[-1][1] == C_
            assert all(a % 4 == 0 and b > a for a, b in s)
            assert all(s[i][1] == s[i + 1][0] for i in range(n - 1))
            assert s == colsharded.column_slices(C_, n)  # deterministic
            # the tail of every multi-chunk slice is one the packed tail kernels take, where one exists
            widths = [(b - a) // 4 for a, b in s]
            assert max(widths) - min(widths) <= 2 * colsharded.CHUNK
    # columns not a multiple of 4: an even split
    assert colsharded.column_slices(10, 3) == [(0, 3), (3, 6), (6, 10)]


def test_exchange_choice_on_cpu():
    """Without CUDA the point-to-point exchange is chosen; asking for the peer
    exchange is refused with a clear error instead of reaching CUDA."""
    sys.path.insert(0, ROOT)
    from stockfish_trainer_b200 import colsharded

    sh = colsharded.ColumnShardedFT(T, C, B, K, device="cpu", kernels=_OracleKernels())
    assert (sh.exchange, sh.prepare, sh.world) == ("p2p", "forward", 1)
    with pytest.raises(ValueError, match="peer exchange"):
        colsharded.ColumnShardedFT(T, C, B, K, device="cpu", kernels=_OracleKernels(), exchange="peer")
    with pytest.raises(ValueError):
        colsharded.ColumnShardedFT(T, C, B, K, device="cpu", kernels=_OracleKernels(), exchange="nvls")


def _worker_dead_rank(rank, world, port, out_dir):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from stockfish_trainer_b200 import colsharded, ddp

    ddp.init_from_env("gloo", timeout_s=5)
    W, bias, idx, g = _inputs()
    sh = colsharded.ColumnShardedFT(T, C, B, K, device="cpu", kernels=_OracleKernels())
    b = B // world
    lo = rank * b
    sh.forward(sh.shard_columns(torch.from_numpy(W)), sh.shard_columns(torch.from_numpy(bias)),
               torch.from_numpy(idx[0, lo:lo + b].copy()), torch.from_numpy(idx[1, lo:lo + b].copy()))
    if rank == 1:
        os._exit(0)  # leaves between the forward and the backward, before its exchange
    try:
        dW, dB = torch.empty(T, sh.width), torch.empty(sh.width)
        sh.backward(torch.from_numpy(g[0, lo:lo + b].copy()), torch.from_numpy(g[1, lo:lo + b].copy()), dW, dB)
        result = "completed"
    except Exception as e:  # gloo reports the missing peer
        result = "error: " + type(e).__name__
    with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as f:
        f.write(result)
    os._exit(0)


def test_dead_rank_is_detected_not_hung(tmp_path):
    """A rank that leaves between steps: the other's next exchange ends with
    an error within the process group's timeout instead of waiting forever."""
    ctx = mp.start_processes(_worker_dead_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=120)
    alive = [p for p in ctx.processes if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung waiting for a dead peer"
    assert (tmp_path / "r0.txt").read_text().startswith("error")
