"""Data-parallel FT step on 2 GPUs (NCCL): forward + concurrent index phase,
row-blocked backward whose gradient allreduce overlaps the next block, as in
bench.py under torchrun.  Skipped when fewer than 2 GPUs are visible.

With two ranks the averaged gradient is exactly (g_0 + g_1) / 2 (one fp32
add, commutative; halving is exact), so the result is compared bit for bit
with per-shard gradients computed by the single-GPU path."""

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
B, C = 4096, 264


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(rank, world):
    from stockfish_trainer_b200 import ddp, positions

    first, n = ddp.shard(B, rank, world)
    white, black, _ = positions.synthetic_batch(n, FS, seed=99, first=first)
    rng = np.random.default_rng(5)
    g = rng.standard_normal((2, B, C), dtype=np.float32)[:, first:first + n]
    return white, black, np.ascontiguousarray(g[0]), np.ascontiguousarray(g[1]), n


def _worker(rank, world, port, out_dir, blocks):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from stockfish_trainer_b200 import ddp, positions
    from stockfish_trainer_b200.feature_transformer import ops

    rt = ddp.init_from_env("nccl", timeout_s=60)
    dev = torch.device("cuda", rt.local_rank)
    T = positions.feature_set_info(FS)[1]
    K = positions.feature_set_info(FS)[2]
    white, black, g0, g1, n = _inputs(rank, world)
    W = torch.from_numpy(np.random.default_rng(3).standard_normal((T, C), dtype=np.float32) * np.float32(0.01)).to(dev)
    bias = torch.zeros(C, device=dev)
    i0, i1 = torch.from_numpy(white).to(dev), torch.from_numpy(black).to(dev)
    o0 = torch.empty(n, C, device=dev)
    o1 = torch.empty_like(o0)
    ws = ops.alloc_workspace(n, K, T, C, 2, dev)
    buf = ddp.GradientBuffer(T, C, dev)
    ops.forward_pair_prepare(i0, i1, W, bias, o0, o1, ws)
    ddp.backward_allreduce_overlapped(torch.from_numpy(g0).to(dev), torch.from_numpy(g1).to(dev), n, K, buf, ws,
                                      world, n_blocks=blocks)
    torch.cuda.synchronize()
    np.save(os.path.join(out_dir, f"w{rank}.npy"), buf.weight.cpu().numpy())
    np.save(os.path.join(out_dir, f"b{rank}.npy"), buf.bias.cpu().numpy())
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("blocks", [1, 4, 7])
def test_two_gpu_overlapped_allreduce_matches_shard_gradients(tmp_path, blocks):
    from stockfish_trainer_b200 import positions
    from stockfish_trainer_b200.feature_transformer import ops

    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), blocks), nprocs=world, join=True,
                       start_method="spawn")
    T = positions.feature_set_info(FS)[1]
    dev = torch.device("cuda", 0)
    shard = []
    for r in range(world):
        white, black, g0, g1, n = _inputs(r, world)
        dW = torch.empty(T, C, device=dev)
        dB = torch.empty(C, device=dev)
        t = lambda a: torch.from_numpy(a).to(dev)
        ops.backward_into(t(white), t(black), t(g0), t(g1), dW, dB, accumulate=False)
        shard.append((dW.cpu().numpy(), dB.cpu().numpy()))
    expect_w = (shard[0][0] + shard[1][0]) / np.float32(2)
    expect_b = (shard[0][1] + shard[1][1]) / np.float32(2)
    for r in range(world):
        np.testing.assert_array_equal(np.load(tmp_path / f"w{r}.npy"), expect_w)
        np.testing.assert_array_equal(np.load(tmp_path / f"b{r}.npy"), expect_b)


def _autograd_worker(rank, world, port, out_dir):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from stockfish_trainer_b200 import ddp, positions

    rt = ddp.init_from_env("nccl", timeout_s=60)
    dev = torch.device("cuda", rt.local_rank)
    T = positions.feature_set_info(FS)[1]
    white, black, g0, g1, n = _inputs(rank, world)
    W = torch.from_numpy(np.random.default_rng(3).standard_normal((T, C), dtype=np.float32) *
                         np.float32(0.01)).to(dev).requires_grad_()
    bias = torch.zeros(C, device=dev, requires_grad=True)
    i0, i1 = torch.from_numpy(white).to(dev), torch.from_numpy(black).to(dev)
    o0, o1 = ddp.SparseLinearPairAllreduce.apply(i0, i1, W, bias, world, 3)
    torch.autograd.backward([o0, o1], [torch.from_numpy(g0).to(dev), torch.from_numpy(g1).to(dev)])
    torch.cuda.synchronize()
    np.save(os.path.join(out_dir, f"w{rank}.npy"), W.grad.cpu().numpy())
    np.save(os.path.join(out_dir, f"b{rank}.npy"), bias.grad.cpu().numpy())
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_allreduce_autograd_function_matches_shard_gradients(tmp_path):
    from stockfish_trainer_b200 import positions
    from stockfish_trainer_b200.feature_transformer import ops

    world = 2
    mp.start_processes(_autograd_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    T = positions.feature_set_info(FS)[1]
    dev = torch.device("cuda", 0)
    shard = []
    for r in range(world):
        white, black, g0, g1, n = _inputs(r, world)
        dW = torch.empty(T, C, device=dev)
        dB = torch.empty(C, device=dev)
        t = lambda a: torch.from_numpy(a).to(dev)
        ops.backward_into(t(white), t(black), t(g0), t(g1), dW, dB, accumulate=False)
        shard.append((dW.cpu().numpy(), dB.cpu().numpy()))
    for r in range(world):
        np.testing.assert_array_equal(np.load(tmp_path / f"w{r}.npy"), (shard[0][0] + shard[1][0]) / np.float32(2))
        np.testing.assert_array_equal(np.load(tmp_path / f"b{r}.npy"), (shard[0][1] + shard[1][1]) / np.float32(2))


def test_allreduce_autograd_function_single_rank_equals_pair_function(cuda):
    """world_size 1: the same outputs and gradients as SparseLinearPairFunction,
    bit for bit, also when one output gets no gradient."""
    from stockfish_trainer_b200 import SparseLinearPairFunction, ddp, positions

    T = positions.feature_set_info(FS)[1]
    white, black, g0, g1, n = _inputs(0, 1)
    i0, i1 = torch.from_numpy(white).to(cuda), torch.from_numpy(black).to(cuda)
    W0 = torch.from_numpy(np.random.default_rng(3).standard_normal((T, C), dtype=np.float32) * np.float32(0.01))
    b0 = torch.from_numpy(np.random.default_rng(4).standard_normal(C, dtype=np.float32))
    for use_g1 in (True, False):
        res = []
        for fn in (lambda *a: SparseLinearPairFunction.apply(*a), lambda *a: ddp.SparseLinearPairAllreduce.apply(*a)):
            W = W0.to(cuda).requires_grad_()
            bias = b0.to(cuda).requires_grad_()
            o0, o1 = fn(i0, i1, W, bias)
            outs, grads = [o0], [torch.from_numpy(g0).to(cuda)]
            if use_g1:
                outs.append(o1)
                grads.append(torch.from_numpy(g1).to(cuda))
            torch.autograd.backward(outs, grads)
            res.append((o0.detach().cpu(), o1.detach().cpu(), W.grad.cpu(), bias.grad.cpu()))
        for a, b in zip(*res):
            if a.shape == res[0][3].shape:
                torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)  # bias grad: float64 column sums either way
            else:
                assert torch.equal(a, b)
