"""Column-sharded FT step (stockfish_trainer_b200/colsharded.py) on the GPU.

* One GPU, every rank emulated: the kernels over the whole batch on each
  rank's column slice (the slices of 2, 4 and 8 ranks at the headline width,
  so two-chunk slices with packed tails are covered) give exactly those
  columns of the whole-table forward and backward.
* One GPU, no process group: the autograd function equals
  SparseLinearPairFunction bit for bit.
* Two GPUs (NCCL; skipped with fewer): each rank's outputs are its positions'
  rows of the one-GPU forward, and its gradient columns are the one-GPU
  full-batch gradient of those columns times 1/2, bit for bit."""

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


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(B, C, seed=5):
    from stockfish_trainer_b200 import positions

    _, T, K = positions.feature_set_info(FS)
    white, black, _ = positions.synthetic_batch(B, FS, seed=seed)
    rng = np.random.default_rng(seed + 1)
    W = (rng.standard_normal((T, C), dtype=np.float32) * np.float32(0.01))
    bias = rng.standard_normal(C, dtype=np.float32)
    g = rng.standard_normal((2, B, C), dtype=np.float32)
    return white, black, W, bias, g, T, K


@pytest.mark.parametrize("world", [2, 4, 8])
def test_every_rank_slice_equals_whole_table_columns(cuda, world):
    from stockfish_trainer_b200 import colsharded
    from stockfish_trainer_b200.feature_transformer import ops

    B, C = 6144, 1048
    white, black, W, bias, g, T, K = _inputs(B, C)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    i0, i1, Wd, bd, g0, g1 = t(white), t(black), t(W), t(bias), t(g[0]), t(g[1])
    o0, o1 = torch.empty(B, C, device=cuda), torch.empty(B, C, device=cuda)
    ws = ops.alloc_workspace(B, K, T, C, 2, cuda)
    dW, dB = torch.empty(T, C, device=cuda), torch.empty(C, device=cuda)
    ops.forward_pair_prepare(i0, i1, Wd, bd, o0, o1, ws)
    ops.backward_apply(g0, g1, B, K, dW, dB, False, ws)
    for c0, c1 in colsharded.column_slices(C, world):
        w = c1 - c0
        y0, y1 = torch.empty(B, w, device=cuda), torch.empty(B, w, device=cuda)
        wsr = ops.alloc_workspace(B, K, T, w, 2, cuda)
        dWr, dBr = torch.empty(T, w, device=cuda), torch.empty(w, device=cuda)
        ops.forward_pair_prepare(i0, i1, Wd[:, c0:c1].contiguous(), bd[c0:c1].contiguous(), y0, y1, wsr)
        ops.backward_apply(g0[:, c0:c1].contiguous(), g1[:, c0:c1].contiguous(), B, K, dWr, dBr, False, wsr)
        assert torch.equal(y0, o0[:, c0:c1]) and torch.equal(y1, o1[:, c0:c1]), (c0, c1)
        assert torch.equal(dWr, dW[:, c0:c1]), (c0, c1)
        torch.testing.assert_close(dBr, dB[c0:c1], rtol=1e-5, atol=1e-6)
    from stockfish_trainer_b200 import _native

    assert _native.device_errors() == 0


def test_single_process_equals_pair_function(cuda):
    from stockfish_trainer_b200 import SparseLinearPairFunction, colsharded

    B, C = 2048, 264
    white, black, W, bias, g, T, K = _inputs(B, C, seed=9)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    i0, i1 = t(white), t(black)
    sh = colsharded.ColumnShardedFT(T, C, B, K, device=cuda)
    assert (sh.world, sh.c0, sh.c1) == (1, 0, C)
    res = []
    for fn in (lambda a, b, w, c: SparseLinearPairFunction.apply(a, b, w, c),
               lambda a, b, w, c: colsharded.SparseLinearPairColumnSharded.apply(a, b, w, c, sh)):
        Wp, bp = t(W).requires_grad_(), t(bias).requires_grad_()
        o0, o1 = fn(i0, i1, Wp, bp)
        torch.autograd.backward([o0, o1], [t(g[0]), t(g[1])])
        res.append((o0.detach(), o1.detach(), Wp.grad, bp.grad))
    for a, b in zip(res[0][:3], res[1][:3]):
        assert torch.equal(a, b)
    torch.testing.assert_close(res[0][3], res[1][3], rtol=1e-5, atol=1e-6)


def _worker(rank, world, port, out_dir, B, C):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from stockfish_trainer_b200 import colsharded, ddp

    rt = ddp.init_from_env("nccl", timeout_s=60)
    dev = torch.device("cuda", rt.local_rank)
    white, black, W, bias, g, T, K = _inputs(B, C)
    b = B // world
    lo = rank * b
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    sh = colsharded.ColumnShardedFT(T, C, B, K, device=dev)
    Wp = sh.shard_columns(t(W)).requires_grad_()
    bp = sh.shard_columns(t(bias)).requires_grad_()
    for _ in range(2):  # two steps: the second reuses every buffer
        Wp.grad = bp.grad = None
        o0, o1 = colsharded.SparseLinearPairColumnSharded.apply(t(white[lo:lo + b]), t(black[lo:lo + b]), Wp, bp, sh)
        torch.autograd.backward([o0, o1], [t(g[0, lo:lo + b]), t(g[1, lo:lo + b])])
    full = sh.gather_columns(Wp.grad)
    torch.cuda.synchronize()
    np.savez(os.path.join(out_dir, f"r{rank}.npz"), o0=o0.detach().cpu().numpy(), o1=o1.detach().cpu().numpy(),
             dW=Wp.grad.cpu().numpy(), dB=bp.grad.cpu().numpy(), c0=sh.c0, c1=sh.c1, full=full.cpu().numpy())
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("C", [1048, 264])
def test_two_gpu_column_sharded_matches_one_gpu(tmp_path, C):
    from stockfish_trainer_b200.feature_transformer import ops

    world, B = 2, 4096
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), B, C), nprocs=world, join=True,
                       start_method="spawn")
    white, black, W, bias, g, T, K = _inputs(B, C)
    dev = torch.device("cuda", 0)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    o0, o1 = torch.empty(B, C, device=dev), torch.empty(B, C, device=dev)
    ws = ops.alloc_workspace(B, K, T, C, 2, dev)
    dW, dB = torch.empty(T, C, device=dev), torch.empty(C, device=dev)
    ops.forward_pair_prepare(t(white), t(black), t(W), t(bias), o0, o1, ws)
    ops.backward_apply(t(g[0]), t(g[1]), B, K, dW, dB, False, ws)
    o0, o1, dW, dB = o0.cpu().numpy(), o1.cpu().numpy(), dW.cpu().numpy(), dB.cpu().numpy()
    b = B // world
    for r in range(world):
        z = np.load(tmp_path / f"r{r}.npz")
        c0, c1 = int(z["c0"]), int(z["c1"])
        np.testing.assert_array_equal(z["o0"], o0[r * b:(r + 1) * b])
        np.testing.assert_array_equal(z["o1"], o1[r * b:(r + 1) * b])
        np.testing.assert_array_equal(z["dW"], dW[:, c0:c1] * np.float32(0.5))
        np.testing.assert_array_equal(z["full"], dW * np.float32(0.5))
        np.testing.assert_allclose(z["dB"], dB[c0:c1] * np.float32(0.5), rtol=1e-5, atol=1e-6)
