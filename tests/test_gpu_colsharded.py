"""Column-sharded FT step (stockfish_trainer_b200/colsharded.py) on the GPU.

* One GPU, every rank emulated: the kernels over the whole batch on each
  rank's column slice (the slices of 2, 4 and 8 ranks at the headline width,
  so two-chunk slices with packed tails are covered) give exactly those
  columns of the whole-table forward and backward.
* One GPU, no process group: the autograd function equals
  SparseLinearPairFunction bit for bit.
* One GPU, the exchange kernel: strided, scaled and bit-for-bit copies with
  the barrier of one rank; a barrier whose other rank never arrives times
  out with the timeout flag instead of hanging.
* Two GPUs (NCCL; skipped with fewer), both exchange paths: each rank's
  outputs are its positions' rows of the one-GPU forward, and its gradient
  columns are the one-GPU full-batch gradient of those columns times 1/2,
  bit for bit."""

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


@pytest.mark.parametrize("exchange,prepare", [("peer", "forward"), ("p2p", "forward"), ("peer", "overlap")])
def test_single_process_equals_pair_function(cuda, exchange, prepare):
    from stockfish_trainer_b200 import SparseLinearPairFunction, colsharded

    B, C = 2048, 264
    white, black, W, bias, g, T, K = _inputs(B, C, seed=9)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    i0, i1 = t(white), t(black)
    sh = colsharded.ColumnShardedFT(T, C, B, K, device=cuda, exchange=exchange, prepare=prepare)
    assert (sh.world, sh.c0, sh.c1, sh.exchange) == (1, 0, C, exchange)
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
    sh.close()


def test_single_process_prefetched_indices(cuda):
    """Index rows sent ahead with prefetch_indices (three steps, the slots
    rotating): the same outputs and gradients as passing them each step."""
    from stockfish_trainer_b200 import colsharded

    B, C = 2048, 264
    white, black, W, bias, g, T, K = _inputs(B, C, seed=13)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    i0, i1 = t(white), t(black)
    res = []
    for prefetch in (False, True):
        sh = colsharded.ColumnShardedFT(T, C, B, K, device=cuda, prepare="overlap")
        Wp, bp = t(W).requires_grad_(), t(bias).requires_grad_()
        if prefetch:
            sh.prefetch_indices(i0, i1)
        steps = []
        for _ in range(3):
            Wp.grad = bp.grad = None
            o0, o1 = colsharded.SparseLinearPairColumnSharded.apply(None if prefetch else i0, None if prefetch else i1,
                                                                    Wp, bp, sh)
            if prefetch:
                sh.prefetch_indices(i0, i1)
            torch.autograd.backward([o0, o1], [t(g[0]), t(g[1])])
            steps.append((o0.detach().clone(), o1.detach().clone(), Wp.grad.clone(), bp.grad.clone()))
        res.append(steps)
        sh.close()
    for a, b in zip(res[0], res[1]):
        for x, y in zip(a, b):
            assert torch.equal(x, y)


def test_explicit_rows_take_precedence_over_a_prefetch(cuda):
    """Rows passed to the step win over different rows sent ahead with
    prefetch_indices (which still land first); with None the prefetched rows
    are used."""
    from stockfish_trainer_b200 import colsharded, positions

    B, C = 1024, 264
    white, black, W, bias, g, T, K = _inputs(B, C, seed=17)
    w2, b2, _ = positions.synthetic_batch(B, FS, seed=18)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    Wd, bd = t(W), t(bias)
    sh = colsharded.ColumnShardedFT(T, C, B, K, device=cuda)
    want_a = [x.clone() for x in sh.forward(Wd, bd, t(white), t(black))]
    want_b = [x.clone() for x in sh.forward(Wd, bd, t(w2), t(b2))]
    sh.prefetch_indices(t(w2), t(b2))
    got = [x.clone() for x in sh.forward(Wd, bd, t(white), t(black))]  # explicit rows win
    assert all(torch.equal(a, b) for a, b in zip(got, want_a))
    sh.prefetch_indices(t(w2), t(b2))
    got = [x.clone() for x in sh.forward(Wd, bd, None, None)]  # the prefetched rows
    assert all(torch.equal(a, b) for a, b in zip(got, want_b))
    sh.close()


def _exchange_buffer(nbytes):
    import ctypes

    from stockfish_trainer_b200 import _native

    p, h = ctypes.c_void_p(0), ctypes.create_string_buffer(64)
    _native.call("nnue_ft_exchange_alloc", nbytes, ctypes.byref(p), h)
    return p.value


@pytest.mark.parametrize("rows,blocks", [(1, 4), (2, 1), (4, 8)])
def test_exchange_copies_and_self_barrier(cuda, rows, blocks):
    """One rank: strided block copies (scaled, and bit-for-bit with scale 1,
    int32 and NaN payloads included), then the barrier with itself; the flag
    words count the epochs.  Every rows-per-warp / grid setting."""
    import ctypes

    from stockfish_trainer_b200 import _native, colsharded

    buf = _exchange_buffer(1 << 20)
    old = {k: _native.get_param(k) for k in ("xchg_rows", "xchg_blocks_per_sm")}
    _native.set_param("xchg_rows", rows)
    _native.set_param("xchg_blocks_per_sm", blocks)
    try:
        flags = colsharded._device_view(buf, (64,), torch.int32, cuda)
        assert int(flags.abs().sum()) == 0  # zeroed at allocation
        rng = np.random.default_rng(3)
        src = torch.from_numpy(rng.standard_normal((37, 24), dtype=np.float32)).to(cuda)
        src[3, 10] = float("nan")  # inside the scale-1 copy
        ints = torch.from_numpy(rng.integers(-2**31, 2**31 - 1, (37, 8), dtype=np.int64).astype(np.int32)).to(cuda)
        dst = torch.full((37, 40), -7.0, device=cuda)
        dst_i = torch.zeros(37, 8, dtype=torch.int32, device=cuda)
        D = colsharded._CopyDesc
        arr = (D * 3)(D(src.data_ptr() + 8 * 4, dst.data_ptr() + 4 * 4, 37, 6, 10, 3, 1.0),
                      D(src.data_ptr(), dst.data_ptr() + 20 * 4, 37, 6, 10, 2, 0.25),
                      D(ints.data_ptr(), dst_i.data_ptr(), 37, 2, 2, 2, 1.0))
        fl = (ctypes.c_void_p * 1)(buf)
        stream = torch.cuda.current_stream(cuda).cuda_stream
        for epoch in (1, 2):
            _native.call("nnue_ft_exchange", arr, 3, fl, 1, 0, 0, epoch, 1000, stream)
        _native.call("nnue_ft_exchange", None, 0, fl, 1, 0, 2, 1, 1000, stream)  # channel 2: its own epochs
        torch.cuda.synchronize()
        assert _native.device_errors() == 0
        want = torch.full((37, 40), -7.0, device=cuda)
        want[:, 4:16] = src[:, 8:20]
        want[:, 20:28] = src[:, 0:8] * 0.25
        got = dst.view(torch.int32)
        assert torch.equal(got[:, :20], want.view(torch.int32)[:, :20])  # bit for bit, the NaN too
        assert torch.equal(dst[:, 20:], want[:, 20:])
        assert torch.equal(dst_i, ints)
        # channel 0 saw epoch 2, channel 2 epoch 1; the block counters are reset
        assert flags[0].item() == 2 and flags[15].item() == 0
        assert flags[32].item() == 1 and flags[47].item() == 0
    finally:
        for k, v in old.items():
            _native.set_param(k, v)
        _native.call("nnue_ft_exchange_free", buf)


def test_exchange_barrier_times_out_without_the_other_rank(cuda):
    """Two ranks' flag words, one process playing rank 0: rank 1 never
    signals, so the bounded wait runs out, raises the timeout flag and the
    launch returns; the context stays usable."""
    import ctypes
    import time

    from stockfish_trainer_b200 import _native

    own, other = _exchange_buffer(4096), _exchange_buffer(4096)
    try:
        fl = (ctypes.c_void_p * 2)(own, other)
        _native.device_errors()  # start from clear flags
        t0 = time.perf_counter()
        _native.call("nnue_ft_exchange", None, 0, fl, 2, 0, 0, 1, 200, torch.cuda.current_stream(cuda).cuda_stream)
        torch.cuda.synchronize()
        assert time.perf_counter() - t0 >= 0.19
        assert _native.device_errors() == _native.DEVERR_EXCHANGE_TIMEOUT
        x = torch.ones(8, device=cuda)
        assert float((x * 2).sum()) == 16.0
    finally:
        _native.call("nnue_ft_exchange_free", own)
        _native.call("nnue_ft_exchange_free", other)


def _worker(rank, world, port, out_dir, B, C, exchange, prepare):
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
    sh = colsharded.ColumnShardedFT(T, C, B, K, device=dev, exchange=exchange, prepare=prepare)
    assert sh.exchange == exchange
    Wp = sh.shard_columns(t(W)).requires_grad_()
    bp = sh.shard_columns(t(bias)).requires_grad_()
    for _ in range(2):  # two steps: the second reuses every buffer
        Wp.grad = bp.grad = None
        o0, o1 = colsharded.SparseLinearPairColumnSharded.apply(t(white[lo:lo + b]), t(black[lo:lo + b]), Wp, bp, sh)
        torch.autograd.backward([o0, o1], [t(g[0, lo:lo + b]), t(g[1, lo:lo + b])])
    full = sh.gather_columns(Wp.grad)
    torch.cuda.synchronize()
    from stockfish_trainer_b200 import _native

    np.savez(os.path.join(out_dir, f"r{rank}.npz"), o0=o0.detach().cpu().numpy(), o1=o1.detach().cpu().numpy(),
             dW=Wp.grad.cpu().numpy(), dB=bp.grad.cpu().numpy(), c0=sh.c0, c1=sh.c1, full=full.cpu().numpy(),
             errors=_native.device_errors())
    sh.close()
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("C,exchange,prepare", [(1048, "peer", "forward"), (264, "peer", "overlap"),
                                                (1048, "p2p", "forward")])
def test_two_gpu_column_sharded_matches_one_gpu(tmp_path, C, exchange, prepare):
    from stockfish_trainer_b200.feature_transformer import ops

    world, B = 2, 4096
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), B, C, exchange, prepare), nprocs=world,
                       join=True, start_method="spawn")
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
        assert int(z["errors"]) == 0
        c0, c1 = int(z["c0"]), int(z["c1"])
        np.testing.assert_array_equal(z["o0"], o0[r * b:(r + 1) * b])
        np.testing.assert_array_equal(z["o1"], o1[r * b:(r + 1) * b])
        np.testing.assert_array_equal(z["dW"], dW[:, c0:c1] * np.float32(0.5))
        np.testing.assert_array_equal(z["full"], dW * np.float32(0.5))
        np.testing.assert_allclose(z["dB"], dB[c0:c1] * np.float32(0.5), rtol=1e-5, atol=1e-6)
