"""Row-block backward on one GPU: ``nnue_ft_backward_apply_rows``, the call the
data-parallel backward makes once per row block (each finished block's
gradient is exchanged while the next block is computed), checked against the
whole-table backward ``nnue_ft_backward_apply`` of the same workspace.

* the table cut into 1, 3, 4 or 7 equal row blocks, and into blocks whose
  bounds isolate hot (heavy) rows, so hot rows land alone, first or last in a
  block;
* the bias gradient produced only by the last block;
* dW prefilled with NaN, so a row that no block writes shows.

Then ``ddp.SparseLinearPairAllreduce`` through autograd over a one-rank NCCL
process group: the row blocks and their collectives run (an average over one
rank), and the gradients equal ``SparseLinearPairFunction``'s bit for bit.
"""

import socket

import numpy as np
import pytest
import torch

from stockfish_trainer_b200 import SparseLinearPairFunction, _native, ddp
from stockfish_trainer_b200.feature_transformer import ops

from _inputs import feature_batch

pytestmark = pytest.mark.gpu

FS = "Full_Threats+HalfKAv2_hm^"
B, C = 16384, 1048


@pytest.fixture(scope="module")
def prepared(cuda):
    white, black, T = feature_batch(B, FS, seed=606)
    K = white.shape[1]
    gen = torch.Generator(device=cuda).manual_seed(607)
    W = torch.randn(T, C, device=cuda, generator=gen) * 0.01
    bias = torch.zeros(C, device=cuda)
    g0 = torch.randn(B, C, device=cuda, generator=gen)
    g1 = torch.randn(B, C, device=cuda, generator=gen)
    i0, i1 = torch.from_numpy(white).to(cuda), torch.from_numpy(black).to(cuda)
    o0, o1 = torch.empty(B, C, device=cuda), torch.empty(B, C, device=cuda)
    ws = ops.alloc_workspace(B, K, T, C, 2, cuda)
    ops.forward_pair_prepare(i0, i1, W, bias, o0, o1, ws)
    ref_w = torch.empty(T, C, device=cuda)
    ref_b = torch.empty(C, device=cuda)
    ops.backward_apply(g0, g1, B, K, ref_w, ref_b, False, ws)
    counts = np.bincount(white[white >= 0], minlength=T) + np.bincount(black[black >= 0], minlength=T)
    heavy = np.flatnonzero(counts > _native.get_param("heavy_threshold"))
    return dict(T=T, K=K, W=W, bias=bias, g0=g0, g1=g1, i0=i0, i1=i1, ws=ws, ref_w=ref_w, ref_b=ref_b,
                heavy=heavy)


def _run_blocks(d, bounds, cuda):
    dW = torch.full((d["T"], C), float("nan"), device=cuda)
    dB = torch.full((C,), float("nan"), device=cuda)
    for i in range(len(bounds) - 1):
        ops.backward_apply_rows(d["g0"], d["g1"], B, d["K"], dW, dB, False, d["ws"], bounds[i], bounds[i + 1],
                                with_bias=i == len(bounds) - 2)
    torch.cuda.synchronize()
    assert _native.device_errors() == 0
    return dW, dB


def _check(d, dW, dB):
    assert not torch.isnan(dW).any(), "a row block left rows unwritten"
    assert torch.equal(dW, d["ref_w"])
    torch.testing.assert_close(dB, d["ref_b"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("n_blocks", [1, 3, 4, 7])
def test_equal_row_blocks_match_whole_backward(prepared, cuda, n_blocks):
    T = prepared["T"]
    bounds = [T * i // n_blocks for i in range(n_blocks + 1)]
    _check(prepared, *_run_blocks(prepared, bounds, cuda))


def test_blocks_split_at_hot_rows(prepared, cuda):
    heavy = prepared["heavy"]
    assert heavy.size >= 4, "the case needs hot rows"
    h = [int(x) for x in heavy[[0, 1, heavy.size // 2, heavy.size - 1]]]
    T = prepared["T"]
    # a hot row alone in its block, one ending a block, one starting a block
    bounds = sorted({0, h[0], h[0] + 1, h[1] + 1, h[2], h[3], T})
    _check(prepared, *_run_blocks(prepared, bounds, cuda))


def test_pair_allreduce_one_rank_group(prepared, cuda):
    import torch.distributed as dist

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                            device_id=cuda)
    try:
        d = prepared
        Wa = d["W"].clone().requires_grad_()
        ba = d["bias"].clone().requires_grad_()
        o0, o1 = ddp.SparseLinearPairAllreduce.apply(d["i0"], d["i1"], Wa, ba, 1, 5)
        torch.autograd.backward([o0, o1], [d["g0"], d["g1"]])
        Wb = d["W"].clone().requires_grad_()
        bb = d["bias"].clone().requires_grad_()
        r0, r1 = SparseLinearPairFunction.apply(d["i0"], d["i1"], Wb, bb)
        torch.autograd.backward([r0, r1], [d["g0"], d["g1"]])
        torch.cuda.synchronize()
        assert torch.equal(o0, r0) and torch.equal(o1, r1)
        assert torch.equal(Wa.grad, Wb.grad)
        assert torch.equal(ba.grad, bb.grad)
    finally:
        dist.destroy_process_group()
