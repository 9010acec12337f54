"""Forward kernel vs the oracle (bit-exact: same fp32 add order as the reference)."""

import numpy as np
import pytest
import torch

import oracle
from stockfish_trainer_b200 import _native
from stockfish_trainer_b200.feature_transformer import ops

from _inputs import feature_batch, random_indices, random_table

pytestmark = pytest.mark.gpu


def _fwd(idx, W, bias, dev):
    out = torch.empty(idx.shape[0], W.shape[1], dtype=torch.float32, device=dev)
    ops.forward_into(torch.from_numpy(idx).to(dev), torch.from_numpy(W).to(dev), torch.from_numpy(bias).to(dev), out)
    return out.cpu().numpy()


@pytest.mark.parametrize("fs,B", [("HalfKAv2_hm^", 1000), ("Full_Threats+HalfKAv2_hm^", 600)])
def test_forward_matches_oracle_bit_exact(cuda, fs, B):
    white, black, T = feature_batch(B, fs, seed=1)
    C = 1048
    W = random_table(T, C, seed=2)
    bias = random_table(1, C, seed=3)[0]
    for idx in (white, black):
        np.testing.assert_array_equal(_fwd(idx, W, bias, cuda), oracle.ft_forward(idx, W, bias))


def test_forward_pair_matches_two_single_calls(cuda):
    white, black, T = feature_batch(700, "Full_Threats+HalfKAv2_hm^", seed=4)
    C = 1048
    W = random_table(T, C, seed=5)
    bias = random_table(1, C, seed=6)[0]
    dW, db = torch.from_numpy(W).to(cuda), torch.from_numpy(bias).to(cuda)
    i0, i1 = torch.from_numpy(white).to(cuda), torch.from_numpy(black).to(cuda)
    o0 = torch.empty(700, C, device=cuda)
    o1 = torch.empty_like(o0)
    ops.forward_pair_into(i0, i1, dW, db, o0, o1)
    np.testing.assert_array_equal(o0.cpu().numpy(), oracle.ft_forward(white, W, bias))
    np.testing.assert_array_equal(o1.cpu().numpy(), oracle.ft_forward(black, W, bias))


@pytest.mark.parametrize("C", [4, 36, 13, 1, 260, 2052])
@pytest.mark.parametrize("K", [1, 7, 32, 33, 70])
def test_forward_shapes_and_holes(cuda, C, K):
    T, B = 300, 257
    idx = random_indices(B, K, T, seed=C * 100 + K)
    W = random_table(T, C, seed=K, std=1.0)
    bias = random_table(1, C, seed=C, std=1.0)[0]
    np.testing.assert_array_equal(_fwd(idx, W, bias, cuda), oracle.ft_forward(idx, W, bias))


@pytest.mark.parametrize("C", [64, 1048, 2052])
def test_forward_misaligned_pointers_use_scalar_path(cuda, C):
    T, B, K = 120, 300, 16
    idx = random_indices(B, K, T, seed=7 + C)
    W = random_table(T, C, seed=8, std=1.0)
    bias = random_table(1, C, seed=9, std=1.0)[0]
    buf = torch.zeros(T * C + 1, device=cuda)
    Wd = buf[1:].view(T, C)  # 4-byte offset: not 16-byte aligned
    Wd.copy_(torch.from_numpy(W))
    out = torch.empty(B, C, device=cuda)
    ops.forward_into(torch.from_numpy(idx).to(cuda), Wd, torch.from_numpy(bias).to(cuda), out)
    np.testing.assert_array_equal(out.cpu().numpy(), oracle.ft_forward(idx, W, bias))


def test_forward_empty_rows_and_batches(cuda):
    T, C = 50, 32
    W = random_table(T, C, seed=1)
    bias = random_table(1, C, seed=2)[0]
    idx = np.full((9, 12), -1, np.int32)
    np.testing.assert_array_equal(_fwd(idx, W, bias, cuda), np.tile(bias, (9, 1)))
    out = torch.empty(0, C, device=cuda)
    ops.forward_into(torch.empty(0, 12, dtype=torch.int32, device=cuda), torch.from_numpy(W).to(cuda),
                     torch.from_numpy(bias).to(cuda), out)
    torch.cuda.synchronize()


@pytest.mark.parametrize(
    "params",
    [
        {"fwd_chunk_vec": 0, "fwd_items_per_warp": 1},
        {"fwd_chunk_vec": 16, "fwd_items_per_warp": 2},
        {"fwd_chunk_vec": 32, "fwd_items_per_warp": 4},
        {"fwd_chunk_vec": 64, "fwd_items_per_warp": 4},
        {"fwd_chunk_vec": 128, "fwd_items_per_warp": 16},
        {"fwd_chunk_vec": 8, "fwd_items_per_warp": 3},
        {"fwd_chunk_vec": 100, "fwd_items_per_warp": 5},
        {"fwd_chunk_vec": 300, "fwd_items_per_warp": 2},
        {"fwd_chunk_vec": 53, "fwd_exact_chunks": 0, "fwd_unroll": 4, "fwd_min_blocks": 3},
        {"fwd_unroll": 8, "fwd_min_blocks": 2},
        {"fwd_unroll": 4, "fwd_min_blocks": 6},
        {"fwd_unroll": 6, "fwd_min_blocks": 5, "fwd_items_per_warp": 7},
        {"fwd_block": 256},
        {"fwd_block": 128, "fwd_items_per_warp": 5},
        {"fwd_groups": 8, "fwd_unroll": 4, "fwd_min_blocks": 6},
        {"fwd_groups": 8},
        {"fwd_groups": 5},
        {"fwd_groups": 1},  # K = 160 read 32 slots at a time: several passes per item
        {"fwd_groups": 5, "fwd_queue_blocks": 8, "fwd_unroll": 4},
        {"fwd_groups": 5, "fwd_queue_blocks": 12, "fwd_unroll": 3},
        {"fwd_groups": 5, "fwd_queue_blocks": 12, "fwd_unroll": 4},
        {"fwd_groups": 5, "fwd_queue_blocks": 16, "fwd_unroll": 2},
        {"fwd_groups": 1, "fwd_queue_blocks": 16, "fwd_unroll": 3, "fwd_items_per_warp": 3},
        {"fwd_groups": 5, "fwd_chunk_vec": 8, "fwd_items_per_warp": 1},
    ],
)
def test_forward_tuning_variants_bit_exact(cuda, params):
    white, _, T = feature_batch(400, "Full_Threats+HalfKAv2_hm^", seed=12)
    C = 1048
    W = random_table(T, C, seed=13)
    bias = random_table(1, C, seed=14)[0]
    old = {k: _native.get_param(k) for k in params}
    try:
        for k, v in params.items():
            _native.set_param(k, v)
        got = _fwd(white, W, bias, cuda)
    finally:
        for k, v in old.items():
            _native.set_param(k, v)
    np.testing.assert_array_equal(got, oracle.ft_forward(white, W, bias))


def test_forward_out_of_range_index_is_skipped_and_flagged(cuda):
    T, C, B, K = 40, 16, 20, 6
    idx = random_indices(B, K, T, seed=3)
    bad = idx.copy()
    bad[2, 0] = T  # one past the table
    bad[5, 3] = -7  # negative other than -1
    W = random_table(T, C, seed=4)
    bias = random_table(1, C, seed=5)[0]
    _native.device_errors(clear=True)
    got = _fwd(bad, W, bias, cuda)
    flags = _native.device_errors(clear=True)
    assert flags & _native.DEVERR_BAD_INDEX
    clean = bad.copy()
    clean[(clean < -1) | (clean >= T)] = -1
    np.testing.assert_array_equal(got, oracle.ft_forward(clean, W, bias))
    # a clean call raises nothing
    _fwd(idx, W, bias, cuda)
    assert _native.device_errors(clear=True) == 0


@pytest.mark.parametrize("C,tail", [(1048, 6), (264, 2), (140, 3), (144, 4), (160, 8), (132, 1)])  # tail 1: not packed
@pytest.mark.parametrize("K", [32, 160])
def test_forward_packed_tail_chunk(cuda, C, tail, K):
    """The narrow last column chunk packed 32 // tail items per warp
    (ft_forward_tail_kernel): every width it is built for, one or five index
    groups per item, a batch that does not fill the last packed group, both
    the single and the pair forward; bit-exact against the oracle and equal
    to the unpacked chunk."""
    assert (C // 4) % 32 == tail
    T, B = 3000, 1001
    idx0 = random_indices(B, K, T, seed=C + K)
    idx1 = random_indices(B, K, T, seed=C + K + 1)
    W = random_table(T, C, seed=K, std=1.0)
    bias = random_table(1, C, seed=C, std=1.0)[0]
    dW, db = torch.from_numpy(W).to(cuda), torch.from_numpy(bias).to(cuda)
    i0, i1 = torch.from_numpy(idx0).to(cuda), torch.from_numpy(idx1).to(cuda)
    results = {}
    for packed in (3, 2, 1, 0):  # large-batch auto, side stream, caller's stream, not packed
        old = _native.get_param("fwd_tail")
        _native.set_param("fwd_tail", packed)
        try:
            o0 = torch.empty(B, C, device=cuda)
            o1 = torch.empty_like(o0)
            ops.forward_pair_into(i0, i1, dW, db, o0, o1)
            single = _fwd(idx0, W, bias, cuda)
            p0, p1 = torch.empty_like(o0), torch.empty_like(o0)  # the prepare form forks a side stream
            ops.forward_pair_prepare(i0, i1, dW, db, p0, p1, ops.alloc_workspace(B, K, T, C, 2, cuda))
            torch.cuda.synchronize()
        finally:
            _native.set_param("fwd_tail", old)
        results[packed] = (o0.cpu().numpy(), o1.cpu().numpy(), single, p0.cpu().numpy(), p1.cpu().numpy())
    np.testing.assert_array_equal(results[1][0], oracle.ft_forward(idx0, W, bias))
    np.testing.assert_array_equal(results[1][1], oracle.ft_forward(idx1, W, bias))
    np.testing.assert_array_equal(results[1][2], results[1][0])
    for packed in (3, 2, 1):
        for a, b in zip(results[packed], results[0]):
            np.testing.assert_array_equal(a, b)
