"""Backward (device CSR build + segment sums + bias column sum) vs the oracle.

dW is bit-exact: each feature's sum runs over positions in ascending order,
like the reference's stable sort + sequential segment kernel, and the two
perspectives are added once, like autograd adds the reference's two dense
gradients.  dB is compared with |a - b| <= 1e-6 + 1e-5 |b| (torch's column
sum order is not reproducible)."""

import numpy as np
import pytest
import torch

import oracle
from stockfish_trainer_b200 import _native
from stockfish_trainer_b200.feature_transformer import ops

from _inputs import feature_batch, random_indices, random_table

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6


def _grads(B, C, seed):
    rng = np.random.default_rng(seed)
    return rng.standard_normal((B, C), dtype=np.float32), rng.standard_normal((B, C), dtype=np.float32)


def _bwd_pair(i0, i1, g0, g1, T, dev, accumulate=False, dW0=None, dB0=None):
    C = g0.shape[1]
    dW = torch.from_numpy(dW0).to(dev) if dW0 is not None else torch.full((T, C), float("nan"), device=dev)
    dB = torch.from_numpy(dB0).to(dev) if dB0 is not None else torch.full((C,), float("nan"), device=dev)
    t = lambda a: None if a is None else torch.from_numpy(a).to(dev)
    ops.backward_into(t(i0), t(i1), t(g0), t(g1), dW, dB, accumulate=accumulate)
    return dW.cpu().numpy(), dB.cpu().numpy()


@pytest.mark.parametrize("fs,B", [("HalfKAv2_hm^", 1500), ("Full_Threats+HalfKAv2_hm^", 800)])
def test_backward_pair_matches_reference_module_gradient(cuda, fs, B):
    white, black, T = feature_batch(B, fs, seed=21)
    C = 1048
    g0, g1 = _grads(B, C, 22)
    dW, dB = _bwd_pair(white, black, g0, g1, T, cuda)
    rW, rB = oracle.ft_backward_pair(white, black, g0, g1, T)
    np.testing.assert_array_equal(dW, rW)
    np.testing.assert_allclose(dB, rB, rtol=RTOL, atol=ATOL)


def test_backward_single_perspective_accumulates_like_reference_kernel(cuda):
    T, C, B, K = 500, 72, 900, 20
    idx = random_indices(B, K, T, seed=5)
    g, _ = _grads(B, C, 6)
    dW0 = random_table(T, C, seed=7, std=1.0)
    dB0 = random_table(1, C, seed=8, std=1.0)[0]
    dW, dB = _bwd_pair(idx, None, g, None, T, cuda, accumulate=True, dW0=dW0, dB0=dB0)
    rW, rB = oracle.ft_backward(idx, g, T, dW0.copy(), dB0.copy())
    np.testing.assert_array_equal(dW, rW)
    np.testing.assert_allclose(dB, rB, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("C", [13, 4, 1, 36, 300])
def test_backward_shapes(cuda, C):
    T, B, K = 200, 333, 33
    i0 = random_indices(B, K, T, seed=C)
    i1 = random_indices(B, K, T, seed=C + 1)
    g0, g1 = _grads(B, C, C + 2)
    dW, dB = _bwd_pair(i0, i1, g0, g1, T, cuda)
    rW, rB = oracle.ft_backward_pair(i0, i1, g0, g1, T)
    np.testing.assert_array_equal(dW, rW)
    np.testing.assert_allclose(dB, rB, rtol=RTOL, atol=ATOL)


def _with_params(params, fn):
    old = {k: _native.get_param(k) for k in params}
    try:
        for k, v in params.items():
            _native.set_param(k, v)
        return fn()
    finally:
        for k, v in old.items():
            _native.set_param(k, v)


@pytest.mark.parametrize(
    "params",
    [
        {"heavy_threshold": 4, "heavy_cap": 3},  # heavy rows overflow to the light path
        {"heavy_threshold": 1, "heavy_cap": 100000},  # nearly every row heavy
        {"heavy_threshold": 10**9},  # no heavy rows
        {},
        {"bwd_exact_chunks": 1},
        {"bwd_chunk_vec": 64, "bwd_exact_chunks": 1},
        {"bwd_chunk_vec": 8},
        {"bwd_chunk_vec": 0},
        {"bwd_chunk_vec": 32},
        {"bwd_chunk_vec": 128},
        {"bwd_chunk_vec": 1000},
        {"sort_blocks_per_sm": 1},
        {"sort_blocks_per_sm": 64},
        {"colsum_parts": 1},
        {"bwd_queue": 0, "bwd_unroll": 2, "bwd_min_blocks": 8},
        {"bwd_queue": 0, "bwd_unroll": 8, "bwd_min_blocks": 4},
        {"bwd_queue": 0, "bwd_unroll": 4, "bwd_min_blocks": 0},
        {"bwd_unroll": 4, "bwd_min_blocks": 5, "bwd_chunk_vec": 64, "bwd_exact_chunks": 1},
        {"bwd_queue": 0, "bwd_block": 256},
        {"bwd_queue": 0, "bwd_block": 128},
        {"bwd_queue": 0, "bwd_block": 64},
        {"bwd_queue": 0, "heavy_threshold": 4, "heavy_cap": 3},
        {"bwd_queue": 2, "bwd_queue_min_blocks": 16, "bwd_queue_min_entries": 0},
        {"bwd_queue": 3, "bwd_queue_min_blocks": 16, "bwd_queue_min_entries": 0},
        {"bwd_queue": 3, "bwd_queue_min_blocks": 12, "bwd_queue_min_entries": 0},
        {"bwd_queue": 4, "bwd_queue_min_blocks": 16, "bwd_queue_min_entries": 0},
        {"bwd_queue": 4, "bwd_queue_min_blocks": 12, "bwd_queue_min_entries": 0},
        {"bwd_queue": 4, "bwd_queue_min_blocks": 8, "bwd_queue_min_entries": 0},
        {"bwd_queue": 6, "bwd_queue_min_blocks": 12, "bwd_queue_min_entries": 0},
        {"bwd_queue": 6, "bwd_queue_min_blocks": 8, "bwd_queue_min_entries": 0},
        {"bwd_queue": 2, "bwd_block": 64, "bwd_queue_min_entries": 0},
        {"bwd_queue": 3, "bwd_block": 64, "bwd_queue_min_entries": 0},
        # rows > 256 entries (the long-row path) and > 32 per perspective (the list path)
        {"bwd_queue": 6, "bwd_queue_min_blocks": 8, "heavy_threshold": 4, "heavy_cap": 3, "bwd_queue_min_entries": 0},
        {"bwd_queue": 2, "heavy_threshold": 10**9, "bwd_queue_min_entries": 0},  # hot rows on the queued path
        {"bwd_queue": 6, "bwd_queue_min_blocks": 8, "bwd_chunk_vec": 8, "bwd_queue_min_entries": 0},
        {"bwd_queue": 2, "bwd_queue_min_entries": 10**9},  # the heuristic picks the batched kernel
        # heavy rows before the packed tail chunk on the side stream, and alone on the caller's stream
        {"bwd_heavy_first": 1, "heavy_threshold": 4, "heavy_cap": 40},
        {"bwd_heavy_first": 2, "heavy_threshold": 4, "heavy_cap": 40},
        {"bwd_heavy_first": 2, "bwd_tail": 1, "heavy_threshold": 4, "heavy_cap": 3},
    ],
)
def test_backward_tuning_and_heavy_rows(cuda, params):
    B, C = 3000, 264
    T = 700
    i0 = random_indices(B, 12, T, seed=31, holes=False)
    i1 = random_indices(B, 12, T, seed=32)
    i0[:, 0] = 5  # a feature every position uses: 3000-long serial segment
    i1[::2, 5] = 699
    g0, g1 = _grads(B, C, 33)
    # duplicates inside a row are legal: each (position, slot) entry counts once
    dW, dB = _with_params(params, lambda: _bwd_pair(i0, i1, g0, g1, T, cuda))
    rW, rB = oracle.ft_backward_pair(i0, i1, g0, g1, T)
    np.testing.assert_array_equal(dW, rW)
    np.testing.assert_allclose(dB, rB, rtol=RTOL, atol=ATOL)


def test_backward_misaligned_gradients_use_scalar_path(cuda):
    T, C, B, K = 400, 2052, 500, 10
    i0 = random_indices(B, K, T, seed=17)
    i1 = random_indices(B, K, T, seed=18)
    i0[:, 0] = 3  # one heavy row
    g0, g1 = _grads(B, C, 19)
    buf = torch.zeros(2 * B * C + 1, device=cuda)
    d0 = buf[1:1 + B * C].view(B, C)  # 4-byte offset: scalar path
    d1 = buf[1 + B * C:].view(B, C)
    d0.copy_(torch.from_numpy(g0))
    d1.copy_(torch.from_numpy(g1))
    dW = torch.empty(T, C, device=cuda)
    dB = torch.empty(C, device=cuda)
    ops.backward_into(torch.from_numpy(i0).to(cuda), torch.from_numpy(i1).to(cuda), d0, d1, dW, dB,
                      accumulate=False)
    rW, rB = oracle.ft_backward_pair(i0, i1, g0, g1, T)
    np.testing.assert_array_equal(dW.cpu().numpy(), rW)
    np.testing.assert_allclose(dB.cpu().numpy(), rB, rtol=RTOL, atol=ATOL)


def test_backward_small_and_large_key_spaces(cuda):
    # T * P keys from 200 to 1.2 M: one scan block to many
    for T, C in ((100, 8), (600_000, 4)):
        B, K = 1200, 9
        i0 = random_indices(B, K, T, seed=T % 97)
        i1 = random_indices(B, K, T, seed=T % 89)
        g0, g1 = _grads(B, C, 3)
        dW, dB = _bwd_pair(i0, i1, g0, g1, T, cuda)
        rW, rB = oracle.ft_backward_pair(i0, i1, g0, g1, T)
        np.testing.assert_array_equal(dW, rW)
        np.testing.assert_allclose(dB, rB, rtol=RTOL, atol=ATOL)


def test_backward_is_deterministic(cuda):
    white, black, T = feature_batch(2000, "Full_Threats+HalfKAv2_hm^", seed=41)
    g0, g1 = _grads(2000, 1048, 42)
    a = _bwd_pair(white, black, g0, g1, T, cuda)
    b = _bwd_pair(white, black, g0, g1, T, cuda)
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])


def test_backward_all_empty(cuda):
    T, C, B, K = 64, 20, 10, 4
    idx = np.full((B, K), -1, np.int32)
    g0, g1 = _grads(B, C, 1)
    dW, dB = _bwd_pair(idx, idx, g0, g1, T, cuda)
    assert np.all(dW == 0)
    np.testing.assert_allclose(dB, g0.astype(np.float64).sum(0) + g1.astype(np.float64).sum(0), rtol=RTOL, atol=ATOL)


def test_backward_bad_index_is_skipped_and_flagged(cuda):
    T, C, B, K = 90, 16, 120, 8
    idx = random_indices(B, K, T, seed=9)
    bad = idx.copy()
    bad[3, 1] = T + 5
    bad[7, 2] = -3
    g0, _ = _grads(B, C, 10)
    _native.device_errors(clear=True)
    dW, dB = _bwd_pair(bad, None, g0, None, T, cuda)
    assert _native.device_errors(clear=True) & _native.DEVERR_BAD_INDEX
    clean = bad.copy()
    clean[(clean < -1) | (clean >= T)] = -1
    rW, rB = oracle.ft_backward(clean, g0, T)
    np.testing.assert_array_equal(dW, rW)


def test_backward_workspace_too_small_raises(cuda):
    T, C, B, K = 50, 8, 10, 4
    idx = torch.from_numpy(random_indices(B, K, T, seed=1)).to(cuda)
    ws = torch.empty(64, dtype=torch.uint8, device=cuda)
    with pytest.raises(_native.NativeError):
        ops.backward_prepare(idx, None, T, C, ws)


def test_forward_pair_prepare_then_apply(cuda):
    """The fused forward + concurrent index phase feeds apply exactly like the
    separate calls."""
    white, black, T = feature_batch(1500, "Full_Threats+HalfKAv2_hm^", seed=71)
    B, C, K = 1500, 1048, white.shape[1]
    rng = np.random.default_rng(72)
    W = torch.from_numpy(rng.standard_normal((T, C), dtype=np.float32) * np.float32(0.01)).to(cuda)
    bias = torch.zeros(C, device=cuda)
    g0, g1 = _grads(B, C, 73)
    i0, i1 = torch.from_numpy(white).to(cuda), torch.from_numpy(black).to(cuda)
    o0 = torch.empty(B, C, device=cuda)
    o1 = torch.empty_like(o0)
    ws = ops.alloc_workspace(B, K, T, C, 2, cuda)
    ops.forward_pair_prepare(i0, i1, W, bias, o0, o1, ws)
    dW = torch.empty(T, C, device=cuda)
    dB = torch.empty(C, device=cuda)
    ops.backward_apply(torch.from_numpy(g0).to(cuda), torch.from_numpy(g1).to(cuda), B, K, dW, dB, False, ws)
    Wn = W.cpu().numpy()
    np.testing.assert_array_equal(o0.cpu().numpy(), oracle.ft_forward(white, Wn, bias.cpu().numpy()))
    rW, rB = oracle.ft_backward_pair(white, black, g0, g1, T)
    np.testing.assert_array_equal(dW.cpu().numpy(), rW)
    np.testing.assert_allclose(dB.cpu().numpy(), rB, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("B,T", [(5000, 50), (9000, 50), (20000, 50), (40000, 500)])
def test_backward_long_segments(cuda, B, T):
    """Segments longer than one warp's sort (256) and than one block's shared
    memory (8192), with repeated positions inside a segment; counted in one
    or several position windows, or (B = 40000: ~320 per key) sorted by the
    block network."""
    C, K = 8, 4
    i0 = random_indices(B, K, T, seed=41)
    i1 = random_indices(B, K, T, seed=42)
    i0[:, 0] = 7  # every position
    i0[::3, 1] = 7  # a third of them twice
    i1[:, 2] = 7
    g0, g1 = _grads(B, C, 43)
    dW, dB = _bwd_pair(i0, i1, g0, g1, T, cuda)
    rW, rB = oracle.ft_backward_pair(i0, i1, g0, g1, T)
    np.testing.assert_array_equal(dW, rW)
    np.testing.assert_allclose(dB, rB, rtol=RTOL, atol=ATOL)



@pytest.mark.parametrize("queue", [0, 2, 6])
def test_backward_gradients_in_reverse_memory_order(cuda, queue):
    """The two perspectives' output gradients as views of one tensor, the
    second below the first in memory: the queued light rows address both from
    the first one's base with a negative distance."""
    B, C, T = 2000, 1048, 24576
    white, black, _ = feature_batch(B, "HalfKAv2_hm^", seed=61)
    g = torch.randn(2, B, C, device=cuda, generator=torch.Generator(device=cuda).manual_seed(62))
    g0, g1 = g[1], g[0]  # perspective 1's gradient sits before perspective 0's
    dW = torch.empty(T, C, device=cuda)
    dB = torch.empty(C, device=cuda)
    t = lambda a: torch.from_numpy(a).to(cuda)
    _with_params({"bwd_queue": queue, "bwd_queue_min_blocks": 8, "bwd_queue_min_entries": 0},
                 lambda: ops.backward_into(t(white), t(black), g0, g1, dW, dB, accumulate=False))
    rW, rB = oracle.ft_backward_pair(white, black, g0.cpu().numpy(), g1.cpu().numpy(), T)
    np.testing.assert_array_equal(dW.cpu().numpy(), rW)
    np.testing.assert_allclose(dB.cpu().numpy(), rB, rtol=RTOL, atol=ATOL)


def test_backward_rejects_max_active_beyond_counters(cuda):
    """The per-segment sort counts repeats of a position in 16-bit counters,
    so max_active >= 65536 is refused instead of mis-sorted."""
    lib = _native.load()
    assert lib.nnue_ft_backward_workspace_size(4, 65536, 100, 8, 2) == 0


@pytest.mark.parametrize("C,tail", [(1048, 6), (264, 2), (140, 3), (144, 4), (160, 8)])
@pytest.mark.parametrize("case", ["plain", "heavy_in_warp", "long_light_rows", "accumulate"])
def test_backward_packed_tail_chunk(cuda, C, tail, case):
    """The light rows' narrow last column chunk packed 32 // tail rows per
    warp (ft_segsum_tail_kernel): every width it is built for; a hot row
    inside a packed warp and rows past the heavy-row cap (both take the
    direct path); accumulate mode.  Bit-exact against the oracle and equal to
    the unpacked chunk."""
    assert (C // 4) % 32 == tail
    T, B, K = 700, 2500, 12
    i0 = random_indices(B, K, T, seed=C + 1)
    i1 = random_indices(B, K, T, seed=C + 2)
    params = {"bwd_queue_min_entries": 0}
    if case in ("heavy_in_warp", "long_light_rows"):
        i0[:, 0] = 17  # hot rows in the middle of a packed group
        i1[::2, 3] = 18
        i1[1::2, 3] = 503
    if case == "long_light_rows":
        params.update(heavy_threshold=4, heavy_cap=1)
    g0, g1 = _grads(B, C, C + 3)
    acc = case == "accumulate"
    dW0 = random_table(T, C, seed=5, std=1.0) if acc else None
    dB0 = random_table(1, C, seed=6, std=1.0)[0] if acc else None
    got = {}
    for packed in (2, 1, 0):  # side stream, caller's stream, not packed
        p = dict(params, bwd_tail=packed)
        got[packed] = _with_params(p, lambda: _bwd_pair(i0, i1, g0, g1, T, cuda, accumulate=acc,
                                                        dW0=None if dW0 is None else dW0.copy(),
                                                        dB0=None if dB0 is None else dB0.copy()))
    if acc:
        rW, rB = oracle.ft_backward(i0, g0, T, dW0.copy(), dB0.copy())
        rW, rB = oracle.ft_backward(i1, g1, T, rW, rB)
    else:
        rW, rB = oracle.ft_backward_pair(i0, i1, g0, g1, T)
    np.testing.assert_array_equal(got[1][0], got[0][0])
    np.testing.assert_array_equal(got[2][0], got[0][0])
    if not acc:
        np.testing.assert_array_equal(got[1][0], rW)
    else:
        np.testing.assert_allclose(got[1][0], rW, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(got[1][1], rB, rtol=RTOL, atol=1e-5)
