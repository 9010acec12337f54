"""int16 quantised forward and the export + quantisation that feeds it,
bit-exact against the oracle (pinned to the reference serializer's
quantisation by tests/golden/quantize_ft.npz and export_weights.npz)."""

import numpy as np
import pytest
import torch

import oracle
from stockfish_trainer_b200.feature_transformer import ops

from _inputs import feature_batch, random_table

pytestmark = pytest.mark.gpu

L1, NP = 1040, 8


def _tables(seed):
    W = random_table(24576, L1 + NP, seed=seed, std=0.01)
    W[:, L1:] = random_table(24576, NP, seed=seed + 1, std=0.3)  # PSQT columns carry larger values
    V = random_table(768, L1 + NP, seed=seed + 2, std=0.002)
    return W, V


def test_export_quantize_matches_reference_path(cuda):
    W, V = _tables(101)
    wq, pq = ops.halfka_export_quantize(torch.from_numpy(W).to(cuda), torch.from_numpy(V).to(cuda), L1)
    export = oracle.halfka_export_weights(W, V)
    np.testing.assert_array_equal(wq.cpu().numpy(), oracle.quantize(export[:, :L1], 255.0, np.int16))
    np.testing.assert_array_equal(pq.cpu().numpy(), oracle.quantize(export[:, L1:], 9600.0, np.int32))


def test_quantize_bias_matches_golden(cuda, golden):
    q = golden("quantize_ft.npz")
    got = ops.quantize_i16(torch.from_numpy(q["bias"]).to(cuda), float(q["ft_quantized_one"]))
    np.testing.assert_array_equal(got.cpu().numpy(), q["q_bias"])
    got = ops.quantize_i16(torch.from_numpy(q["weight"]).to(cuda), float(q["ft_quantized_one"]))
    np.testing.assert_array_equal(got.cpu().numpy(), q["q_weight"])


@pytest.mark.parametrize("map_training", [True, False])
def test_quantized_forward_bit_exact(cuda, map_training):
    white, black, _ = feature_batch(2000, "HalfKAv2_hm^", seed=111)
    W, V = _tables(112)
    export = oracle.halfka_export_weights(W, V)
    wq = oracle.quantize(export[:, :L1], 255.0, np.int16)
    pq = oracle.quantize(export[:, L1:], 9600.0, np.int32)
    bq = oracle.quantize(random_table(1, L1, seed=113, std=0.05)[0], 255.0, np.int16)
    if not map_training:
        white = np.where(white >= 0, oracle.halfka_export_rows(np.maximum(white, 0)), -1).astype(np.int32)
        black = np.where(black >= 0, oracle.halfka_export_rows(np.maximum(black, 0)), -1).astype(np.int32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    a0, a1, p0, p1 = ops.quantized_forward_pair(t(white), t(black), t(wq), t(pq), t(bq), map_training)
    for idx, acc, ps in ((white, a0, p0), (black, a1, p1)):
        ra, rp = oracle.ft_quantized_forward(idx, wq, pq, bq, map_training)
        np.testing.assert_array_equal(acc.cpu().numpy(), ra)
        np.testing.assert_array_equal(ps.cpu().numpy(), rp)


def test_quantized_forward_wraps_like_int16(cuda):
    rng = np.random.default_rng(5)
    Tq, L, P_, B, K = 64, 16, 4, 200, 40
    wq = rng.integers(-32768, 32767, size=(Tq, L), dtype=np.int16)
    pq = rng.integers(-2**31, 2**31 - 1, size=(Tq, P_), dtype=np.int64).astype(np.int32)
    bq = rng.integers(-32768, 32767, size=L, dtype=np.int16)
    idx = rng.integers(-1, Tq, size=(B, K)).astype(np.int32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    acc, ps = ops.quantized_forward_pair(t(idx), None, t(wq), t(pq), t(bq), False)
    ra, rp = oracle.ft_quantized_forward(idx, wq, pq, bq, False)
    np.testing.assert_array_equal(acc.cpu().numpy(), ra)
    np.testing.assert_array_equal(ps.cpu().numpy(), rp)


def test_quantized_forward_full_size(cuda):
    """The int16 configuration at full size: HalfKAv2_hm^, B = 65536 positions,
    both perspectives, export tables 22528 x (1040 int16 + 8 int32), every
    accumulator and PSQT value."""
    white, black, _ = feature_batch(65536, "HalfKAv2_hm^", seed=2024)
    W, V = _tables(2025)
    export = oracle.halfka_export_weights(W, V)
    wq = oracle.quantize(export[:, :L1], 255.0, np.int16)
    pq = oracle.quantize(export[:, L1:], 9600.0, np.int32)
    bq = oracle.quantize(random_table(1, L1, seed=2026, std=0.05)[0], 255.0, np.int16)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    a0, a1, p0, p1 = ops.quantized_forward_pair(t(white), t(black), t(wq), t(pq), t(bq), True)
    for idx, acc, ps in ((white, a0, p0), (black, a1, p1)):
        ra, rp = oracle.ft_quantized_forward(idx, wq, pq, bq, True)
        np.testing.assert_array_equal(acc.cpu().numpy(), ra)
        np.testing.assert_array_equal(ps.cpu().numpy(), rp)
