"""Headline configuration (Full_Threats+HalfKAv2_hm^, B = 65536, L1 = 1040 + 8
PSQT, T = 85296) checked through properties that do not need a full CPU
recomputation: sampled positions / feature rows bit-exact against the oracle,
and column-sum identities in float64."""

import numpy as np
import pytest
import torch

import oracle
from stockfish_trainer_b200.feature_transformer import ops

from _inputs import feature_batch

pytestmark = pytest.mark.gpu

B, C = 65536, 1048


@pytest.fixture(scope="module")
def full(cuda):
    white, black, T = feature_batch(B, "Full_Threats+HalfKAv2_hm^", seed=2024)
    gen = torch.Generator(device=cuda).manual_seed(7)
    W = torch.randn(T, C, device=cuda, generator=gen) * 0.01
    bias = torch.zeros(C, device=cuda)
    g0 = torch.randn(B, C, device=cuda, generator=gen)
    g1 = torch.randn(B, C, device=cuda, generator=gen)
    i0, i1 = torch.from_numpy(white).to(cuda), torch.from_numpy(black).to(cuda)
    return dict(white=white, black=black, T=T, W=W, bias=bias, g0=g0, g1=g1, i0=i0, i1=i1)


def test_fullsize_forward_sampled_rows(full, cuda):
    o0 = torch.empty(B, C, device=cuda)
    o1 = torch.empty_like(o0)
    ops.forward_pair_into(full["i0"], full["i1"], full["W"], full["bias"], o0, o1)
    rows = np.random.default_rng(0).choice(B, 300, replace=False)
    W = full["W"].cpu().numpy()
    bias = full["bias"].cpu().numpy()
    for idx, out in ((full["white"], o0), (full["black"], o1)):
        np.testing.assert_array_equal(out[torch.from_numpy(rows).to(cuda)].cpu().numpy(),
                                      oracle.ft_forward(idx[rows], W, bias))


def test_fullsize_backward_sampled_features_and_sums(full, cuda):
    T = full["T"]
    dW = torch.empty(T, C, device=cuda)
    dB = torch.empty(C, device=cuda)
    ops.backward_into(full["i0"], full["i1"], full["g0"], full["g1"], dW, dB, accumulate=False)
    torch.cuda.synchronize()
    white, black = full["white"], full["black"]
    counts = np.bincount(np.concatenate([white[white >= 0], black[black >= 0]]), minlength=T)
    hot = np.argsort(counts)[-8:]  # includes the own-king rows (thousands of positions)
    rng = np.random.default_rng(1)
    sample = np.unique(np.concatenate([hot, rng.choice(T, 120, replace=False)]))
    keep = np.isin(white, sample)
    w_sub = np.where(keep, white, -1).astype(np.int32)
    keep = np.isin(black, sample)
    b_sub = np.where(keep, black, -1).astype(np.int32)
    g0 = full["g0"].cpu().numpy()
    g1 = full["g1"].cpu().numpy()
    rW, _ = oracle.ft_backward_pair(w_sub, b_sub, g0, g1, T)
    np.testing.assert_array_equal(dW[torch.from_numpy(sample).to(cuda)].cpu().numpy(), rW[sample])
    # bias gradient = column sums of both perspectives
    ref_b = g0.astype(np.float64).sum(0) + g1.astype(np.float64).sum(0)
    np.testing.assert_allclose(dB.cpu().numpy(), ref_b, rtol=1e-5, atol=1e-3)
    # sum over all feature rows of dW = sum_b n_active(b) * dOut[b] (float64)
    n0 = (white >= 0).sum(1).astype(np.float64)
    n1 = (black >= 0).sum(1).astype(np.float64)
    lhs = dW.double().sum(0).cpu().numpy()
    rhs = (n0[:, None] * g0).sum(0) + (n1[:, None] * g1).sum(0)
    np.testing.assert_allclose(lhs, rhs, rtol=1e-6, atol=1e-2)
