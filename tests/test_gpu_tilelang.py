"""The reference's own TileLang kernels as the GPU checker of the fp32 math.

``oracle/_ref/ref_feature_transformer`` is the reference's feature-transformer
package (``src/model/modules/feature_transformer/{__init__,functions,kernel}.py``)
staged byte for byte by ``oracle/build.py``.  Its ``SparseLinearFunction``
runs the TileLang forward (``kernel.py:66-105``) and backward
(``kernel.py:108-188``, bias gradient ``:269``), JIT-compiled for this GPU and
autotuned at the first call.  Each case drives it the way the reference's
composed module does (two calls sharing one table, autograd summing the two
dense weight gradients, ``composed.py:52-53``) and compares it with:

* this library's timed path (``forward_pair_prepare`` + ``backward_apply``,
  the calls ``bench.py`` times), and
* the C oracle.

Forward outputs and the weight gradient must match bit for bit (same fp32
adds in the same order).  The bias gradient is a column sum: the reference
takes it with torch's fp32 ``sum(dim=0)`` (``kernel.py:269``), whose order
torch chooses, while this library sums in float64 and rounds once.  Both are
checked against float64 column sums S0, S1 of the two perspectives: this
library's against fp32(S0) + fp32(S1) (each perspective rounded once and the
two added in fp32, as autograd adds the reference's two gradients) within
|a - x| <= 1e-6 + 1e-5 |x|; the reference's against S0 + S1 within the error
bound of pairwise fp32 summation plus the final add,
1e-6 + ceil(log2 B) * 2^-24 * sum|terms| + 2^-24 |S0 + S1| (Higham,
"Accuracy and Stability of Numerical Algorithms", 2nd ed., section 4.2).
"""

import math

import numpy as np
import pytest
import torch

import oracle
from oracle import tilelang_ref
from stockfish_trainer_b200.feature_transformer import ops

from _inputs import feature_batch, random_indices, random_table

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6
C = 1048


@pytest.fixture(scope="module")
def ref():
    return tilelang_ref.load()


def _ours(i0, i1, W, bias, g0, g1):
    """This library's timed path: forward of both perspectives with the
    backward's index phase beside it, then the segment sums (dense dW, dB)."""
    B, K = i0.shape
    T = W.shape[0]
    out0, out1 = torch.empty(B, C, device=W.device), torch.empty(B, C, device=W.device)
    ws = ops.alloc_workspace(B, K, T, C, 2, W.device)
    ops.forward_pair_prepare(i0, i1, W, bias, out0, out1, ws)
    dW = torch.empty_like(W)
    dB = torch.empty(C, device=W.device)
    ops.backward_apply(g0, g1, B, K, dW, dB, False, ws)
    return out0, out1, dW, dB


def _compare(ref, white, black, T, seed, with_oracle=True):
    dev = torch.device("cuda", 0)
    B = white.shape[0]
    W = torch.from_numpy(random_table(T, C, seed=seed)).to(dev)
    bias = torch.from_numpy(random_table(1, C, seed=seed + 1)[0]).to(dev)
    rng = np.random.default_rng(seed + 2)
    g0 = torch.from_numpy(rng.standard_normal((B, C), dtype=np.float32)).to(dev)
    g1 = torch.from_numpy(rng.standard_normal((B, C), dtype=np.float32)).to(dev)
    i0, i1 = torch.from_numpy(white).to(dev), torch.from_numpy(black).to(dev)

    r0, r1, rW, rB = tilelang_ref.reference_pair_step(ref, i0, i1, W, bias, g0, g1)
    o0, o1, dW, dB = _ours(i0, i1, W, bias, g0, g1)
    torch.cuda.synchronize()
    assert torch.equal(o0, r0), "forward (perspective 0) differs from the reference TileLang kernel"
    assert torch.equal(o1, r1), "forward (perspective 1) differs from the reference TileLang kernel"
    assert torch.equal(dW, rW), "weight gradient differs from the reference TileLang kernels"
    s0, s1 = g0.double().sum(0), g1.double().sum(0)
    # each perspective's gradient rounded once to fp32, added once in fp32
    torch.testing.assert_close(dB, s0.float() + s1.float(), rtol=RTOL, atol=ATOL)
    u = 2.0 ** -24
    mass = g0.double().abs().sum(0) + g1.double().abs().sum(0)
    bound = 1e-6 + math.ceil(math.log2(B)) * u * mass + u * (s0 + s1).abs()
    assert bool(((rB.double() - (s0 + s1)).abs() <= bound).all()), "reference bias gradient outside the fp32 bound"
    if with_oracle:
        Wn, bn = W.cpu().numpy(), bias.cpu().numpy()
        np.testing.assert_array_equal(r0.cpu().numpy(), oracle.ft_forward(white, Wn, bn))
        np.testing.assert_array_equal(r1.cpu().numpy(), oracle.ft_forward(black, Wn, bn))
        oW, oB = oracle.ft_backward_pair(white, black, g0.cpu().numpy(), g1.cpu().numpy(), T)
        np.testing.assert_array_equal(rW.cpu().numpy(), oW)
        np.testing.assert_allclose(dB.cpu().numpy(), oB, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("feature_set,B,seed", [
    ("HalfKAv2_hm^", 1000, 11),
    ("Full_Threats+HalfKAv2_hm^", 1500, 21),
])
def test_tilelang_matches_on_encoded_positions(ref, feature_set, B, seed):
    white, black, T = feature_batch(B, feature_set, seed=seed)
    _compare(ref, white, black, T, seed + 100)


def test_tilelang_matches_with_holes_and_repeats(ref):
    """-1 anywhere in a row, a feature repeated inside one row, and a hot
    feature shared by every position (one long segment)."""
    T, K, B = 24576, 32, 700
    white = random_indices(B, K, T, seed=31, holes=True)
    black = random_indices(B, K, T, seed=32, holes=True)
    white[::3, 0] = 77  # hot row, in every third position
    black[:, 5] = 77
    white[5, 1:4] = 4242  # the same feature three times in one row
    _compare(ref, white, black, T, 33)


def test_tilelang_matches_at_headline_size(ref):
    """Full_Threats+HalfKAv2_hm^, B = 65536, K = 160, T = 85296, C = 1048:
    the bench's headline configuration, every output and every gradient row."""
    white, black, T = feature_batch(65536, "Full_Threats+HalfKAv2_hm^", seed=2024)
    _compare(ref, white, black, T, 2025, with_oracle=False)


def test_tilelang_matches_halfka_16384(ref):
    """HalfKAv2_hm^, B = 16384 (the bench's HalfKA configuration)."""
    white, black, T = feature_batch(16384, "HalfKAv2_hm^", seed=7)
    _compare(ref, white, black, T, 8, with_oracle=False)
