"""Fused FT epilogue (nnue_ft_epilogue_forward / _backward through
TransformInputsFunction) vs the PyTorch fp32 oracle of model.py:93-115 and its
autograd gradients: bit for bit, zero signs included."""

import numpy as np
import pytest
import torch

from oracle import epilogue as oracle_epi
from stockfish_trainer_b200 import _native
from stockfish_trainer_b200.feature_transformer import transform_inputs

pytestmark = pytest.mark.gpu


def _bits(t):
    return np.ascontiguousarray(t.detach().cpu().numpy(), dtype=np.float32).view(np.int32)


def _inputs(B, L1, NP, seed, specials=True):
    g = torch.Generator().manual_seed(seed)
    wp = torch.randn(B, L1 + NP, generator=g) * 0.8 + 0.4
    bp = torch.randn(B, L1 + NP, generator=g) * 0.8 + 0.4
    if specials and L1 >= 6:
        wp[0, :6] = torch.tensor([0.0, 1.0, -0.0, 1.5, -0.25, 0.5])
        bp[min(1, B - 1), :6] = torch.tensor([1.0, 0.0, 2.0, -0.0, 0.999, 1e-30])
    us = (torch.rand(B, 1, generator=g) < 0.5).float()
    pidx = torch.randint(0, NP, (B,), generator=g)
    d_l0 = torch.randn(B, L1, generator=g)
    d_psqt = torch.randn(B, 1, generator=g)
    if specials:
        d_l0[0, :2] = torch.tensor([-0.0, 0.0])
        d_psqt[0, 0] = -0.0
    return wp, bp, us, pidx, d_l0, d_psqt


def _run(wp, bp, us, pidx, d_l0, d_psqt, L1, dev):
    wpd = wp.to(dev).requires_grad_()
    bpd = bp.to(dev).requires_grad_()
    l0, psqt = transform_inputs(wpd, bpd, us.to(dev), pidx.to(dev), L1)
    torch.autograd.backward([l0, psqt], [d_l0.to(dev), d_psqt.to(dev)])
    torch.cuda.synchronize()
    return l0, psqt, wpd.grad, bpd.grad


@pytest.mark.parametrize("B,L1,NP", [(2048, 1040, 8), (100, 24, 8), (77, 18, 3), (5, 2, 1)])
def test_epilogue_matches_torch_graph(cuda, B, L1, NP):
    wp, bp, us, pidx, d_l0, d_psqt = _inputs(B, L1, NP, seed=B + L1)
    got = _run(wp, bp, us, pidx, d_l0, d_psqt, L1, cuda)
    want = oracle_epi.forward_backward(wp, bp, us, pidx, L1, d_l0, d_psqt)
    for g, w, name in zip(got, want, ("l0", "psqt", "d_wp", "d_bp")):
        np.testing.assert_array_equal(_bits(g), _bits(w), err_msg=name)


def test_epilogue_only_psqt_used(cuda):
    """l0 unused: autograd hands the backward a zero l0 gradient."""
    wp, bp, us, pidx, _, d_psqt = _inputs(64, 1040, 8, seed=3)
    wpd = wp.to(cuda).requires_grad_()
    bpd = bp.to(cuda).requires_grad_()
    _, psqt = transform_inputs(wpd, bpd, us.to(cuda), pidx.to(cuda), 1040)
    psqt.backward(d_psqt.to(cuda))
    wpc = wp.clone().requires_grad_()
    bpc = bp.clone().requires_grad_()
    _, ps = oracle_epi.transform(wpc, bpc, us, pidx, 1040)
    ps.backward(d_psqt)
    np.testing.assert_array_equal(_bits(wpd.grad), _bits(wpc.grad))
    np.testing.assert_array_equal(_bits(bpd.grad), _bits(bpc.grad))


def test_epilogue_misaligned_uses_scalar_path(cuda):
    B, L1, NP = 50, 1040, 8
    wp, bp, us, pidx, d_l0, d_psqt = _inputs(B, L1, NP, seed=11)
    buf = torch.zeros(2, B * (L1 + NP) + 1, device=cuda)
    wv = buf[0, 1:].view(B, L1 + NP)  # 4-byte offset
    bv = buf[1, 1:].view(B, L1 + NP)
    wv.copy_(wp)
    bv.copy_(bp)
    l0, psqt = transform_inputs(wv, bv, us.to(cuda), pidx.to(cuda), L1)
    want_l0, want_psqt = oracle_epi.transform(wp, bp, us, pidx, L1)
    np.testing.assert_array_equal(_bits(l0), _bits(want_l0))
    np.testing.assert_array_equal(_bits(psqt), _bits(want_psqt))


def test_epilogue_nan_propagates_like_torch(cuda):
    wp, bp, us, pidx, d_l0, d_psqt = _inputs(16, 24, 8, seed=5)
    wp[3, 2] = float("nan")
    bp[4, 20] = float("nan")
    got = _run(wp, bp, us, pidx, d_l0, d_psqt, 24, cuda)
    want = oracle_epi.forward_backward(wp, bp, us, pidx, 24, d_l0, d_psqt)
    for g, w in zip(got, want):
        g, w = g.detach().cpu().numpy(), w.numpy()
        np.testing.assert_array_equal(np.isnan(g), np.isnan(w))
        np.testing.assert_array_equal(np.where(np.isnan(g), 0, g), np.where(np.isnan(w), 0, w))


def test_epilogue_bad_psqt_index_is_flagged(cuda):
    wp, bp, us, pidx, d_l0, d_psqt = _inputs(8, 24, 8, seed=9)
    pidx[2] = 8  # out of range
    _native.device_errors(clear=True)
    l0, psqt = transform_inputs(wp.to(cuda), bp.to(cuda), us.to(cuda), pidx.to(cuda), 24)
    torch.cuda.synchronize()
    assert _native.device_errors(clear=True) & _native.DEVERR_BAD_PSQT_INDEX
    assert float(psqt[2, 0]) == 0.0
