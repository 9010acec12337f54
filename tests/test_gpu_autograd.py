"""The reference-facing API: SparseLinearFunction, the pair function and the
kernel factories, driven through autograd like the reference's module does
(src/model/modules/features/composed.py:49-54, halfka_v2_hm.py:69-70)."""

import numpy as np
import pytest
import torch

import oracle
from stockfish_trainer_b200 import (
    SparseLinearFunction,
    SparseLinearPairFunction,
    make_sparse_input_linear_backward_kernel,
    make_sparse_input_linear_forward_kernel,
)

from _inputs import feature_batch, random_table

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6


def test_sparse_linear_function_autograd(cuda):
    white, _, T = feature_batch(900, "HalfKAv2_hm^", seed=51)
    C = 1048
    W = random_table(T, C, seed=52)
    bias = random_table(1, C, seed=53)[0]
    g = np.random.default_rng(54).standard_normal((900, C), dtype=np.float32)
    Wt = torch.from_numpy(W).to(cuda).requires_grad_()
    bt = torch.from_numpy(bias).to(cuda).requires_grad_()
    out = SparseLinearFunction.apply(torch.from_numpy(white).to(cuda), Wt, bt)
    np.testing.assert_array_equal(out.detach().cpu().numpy(), oracle.ft_forward(white, W, bias))
    out.backward(torch.from_numpy(g).to(cuda))
    rW, rB = oracle.ft_backward(white, g, T)
    np.testing.assert_array_equal(Wt.grad.cpu().numpy(), rW)
    np.testing.assert_allclose(bt.grad.cpu().numpy(), rB, rtol=RTOL, atol=ATOL)


def test_sparse_linear_function_rejects_reference_violations(cuda):
    W = torch.zeros(10, 8, device=cuda)
    b = torch.zeros(8, device=cuda)
    with pytest.raises(AssertionError):
        SparseLinearFunction.apply(torch.zeros(2, 3, dtype=torch.int64, device=cuda), W, b)
    with pytest.raises(AssertionError):
        SparseLinearFunction.apply(torch.zeros(2, 3, dtype=torch.int32), W, b)
    with pytest.raises(AssertionError):
        SparseLinearFunction.apply(torch.zeros(3, 2, dtype=torch.int32, device=cuda).t(), W, b)


def test_pair_function_equals_two_reference_calls(cuda):
    """One pair call == the reference's two SparseLinearFunction calls on a
    shared table, outputs and summed gradients bit for bit."""
    white, black, T = feature_batch(1200, "Full_Threats+HalfKAv2_hm^", seed=61)
    C = 1048
    W = torch.from_numpy(random_table(T, C, seed=62)).to(cuda)
    bias = torch.from_numpy(random_table(1, C, seed=63)[0]).to(cuda)
    rng = np.random.default_rng(64)
    g0 = torch.from_numpy(rng.standard_normal((1200, C), dtype=np.float32)).to(cuda)
    g1 = torch.from_numpy(rng.standard_normal((1200, C), dtype=np.float32)).to(cuda)
    i0, i1 = torch.from_numpy(white).to(cuda), torch.from_numpy(black).to(cuda)

    Wa, ba = W.clone().requires_grad_(), bias.clone().requires_grad_()
    o0, o1 = SparseLinearPairFunction.apply(i0, i1, Wa, ba)
    torch.autograd.backward([o0, o1], [g0, g1])

    Wb, bb = W.clone().requires_grad_(), bias.clone().requires_grad_()
    r0 = SparseLinearFunction.apply(i0, Wb, bb)
    r1 = SparseLinearFunction.apply(i1, Wb, bb)
    torch.autograd.backward([r0, r1], [g0, g1])

    assert torch.equal(o0, r0) and torch.equal(o1, r1)
    assert torch.equal(Wa.grad, Wb.grad)
    torch.testing.assert_close(ba.grad, bb.grad, rtol=RTOL, atol=ATOL)


def test_pair_function_one_output_unused(cuda):
    white, black, T = feature_batch(300, "HalfKAv2_hm^", seed=71)
    C = 64
    W = torch.from_numpy(random_table(T, C, seed=72)).to(cuda).requires_grad_()
    b = torch.zeros(C, device=cuda, requires_grad=True)
    o0, o1 = SparseLinearPairFunction.apply(torch.from_numpy(white).to(cuda), torch.from_numpy(black).to(cuda), W, b)
    g = torch.ones_like(o1)
    o1.backward(g)
    rW, rB = oracle.ft_backward(black, g.cpu().numpy(), T)
    np.testing.assert_array_equal(W.grad.cpu().numpy(), rW)


def test_kernel_factories_follow_reference_contract(cuda):
    """forward kernel WRITES output; backward kernel ACCUMULATES (kernel.py:184-186, :269)."""
    white, _, T = feature_batch(500, "HalfKAv2_hm^", seed=81)
    C = 1048
    W = random_table(T, C, seed=82)
    bias = random_table(1, C, seed=83)[0]
    fwd = make_sparse_input_linear_forward_kernel(32, C)
    bwd = make_sparse_input_linear_backward_kernel(32, C)
    assert make_sparse_input_linear_forward_kernel(32, C) is fwd
    idx = torch.from_numpy(white).to(cuda)
    out = torch.full((500, C), 7.0, device=cuda)
    fwd(idx, torch.from_numpy(W).to(cuda), torch.from_numpy(bias).to(cuda), out)
    np.testing.assert_array_equal(out.cpu().numpy(), oracle.ft_forward(white, W, bias))

    g = np.random.default_rng(84).standard_normal((500, C), dtype=np.float32)
    wg0 = random_table(T, C, seed=85, std=1.0)
    bg0 = random_table(1, C, seed=86, std=1.0)[0]
    wg, bg = torch.from_numpy(wg0).to(cuda), torch.from_numpy(bg0).to(cuda)
    bwd(idx, wg, bg, torch.from_numpy(g).to(cuda))
    rW, rB = oracle.ft_backward(white, g, T, wg0.copy(), bg0.copy())
    np.testing.assert_array_equal(wg.cpu().numpy(), rW)
    np.testing.assert_allclose(bg.cpu().numpy(), rB, rtol=RTOL, atol=ATOL)


def test_module_level_gradients_of_factorised_table(cuda):
    """composed.py:50 + halfka_v2_hm.py:69-70: merged = cat(threat, halfka + virtual.repeat(32, 1)).
    The threat / HalfKA slices of dW and the virtual gradient (sum over 32 buckets)."""
    white, black, T = feature_batch(600, "Full_Threats+HalfKAv2_hm^", seed=91)
    C = 24
    rng = np.random.default_rng(92)
    thr = torch.from_numpy(rng.standard_normal((60720, C), dtype=np.float32) * 0.01).to(cuda).requires_grad_()
    hka = torch.from_numpy(rng.standard_normal((24576, C), dtype=np.float32) * 0.01).to(cuda).requires_grad_()
    vir = torch.zeros(768, C, device=cuda, requires_grad=True)
    bias = torch.zeros(C, device=cuda, requires_grad=True)
    merged = torch.cat([thr, hka + vir.repeat(32, 1)], dim=0)
    o0, o1 = SparseLinearPairFunction.apply(torch.from_numpy(white).to(cuda), torch.from_numpy(black).to(cuda),
                                            merged, bias)
    g0 = rng.standard_normal((600, C), dtype=np.float32)
    g1 = rng.standard_normal((600, C), dtype=np.float32)
    torch.autograd.backward([o0, o1], [torch.from_numpy(g0).to(cuda), torch.from_numpy(g1).to(cuda)])
    rW, _ = oracle.ft_backward_pair(white, black, g0, g1, T)
    np.testing.assert_array_equal(thr.grad.cpu().numpy(), rW[:60720])
    np.testing.assert_array_equal(hka.grad.cpu().numpy(), rW[60720:])
    # The virtual gradient is torch's repeat-backward (reference module code,
    # not this library): feed the oracle's dW through the same graph and the
    # two must agree bit for bit.
    rW_t = torch.from_numpy(rW).to(cuda)

    class _OracleGrad(torch.autograd.Function):
        @staticmethod
        def forward(ctx, m):
            return m.sum()

        @staticmethod
        def backward(ctx, g):
            return rW_t

    vir2 = torch.zeros(768, C, device=cuda, requires_grad=True)
    merged2 = torch.cat([thr.detach(), hka.detach() + vir2.repeat(32, 1)], dim=0)
    _OracleGrad.apply(merged2).backward()
    assert torch.equal(vir.grad, vir2.grad)
    rV = rW[60720:].astype(np.float64).reshape(32, 768, C).sum(0)
    np.testing.assert_allclose(vir.grad.cpu().numpy(), rV, rtol=1e-4, atol=1e-5)
