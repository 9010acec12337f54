"""The FT's torch.library custom operators on the GPU: the same results as the
autograd functions (bit for bit), a torch.compile'd module using them with
fullgraph=True (a graph break would raise), and torch.library.opcheck of the
schema, the autograd registration and the fake implementations."""

import numpy as np
import pytest
import torch

from stockfish_trainer_b200 import SparseLinearFunction, SparseLinearPairFunction
from stockfish_trainer_b200.feature_transformer import sparse_linear, sparse_linear_pair

from _inputs import feature_batch, random_table

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6


def _inputs(cuda, B=1200, fs="Full_Threats+HalfKAv2_hm^", C=1048, seed=81):
    white, black, T = feature_batch(B, fs, seed=seed)
    W = torch.from_numpy(random_table(T, C, seed=seed + 1)).to(cuda)
    bias = torch.from_numpy(random_table(1, C, seed=seed + 2)[0]).to(cuda)
    rng = np.random.default_rng(seed + 3)
    g0 = torch.from_numpy(rng.standard_normal((B, C), dtype=np.float32)).to(cuda)
    g1 = torch.from_numpy(rng.standard_normal((B, C), dtype=np.float32)).to(cuda)
    return torch.from_numpy(white).to(cuda), torch.from_numpy(black).to(cuda), W, bias, g0, g1


def _grads(fn, W, bias, g0, g1):
    Wp, bp = W.clone().requires_grad_(), bias.clone().requires_grad_()
    o0, o1 = fn(Wp, bp)
    torch.autograd.backward([o0, o1], [g0, g1])
    return o0.detach(), o1.detach(), Wp.grad, bp.grad


def test_ops_equal_autograd_functions(cuda):
    i0, i1, W, bias, g0, g1 = _inputs(cuda)
    ref = _grads(lambda w, b: SparseLinearPairFunction.apply(i0, i1, w, b), W, bias, g0, g1)
    got = _grads(lambda w, b: sparse_linear_pair(i0, i1, w, b), W, bias, g0, g1)
    one = _grads(lambda w, b: (sparse_linear(i0, w, b), sparse_linear(i1, w, b)), W, bias, g0, g1)
    two = _grads(lambda w, b: (SparseLinearFunction.apply(i0, w, b), SparseLinearFunction.apply(i1, w, b)),
                 W, bias, g0, g1)
    for a, r in ((got, ref), (one, two), (one, ref)):
        assert torch.equal(a[0], r[0]) and torch.equal(a[1], r[1]) and torch.equal(a[2], r[2])
        torch.testing.assert_close(a[3], r[3], rtol=RTOL, atol=ATOL)


class _FT(torch.nn.Module):
    def __init__(self, W, bias, pair):
        super().__init__()
        self.weight = torch.nn.Parameter(W.clone())
        self.bias = torch.nn.Parameter(bias.clone())
        self.pair = pair

    def forward(self, i0, i1):
        if self.pair:
            o0, o1 = sparse_linear_pair(i0, i1, self.weight, self.bias)
        else:
            o0, o1 = sparse_linear(i0, self.weight, self.bias), sparse_linear(i1, self.weight, self.bias)
        # a little of the surrounding model, so the compiled graph has more than the op
        return torch.clamp(o0, 0.0, 1.0) * torch.clamp(o1, 0.0, 1.0)


@pytest.mark.parametrize("pair", [True, False])
def test_torch_compile_fullgraph(cuda, pair):
    torch._dynamo.reset()
    i0, i1, W, bias, g0, _ = _inputs(cuda, B=700, seed=91)
    eager = _FT(W, bias, pair).to(cuda)
    compiled = torch.compile(_FT(W, bias, pair).to(cuda), fullgraph=True)
    y_e = eager(i0, i1)
    y_c = compiled(i0, i1)
    y_e.backward(g0)
    y_c.backward(g0)
    assert torch.equal(y_e, y_c)
    assert torch.equal(eager.weight.grad, compiled.weight.grad)
    torch.testing.assert_close(eager.bias.grad, compiled.bias.grad, rtol=RTOL, atol=ATOL)


def test_opcheck(cuda):
    i0, i1, W, bias, _, _ = _inputs(cuda, B=300, fs="HalfKAv2_hm^", C=264, seed=101)
    utils = ("test_schema", "test_autograd_registration", "test_faketensor")
    torch.library.opcheck(torch.ops.nnue_ft.sparse_linear.default, (i0, W.requires_grad_(), bias), test_utils=utils)
    torch.library.opcheck(torch.ops.nnue_ft.sparse_linear_pair.default, (i0, i1, W, bias), test_utils=utils)
