"""Full-size configurations, every tensor element, through the calls the bench
times (``forward_pair_prepare``: forward of both perspectives with the
backward's index phase beside it, then ``backward_apply``: the segment sums
into a dense weight gradient and the bias gradient), against the C oracle
(OpenMP) on the same inputs.

* Full_Threats+HalfKAv2_hm^, B = 65536, K = 160, T = 85296, C = 1048 (the
  headline);
* HalfKAv2_hm^, B = 16384, K = 32, T = 24576, C = 1048.

Two steps run back to back on one workspace, the second on other output
gradients, so anything the first step leaves behind in the workspace or in
the outputs would show.  Outputs and dW are compared bit for bit, dB within
|a - b| <= 1e-6 + 1e-5 |b|."""

import numpy as np
import pytest
import torch

import oracle
from stockfish_trainer_b200.feature_transformer import ops

from _inputs import feature_batch

pytestmark = pytest.mark.gpu

C = 1048
RTOL, ATOL = 1e-5, 1e-6


@pytest.mark.parametrize("feature_set,B,seed", [
    ("Full_Threats+HalfKAv2_hm^", 65536, 2024),
    ("HalfKAv2_hm^", 16384, 77),
])
def test_timed_path_every_element(cuda, feature_set, B, seed):
    white, black, T = feature_batch(B, feature_set, seed=seed)
    K = white.shape[1]
    gen = torch.Generator(device=cuda).manual_seed(seed + 1)
    W = torch.randn(T, C, device=cuda, generator=gen) * 0.01
    bias = torch.randn(C, device=cuda, generator=gen) * 0.01
    i0, i1 = torch.from_numpy(white).to(cuda), torch.from_numpy(black).to(cuda)
    o0 = torch.empty(B, C, device=cuda)
    o1 = torch.empty_like(o0)
    dW = torch.empty(T, C, device=cuda)
    dB = torch.empty(C, device=cuda)
    ws = ops.alloc_workspace(B, K, T, C, 2, cuda)
    Wn, bn = W.cpu().numpy(), bias.cpu().numpy()
    ref0 = oracle.ft_forward(white, Wn, bn)
    ref1 = oracle.ft_forward(black, Wn, bn)
    for step in range(2):
        g0 = torch.randn(B, C, device=cuda, generator=gen)
        g1 = torch.randn(B, C, device=cuda, generator=gen)
        ops.forward_pair_prepare(i0, i1, W, bias, o0, o1, ws)
        ops.backward_apply(g0, g1, B, K, dW, dB, False, ws)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(o0.cpu().numpy(), ref0, err_msg=f"forward 0, step {step}")
        np.testing.assert_array_equal(o1.cpu().numpy(), ref1, err_msg=f"forward 1, step {step}")
        rW, rB = oracle.ft_backward_pair(white, black, g0.cpu().numpy(), g1.cpu().numpy(), T)
        np.testing.assert_array_equal(dW.cpu().numpy(), rW, err_msg=f"weight gradient, step {step}")
        np.testing.assert_allclose(dB.cpu().numpy(), rB, rtol=RTOL, atol=ATOL, err_msg=f"bias gradient, step {step}")
