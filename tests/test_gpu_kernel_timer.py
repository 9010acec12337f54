"""The library's per-launch kernel timer (nnue_ft_kernel_timer_arm / _read):
every launch of an armed gather kernel class is bracketed by an event pair on
its own stream, unarmed classes record nothing, launches beyond the capacity
are not recorded, and timing changes no result."""

import pytest
import torch

from stockfish_trainer_b200 import _native
from stockfish_trainer_b200.feature_transformer import ops

from _inputs import feature_batch

pytestmark = pytest.mark.gpu


def _step(i0, i1, W, bias, out0, out1, g0, g1, dW, dB, ws, B, K):
    ops.forward_pair_prepare(i0, i1, W, bias, out0, out1, ws)
    ops.backward_apply(g0, g1, B, K, dW, dB, False, ws)


def test_kernel_timer_records_each_armed_launch(cuda):
    B, C = 2048, 1048
    white, black, T = feature_batch(B, "Full_Threats+HalfKAv2_hm^", seed=5)
    K = white.shape[1]
    g = torch.Generator(device=cuda).manual_seed(3)
    W = torch.randn(T, C, device=cuda, generator=g) * 0.01
    bias = torch.zeros(C, device=cuda)
    g0 = torch.randn(B, C, device=cuda, generator=g)
    g1 = torch.randn(B, C, device=cuda, generator=g)
    i0, i1 = torch.from_numpy(white).to(cuda), torch.from_numpy(black).to(cuda)
    out0, out1 = torch.empty(B, C, device=cuda), torch.empty(B, C, device=cuda)
    dW, dB = torch.empty(T, C, device=cuda), torch.empty(C, device=cuda)
    ws = ops.alloc_workspace(B, K, T, C, 2, cuda)
    args = (i0, i1, W, bias, out0, out1, g0, g1, dW, dB, ws, B, K)

    _step(*args)
    torch.cuda.synchronize()
    ref = (out0.clone(), out1.clone(), dW.clone(), dB.clone())

    try:
        _native.kernel_timer_arm([_native.TIMED_FORWARD, _native.TIMED_LIGHT_ROWS], 3)
        for _ in range(2):
            _step(*args)
        fwd = _native.kernel_timer_read(_native.TIMED_FORWARD)
        light = _native.kernel_timer_read(_native.TIMED_LIGHT_ROWS)
        heavy = _native.kernel_timer_read(_native.TIMED_HEAVY_ROWS)
    finally:
        _native.kernel_timer_arm((), 0)
    # 4 armed launches, capacity 3: forward, light, forward recorded
    assert len(fwd) == 2 and len(light) == 1 and heavy == []
    assert all(t > 0.0 for t in fwd + light)
    torch.cuda.synchronize()
    for a, b in zip(ref, (out0, out1, dW, dB)):
        assert torch.equal(a, b)
    assert _native.device_errors() == 0
