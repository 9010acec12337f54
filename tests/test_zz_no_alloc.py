"""The allocation-free backward entry point (nnue_ft_backward_noalloc).

Some callers cannot allocate device memory per call -- a search or inference
loop that runs on a fixed memory budget, or a host that only reaches the GPU
through the C ABI with tensors owned by another framework and nothing to hand
over as a workspace.  For them the library keeps one fixed scratch array per
GPU.  This test calls that entry point directly through the C ABI and checks
it against the regular workspace entry point (nnue_ft_backward), twice in a
row: the second call has another shape (feature set, batch and width), so the
scratch layout moves and anything the first call left in the array lands in
different fields.  It lives in its own file, named to be collected last, and
passes both alone in a fresh process and after the other tests.
"""

import ctypes

import numpy as np
import pytest
import torch

from stockfish_trainer_b200 import _native, positions
from stockfish_trainer_b200.feature_transformer import ops

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6


def _call_noalloc(i0, i1, g0, g1, T, dW, dB, accumulate):
    lib = _native.load()
    B, K = i0.shape
    C = dW.shape[1]
    stream = torch.cuda.current_stream(i0.device).cuda_stream
    return lib.nnue_ft_backward_noalloc(i0.data_ptr(), i1.data_ptr(), B, K, g0.data_ptr(), g1.data_ptr(), 2, T, C,
                                        dW.data_ptr(), dB.data_ptr(), int(accumulate), stream)


def _call_workspace(i0, i1, g0, g1, T, dW, dB, accumulate):
    lib = _native.load()
    B, K = i0.shape
    C = dW.shape[1]
    ws = ops.alloc_workspace(B, K, T, C, 2, i0.device)
    stream = torch.cuda.current_stream(i0.device).cuda_stream
    return lib.nnue_ft_backward(i0.data_ptr(), i1.data_ptr(), B, K, g0.data_ptr(), g1.data_ptr(), 2, T, C,
                                dW.data_ptr(), dB.data_ptr(), int(accumulate), ws.data_ptr(), ws.numel(), stream)


@pytest.mark.parametrize("first,second", [
    (("HalfKAv2_hm^", 2048, 1048), ("Full_Threats+HalfKAv2_hm^", 768, 264)),
    (("Full_Threats+HalfKAv2_hm^", 768, 1048), ("HalfKAv2_hm^", 1500, 520)),
])
def test_noalloc_backward_matches_workspace_backward_twice(cuda, first, second):
    lib = _native.load()
    for call, (fs, B, C) in enumerate((first, second)):  # two calls in a row, different shapes
        seed = 11 + call
        T = positions.feature_set_info(fs)[1]
        assert lib.nnue_ft_backward_workspace_size(B, positions.feature_set_info(fs)[2], T, C, 2) <= \
            lib.nnue_ft_noalloc_scratch_bytes()
        white, black, _ = positions.synthetic_batch(B, fs, seed=seed)
        rng = np.random.default_rng(seed)
        g0 = torch.from_numpy(rng.standard_normal((B, C), dtype=np.float32)).to(cuda)
        g1 = torch.from_numpy(rng.standard_normal((B, C), dtype=np.float32)).to(cuda)
        i0, i1 = torch.from_numpy(white).to(cuda), torch.from_numpy(black).to(cuda)
        dW = torch.full((T, C), float("nan"), device=cuda)
        dB = torch.full((C,), float("nan"), device=cuda)
        rW = torch.full((T, C), float("nan"), device=cuda)
        rB = torch.full((C,), float("nan"), device=cuda)
        assert _call_noalloc(i0, i1, g0, g1, T, dW, dB, accumulate=False) == 0, _native.last_error()
        assert _call_workspace(i0, i1, g0, g1, T, rW, rB, accumulate=False) == 0, _native.last_error()
        torch.cuda.synchronize()
        assert torch.equal(dW, rW), f"call {call}: weight gradient differs"
        torch.testing.assert_close(dB, rB, rtol=RTOL, atol=ATOL)
    assert _native.device_errors(clear=True) == 0


def test_noalloc_backward_accumulates_like_workspace_backward(cuda):
    fs, B, C = "HalfKAv2_hm^", 1024, 264
    T = positions.feature_set_info(fs)[1]
    white, black, _ = positions.synthetic_batch(B, fs, seed=21)
    rng = np.random.default_rng(21)
    g0 = torch.from_numpy(rng.standard_normal((B, C), dtype=np.float32)).to(cuda)
    g1 = torch.from_numpy(rng.standard_normal((B, C), dtype=np.float32)).to(cuda)
    i0, i1 = torch.from_numpy(white).to(cuda), torch.from_numpy(black).to(cuda)
    start = torch.from_numpy(rng.standard_normal((T, C), dtype=np.float32)).to(cuda)
    dW, rW = start.clone(), start.clone()
    dB, rB = torch.ones(C, device=cuda), torch.ones(C, device=cuda)
    assert _call_noalloc(i0, i1, g0, g1, T, dW, dB, accumulate=True) == 0, _native.last_error()
    assert _call_workspace(i0, i1, g0, g1, T, rW, rB, accumulate=True) == 0, _native.last_error()
    torch.cuda.synchronize()
    assert torch.equal(dW, rW)
    torch.testing.assert_close(dB, rB, rtol=RTOL, atol=ATOL)


def test_noalloc_backward_rejects_sizes_beyond_its_scratch(cuda):
    lib = _native.load()
    B, K, T, C = 65536, 160, 85296, 1048
    assert lib.nnue_ft_backward_workspace_size(B, K, T, C, 2) > lib.nnue_ft_noalloc_scratch_bytes()
    dummy = ctypes.c_void_p(256)  # never dereferenced: the size check fails first
    rc = lib.nnue_ft_backward_noalloc(dummy, dummy, B, K, dummy, dummy, 2, T, C, dummy, dummy, 0, None)
    assert rc == _native.NNUE_ERR_UNSUPPORTED
    assert "scratch" in _native.last_error()
