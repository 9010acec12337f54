"""The FT's torch.library custom operators (namespace nnue_ft) on CPU: they
register at import, and their fake (shape-only) implementations give the
shapes torch.compile traces with -- no GPU needed."""

import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import stockfish_trainer_b200.feature_transformer as ft
from stockfish_trainer_b200.feature_transformer import ops


def test_ops_are_registered():
    for name in ("sparse_linear", "sparse_linear_backward", "sparse_linear_pair", "sparse_linear_pair_backward"):
        assert hasattr(torch.ops.nnue_ft, name)
    assert ft.sparse_linear is not None and ft.sparse_linear_pair is not None


def test_fake_shapes():
    B, K, T, C = 64, 160, 85296, 1048
    with FakeTensorMode():
        idx = torch.empty(B, K, dtype=torch.int32)
        W = torch.empty(T, C)
        b = torch.empty(C)
        out = torch.ops.nnue_ft.sparse_linear(idx, W, b)
        assert tuple(out.shape) == (B, C) and out.dtype == torch.float32
        dW, dB = torch.ops.nnue_ft.sparse_linear_backward(idx, out, T)
        assert tuple(dW.shape) == (T, C) and tuple(dB.shape) == (C,)
        o0, o1, ws = torch.ops.nnue_ft.sparse_linear_pair(idx, idx, W, b)
        assert tuple(o0.shape) == (B, C) and tuple(o1.shape) == (B, C)
        assert ws.dtype == torch.uint8 and ws.numel() == ops.workspace_bytes(B, K, T, C, 2)
        dW, dB = torch.ops.nnue_ft.sparse_linear_pair_backward(o0, o1, ws, B, K, T)
        assert tuple(dW.shape) == (T, C) and tuple(dB.shape) == (C,)
