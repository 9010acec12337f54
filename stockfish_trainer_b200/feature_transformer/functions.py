"""Autograd functions with the reference's interface.

``SparseLinearFunction`` keeps the signature, input assertions and return
values of src/model/modules/feature_transformer/functions.py:10-72, so
``ComposedFeatureTransformer`` (src/model/modules/features/composed.py:49-54)
and everything above it run unchanged.

``SparseLinearPairFunction`` is the two-perspective form of the same op: both
perspectives share one table, the forward is one launch and the backward
writes ONE dense weight gradient, dW = dW_white + dW_black, bit-identical to
the reference's two per-perspective gradients summed by autograd.
"""

from __future__ import annotations

import torch
from torch import autograd

from . import ops
from .kernel import make_sparse_input_linear_backward_kernel, make_sparse_input_linear_forward_kernel


def _check_inputs(feature_indices, weight, bias):
    # functions.py:15-28
    assert len(feature_indices.shape) == 2
    assert feature_indices.dtype == torch.int32
    assert len(weight.shape) == 2
    assert weight.dtype == torch.float32
    assert len(bias.shape) == 1
    assert bias.dtype == torch.float32
    assert feature_indices.is_cuda
    assert weight.is_cuda
    assert bias.is_cuda
    assert weight.device == feature_indices.device
    assert bias.device == feature_indices.device
    assert feature_indices.is_contiguous()
    assert weight.is_contiguous()
    assert bias.is_contiguous()


@torch.compiler.disable
def _forward(feature_indices, weight, bias):
    out = torch.empty(feature_indices.shape[0], weight.shape[1], dtype=torch.float32, device=feature_indices.device)
    kernel = make_sparse_input_linear_forward_kernel(feature_indices.shape[1], weight.shape[1])
    kernel(feature_indices, weight, bias, out)
    return out


@torch.compiler.disable
def _backward(idx0, idx1, grad0, grad1, num_inputs, output_size):
    device = idx0.device
    # Every row is written (untouched rows get 0), so empty() replaces the
    # reference's zeros() + read-modify-write.
    weight_grad = torch.empty(num_inputs, output_size, dtype=torch.float32, device=device)
    bias_grad = torch.empty(output_size, dtype=torch.float32, device=device)
    ops.backward_into(idx0, idx1, grad0, grad1, weight_grad, bias_grad, accumulate=False)
    return weight_grad, bias_grad


class SparseLinearFunction(autograd.Function):
    @staticmethod
    def forward(ctx, feature_indices, weight, bias):
        ctx.save_for_backward(feature_indices, weight, bias)
        _check_inputs(feature_indices, weight, bias)
        return _forward(feature_indices, weight, bias)

    @staticmethod
    def backward(ctx, grad_output):
        assert not ctx.needs_input_grad[0]
        grad_output = grad_output.contiguous()
        feature_indices, weight, _bias = ctx.saved_tensors
        weight_grad, bias_grad = _backward(feature_indices, None, grad_output, None, weight.shape[0], weight.shape[1])
        return None, weight_grad, bias_grad


@torch.compiler.disable
def _forward_pair(idx0, idx1, weight, bias):
    B, K = idx0.shape
    T, C = weight.shape
    out0 = torch.empty(B, C, dtype=torch.float32, device=idx0.device)
    out1 = torch.empty_like(out0)
    # The backward's index-only phase (sorted position lists per feature) runs
    # during the forward, on the library's side stream; its workspace lives
    # until the backward consumes it.
    ws = ops.alloc_workspace(B, K, T, C, 2, idx0.device)
    ops.forward_pair_prepare(idx0, idx1, weight, bias, out0, out1, ws)
    return out0, out1, ws


@torch.compiler.disable
def _backward_pair_apply(grad0, grad1, batch, max_active, num_inputs, output_size, ws):
    weight_grad = torch.empty(num_inputs, output_size, dtype=torch.float32, device=grad0.device)
    bias_grad = torch.empty(output_size, dtype=torch.float32, device=grad0.device)
    ops.backward_apply(grad0, grad1, batch, max_active, weight_grad, bias_grad, False, ws)
    return weight_grad, bias_grad


class SparseLinearPairFunction(autograd.Function):
    """(idx_white, idx_black, weight, bias) -> (out_white, out_black)."""

    @staticmethod
    def forward(ctx, feature_indices_0, feature_indices_1, weight, bias):
        _check_inputs(feature_indices_0, weight, bias)
        _check_inputs(feature_indices_1, weight, bias)
        assert feature_indices_0.shape == feature_indices_1.shape
        ctx.save_for_backward(feature_indices_0, feature_indices_1, weight)
        out0, out1, ws = _forward_pair(feature_indices_0, feature_indices_1, weight, bias)
        ctx.workspace = ws
        return out0, out1

    @staticmethod
    def backward(ctx, grad0, grad1):
        assert not ctx.needs_input_grad[0] and not ctx.needs_input_grad[1]
        idx0, idx1, weight = ctx.saved_tensors
        ws, ctx.workspace = ctx.workspace, None
        T, C = weight.shape
        B, K = idx0.shape
        if grad0 is None and grad1 is None:
            return None, None, None, None
        if grad0 is None:
            weight_grad, bias_grad = _backward(idx1, None, grad1.contiguous(), None, T, C)
        elif grad1 is None:
            weight_grad, bias_grad = _backward(idx0, None, grad0.contiguous(), None, T, C)
        else:
            weight_grad, bias_grad = _backward_pair_apply(grad0.contiguous(), grad1.contiguous(), B, K, T, C, ws)
        return None, None, weight_grad, bias_grad
