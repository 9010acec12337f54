"""The FT as ``torch.library`` custom operators (namespace ``nnue_ft``).

The reference keeps ``torch.compile`` away from its op with
``@torch.compiler.disable`` (src/model/modules/feature_transformer/kernel.py:301,
315), so a compiled trainer (src/train/common.py:189) breaks its graph at every
FT call.  Registered as custom operators with fake (shape-only)
implementations and an autograd formula, the same kernels are opaque nodes
that ``torch.compile`` traces through without a graph break:

* ``nnue_ft::sparse_linear(feature_indices, weight, bias) -> output`` and its
  backward ``nnue_ft::sparse_linear_backward(feature_indices, grad_output,
  num_inputs) -> (weight_grad, bias_grad)``: one perspective, the semantics of
  ``SparseLinearFunction`` (functions.py:10-72);
* ``nnue_ft::sparse_linear_pair(idx_0, idx_1, weight, bias) -> (out_0, out_1,
  workspace)`` and ``nnue_ft::sparse_linear_pair_backward(grad_0, grad_1,
  workspace, batch, max_active, num_inputs) -> (weight_grad, bias_grad)``: both
  perspectives on one table, the backward's index phase run during the forward
  (its result travels in ``workspace``), one dense weight gradient -- the
  semantics of ``SparseLinearPairFunction``.

``sparse_linear`` / ``sparse_linear_pair`` below are the user-facing calls.
Results equal the autograd functions' bit for bit (the same kernels).
"""

from __future__ import annotations

import torch

from . import ops

_NS = "nnue_ft"


def _empty_like_rows(n: int, cols: int, like: torch.Tensor) -> torch.Tensor:
    return torch.empty(n, cols, dtype=torch.float32, device=like.device)


# ---- one perspective -----------------------------------------------------
@torch.library.custom_op(f"{_NS}::sparse_linear", mutates_args=())
def _sparse_linear(feature_indices: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    out = _empty_like_rows(feature_indices.shape[0], weight.shape[1], weight)
    ops.forward_into(feature_indices, weight, bias, out)
    return out


@_sparse_linear.register_fake
def _(feature_indices, weight, bias):
    return feature_indices.new_empty(feature_indices.shape[0], weight.shape[1], dtype=torch.float32)


@torch.library.custom_op(f"{_NS}::sparse_linear_backward", mutates_args=())
def _sparse_linear_backward(feature_indices: torch.Tensor, grad_output: torch.Tensor,
                            num_inputs: int) -> tuple[torch.Tensor, torch.Tensor]:
    C = grad_output.shape[1]
    weight_grad = _empty_like_rows(num_inputs, C, grad_output)
    bias_grad = torch.empty(C, dtype=torch.float32, device=grad_output.device)
    ops.backward_into(feature_indices, None, grad_output.contiguous(), None, weight_grad, bias_grad,
                      accumulate=False)
    return weight_grad, bias_grad


@_sparse_linear_backward.register_fake
def _(feature_indices, grad_output, num_inputs):
    C = grad_output.shape[1]
    return (grad_output.new_empty(num_inputs, C, dtype=torch.float32),
            grad_output.new_empty(C, dtype=torch.float32))


def _sl_setup(ctx, inputs, output):
    feature_indices, weight, _bias = inputs
    ctx.save_for_backward(feature_indices)
    ctx.num_inputs = weight.shape[0]


def _sl_backward(ctx, grad_output):
    (feature_indices,) = ctx.saved_tensors
    weight_grad, bias_grad = _sparse_linear_backward(feature_indices, grad_output.contiguous(), ctx.num_inputs)
    return None, weight_grad, bias_grad


_sparse_linear.register_autograd(_sl_backward, setup_context=_sl_setup)


# ---- both perspectives ---------------------------------------------------
@torch.library.custom_op(f"{_NS}::sparse_linear_pair", mutates_args=())
def _sparse_linear_pair(feature_indices_0: torch.Tensor, feature_indices_1: torch.Tensor, weight: torch.Tensor,
                        bias: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    B, K = feature_indices_0.shape
    T, C = weight.shape
    out0 = _empty_like_rows(B, C, weight)
    out1 = _empty_like_rows(B, C, weight)
    ws = ops.alloc_workspace(B, K, T, C, 2, weight.device)
    ops.forward_pair_prepare(feature_indices_0, feature_indices_1, weight, bias, out0, out1, ws)
    return out0, out1, ws


@_sparse_linear_pair.register_fake
def _(feature_indices_0, feature_indices_1, weight, bias):
    B, K = feature_indices_0.shape
    T, C = weight.shape
    n_ws = ops.workspace_bytes(int(B), int(K), int(T), int(C), 2)
    return (weight.new_empty(B, C), weight.new_empty(B, C), weight.new_empty(n_ws, dtype=torch.uint8))


@torch.library.custom_op(f"{_NS}::sparse_linear_pair_backward", mutates_args=())
def _sparse_linear_pair_backward(grad_0: torch.Tensor, grad_1: torch.Tensor, workspace: torch.Tensor, batch: int,
                                 max_active: int, num_inputs: int) -> tuple[torch.Tensor, torch.Tensor]:
    C = grad_0.shape[1]
    weight_grad = _empty_like_rows(num_inputs, C, grad_0)
    bias_grad = torch.empty(C, dtype=torch.float32, device=grad_0.device)
    ops.backward_apply(grad_0.contiguous(), grad_1.contiguous(), batch, max_active, weight_grad, bias_grad, False,
                       workspace)
    return weight_grad, bias_grad


@_sparse_linear_pair_backward.register_fake
def _(grad_0, grad_1, workspace, batch, max_active, num_inputs):
    C = grad_0.shape[1]
    return grad_0.new_empty(num_inputs, C), grad_0.new_empty(C)


def _slp_setup(ctx, inputs, output):
    feature_indices_0, _i1, weight, _bias = inputs
    ctx.save_for_backward(output[2])
    ctx.shape = (feature_indices_0.shape[0], feature_indices_0.shape[1], weight.shape[0])


def _slp_backward(ctx, grad_0, grad_1, _grad_ws):
    (ws,) = ctx.saved_tensors
    B, K, T = ctx.shape
    # an output that received no gradient counts as zeros
    if grad_0 is None:
        grad_0 = torch.zeros_like(grad_1)
    if grad_1 is None:
        grad_1 = torch.zeros_like(grad_0)
    weight_grad, bias_grad = _sparse_linear_pair_backward(grad_0, grad_1, ws, B, K, T)
    return None, None, weight_grad, bias_grad


_sparse_linear_pair.register_autograd(_slp_backward, setup_context=_slp_setup)


def sparse_linear(feature_indices: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """``SparseLinearFunction.apply`` as a custom operator (traceable by
    ``torch.compile`` without a graph break)."""
    return torch.ops.nnue_ft.sparse_linear(feature_indices, weight, bias)


def sparse_linear_pair(feature_indices_0: torch.Tensor, feature_indices_1: torch.Tensor, weight: torch.Tensor,
                       bias: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """``SparseLinearPairFunction.apply`` as a custom operator."""
    out0, out1, _ws = torch.ops.nnue_ft.sparse_linear_pair(feature_indices_0, feature_indices_1, weight, bias)
    return out0, out1
