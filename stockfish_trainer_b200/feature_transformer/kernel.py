"""Kernel factories with the reference's names and calling conventions.

Reference: src/model/modules/feature_transformer/kernel.py:301-319.

* ``make_sparse_input_linear_forward_kernel(max_active, output_size)``
  returns ``fn(input_indices, weight, bias, output)`` that WRITES ``output``.
* ``make_sparse_input_linear_backward_kernel(max_active, output_size)``
  returns ``fn(input_indices, weight_grad, bias_grad, output_grad)`` that
  ACCUMULATES into ``weight_grad`` (touched rows only) and ``bias_grad``,
  exactly like the reference kernel (kernel.py:184-186, :269).

There is no autotuning step (the reference tunes TileLang thread counts on
the first call, kernel.py:200-218): the sm_100a kernels have one schedule,
so the backward may run on any thread, including autograd's.

The native calls go through ``ops``; every entry launches on the calling
thread's current CUDA stream of the tensors' device and never synchronises.
"""

from __future__ import annotations

from collections.abc import Callable

import torch

from . import ops

SparseInputLinearForwardKernel = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor], None]
SparseInputLinearBackwardKernel = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor], None]


class _ForwardKernel:
    def __init__(self, max_active_indices: int, output_size: int):
        self.max_active_indices = max_active_indices
        self.output_size = output_size

    def __call__(self, input_indices, weight, bias, output) -> None:
        if input_indices.shape[1] != self.max_active_indices or weight.shape[1] != self.output_size:
            raise ValueError("tensor shapes do not match the kernel's (max_active, output_size)")
        ops.forward_into(input_indices, weight, bias, output)


class _BackwardKernel:
    def __init__(self, max_active_indices: int, output_size: int):
        self.max_active_indices = max_active_indices
        self.output_size = output_size

    def __call__(self, input_indices, weight_grad, bias_grad, output_grad) -> None:
        if input_indices.shape[1] != self.max_active_indices or weight_grad.shape[1] != self.output_size:
            raise ValueError("tensor shapes do not match the kernel's (max_active, output_size)")
        ops.backward_into(input_indices, None, output_grad, None, weight_grad, bias_grad, accumulate=True)


_forward_kernel_cache: dict[tuple[int, int], _ForwardKernel] = {}
_backward_kernel_cache: dict[tuple[int, int], _BackwardKernel] = {}


@torch.compiler.disable(recursive=False)
def make_sparse_input_linear_forward_kernel(max_active_indices: int, output_size: int) -> SparseInputLinearForwardKernel:
    key = (max_active_indices, output_size)
    if key not in _forward_kernel_cache:
        _forward_kernel_cache[key] = _ForwardKernel(max_active_indices, output_size)
    return _forward_kernel_cache[key]


@torch.compiler.disable(recursive=False)
def make_sparse_input_linear_backward_kernel(max_active_indices: int, output_size: int) -> SparseInputLinearBackwardKernel:
    key = (max_active_indices, output_size)
    if key not in _backward_kernel_cache:
        _backward_kernel_cache[key] = _BackwardKernel(max_active_indices, output_size)
    return _backward_kernel_cache[key]
