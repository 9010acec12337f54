"""Module-level drop-in for ComposedFeatureTransformer
(reference src/model/modules/features/composed.py).

The reference rebuilds the whole merged table every step,
``torch.cat([f.merged_weight() for f in features])`` (composed.py:50), where
HalfKav2Hm's merged_weight is ``weight + virtual_weight.repeat(32, 1)``
(halfka_v2_hm.py:69-70), then calls the FT op once per perspective, and
autograd splits the merged gradient back into the per-feature parameters.
Here the FT kernels read the per-feature tables where they are
(``nnue_ft_forward_pair_tables``), the HalfKA table plus its virtual rows is
formed in one pass without the repeat (``nnue_ft_merge_virtual``), and the
backward writes each feature's weight gradient directly
(``nnue_ft_backward_apply_tables``); the virtual-weight gradient is torch's
own repeat backward of the HalfKA gradient, exactly as in the reference
graph.  Outputs and every gradient are bit-identical to the reference module
running SparseLinearFunction on the merged table.
"""

from __future__ import annotations

import math

import torch
from torch import autograd, nn

from . import ops


class MergeVirtualFunction(autograd.Function):
    """weight + virtual_weight.repeat(k, 1) with the reference graph's
    gradients (AddBackward passes the gradient through, RepeatBackward sums
    the k copies)."""

    @staticmethod
    def forward(ctx, weight, virtual_weight):
        ctx.reps = weight.shape[0] // virtual_weight.shape[0]
        ctx.vshape = virtual_weight.shape
        return ops.merge_virtual(weight, virtual_weight)

    @staticmethod
    def backward(ctx, grad):
        d_virtual = None
        if ctx.needs_input_grad[1]:
            with torch.enable_grad():
                v = torch.zeros(ctx.vshape, dtype=grad.dtype, device=grad.device, requires_grad=True)
                (d_virtual,) = autograd.grad(v.repeat(ctx.reps, 1), v, grad)
        return grad, d_virtual


class ComposedSparseLinearFunction(autograd.Function):
    """(idx_white, idx_black, bias, *tables) -> (out_white, out_black): the
    two SparseLinearFunction calls of composed.py:51-54 on the row-wise
    concatenation of ``tables``, without materialising it."""

    @staticmethod
    def forward(ctx, feature_indices_0, feature_indices_1, bias, *tables):
        B, K = feature_indices_0.shape
        C = bias.shape[0]
        T = sum(t.shape[0] for t in tables)
        out0 = torch.empty(B, C, dtype=torch.float32, device=bias.device)
        out1 = torch.empty_like(out0)
        ws = ops.alloc_workspace(B, K, T, C, 2, bias.device)
        ops.forward_pair_tables_prepare(feature_indices_0, feature_indices_1, list(tables), bias, out0, out1, ws)
        ctx.workspace = ws
        ctx.meta = (B, K, [t.shape for t in tables])
        return out0, out1

    @staticmethod
    def backward(ctx, grad0, grad1):
        B, K, shapes = ctx.meta
        ws, ctx.workspace = ctx.workspace, None
        dev = ws.device
        C = shapes[0][1]
        grad0 = torch.zeros(B, C, device=dev) if grad0 is None else grad0.contiguous()
        grad1 = torch.zeros(B, C, device=dev) if grad1 is None else grad1.contiguous()
        weight_grads = [torch.empty(s, dtype=torch.float32, device=dev) for s in shapes]
        bias_grad = torch.empty(C, dtype=torch.float32, device=dev)
        ops.backward_apply_tables(grad0, grad1, B, K, weight_grads, bias_grad, ws)
        return (None, None, bias_grad, *weight_grads)


def _feature_table(f):
    """The feature's table as the FT reads it: HalfKav2Hm-style features
    (``weight`` + ``virtual_weight`` repeated NUM_BUCKETS times) go through
    MergeVirtualFunction; every other feature supplies ``merged_weight()``
    (for FullThreats that is the weight parameter itself)."""
    w = getattr(f, "weight", None)
    v = getattr(f, "virtual_weight", None)
    reps = getattr(f, "NUM_BUCKETS", None)
    if w is not None and v is not None and reps and w.shape[0] == v.shape[0] * reps:
        return MergeVirtualFunction.apply(w, v)
    return f.merged_weight()


class ComposedFeatureTransformer(nn.Module):
    """Same constructor, parameters, attributes and methods as the
    reference's ComposedFeatureTransformer (composed.py:8-81); forward runs
    the table-set kernels."""

    def __init__(self, features):
        super().__init__()
        self.features = nn.ModuleList(features)
        self.num_outputs = features[0].num_outputs
        self.bias = nn.Parameter(torch.empty(self.num_outputs, dtype=torch.float32))
        self.NUM_INPUTS = sum(f.NUM_INPUTS for f in features)
        self.MAX_ACTIVE_FEATURES = sum(f.MAX_ACTIVE_FEATURES for f in features)
        self.NUM_REAL_FEATURES = sum(f.NUM_REAL_FEATURES for f in features)
        self.FEATURE_NAME = "+".join(f.FEATURE_NAME for f in features)
        self.INPUT_FEATURE_NAME = "+".join(f.INPUT_FEATURE_NAME for f in features)
        h = 0
        for f in features:  # composed.py:34-39
            h = ((h << 1) | (h >> 31)) & 0xFFFFFFFF
            h ^= f.HASH
        self.HASH = h
        sigma = math.sqrt(1 / self.NUM_INPUTS)
        with torch.no_grad():
            self.bias.uniform_(-sigma, sigma)

    def forward(self, feature_indices_0, feature_indices_1):
        tables = [_feature_table(f) for f in self.features]
        return ComposedSparseLinearFunction.apply(feature_indices_0, feature_indices_1, self.bias, *tables)

    @torch.no_grad()
    def coalesce(self) -> None:
        for f in self.features:
            f.coalesce()

    @torch.no_grad()
    def init_weights(self, num_psqt_buckets: int, nnue2score: float) -> None:
        for f in self.features:
            f.init_weights(num_psqt_buckets, nnue2score)
        L1 = self.num_outputs - num_psqt_buckets
        for i in range(num_psqt_buckets):
            self.bias[L1 + i] = 0.0

    @torch.no_grad()
    def get_export_weights(self) -> torch.Tensor:
        return torch.cat([f.get_export_weights() for f in self.features], dim=0)

    @torch.no_grad()
    def load_export_weights(self, export_weight: torch.Tensor) -> None:
        offset = 0
        for f in self.features:
            n = f.NUM_REAL_FEATURES
            f.load_export_weights(export_weight[offset: offset + n])
            offset += n

    def clip_weights(self, quantization) -> None:
        for f in self.features:
            f.clip_weights(quantization)
