"""FT epilogue: NNUEModel._transform_inputs after the feature transformer
(reference src/model/model.py:93-115) as one fused kernel each way.

``transform_inputs(wp, bp, us, psqt_indices, L1)`` returns ``(l0_, psqt)``
exactly like the reference's tensor code (split, clamp to [0, 1], pairwise
product of the two halves, perspective order by ``us``, x 127/128, PSQT
bucket gather, (w - b) * (us - 0.5)), and its backward returns the gradients
torch autograd would, bit for bit.  ``wp`` / ``bp`` are the two FT outputs
[B, L1 + n_psqt]; ``us`` is the [B, 1] float side-to-move tensor and
``psqt_indices`` the [B] int64 bucket indices, as the reference's loader
produces them (src/data/loader.py:67-84).
"""

from __future__ import annotations

import torch

from .. import _native


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def _check_inputs(wp, bp, us, psqt_indices, l1):
    for name, t in (("wp", wp), ("bp", bp)):
        if t.dtype != torch.float32 or t.dim() != 2 or not t.is_cuda or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous 2-D fp32 CUDA tensor")
    if wp.shape != bp.shape or wp.device != bp.device:
        raise ValueError("wp and bp must have the same shape and device")
    if not (0 < l1 <= wp.shape[1]) or l1 % 2:
        raise ValueError(f"L1 = {l1} must be even and at most the FT width {wp.shape[1]}")
    B = wp.shape[0]
    if us.numel() != B or us.dtype != torch.float32 or us.device != wp.device:
        raise ValueError("us must hold one fp32 value per position, on the FT's device")
    if psqt_indices.numel() != B or psqt_indices.dtype != torch.int64 or psqt_indices.device != wp.device:
        raise ValueError("psqt_indices must hold one int64 index per position, on the FT's device")


class TransformInputsFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, wp, bp, us, psqt_indices, l1):
        _check_inputs(wp, bp, us, psqt_indices, l1)
        B, width = wp.shape
        us_flat = us.reshape(-1).contiguous()
        pidx = psqt_indices.reshape(-1).contiguous()
        l0 = torch.empty(B, l1, dtype=torch.float32, device=wp.device)
        psqt = torch.empty(B, 1, dtype=torch.float32, device=wp.device)
        with torch.cuda.device(wp.device):
            _native.call("nnue_ft_epilogue_forward", wp.data_ptr(), bp.data_ptr(), B, l1, width - l1,
                         us_flat.data_ptr(), pidx.data_ptr(), l0.data_ptr(), psqt.data_ptr(), _stream(wp.device))
        ctx.save_for_backward(wp, bp, us_flat, pidx)
        ctx.l1 = l1
        return l0, psqt

    @staticmethod
    def backward(ctx, d_l0, d_psqt):
        wp, bp, us_flat, pidx = ctx.saved_tensors
        B, width = wp.shape
        d_wp = torch.empty_like(wp)
        d_bp = torch.empty_like(bp)
        g0 = None if d_l0 is None else d_l0.contiguous()
        g1 = None if d_psqt is None else d_psqt.reshape(-1).contiguous()
        with torch.cuda.device(wp.device):
            _native.call("nnue_ft_epilogue_backward", wp.data_ptr(), bp.data_ptr(), B, ctx.l1, width - ctx.l1,
                         us_flat.data_ptr(), pidx.data_ptr(), 0 if g0 is None else g0.data_ptr(),
                         0 if g1 is None else g1.data_ptr(), d_wp.data_ptr(), d_bp.data_ptr(), _stream(wp.device))
        return d_wp, d_bp, None, None, None


def transform_inputs(wp: torch.Tensor, bp: torch.Tensor, us: torch.Tensor, psqt_indices: torch.Tensor, l1: int):
    """Drop-in for the tensor code of model.py:94-115 (everything after
    ``wp, bp = self.input(white_indices, black_indices)``)."""
    return TransformInputsFunction.apply(wp, bp, us, psqt_indices, l1)
