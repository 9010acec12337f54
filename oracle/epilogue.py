"""ORACLE -- TEST INFRASTRUCTURE ONLY.

fp32 PyTorch (CPU) restatement of the FT epilogue in
NNUEModel._transform_inputs (src/model/model.py:93-115), the checker for
``nnue_ft_epilogue_forward`` / ``_backward``: the same tensor operations in
the same order, differentiated by torch autograd.
"""

from __future__ import annotations

import torch


def transform(wp: torch.Tensor, bp: torch.Tensor, us: torch.Tensor, psqt_indices: torch.Tensor, l1: int):
    """model.py:93-115 after ``self.input(...)``: returns (l0_, psqt)."""
    w, wpsqt = torch.split(wp, l1, dim=1)
    b, bpsqt = torch.split(bp, l1, dim=1)
    chunk = l1 // 2
    us_bool = us.bool()
    w_c = torch.clamp(w, 0.0, 1.0).reshape(-1, 2, chunk)
    b_c = torch.clamp(b, 0.0, 1.0).reshape(-1, 2, chunk)
    w_pw = w_c[:, 0, :] * w_c[:, 1, :]
    b_pw = b_c[:, 0, :] * b_c[:, 1, :]
    l0_ = torch.cat([torch.where(us_bool, w_pw, b_pw), torch.where(us_bool, b_pw, w_pw)], dim=1) * (127 / 128)
    idx = psqt_indices.unsqueeze(dim=1)
    psqt = (wpsqt.gather(1, idx) - bpsqt.gather(1, idx)) * (us - 0.5)
    return l0_, psqt


def forward_backward(wp, bp, us, psqt_indices, l1, d_l0, d_psqt):
    """Forward outputs and the autograd gradients w.r.t. wp and bp."""
    wp = wp.detach().clone().requires_grad_()
    bp = bp.detach().clone().requires_grad_()
    l0_, psqt = transform(wp, bp, us, psqt_indices, l1)
    torch.autograd.backward([l0_, psqt], [d_l0, d_psqt])
    return l0_.detach(), psqt.detach(), wp.grad, bp.grad
