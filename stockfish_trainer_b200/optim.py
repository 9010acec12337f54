"""Ranger22 for the FT parameters, one fused kernel per parameter.

The reference (src/ranger22/optimizer.py) trains every parameter with
Ranger22 configured as in src/train/common.py:155-169 (no gradient
centralisation, no AGC, no softplus, no weight decay, PNM momentum, norm loss,
lookahead every 5 steps).  In that configuration ``Ranger22.step`` takes its
fused path (:307-551): per-step scalars computed once per group (:398-418),
then per parameter a torch.compile'd EMA + norm-loss + PNM update
(:48-107), then the lookahead blend (:569-597).  Here the update and, on
merge steps, the blend are one kernel per parameter
(``nnue_ft_ranger22_step``): it reads p, grad, variance_ma, the two grad EMAs
(and the slow copy) once and writes p, variance_ma, the current EMA (and the
slow copy).

``Ranger22FT`` keeps the reference's state layout (``step``, ``grad_ma``,
``variance_ma``, ``neg_grad_ma``, ``max_variance_ma``, ``lookahead_params``)
so checkpoints move between the two.  Only the trainer's configuration is
supported; anything else raises ``NotImplementedError`` instead of silently
changing the update rule.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _native


def ranger22_scalars(lr: float, step: int, betas=(0.9, 0.999), eps: float = 1e-7, normloss_factor: float = 1e-4,
                     momentum_pnm: bool = True) -> list[float]:
    """The 12 per-step constants of optimizer.py:398-418 / 211-245, in that
    order: lr, inv_sqrt_bc2, eps, two_nl_factor, noise_norm_recip, pnm_a,
    pnm_b, step_size, beta2, 1 - beta2, beta1^2, 1 - beta1^2 (computed in
    float64 like the reference, handed to the kernel as fp32)."""
    beta1, beta2 = betas
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    return [lr, 1.0 / math.sqrt(bc2), eps, 2.0 * normloss_factor,
            1.0 / math.sqrt((1.0 + beta2) ** 2 + beta2 ** 2), float(1 + momentum_pnm), float(-momentum_pnm),
            lr / bc1, beta2, 1.0 - beta2, beta1 * beta1, 1.0 - beta1 * beta1]


def ranger22_update_(p: torch.Tensor, grad: torch.Tensor, variance_ma: torch.Tensor, gma_cur: torch.Tensor,
                     gma_prev: torch.Tensor, scalars, lookahead: torch.Tensor | None = None, merge: bool = False,
                     lookahead_alpha: float = 0.5) -> None:
    """One Ranger22 update of a 1-D or 2-D fp32 CUDA parameter, in place
    (norm per row for 2-D, over the whole vector for 1-D); with ``merge`` the
    lookahead blend of the same step follows in the same pass."""
    if p.dim() not in (1, 2):
        raise ValueError(f"Ranger22 fused update supports 1-D and 2-D parameters, got shape {tuple(p.shape)}")
    tensors = {"param": p, "grad": grad, "variance_ma": variance_ma, "gma_cur": gma_cur, "gma_prev": gma_prev}
    if merge:
        if lookahead is None:
            raise ValueError("merge=True needs the lookahead tensor")
        tensors["lookahead"] = lookahead
    for name, t in tensors.items():
        if t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous() or t.shape != p.shape \
                or t.device != p.device:
            raise ValueError(f"{name} must be a contiguous fp32 CUDA tensor shaped like the parameter")
    if len(scalars) != 12:
        raise ValueError("scalars must hold the 12 per-step constants")
    rows, cols = (p.shape[0], p.shape[1]) if p.dim() == 2 else (1, p.shape[0])
    host = (ctypes.c_float * 12)(*[float(x) for x in scalars])
    with torch.cuda.device(p.device):
        _native.call("nnue_ft_ranger22_step", p.data_ptr(), grad.data_ptr(), variance_ma.data_ptr(),
                     gma_cur.data_ptr(), gma_prev.data_ptr(), lookahead.data_ptr() if merge else 0, rows, cols,
                     ctypes.addressof(host), 1 if merge else 0, float(lookahead_alpha),
                     torch.cuda.current_stream(p.device).cuda_stream)


class Ranger22FT(torch.optim.Optimizer):
    """Ranger22 in the reference trainer's configuration, every 1-D / 2-D
    fp32 CUDA parameter updated by the fused kernel.

    Constructor arguments mirror ``Ranger22(...)`` as called in
    src/train/common.py:155-169; options the fused path of the reference does
    not take (gradient centralisation, AGC, softplus, weight decay, MADGRAD,
    AdaBelief, warm-up / warm-down schedules) must stay off."""

    def __init__(self, params, lr, betas=(0.9, 0.999), eps=1e-7, lookahead_active=True, lookahead_mergetime=5,
                 lookahead_blending_alpha=0.5, normloss_active=True, normloss_factor=1e-4, momentum_type="pnm",
                 using_gc=False, using_normgc=False, weight_decay=0.0, use_adaptive_gradient_clipping=False,
                 softplus=False, use_madgrad=False, use_adabelief=False, use_warmup=False, warmdown_active=False,
                 **ignored):
        unsupported = {
            "using_gc": using_gc, "using_normgc": using_normgc, "weight_decay": weight_decay != 0.0,
            "use_adaptive_gradient_clipping": use_adaptive_gradient_clipping, "softplus": softplus,
            "use_madgrad": use_madgrad, "use_adabelief": use_adabelief, "use_warmup": use_warmup,
            "warmdown_active": warmdown_active, "normloss_active": not normloss_active,
            "momentum_type": momentum_type != "pnm",
        }
        bad = [k for k, v in unsupported.items() if v]
        if bad:
            raise NotImplementedError(f"Ranger22FT implements the trainer's fused path only; unsupported: {bad}")
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=0.0))
        self.eps = eps
        self.normloss_factor = normloss_factor
        self.momentum_pnm = True  # momentum_type == "pnm"; used as a number like upstream
        self.lookahead_active = lookahead_active
        self.lookahead_mergetime = lookahead_mergetime
        self.lookahead_alpha = lookahead_blending_alpha
        self.lookahead_step = 0

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            for p in group["params"]:
                if p.grad is None:
                    continue
                state = self.state[p]
                if len(state) == 0:
                    state["step"] = 0
                    for key in ("grad_ma", "variance_ma", "neg_grad_ma", "max_variance_ma"):
                        state[key] = torch.zeros_like(p, memory_format=torch.preserve_format)
                    if self.lookahead_active:
                        state["lookahead_params"] = p.detach().clone()
                state["step"] += 1
        merge = False
        if self.lookahead_active:
            self.lookahead_step += 1
            if self.lookahead_step >= self.lookahead_mergetime:
                self.lookahead_step = 0
                merge = True
        for group in self.param_groups:
            with_grad = [p for p in group["params"] if p.grad is not None]
            if not with_grad:
                continue
            step = self.state[with_grad[0]]["step"]
            scalars = ranger22_scalars(float(group["lr"]), step, group["betas"], float(group["eps"]),
                                       self.normloss_factor, self.momentum_pnm)
            for p in with_grad:
                if p.grad.is_sparse:
                    raise NotImplementedError("sparse gradients are not supported")
                state = self.state[p]
                if state["step"] % 2 == 1:
                    gma_cur, gma_prev = state["grad_ma"], state["neg_grad_ma"]
                else:
                    gma_cur, gma_prev = state["neg_grad_ma"], state["grad_ma"]
                ranger22_update_(p.data, p.grad, state["variance_ma"], gma_cur, gma_prev, scalars,
                                 state.get("lookahead_params"), merge, self.lookahead_alpha)
        return loss
