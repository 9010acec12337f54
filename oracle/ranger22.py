"""ORACLE -- TEST INFRASTRUCTURE ONLY.

numpy restatement of one Ranger22 parameter update in the reference
trainer's configuration, the checker for ``nnue_ft_ranger22_step``.

Follows src/ranger22/optimizer.py:79-107 (_compiled_full_update_2d; the 1-D
form :48-76 takes the norm over the whole vector) operation by operation in
float32, with the row norm taken in float64 and rounded once, and the
lookahead blend of :569-597 (torch.lerp's two-branch formula, weight
1 - alpha, then lookahead = p).  Scalars come from ``scalars()``, which
restates optimizer.py:398-418.
"""

from __future__ import annotations

import math

import numpy as np

f32 = np.float32


def scalars(lr, step, betas=(0.9, 0.999), eps=1e-7, normloss_factor=1e-4, momentum_pnm=True):
    """optimizer.py:398-418 -> the 12 constants of the compiled update, fp32."""
    beta1, beta2 = betas
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    vals = [lr, 1.0 / math.sqrt(bc2), eps, 2.0 * normloss_factor,
            1.0 / math.sqrt((1.0 + beta2) ** 2 + beta2 ** 2), float(1 + momentum_pnm), float(-momentum_pnm),
            lr / bc1, beta2, 1.0 - beta2, beta1 * beta1, 1.0 - beta1 * beta1]
    return np.array(vals, dtype=np.float32)


def _lerp(start, end, w):
    d = (end - start).astype(f32)
    if w < f32(0.5):
        return (start + (w * d).astype(f32)).astype(f32)
    return (end - (d * (f32(1.0) - w)).astype(f32)).astype(f32)


def update(p, grad, variance_ma, gma_cur, gma_prev, sc, lookahead=None, merge=False, alpha=0.5):
    """In-place update of float32 arrays (1-D or 2-D); returns nothing."""
    lr, inv_sqrt_bc2, eps, two_nl, noise_recip, pnm_a, pnm_b, step_size, beta2, omb2, b1sq, omb1sq = [f32(x) for x in sc]
    rows = p.reshape(1, -1) if p.ndim == 1 else p
    u = np.sqrt(np.sum(rows.astype(np.float64) ** 2, axis=1)).astype(f32)[:, None]
    corr = (two_nl * (f32(1.0) - (f32(1.0) / (u + eps).astype(f32)).astype(f32)).astype(f32)).astype(f32)
    pscale = (f32(1.0) - (lr * corr).astype(f32)).astype(f32)
    g = grad.reshape(rows.shape)
    v = variance_ma.reshape(rows.shape)
    m = gma_cur.reshape(rows.shape)
    mp = gma_prev.reshape(rows.shape)
    v[...] = ((v * beta2).astype(f32) + ((g * g).astype(f32) * omb2).astype(f32)).astype(f32)
    m[...] = ((m * b1sq).astype(f32) + (g * omb1sq).astype(f32)).astype(f32)
    denom = ((np.sqrt(v).astype(f32) * inv_sqrt_bc2).astype(f32) + eps).astype(f32)
    pn = (((m * pnm_a).astype(f32) + (mp * pnm_b).astype(f32)).astype(f32) * noise_recip).astype(f32)
    x = (rows * pscale).astype(f32)
    x = (x - ((pn / denom).astype(f32) * step_size).astype(f32)).astype(f32)
    if merge:
        la = lookahead.reshape(rows.shape)
        x = _lerp(x, la, f32(1.0) - f32(alpha))
        la[...] = x
    rows[...] = x
