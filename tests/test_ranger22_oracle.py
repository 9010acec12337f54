"""The Ranger22 oracle (oracle/ranger22.py) replays seven steps of the
reference optimizer (tests/golden/ranger22_steps.npz, produced by
src/ranger22 itself) on a 2-D and a 1-D parameter.  The reference's CPU path
orders a few operations differently (denominator divided by sqrt(bc2) instead
of multiplied by its inverse, addcdiv), so the comparison carries a float32
tolerance."""

import os

import numpy as np

from oracle import ranger22

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ranger22_steps.npz")


def _replay(p0, grads, lr):
    p = p0.astype(np.float32).copy()
    st = {k: np.zeros_like(p) for k in ("grad_ma", "neg_grad_ma", "variance_ma")}
    la = p.copy()
    la_step = 0
    for s, g in enumerate(grads, start=1):
        cur, prev = ("grad_ma", "neg_grad_ma") if s % 2 == 1 else ("neg_grad_ma", "grad_ma")
        la_step += 1
        merge = la_step >= 5
        if merge:
            la_step = 0
        ranger22.update(p, g.astype(np.float32), st["variance_ma"], st[cur], st[prev], ranger22.scalars(lr, s),
                        la, merge, 0.5)
    return p, st, la


def test_oracle_replays_reference_ranger22_steps():
    z = np.load(GOLD)
    for name, p0, grads in (("w", z["w0"], z["gw"]), ("b", z["b0"], z["gb"])):
        p, st, la = _replay(p0, grads, float(z["lr"]))
        np.testing.assert_allclose(p, z[name], rtol=1e-5, atol=1e-7)
        np.testing.assert_allclose(la, z[f"{name}_lookahead_params"], rtol=1e-5, atol=1e-7)
        for key in ("grad_ma", "neg_grad_ma", "variance_ma"):
            np.testing.assert_allclose(st[key], z[f"{name}_{key}"], rtol=1e-5, atol=1e-9)


def test_oracle_scalars_follow_reference_formulas():
    s = ranger22.scalars(1e-3, 3)
    assert s.dtype == np.float32 and s.shape == (12,)
    assert np.isclose(s[7], 1e-3 / (1 - 0.9 ** 3))
    assert s[5] == 2.0 and s[6] == -1.0  # upstream's boolean PNM factor
