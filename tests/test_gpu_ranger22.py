"""Fused Ranger22 update (nnue_ft_ranger22_step) vs the numpy oracle, and the
Ranger22FT optimizer vs seven steps of the reference optimizer.

Elementwise state (variance_ma, the grad EMA, the lookahead copy) follows the
oracle's fp32 operation order and is compared bit for bit; the parameter also
depends on the row norm, whose fp64 summation order differs, so it carries a
float32 tolerance."""

import os

import numpy as np
import pytest
import torch

from oracle import ranger22 as oracle_r22
from stockfish_trainer_b200 import optim

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ranger22_steps.npz")


def _state(shape, seed):
    rng = np.random.default_rng(seed)
    p = (rng.standard_normal(shape) * 0.05).astype(np.float32)
    g = rng.standard_normal(shape).astype(np.float32)
    v = np.abs(rng.standard_normal(shape) * 1e-3).astype(np.float32)
    m = (rng.standard_normal(shape) * 1e-2).astype(np.float32)
    mp = (rng.standard_normal(shape) * 1e-2).astype(np.float32)
    la = (p + rng.standard_normal(shape).astype(np.float32) * 1e-3).astype(np.float32)
    return p, g, v, m, mp, la


@pytest.mark.parametrize("shape", [(300, 1048), (7, 13), (1048,), (20001,), (5, 9000), (3,), (64, 32)])
@pytest.mark.parametrize("merge", [False, True])
def test_fused_update_matches_oracle(cuda, shape, merge):
    p, g, v, m, mp, la = _state(shape, seed=sum(shape) + merge)
    sc = oracle_r22.scalars(8.75e-4, 4)
    t = lambda a: torch.from_numpy(a.copy()).to(cuda)
    dp, dg, dv, dm, dmp, dla = t(p), t(g), t(v), t(m), t(mp), t(la)
    optim.ranger22_update_(dp, dg, dv, dm, dmp, sc.tolist(), dla, merge, 0.5)
    torch.cuda.synchronize()
    oracle_r22.update(p, g, v, m, mp, sc, la, merge, 0.5)
    np.testing.assert_array_equal(dv.cpu().numpy(), v)
    np.testing.assert_array_equal(dm.cpu().numpy(), m)
    np.testing.assert_allclose(dp.cpu().numpy(), p, rtol=1e-6, atol=1e-9)
    np.testing.assert_allclose(dla.cpu().numpy(), la, rtol=1e-6, atol=1e-9)
    np.testing.assert_array_equal(dg.cpu().numpy(), g)  # read-only inputs untouched
    np.testing.assert_array_equal(dmp.cpu().numpy(), mp)


def test_misaligned_rows_use_scalar_path(cuda):
    p, g, v, m, mp, la = _state((9, 40), seed=3)
    sc = oracle_r22.scalars(1e-3, 2)
    buf = torch.zeros(6, 9 * 40 + 1, device=cuda)
    views = [buf[i, 1:].view(9, 40) for i in range(6)]  # 4-byte offset: not 16-byte aligned
    for view, a in zip(views, (p, g, v, m, mp, la)):
        view.copy_(torch.from_numpy(a))
    optim.ranger22_update_(*views[:5], sc.tolist(), views[5], True, 0.5)
    torch.cuda.synchronize()
    oracle_r22.update(p, g, v, m, mp, sc, la, True, 0.5)
    np.testing.assert_array_equal(views[2].cpu().numpy(), v)
    np.testing.assert_allclose(views[0].cpu().numpy(), p, rtol=1e-6, atol=1e-9)


def test_optimizer_replays_reference_steps(cuda):
    z = np.load(GOLD)
    w = torch.nn.Parameter(torch.from_numpy(z["w0"]).to(cuda))
    b = torch.nn.Parameter(torch.from_numpy(z["b0"]).to(cuda))
    opt = optim.Ranger22FT([{"params": [w, b]}], lr=float(z["lr"]), betas=(0.9, 0.999), eps=1.0e-7)
    for s in range(z["gw"].shape[0]):
        w.grad = torch.from_numpy(z["gw"][s]).to(cuda)
        b.grad = torch.from_numpy(z["gb"][s]).to(cuda)
        opt.step()
    torch.cuda.synchronize()
    np.testing.assert_allclose(w.detach().cpu().numpy(), z["w"], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(b.detach().cpu().numpy(), z["b"], rtol=1e-5, atol=1e-7)
    for name, p in (("w", w), ("b", b)):
        st = opt.state[p]
        for key in ("grad_ma", "neg_grad_ma", "variance_ma", "lookahead_params"):
            np.testing.assert_allclose(st[key].cpu().numpy(), z[f"{name}_{key}"], rtol=1e-5, atol=1e-9)

