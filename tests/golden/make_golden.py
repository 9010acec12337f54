"""Generate the golden fixtures in this directory from the REFERENCE itself.

Run once, in a container that has the reference checkout (it is not present
on the GPU box, so the tests only read the committed ``.npz`` outputs):

    python tests/golden/make_golden.py /path/to/stockfish-trainer

python-chess is not installed, so a stand-in ``chess`` module exposing the
public constants the reference uses (PAWN..KING = 1..6, WHITE = True,
BLACK = False, Piece(piece_type, color)) is registered before the import.

Fixtures and the reference code that produced them:
  halfka_idx.npz              src/model/modules/features/halfka_v2_hm.py:28-37 (_halfka_idx)
  sorted_backward_inputs.npz  src/model/modules/feature_transformer/kernel.py:108-138
  quantize_ft.npz             src/model/quantize.py:76-93 (quantize_feature_transformer)
  export_weights.npz          src/model/modules/features/halfka_v2_hm.py:100-134 (get_export_weights)
  composed_sizes.npz          src/model/modules/features/composed.py:24-26, full_threats.py, halfka_v2_hm.py
  ranger22_steps.npz          src/ranger22/optimizer.py (Ranger22.step, configured as src/train/common.py:155-169)
  transform_inputs.npz        src/model/model.py:86-115 (NNUEModel._transform_inputs, forward + autograd backward)
"""

from __future__ import annotations

import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _install_chess_stub() -> None:
    chess = types.ModuleType("chess")
    chess.PAWN, chess.KNIGHT, chess.BISHOP, chess.ROOK, chess.QUEEN, chess.KING = range(1, 7)
    chess.WHITE, chess.BLACK = True, False

    class Piece:
        def __init__(self, piece_type, color):
            self.piece_type = piece_type
            self.color = color

    chess.Piece = Piece
    sys.modules["chess"] = chess


def main(ref_root: str) -> None:
    _install_chess_stub()
    sys.path.insert(0, ref_root)
    import chess  # the stub
    from src.model.modules.features import halfka_v2_hm, full_threats, composed
    from src.model.modules.feature_transformer import kernel
    from src.model.quantize import QuantizationConfig, QuantizationManager

    # --- HalfKA index table: [pov(white=0, black=1)][ksq][sq][piece id] -------
    table = np.zeros((2, 64, 64, 12), dtype=np.int32)
    for pov in range(2):
        for ksq in range(64):
            for sq in range(64):
                for pid in range(12):
                    p = chess.Piece(pid // 2 + 1, pid % 2 == 0)
                    table[pov, ksq, sq, pid] = halfka_v2_hm._halfka_idx(pov == 0, ksq, sq, p)
    np.savez_compressed(os.path.join(HERE, "halfka_idx.npz"), table=table)

    # --- backward preprocessing --------------------------------------------
    g = torch.Generator().manual_seed(1234)
    cases = {}

    def rows_unique(B, K, T, fill, compact=True):
        idx = torch.full((B, K), -1, dtype=torch.int32)
        for b in range(B):
            n = int(torch.randint(0, K + 1, (1,), generator=g))
            n = max(0, min(n, int(K * fill)))
            vals = torch.randperm(T, generator=g)[:n].to(torch.int32)
            if compact:
                idx[b, :n] = vals
            else:
                pos = torch.randperm(K, generator=g)[:n]
                idx[b, pos] = vals
        return idx

    cases["compact"] = (rows_unique(96, 12, 40, 1.0), 40)
    cases["holes"] = (rows_unique(80, 16, 300, 0.8, compact=False), 300)
    cases["empty"] = (torch.full((7, 5), -1, dtype=torch.int32), 10)
    hot = rows_unique(200, 6, 1000, 1.0)
    hot[:, 0] = 3  # one feature touched by every position
    hot[::3, 1] = 999
    cases["hot"] = (hot, 1000)
    out = {}
    for name, (idx, T) in cases.items():
        flat_bid = kernel._get_flat_batch_indices(idx.shape[0], idx.shape[1], idx.device)
        sb, sf, sc, ss = kernel._build_sorted_backward_inputs(idx, flat_bid)
        out[f"{name}_idx"] = idx.numpy()
        out[f"{name}_T"] = np.int64(T)
        out[f"{name}_sorted_bid"] = sb.numpy()
        out[f"{name}_seg_feat"] = sf.numpy()
        out[f"{name}_seg_count"] = sc.numpy()
        out[f"{name}_seg_start"] = ss.numpy()
    np.savez_compressed(os.path.join(HERE, "sorted_backward_inputs.npz"), names=np.array(list(cases)), **out)

    # --- FT quantisation -----------------------------------------------------
    qm = QuantizationManager(QuantizationConfig())
    gq = torch.Generator().manual_seed(77)
    L1, NP, R = 64, 8, 300
    bias = torch.randn(L1, generator=gq) * 0.05
    weight = torch.randn(R, L1, generator=gq) * 0.01
    psqt = torch.randn(R, NP, generator=gq) * 0.2
    # exact half-way cases: k / 510 * 255 = k / 2 -> ties to even
    weight[0, :] = torch.arange(L1, dtype=torch.float32) / 510.0
    weight[1, :] = -torch.arange(L1, dtype=torch.float32) / 510.0
    bias[:16] = torch.arange(16, dtype=torch.float32) / 510.0
    psqt[0, :] = torch.tensor([0.5, 1.5, 2.5, -0.5, -1.5, 3.5, 0.0, 7.5]) / 9600.0
    qb, qw, qp = qm.quantize_feature_transformer(bias, weight, psqt)
    np.savez_compressed(
        os.path.join(HERE, "quantize_ft.npz"),
        bias=bias.numpy(), weight=weight.numpy(), psqt=psqt.numpy(),
        q_bias=qb.numpy(), q_weight=qw.numpy(), q_psqt=qp.numpy(),
        ft_quantized_one=np.float64(qm.ft_quantized_one),
        psqt_scale=np.float64(qm.nnue2score * qm.weight_scale_out),
    )

    # --- HalfKA export remap (24576 -> 22528 rows) --------------------------
    torch.manual_seed(5)
    feat = halfka_v2_hm.HalfKav2Hm(1)
    with torch.no_grad():
        feat.virtual_weight.normal_()
    export = feat.get_export_weights()
    np.savez_compressed(
        os.path.join(HERE, "export_weights.npz"),
        weight=feat.weight.detach().numpy(), virtual=feat.virtual_weight.detach().numpy(),
        export=export.numpy(),
    )

    # --- composed feature-set sizes -----------------------------------------
    ft = composed.combine_input_features(full_threats.FullThreats, halfka_v2_hm.HalfKav2Hm)(16)
    np.savez_compressed(
        os.path.join(HERE, "composed_sizes.npz"),
        num_inputs=np.int64(ft.NUM_INPUTS), max_active=np.int64(ft.MAX_ACTIVE_FEATURES),
        num_real=np.int64(ft.NUM_REAL_FEATURES), hash=np.int64(ft.HASH),
        halfka_inputs=np.int64(halfka_v2_hm.HalfKav2Hm.NUM_INPUTS),
        threat_inputs=np.int64(full_threats.FullThreats.NUM_INPUTS),
    )
    ranger22_fixture(ref_root)
    transform_inputs_fixture(ref_root)
    print("fixtures written to", HERE)


def transform_inputs_fixture(ref_root: str) -> None:
    """NNUEModel._transform_inputs on given FT outputs (the FT call is stubbed
    to return them), forward and autograd backward, small L1."""
    if "chess" not in sys.modules:
        _install_chess_stub()
    if ref_root not in sys.path:
        sys.path.insert(0, ref_root)
    from src.model.model import NNUEModel

    B, L1, NP = 40, 24, 8
    gen = torch.Generator().manual_seed(7)
    wp = torch.randn(B, L1 + NP, generator=gen) * 0.8 + 0.4
    bp = torch.randn(B, L1 + NP, generator=gen) * 0.8 + 0.4
    wp[0, :6] = torch.tensor([0.0, 1.0, -0.0, 1.5, -0.25, 0.5])  # clamp edges
    bp[1, :6] = torch.tensor([1.0, 0.0, 2.0, -0.0, 0.999, 1e-30])
    us = (torch.rand(B, 1, generator=gen) < 0.5).float()
    pidx = torch.randint(0, NP, (B,), generator=gen)
    d_l0 = torch.randn(B, L1, generator=gen)
    d_l0[2, :4] = torch.tensor([-0.0, 0.0, -1.0, 1.0])
    d_psqt = torch.randn(B, 1, generator=gen)
    d_psqt[3, 0] = -0.0

    class _Stub:
        pass

    stub = _Stub()
    stub.L1 = L1
    wpg, bpg = wp.clone().requires_grad_(), bp.clone().requires_grad_()
    stub.input = lambda wi, bi: (wpg, bpg)
    l0, psqt = NNUEModel._transform_inputs(stub, us, None, None, pidx)
    torch.autograd.backward([l0, psqt], [d_l0, d_psqt])
    np.savez_compressed(os.path.join(HERE, "transform_inputs.npz"), wp=wp.numpy(), bp=bp.numpy(), us=us.numpy(),
                        psqt_indices=pidx.numpy(), d_l0=d_l0.numpy(), d_psqt=d_psqt.numpy(),
                        l0=l0.detach().numpy(), psqt=psqt.detach().numpy(), d_wp=wpg.grad.numpy(),
                        d_bp=bpg.grad.numpy(), l1=np.int64(L1))


def ranger22_fixture(ref_root: str) -> None:
    """Seven Ranger22 steps (one lookahead merge at step 5) on a 2-D and a 1-D
    CPU parameter with the trainer's configuration; CPU tensors take the
    reference's baseline-equivalent path (optimizer.py:606-659)."""
    if ref_root not in sys.path:
        sys.path.insert(0, ref_root)
    from src.ranger22 import Ranger22

    gen = torch.Generator().manual_seed(22)
    w = torch.nn.Parameter(torch.randn(6, 20, generator=gen) * 0.1)
    b = torch.nn.Parameter(torch.randn(20, generator=gen) * 0.1)
    w0, b0 = w.detach().clone(), b.detach().clone()
    opt = Ranger22([{"params": [w, b]}], lr=8.75e-4, betas=(0.9, 0.999), eps=1.0e-7, using_gc=False,
                   using_normgc=False, weight_decay=0.0, num_batches_per_epoch=100, num_epochs=10,
                   warmdown_active=False, use_warmup=False, use_adaptive_gradient_clipping=False, softplus=False,
                   pnm_momentum_factor=0.0)
    steps = 7
    gw = torch.randn(steps, 6, 20, generator=gen)
    gb = torch.randn(steps, 20, generator=gen)
    for s in range(steps):
        w.grad = gw[s].clone()
        b.grad = gb[s].clone()
        opt.step()
    out = {"w0": w0.numpy(), "b0": b0.numpy(), "gw": gw.numpy(), "gb": gb.numpy(), "lr": np.float64(8.75e-4),
           "w": w.detach().numpy(), "b": b.detach().numpy()}
    for name, p in (("w", w), ("b", b)):
        st = opt.state[p]
        for key in ("grad_ma", "neg_grad_ma", "variance_ma", "lookahead_params"):
            out[f"{name}_{key}"] = st[key].numpy()
    np.savez_compressed(os.path.join(HERE, "ranger22_steps.npz"), **out)


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: python tests/golden/make_golden.py REFERENCE_CHECKOUT [ranger22|transform_inputs]")
    if len(sys.argv) > 2 and sys.argv[2] == "ranger22":
        ranger22_fixture(sys.argv[1])
    elif len(sys.argv) > 2 and sys.argv[2] == "transform_inputs":
        transform_inputs_fixture(sys.argv[1])
    else:
        main(sys.argv[1])
