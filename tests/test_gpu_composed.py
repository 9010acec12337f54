"""Module-level composed FT (feature_transformer/composed.py) vs the
reference module's graph: torch.cat of the per-feature tables (HalfKA plus
its virtual rows repeated 32 times) fed to the FT op twice, gradients split
back by autograd.  Outputs and all parameter gradients must be bit-identical;
the weight gradients are also checked against the oracle."""

import math

import numpy as np
import pytest
import torch
from torch import nn

import oracle
from stockfish_trainer_b200.feature_transformer import SparseLinearPairFunction
from stockfish_trainer_b200.feature_transformer.composed import ComposedFeatureTransformer

from _inputs import feature_batch

pytestmark = pytest.mark.gpu


class _Threats(nn.Module):
    """Parameters and interface of FullThreats (full_threats.py)."""
    HASH = 0x8F234CB8
    FEATURE_NAME = INPUT_FEATURE_NAME = "Full_Threats"
    NUM_INPUTS = NUM_REAL_FEATURES = 60720
    MAX_ACTIVE_FEATURES = 128

    def __init__(self, num_outputs):
        super().__init__()
        self.num_outputs = num_outputs
        self.weight = nn.Parameter(torch.empty(self.NUM_INPUTS, num_outputs))
        with torch.no_grad():
            self.weight.uniform_(-math.sqrt(1 / self.NUM_INPUTS), math.sqrt(1 / self.NUM_INPUTS))

    def merged_weight(self):
        return self.weight


class _HalfKA(nn.Module):
    """Parameters and interface of HalfKav2Hm (halfka_v2_hm.py:40-70)."""
    HASH = 0x7F234CB8
    FEATURE_NAME = "HalfKAv2_hm^"
    INPUT_FEATURE_NAME = "HalfKAv2_hm"
    NUM_INPUTS, NUM_BUCKETS, NUM_REAL_FEATURES, MAX_ACTIVE_FEATURES = 24576, 32, 22528, 32

    def __init__(self, num_outputs):
        super().__init__()
        self.num_outputs = num_outputs
        self.weight = nn.Parameter(torch.empty(self.NUM_INPUTS, num_outputs))
        self.virtual_weight = nn.Parameter(torch.zeros(768, num_outputs))
        with torch.no_grad():
            self.weight.uniform_(-math.sqrt(1 / self.NUM_INPUTS), math.sqrt(1 / self.NUM_INPUTS))

    def merged_weight(self):
        return self.weight + self.virtual_weight.repeat(self.NUM_BUCKETS, 1)


def _modules(C, dev, seed):
    torch.manual_seed(seed)
    feats = [_Threats(C), _HalfKA(C)]
    with torch.no_grad():
        feats[1].virtual_weight.normal_(0, 0.01)
    m = ComposedFeatureTransformer(feats).to(dev)
    return m, feats


@pytest.mark.parametrize("C,B", [(72, 700), (30, 257)])
def test_composed_module_matches_reference_graph(cuda, C, B):
    white, black, T = feature_batch(B, "Full_Threats+HalfKAv2_hm^", seed=C)
    assert T == 60720 + 24576
    m, feats = _modules(C, cuda, seed=C)
    i0, i1 = torch.from_numpy(white).to(cuda), torch.from_numpy(black).to(cuda)
    g = torch.Generator().manual_seed(1)
    d0 = torch.randn(B, C, generator=g).to(cuda)
    d1 = torch.randn(B, C, generator=g).to(cuda)

    out0, out1 = m(i0, i1)
    torch.autograd.backward([out0, out1], [d0, d1])
    got = [out0.detach(), out1.detach(), m.bias.grad, feats[0].weight.grad, feats[1].weight.grad,
           feats[1].virtual_weight.grad]
    for p in m.parameters():
        p.grad = None

    merged = torch.cat([f.merged_weight() for f in feats], dim=0)  # the reference module's graph
    r0, r1 = SparseLinearPairFunction.apply(i0, i1, merged, m.bias)
    torch.autograd.backward([r0, r1], [d0, d1])
    want = [r0.detach(), r1.detach(), m.bias.grad, feats[0].weight.grad, feats[1].weight.grad,
            feats[1].virtual_weight.grad]
    names = ["out_white", "out_black", "bias_grad", "threat_weight_grad", "halfka_weight_grad", "virtual_grad"]
    for a, b, name in zip(got, want, names):
        assert a.shape == b.shape, name
        np.testing.assert_array_equal(a.cpu().numpy().view(np.int32), b.cpu().numpy().view(np.int32), err_msg=name)

    # the merged weight gradient against the oracle (ascending-position sums, perspectives added once)
    rW, _ = oracle.ft_backward_pair(white, black, d0.cpu().numpy(), d1.cpu().numpy(), T)
    np.testing.assert_array_equal(np.concatenate([got[3].cpu().numpy(), got[4].cpu().numpy()]), rW)


def test_composed_module_attributes_follow_reference(cuda):
    m, feats = _modules(16, cuda, seed=3)
    assert m.NUM_INPUTS == 85296 and m.MAX_ACTIVE_FEATURES == 160 and m.NUM_REAL_FEATURES == 60720 + 22528
    assert m.FEATURE_NAME == "Full_Threats+HalfKAv2_hm^"
    h = 0
    for f in feats:
        h = ((h << 1) | (h >> 31)) & 0xFFFFFFFF
        h ^= f.HASH
    assert m.HASH == h
