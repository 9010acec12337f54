"""Host-side logic of the Ranger22FT optimizer (no GPU needed)."""

import math

import pytest
import torch

from oracle import ranger22 as oracle_r22
from stockfish_trainer_b200 import optim


def test_unsupported_configuration_is_refused():
    for kwargs in ({"using_gc": True}, {"weight_decay": 1e-4}, {"softplus": True}, {"use_warmup": True},
                   {"use_adaptive_gradient_clipping": True}, {"momentum_type": "classic"}):
        with pytest.raises(NotImplementedError):
            optim.Ranger22FT([torch.nn.Parameter(torch.zeros(3))], lr=1e-3, **kwargs)


def test_scalars_match_oracle_restatement():
    for step in (1, 2, 7, 1000):
        a = optim.ranger22_scalars(8.75e-4, step)
        b = oracle_r22.scalars(8.75e-4, step)
        assert len(a) == 12
        for x, y in zip(a, b):
            assert math.isclose(float(x), float(y), rel_tol=1e-7)


def test_update_rejects_bad_tensors():
    p = torch.zeros(4, 8)
    with pytest.raises(ValueError):  # CPU tensors are refused before any native call
        optim.ranger22_update_(p, p, p, p, p, [0.0] * 12)
    with pytest.raises(ValueError):
        optim.ranger22_update_(torch.zeros(2, 2, 2), p, p, p, p, [0.0] * 12)
