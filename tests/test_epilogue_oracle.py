"""The epilogue oracle (oracle/epilogue.py) reproduces the reference's own
NNUEModel._transform_inputs (tests/golden/transform_inputs.npz, produced by
src/model/model.py itself with the FT call stubbed), forward and autograd
backward, bit for bit (zero signs included)."""

import os

import numpy as np
import torch

from oracle import epilogue

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "transform_inputs.npz")


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.int32)


def test_oracle_matches_reference_transform_inputs():
    z = np.load(GOLD)
    t = lambda k: torch.from_numpy(z[k])
    l0, psqt, d_wp, d_bp = epilogue.forward_backward(t("wp"), t("bp"), t("us"), t("psqt_indices"), int(z["l1"]),
                                                     t("d_l0"), t("d_psqt"))
    for got, key in ((l0, "l0"), (psqt, "psqt"), (d_wp, "d_wp"), (d_bp, "d_bp")):
        np.testing.assert_array_equal(_bits(got.numpy()), _bits(z[key]), err_msg=key)
