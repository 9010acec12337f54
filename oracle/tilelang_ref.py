"""ORACLE -- TEST INFRASTRUCTURE ONLY.

Loads the reference's own feature-transformer package (``SparseLinearFunction``
and its TileLang kernels, ``src/model/modules/feature_transformer/``), staged
unmodified into ``oracle/_ref/ref_feature_transformer/`` by
``oracle/build.py``.  Used as the GPU checker of the fp32 forward and weight
gradient and as the GPU bar of the bench; never by the product package.
"""

from __future__ import annotations

import os
import sys

from . import build as _build


class ReferenceUnavailable(RuntimeError):
    pass


def load():
    """The staged reference package (a module exposing ``SparseLinearFunction``
    and ``kernel``).  Raises ReferenceUnavailable when it was not staged or its
    files differ from the manifest."""
    pkg_dir = _build.staged_reference()
    if pkg_dir is None:
        raise ReferenceUnavailable(
            "the reference feature-transformer package is not staged under oracle/_ref "
            "(run: python oracle/build.py --reference <reference checkout>)")
    parent = os.path.dirname(pkg_dir)
    if parent not in sys.path:
        sys.path.insert(0, parent)
    import importlib

    return importlib.import_module(_build.REF_PKG)


def reference_pair_step(ref, i0, i1, W, bias, g0, g1):
    """One fwd + bwd of both perspectives exactly as the reference's composed
    module drives the op (``composed.py:52-53``): two ``SparseLinearFunction``
    calls sharing one table, autograd summing the two dense weight gradients.
    Returns (out0, out1, dW, dB)."""
    Wr = W.detach().requires_grad_()
    br = bias.detach().requires_grad_()
    o0 = ref.SparseLinearFunction.apply(i0, Wr, br)
    o1 = ref.SparseLinearFunction.apply(i1, Wr, br)
    import torch

    torch.autograd.backward([o0, o1], [g0, g1])
    return o0.detach(), o1.detach(), Wr.grad, br.grad
