"""Drop-in for src/model/modules/feature_transformer (reference __init__.py:1-5)."""

from .epilogue import TransformInputsFunction, transform_inputs
from .functions import SparseLinearFunction, SparseLinearPairFunction
from .kernel import make_sparse_input_linear_backward_kernel, make_sparse_input_linear_forward_kernel
from .library import sparse_linear, sparse_linear_pair

__all__ = [
    "TransformInputsFunction",
    "transform_inputs",
    "SparseLinearFunction",
    "SparseLinearPairFunction",
    "make_sparse_input_linear_forward_kernel",
    "make_sparse_input_linear_backward_kernel",
    "sparse_linear",
    "sparse_linear_pair",
]
