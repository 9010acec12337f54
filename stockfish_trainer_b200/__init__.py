"""B200-native (sm_100a) sparse NNUE feature transformer.

A drop-in for the hot path of rgodha24/stockfish-trainer's
``src/model/modules/feature_transformer``: ``SparseLinearFunction`` and the
kernel factories keep the reference's names and semantics, backed by
hand-written CUDA kernels behind a C ABI (include/nnue_ft.h).

Submodules
  feature_transformer  autograd functions, kernel factories, tensor ops
  positions            seeded synthetic positions + feature-index encoder
  ddp                  torchrun data-parallel step with the FT gradient allreduce
  build                in-tree build of libnnue_ft.so
"""

from .feature_transformer import (
    SparseLinearFunction,
    SparseLinearPairFunction,
    make_sparse_input_linear_backward_kernel,
    make_sparse_input_linear_forward_kernel,
)

__all__ = [
    "SparseLinearFunction",
    "SparseLinearPairFunction",
    "make_sparse_input_linear_forward_kernel",
    "make_sparse_input_linear_backward_kernel",
]
