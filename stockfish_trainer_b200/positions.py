"""Seeded synthetic positions and their feature indices (native, host side).

Stands in for the reference's data path (binpack decode + the Rust feature
encoder, src/rust/feature_extraction.rs) when no training data is available:
``generate_positions`` draws boards, ``encode`` turns them into the int32
``[B, K]`` index tensors, compacted and -1 padded, that the loader hands to
the feature transformer (src/data/device.py:76-77).

Feature-set names follow the reference (src/model/modules/features/__init__.py):
"HalfKAv2_hm^", "Full_Threats", "Full_Threats+HalfKAv2_hm^" (the trailing
"^" marks the factorised training variant and does not change indices).
"""

from __future__ import annotations

import numpy as np

from . import _native

HALFKA_INPUTS = 24576
FULL_THREATS_INPUTS = 60720

_FEATURE_SETS = {
    "HalfKAv2_hm": (0, HALFKA_INPUTS, 32),
    "Full_Threats": (1, FULL_THREATS_INPUTS, 128),
    "Full_Threats+HalfKAv2_hm": (2, FULL_THREATS_INPUTS + HALFKA_INPUTS, 160),
}


def feature_set_info(name: str) -> tuple[int, int, int]:
    """(native id, num_inputs, max_active) for a feature-set name."""
    key = name.replace("^", "")
    if key not in _FEATURE_SETS:
        raise ValueError(f"unknown feature set {name!r}")
    return _FEATURE_SETS[key]


def generate_positions(n: int, seed: int = 0, first: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """Boards [n, 64] uint8 (piece id or 12 = empty) and side to move [n] uint8.

    Position i depends only on (seed, first + i), so any slice can be
    regenerated independently (e.g. per DDP rank)."""
    board = np.empty((n, 64), dtype=np.uint8)
    stm = np.empty(n, dtype=np.uint8)
    _native.call("nnue_generate_positions", seed & (2**64 - 1), first, n, board.ctypes.data, stm.ctypes.data)
    return board, stm


def encode(board: np.ndarray, feature_set: str, nthreads: int = 0):
    """White and black index arrays [n, K] int32 plus active counts [n]."""
    fid, _, K = feature_set_info(feature_set)
    board = np.ascontiguousarray(board, dtype=np.uint8)
    n = board.shape[0]
    white = np.empty((n, K), dtype=np.int32)
    black = np.empty((n, K), dtype=np.int32)
    wc = np.empty(n, dtype=np.int32)
    bc = np.empty(n, dtype=np.int32)
    _native.call("nnue_encode_features", board.ctypes.data, n, fid, white.ctypes.data, black.ctypes.data,
                 wc.ctypes.data, bc.ctypes.data, nthreads)
    return white, black, wc, bc


def encode_device(board, feature_set: str, with_counts: bool = False, out=None):
    """The same index rows as ``encode``, computed on the GPU from a uint8
    ``[n, 64]`` board tensor in device memory (nnue_ft_encode_features), on
    the current stream: returns white and black ``[n, K]`` int32 device
    tensors (+ counts), written into ``out = (white, black)`` when given.  A
    loader can ship boards (64 bytes per position) instead of index rows
    (4 * K bytes per perspective).  Rejected positions get all -1 rows and
    raise the device error flag DEVERR_BAD_POSITION."""
    import torch

    fid, _, K = feature_set_info(feature_set)
    if board.dtype != torch.uint8 or board.dim() != 2 or board.shape[1] != 64 or not board.is_contiguous():
        raise ValueError("board must be a contiguous [n, 64] uint8 tensor")
    if not board.is_cuda:
        raise ValueError("encode_device needs a CUDA tensor")
    n, dev = board.shape[0], board.device
    if out is not None:
        white, black = out
        for t in (white, black):
            if t.dtype != torch.int32 or tuple(t.shape) != (n, K) or not t.is_contiguous() or t.device != dev:
                raise ValueError(f"out tensors must be contiguous [{n}, {K}] int32 on {dev}")
    else:
        white = torch.empty(n, K, dtype=torch.int32, device=dev)
        black = torch.empty(n, K, dtype=torch.int32, device=dev)
    wc = torch.empty(n, dtype=torch.int32, device=dev) if with_counts else None
    bc = torch.empty(n, dtype=torch.int32, device=dev) if with_counts else None
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        _native.call("nnue_ft_encode_features", board.data_ptr(), n, fid, white.data_ptr(), black.data_ptr(),
                     wc.data_ptr() if wc is not None else None, bc.data_ptr() if bc is not None else None, stream)
    return (white, black, wc, bc) if with_counts else (white, black)


def synthetic_batch(n: int, feature_set: str, seed: int = 0, first: int = 0):
    """(white [n, K], black [n, K], side to move [n]) for n seeded positions."""
    board, stm = generate_positions(n, seed, first)
    white, black, _, _ = encode(board, feature_set)
    return white, black, stm


def threat_table_total() -> int:
    return int(_native.load().nnue_threat_table_total())
