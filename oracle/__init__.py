"""ORACLE -- TEST INFRASTRUCTURE ONLY.

CPU restatement of rgodha24/stockfish-trainer's sparse feature-transformer
path, used as the checker in ``tests/``, in ``__graft_entry__.smoke()`` and as
the timed CPU baseline of ``bench.py``.  Nothing in the product package
imports it.

* ``ft_oracle.c`` (built by ``build.py``) -- forward, backward (reference
  summation order), quantised int16 forward, quantisation, export row map.
* ``features.py`` -- feature-index functions (HalfKAv2_hm, Full_Threats).

All arrays are numpy; functions mirror the reference semantics noted in the C
source (src/model/modules/feature_transformer/kernel.py and functions.py,
src/model/quantize.py, src/model/modules/features/halfka_v2_hm.py).
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import build as _build

_lib = None

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = _build.build()
        L = ctypes.CDLL(path)
        L.oracle_max_threads.restype = ctypes.c_int
        L.oracle_ft_forward.restype = _I64
        L.oracle_ft_forward.argtypes = [_P, _I64, _I32, _P, _I64, _I32, _P, _P, ctypes.c_int]
        L.oracle_ft_sorted_backward_inputs.restype = _I64
        L.oracle_ft_sorted_backward_inputs.argtypes = [_P, _I64, _I32, _I64, _P, _P, _P, _P, _P]
        L.oracle_ft_backward.restype = None
        L.oracle_ft_backward.argtypes = [_P, _I64, _I32, _P, _I64, _I32, _P, _P, ctypes.c_int]
        L.oracle_halfka_export_row.restype = _I32
        L.oracle_halfka_export_row.argtypes = [_I32]
        L.oracle_quantize_i16.argtypes = [_P, _I64, ctypes.c_float, _P]
        L.oracle_quantize_i32.argtypes = [_P, _I64, ctypes.c_float, _P]
        L.oracle_ft_quantized_forward.restype = _I64
        L.oracle_ft_quantized_forward.argtypes = [_P, _I64, _I32, _P, _P, _I64, _I32, _I32, _P,
                                                  ctypes.c_int, _P, _P, ctypes.c_int]
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _c(a, dtype) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def ft_forward(idx, weight, bias, nthreads: int = 0) -> np.ndarray:
    """out[b] = bias + sum_k W[idx[b, k]] (ascending k, -1 skipped)."""
    idx = _c(idx, np.int32)
    weight = _c(weight, np.float32)
    bias = _c(bias, np.float32)
    B, K = idx.shape
    T, C = weight.shape
    out = np.empty((B, C), dtype=np.float32)
    bad = lib().oracle_ft_forward(_ptr(idx), B, K, _ptr(weight), T, C, _ptr(bias), _ptr(out), nthreads)
    if bad:
        raise ValueError(f"{bad} feature indices outside [-1, {T})")
    return out


def sorted_backward_inputs(idx, num_inputs: int):
    """kernel.py:108-138: (sorted_bid, seg_feat, seg_count, seg_start), int32."""
    idx = _c(idx, np.int32)
    B, K = idx.shape
    n = max(B * K, 1)
    sb = np.empty(n, np.int32)
    sf = np.empty(max(num_inputs, 1), np.int32)
    sc = np.empty_like(sf)
    ss = np.empty_like(sf)
    nnz = ctypes.c_int64(0)
    u = lib().oracle_ft_sorted_backward_inputs(_ptr(idx), B, K, num_inputs, _ptr(sb), _ptr(sf),
                                               _ptr(sc), _ptr(ss), ctypes.byref(nnz))
    return sb[: nnz.value].copy(), sf[:u].copy(), sc[:u].copy(), ss[:u].copy()


def ft_backward(idx, grad_output, num_inputs: int, weight_grad=None, bias_grad=None, nthreads: int = 0):
    """Reference backward for one perspective, ACCUMULATING like kernel.py:167-186/:269.

    ``weight_grad`` / ``bias_grad`` default to zeros (what functions.py:62-65
    allocates).  Returns (weight_grad, bias_grad)."""
    idx = _c(idx, np.int32)
    g = _c(grad_output, np.float32)
    B, K = idx.shape
    C = g.shape[1]
    dW = np.zeros((num_inputs, C), np.float32) if weight_grad is None else weight_grad
    dB = np.zeros(C, np.float32) if bias_grad is None else bias_grad
    assert dW.flags.c_contiguous and dW.dtype == np.float32
    assert dB.flags.c_contiguous and dB.dtype == np.float32
    lib().oracle_ft_backward(_ptr(idx), B, K, _ptr(g), num_inputs, C, _ptr(dW), _ptr(dB), nthreads)
    return dW, dB


def ft_backward_pair(idx0, idx1, grad0, grad1, num_inputs: int, nthreads: int = 0):
    """Module-level gradient of the reference's two calls sharing one table
    (composed.py:49-54): each perspective's backward starts from zeros and
    autograd adds the two dense results once."""
    dW0, dB0 = ft_backward(idx0, grad0, num_inputs, nthreads=nthreads)
    dW1, dB1 = ft_backward(idx1, grad1, num_inputs, nthreads=nthreads)
    return dW0 + dW1, dB0 + dB1


def halfka_export_rows(rows) -> np.ndarray:
    """halfka_v2_hm.py:100-134 row map, training (24576) -> export (22528)."""
    r = np.asarray(rows, dtype=np.int64)
    bucket, plane, sq = r // 768, (r % 768) // 64, r % 64
    return (bucket * 704 + np.minimum(plane, 10) * 64 + sq).astype(np.int32)


def quantize(x, scale: float, dtype) -> np.ndarray:
    """quantize.py:83-89: x.mul(scale).round() in fp32 (half to even)."""
    x = _c(x, np.float32)
    out = np.empty(x.shape, dtype=dtype)
    if dtype == np.int16:
        lib().oracle_quantize_i16(_ptr(x), x.size, scale, _ptr(out))
    elif dtype == np.int32:
        lib().oracle_quantize_i32(_ptr(x), x.size, scale, _ptr(out))
    else:
        raise TypeError(dtype)
    return out


def ft_quantized_forward(idx, wq, pq, bias_q, map_training: bool, nthreads: int = 0):
    """int16 accumulators (two's-complement wrap) + int32 PSQT, per position."""
    idx = _c(idx, np.int32)
    wq = _c(wq, np.int16)
    pq = _c(pq, np.int32)
    bias_q = _c(bias_q, np.int16)
    B, K = idx.shape
    Tq, L1 = wq.shape
    NP = pq.shape[1]
    acc = np.empty((B, L1), np.int16)
    ps = np.empty((B, NP), np.int32)
    bad = lib().oracle_ft_quantized_forward(_ptr(idx), B, K, _ptr(wq), _ptr(pq), Tq, L1, NP, _ptr(bias_q),
                                            int(map_training), _ptr(acc), _ptr(ps), nthreads)
    if bad:
        raise ValueError(f"{bad} feature indices out of range")
    return acc, ps


def halfka_export_weights(weight, virtual) -> np.ndarray:
    """get_export_weights (halfka_v2_hm.py:100-134): coalesce the virtual rows
    (fp32 add, as ``weight + virtual.repeat(32, 1)``) and merge the two king
    planes into plane 10 (own king only at the bucket's king square)."""
    weight = _c(weight, np.float32)
    virtual = _c(virtual, np.float32)
    coalesced = weight + np.tile(virtual, (32, 1))
    export = np.zeros((32 * 704, weight.shape[1]), np.float32)
    inv = inverse_king_buckets()
    for b in range(32):
        s, d = b * 768, b * 704
        export[d : d + 640] = coalesced[s : s + 640]
        export[d + 640 : d + 704] = coalesced[s + 704 : s + 768]
        export[d + 640 + inv[b]] = coalesced[s + 640 + inv[b]]
    return export


def inverse_king_buckets() -> list[int]:
    from .features import KING_BUCKETS

    inv = [0] * 32
    for sq, bucket in enumerate(KING_BUCKETS):
        if bucket >= 0:
            inv[bucket] = sq
    return inv


__all__ = [
    "lib", "max_threads", "ft_forward", "ft_backward", "ft_backward_pair", "sorted_backward_inputs",
    "halfka_export_rows", "halfka_export_weights", "quantize", "ft_quantized_forward",
    "inverse_king_buckets",
]
