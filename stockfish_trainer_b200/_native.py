"""ctypes binding of ``libnnue_ft.so`` (C ABI declared in include/nnue_ft.h).

The library is built in-tree by ``stockfish_trainer_b200.build`` (and by
``__graft_entry__.build()``).  There is no fallback: if the library cannot be
loaded every entry point raises, so a missing build can never silently turn
into a different implementation.
"""

from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_U64 = ctypes.c_uint64
_SZ = ctypes.c_size_t

NNUE_OK = 0
NNUE_ERR_INVALID_ARGUMENT = -1
NNUE_ERR_UNSUPPORTED = -2
NNUE_ERR_WORKSPACE = -3
NNUE_ERR_CUDA = -4
DEVERR_BAD_INDEX = 1
DEVERR_BAD_QUANT_INDEX = 2
DEVERR_BAD_PSQT_INDEX = 8
DEVERR_BAD_POSITION = 16
DEVERR_EXCHANGE_TIMEOUT = 32

_SIGNATURES = {
    "nnue_ft_version": (_I32, []),
    "nnue_ft_launch_count": (_U64, []),
    "nnue_ft_kernel_timer_arm": (_I32, [ctypes.c_uint32, _I32]),
    "nnue_ft_kernel_timer_read": (_I32, [_I32, ctypes.POINTER(ctypes.c_float), _I32, ctypes.POINTER(_I32)]),
    "nnue_ft_last_error": (ctypes.c_char_p, []),
    "nnue_ft_device_errors": (_I32, [ctypes.POINTER(ctypes.c_uint32), _I32]),
    "nnue_ft_set_param": (_I32, [ctypes.c_char_p, _I64]),
    "nnue_ft_get_param": (_I64, [ctypes.c_char_p]),
    "nnue_ft_forward": (_I32, [_P, _I64, _I32, _P, _I64, _I32, _P, _P, _P]),
    "nnue_ft_forward_pair": (_I32, [_P, _P, _I64, _I32, _P, _I64, _I32, _P, _P, _P, _P]),
    "nnue_ft_forward_pair_prepare": (_I32, [_P, _P, _I64, _I32, _P, _I64, _I32, _P, _P, _P, _P, _SZ, _P]),
    "nnue_ft_backward_workspace_size": (_SZ, [_I64, _I32, _I64, _I32, _I32]),
    "nnue_ft_backward": (_I32, [_P, _P, _I64, _I32, _P, _P, _I32, _I64, _I32, _P, _P, _I32, _P, _SZ, _P]),
    "nnue_ft_backward_apply_rows": (
        _I32, [_P, _P, _I64, _I32, _I32, _I64, _I32, _P, _P, _I32, _I64, _I64, _I32, _P, _SZ, _P]),
    "nnue_ft_backward_noalloc": (_I32, [_P, _P, _I64, _I32, _P, _P, _I32, _I64, _I32, _P, _P, _I32, _P]),
    "nnue_ft_noalloc_scratch_bytes": (_SZ, []),
    "nnue_ft_backward_prepare": (_I32, [_P, _P, _I64, _I32, _I32, _I64, _I32, _P, _SZ, _P]),
    "nnue_ft_backward_apply": (_I32, [_P, _P, _I64, _I32, _I32, _I64, _I32, _P, _P, _I32, _P, _SZ, _P]),
    "nnue_ft_quantized_forward_pair": (
        _I32, [_P, _P, _I32, _I64, _I32, _P, _P, _I64, _I32, _I32, _P, _I32, _P, _P, _P, _P, _P]),
    "nnue_ft_halfka_export_quantize": (_I32, [_P, _P, _I32, _I32, ctypes.c_float, ctypes.c_float, _P, _P, _P]),
    "nnue_ft_quantize_i16": (_I32, [_P, _I64, ctypes.c_float, _P, _P]),
    "nnue_ft_ranger22_step": (_I32, [_P, _P, _P, _P, _P, _P, _I64, _I64, _P, _I32, ctypes.c_float, _P]),
    "nnue_ft_epilogue_forward": (_I32, [_P, _P, _I64, _I32, _I32, _P, _P, _P, _P, _P]),
    "nnue_ft_forward_pair_tables": (_I32, [_P, _P, _I64, _I32, _P, _P, _I32, _I32, _P, _P, _P, _P]),
    "nnue_ft_forward_pair_tables_prepare": (_I32, [_P, _P, _I64, _I32, _P, _P, _I32, _I32, _P, _P, _P, _P, _SZ,
                                                    _P]),
    "nnue_ft_backward_apply_tables": (_I32, [_P, _P, _I64, _I32, _P, _P, _I32, _I32, _P, _I32, _P, _SZ, _P]),
    "nnue_ft_merge_virtual": (_I32, [_P, _I64, _P, _I64, _I32, _P, _P]),
    "nnue_ft_epilogue_backward": (_I32, [_P, _P, _I64, _I32, _I32, _P, _P, _P, _P, _P, _P, _P]),
    "nnue_ft_gather_probe": (_I32, [_P, _I64, _P, _I32, _I32, _P, _P]),
    "nnue_threat_table_total": (_I32, []),
    "nnue_generate_positions": (_I32, [_U64, _I64, _I64, _P, _P]),
    "nnue_encode_features": (_I32, [_P, _I64, _I32, _P, _P, _P, _P, _I32]),
    "nnue_ft_encode_features": (_I32, [_P, _I64, _I32, _P, _P, _P, _P, _P]),
    "nnue_ft_exchange_alloc": (_I32, [_SZ, ctypes.POINTER(_P), _P]),
    "nnue_ft_exchange_free": (_I32, [_P]),
    "nnue_ft_exchange_open": (_I32, [_P, ctypes.POINTER(_P)]),
    "nnue_ft_exchange_close": (_I32, [_P]),
    "nnue_ft_exchange": (_I32, [_P, _I32, _P, _I32, _I32, _I32, ctypes.c_uint32, _I32, _P]),
}

_lib = None
_lock = threading.Lock()


class NativeError(RuntimeError):
    """A C-ABI call returned a negative status."""

    def __init__(self, func: str, code: int, message: str):
        super().__init__(f"{func} failed with status {code}: {message}")
        self.code = code


def lib_path() -> str:
    return _build.LIB_PATH


def load(build_if_missing: bool | None = None) -> ctypes.CDLL:
    """Load (building first if allowed and needed) the native library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if build_if_missing is None:
            build_if_missing = os.environ.get("NNUE_FT_NO_BUILD", "0") != "1"
        path = lib_path()
        if build_if_missing:
            path = _build.build()
        if not os.path.exists(path):
            raise ImportError(
                f"{path} is missing: build it with `python -m stockfish_trainer_b200.build` "
                "(there is no non-native implementation of this path)")
        L = ctypes.CDLL(path)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def last_error() -> str:
    msg = load().nnue_ft_last_error()
    return msg.decode() if msg else ""


def check(func: str, rc: int) -> None:
    if rc != NNUE_OK:
        raise NativeError(func, rc, last_error())


def call(func: str, *args) -> int:
    rc = getattr(load(), func)(*args)
    check(func, rc)
    return rc


def launch_count() -> int:
    """Kernels launched by the native library so far (process-wide)."""
    return int(load().nnue_ft_launch_count())


TIMED_FORWARD, TIMED_LIGHT_ROWS, TIMED_HEAVY_ROWS = 0, 1, 2


def kernel_timer_arm(kernels, capacity: int) -> None:
    """Time every launch of the given kernel classes (TIMED_* values) with a
    CUDA event pair on its own stream, up to `capacity` launches in total;
    an empty `kernels` disarms."""
    mask = 0
    for k in kernels:
        mask |= 1 << int(k)
    call("nnue_ft_kernel_timer_arm", mask, int(capacity))


def kernel_timer_read(kernel: int, max_launches: int = 4096) -> list:
    """Durations (ms) of the timed launches of one kernel class, in order."""
    buf = (ctypes.c_float * max(max_launches, 1))()
    n = _I32(0)
    call("nnue_ft_kernel_timer_read", int(kernel), buf, int(max_launches), ctypes.byref(n))
    return [float(buf[i]) for i in range(min(n.value, max_launches))]


def set_param(name: str, value: int) -> None:
    call("nnue_ft_set_param", name.encode(), int(value))


def get_param(name: str) -> int:
    return int(load().nnue_ft_get_param(name.encode()))


def device_errors(clear: bool = True) -> int:
    """Sticky device error flags of the current device (synchronises)."""
    flags = ctypes.c_uint32(0)
    call("nnue_ft_device_errors", ctypes.byref(flags), int(clear))
    return int(flags.value)
