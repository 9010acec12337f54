"""The C-ABI library loads, exports every symbol the header declares, and
rejects bad arguments on the host before touching a GPU."""

import ctypes
import os
import re

import pytest

from stockfish_trainer_b200 import _native

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "nnue_ft.h")


def _declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nnue_\w+)\s*\(", text)))


def test_header_declares_functions():
    names = _declared_functions()
    assert "nnue_ft_forward" in names and "nnue_ft_backward" in names
    assert len(names) >= 15


def test_library_exports_every_declared_symbol():
    lib = _native.load()
    for name in _declared_functions():
        assert hasattr(lib, name), name
    assert set(_declared_functions()) == set(_native.exported_symbols())


def test_version_and_params():
    lib = _native.load()
    assert lib.nnue_ft_version() >= 100
    old = _native.get_param("fwd_chunk_vec")
    _native.set_param("fwd_chunk_vec", 32)
    assert _native.get_param("fwd_chunk_vec") == 32
    _native.set_param("fwd_chunk_vec", old)
    with pytest.raises(_native.NativeError):
        _native.set_param("no_such_knob", 1)
    with pytest.raises(_native.NativeError):
        _native.set_param("fwd_items_per_warp", 0)


def _documented_knobs():
    text = open(HEADER).read()
    block = re.search(r"/\* Tuning knobs \(names: (.*?)\);", text, flags=re.S).group(1)
    return re.findall(r'"(\w+)"', block)


def test_every_documented_knob_is_readable():
    knobs = _documented_knobs()
    assert len(knobs) == len(set(knobs)) >= 20
    for name in knobs:
        v = _native.get_param(name)
        _native.set_param(name, v)  # the default is inside its own range
        assert _native.get_param(name) == v


def test_host_side_argument_errors():
    lib = _native.load()
    # null pointers -> INVALID_ARGUMENT before any CUDA call
    rc = lib.nnue_ft_forward(None, 4, 8, None, 10, 16, None, None, None)
    assert rc == _native.NNUE_ERR_INVALID_ARGUMENT
    assert "null" in _native.last_error()
    rc = lib.nnue_ft_forward(None, 4, 8, None, 10, 0, None, None, None)
    assert rc == _native.NNUE_ERR_INVALID_ARGUMENT
    # n_persp must be 1 or 2
    assert lib.nnue_ft_backward_workspace_size(4, 8, 10, 16, 3) == 0
    # workspace checks
    size = lib.nnue_ft_backward_workspace_size(4, 8, 10, 16, 2)
    assert size > 0
    buf = ctypes.c_void_p(256)  # never dereferenced: the size check fails first
    rc = lib.nnue_ft_backward_prepare(ctypes.c_void_p(256), ctypes.c_void_p(512), 4, 8, 2, 10, 16, buf, size - 1, None)
    assert rc == _native.NNUE_ERR_WORKSPACE
    # sizes beyond the documented limits
    assert lib.nnue_ft_backward_workspace_size(2**31, 160, 10, 16, 2) == 0
    assert lib.nnue_ft_backward_workspace_size(16, 160, 2**30, 16, 2) == 0
    # quantised forward shape rules
    rc = lib.nnue_ft_quantized_forward_pair(None, None, 1, 4, 8, None, None, 10, 12, 8, None, 0, None, None, None,
                                            None, None)
    assert rc == _native.NNUE_ERR_UNSUPPORTED


def test_workspace_size_grows_with_batch():
    lib = _native.load()
    a = lib.nnue_ft_backward_workspace_size(1024, 160, 85296, 1048, 2)
    b = lib.nnue_ft_backward_workspace_size(4096, 160, 85296, 1048, 2)
    assert 0 < a < b


def test_kernel_timer_arguments():
    lib = _native.load()
    # bad mask / capacity are rejected before any CUDA call
    assert lib.nnue_ft_kernel_timer_arm(8, 4) == _native.NNUE_ERR_INVALID_ARGUMENT
    assert lib.nnue_ft_kernel_timer_arm(1, -1) == _native.NNUE_ERR_INVALID_ARGUMENT
    assert lib.nnue_ft_kernel_timer_arm(1, 0) == _native.NNUE_ERR_INVALID_ARGUMENT
    # disarming with nothing armed is a no-op
    _native.kernel_timer_arm((), 0)
    n = ctypes.c_int32(-1)
    assert lib.nnue_ft_kernel_timer_read(3, None, 0, ctypes.byref(n)) == _native.NNUE_ERR_INVALID_ARGUMENT
    assert _native.kernel_timer_read(_native.TIMED_LIGHT_ROWS) == []
