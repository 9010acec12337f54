"""Tensor-level wrappers of the C ABI (include/nnue_ft.h).

Each function validates its tensors, makes the tensors' device current and
enqueues the native kernels on that device's current CUDA stream.  Memory
(outputs, dense gradients, backward workspace) comes from PyTorch's caching
allocator; the native code allocates nothing.
"""

from __future__ import annotations

import torch

from .. import _native


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _check(t: torch.Tensor, name: str, dtype: torch.dtype, ndim: int, device: torch.device | None = None):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if t.dim() != ndim:
        raise ValueError(f"{name} must be {ndim}-D, got shape {tuple(t.shape)}")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if device is not None and t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")


def forward_into(idx: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, out: torch.Tensor) -> None:
    """out = bias + sum of weight rows (kernel.py:89-103), one perspective."""
    _check(idx, "feature_indices", torch.int32, 2)
    dev = idx.device
    _check(weight, "weight", torch.float32, 2, dev)
    _check(bias, "bias", torch.float32, 1, dev)
    _check(out, "output", torch.float32, 2, dev)
    B, K = idx.shape
    T, C = weight.shape
    if bias.shape[0] != C or tuple(out.shape) != (B, C):
        raise ValueError("bias / output shapes do not match weight and indices")
    with torch.cuda.device(dev):
        _native.call("nnue_ft_forward", idx.data_ptr(), B, K, weight.data_ptr(), T, C, bias.data_ptr(),
                     out.data_ptr(), _stream_ptr(dev))


def forward_pair_into(idx0, idx1, weight, bias, out0, out1) -> None:
    """Both perspectives in one launch (composed.py:49-54 makes two calls)."""
    _check(idx0, "feature_indices_0", torch.int32, 2)
    dev = idx0.device
    _check(idx1, "feature_indices_1", torch.int32, 2, dev)
    _check(weight, "weight", torch.float32, 2, dev)
    _check(bias, "bias", torch.float32, 1, dev)
    _check(out0, "output_0", torch.float32, 2, dev)
    _check(out1, "output_1", torch.float32, 2, dev)
    if idx0.shape != idx1.shape:
        raise ValueError("both perspectives need the same [batch, max_active] shape")
    B, K = idx0.shape
    T, C = weight.shape
    if bias.shape[0] != C or tuple(out0.shape) != (B, C) or tuple(out1.shape) != (B, C):
        raise ValueError("bias / output shapes do not match weight and indices")
    with torch.cuda.device(dev):
        _native.call("nnue_ft_forward_pair", idx0.data_ptr(), idx1.data_ptr(), B, K, weight.data_ptr(), T, C,
                     bias.data_ptr(), out0.data_ptr(), out1.data_ptr(), _stream_ptr(dev))


def forward_pair_prepare(idx0, idx1, weight, bias, out0, out1, workspace: torch.Tensor) -> None:
    """forward_pair_into + backward_prepare (two perspectives) in one call: the
    index-only backward phase runs on the library's side stream while the
    forward gathers, and the current stream waits for both."""
    _check(idx0, "feature_indices_0", torch.int32, 2)
    dev = idx0.device
    _check(idx1, "feature_indices_1", torch.int32, 2, dev)
    _check(weight, "weight", torch.float32, 2, dev)
    _check(bias, "bias", torch.float32, 1, dev)
    _check(out0, "output_0", torch.float32, 2, dev)
    _check(out1, "output_1", torch.float32, 2, dev)
    if idx0.shape != idx1.shape:
        raise ValueError("both perspectives need the same [batch, max_active] shape")
    B, K = idx0.shape
    T, C = weight.shape
    if bias.shape[0] != C or tuple(out0.shape) != (B, C) or tuple(out1.shape) != (B, C):
        raise ValueError("bias / output shapes do not match weight and indices")
    with torch.cuda.device(dev):
        _native.call("nnue_ft_forward_pair_prepare", idx0.data_ptr(), idx1.data_ptr(), B, K, weight.data_ptr(), T, C,
                     bias.data_ptr(), out0.data_ptr(), out1.data_ptr(), workspace.data_ptr(), workspace.numel(),
                     _stream_ptr(dev))


def workspace_bytes(batch: int, max_active: int, num_inputs: int, output_size: int, n_persp: int) -> int:
    n = int(_native.load().nnue_ft_backward_workspace_size(batch, max_active, num_inputs, output_size, n_persp))
    if n == 0:
        raise _native.NativeError("nnue_ft_backward_workspace_size", _native.NNUE_ERR_INVALID_ARGUMENT,
                                  _native.last_error())
    return n


def alloc_workspace(batch, max_active, num_inputs, output_size, n_persp, device) -> torch.Tensor:
    nbytes = workspace_bytes(batch, max_active, num_inputs, output_size, n_persp)
    # the caching allocator returns 512-byte aligned blocks; the ABI needs 256
    return torch.empty(nbytes, dtype=torch.uint8, device=device)


def backward_prepare(idx0, idx1, num_inputs: int, output_size: int, workspace: torch.Tensor) -> None:
    """Sorted position lists per feature (kernel.py:108-138, on the device)."""
    _check(idx0, "feature_indices_0", torch.int32, 2)
    dev = idx0.device
    P = 1 if idx1 is None else 2
    if P == 2:
        _check(idx1, "feature_indices_1", torch.int32, 2, dev)
        if idx1.shape != idx0.shape:
            raise ValueError("both perspectives need the same [batch, max_active] shape")
    B, K = idx0.shape
    with torch.cuda.device(dev):
        _native.call("nnue_ft_backward_prepare", idx0.data_ptr(), 0 if idx1 is None else idx1.data_ptr(), B, K, P,
                     num_inputs, output_size, workspace.data_ptr(), workspace.numel(), _stream_ptr(dev))


def backward_apply(grad0, grad1, batch: int, max_active: int, weight_grad, bias_grad, accumulate: bool,
                   workspace: torch.Tensor) -> None:
    """Segment sums into weight_grad plus the bias column sum (kernel.py:167-186, :269)."""
    dev = weight_grad.device
    _check(weight_grad, "weight_grad", torch.float32, 2, dev)
    _check(bias_grad, "bias_grad", torch.float32, 1, dev)
    _check(grad0, "grad_output_0", torch.float32, 2, dev)
    P = 1 if grad1 is None else 2
    if P == 2:
        _check(grad1, "grad_output_1", torch.float32, 2, dev)
    T, C = weight_grad.shape
    if tuple(grad0.shape) != (batch, C) or (P == 2 and tuple(grad1.shape) != (batch, C)) or bias_grad.shape[0] != C:
        raise ValueError("gradient shapes do not match")
    with torch.cuda.device(dev):
        _native.call("nnue_ft_backward_apply", grad0.data_ptr(), 0 if grad1 is None else grad1.data_ptr(), batch,
                     max_active, P, T, C, weight_grad.data_ptr(), bias_grad.data_ptr(), int(bool(accumulate)),
                     workspace.data_ptr(), workspace.numel(), _stream_ptr(dev))


def backward_apply_rows(grad0, grad1, batch: int, max_active: int, weight_grad, bias_grad, accumulate: bool,
                        workspace: torch.Tensor, row_begin: int, row_end: int, with_bias: bool) -> None:
    """backward_apply for weight-gradient rows [row_begin, row_end) only; the
    bias gradient is produced when ``with_bias``."""
    dev = weight_grad.device
    _check(weight_grad, "weight_grad", torch.float32, 2, dev)
    _check(grad0, "grad_output_0", torch.float32, 2, dev)
    if with_bias:
        _check(bias_grad, "bias_grad", torch.float32, 1, dev)
    P = 1 if grad1 is None else 2
    if P == 2:
        _check(grad1, "grad_output_1", torch.float32, 2, dev)
    T, C = weight_grad.shape
    with torch.cuda.device(dev):
        _native.call("nnue_ft_backward_apply_rows", grad0.data_ptr(), 0 if grad1 is None else grad1.data_ptr(),
                     batch, max_active, P, T, C, weight_grad.data_ptr(), bias_grad.data_ptr() if with_bias else 0,
                     int(bool(accumulate)), row_begin, row_end, int(bool(with_bias)), workspace.data_ptr(),
                     workspace.numel(), _stream_ptr(dev))


def backward_into(idx0, idx1, grad0, grad1, weight_grad, bias_grad, accumulate: bool,
                  workspace: torch.Tensor | None = None) -> None:
    """Full backward for one (idx1 is None) or two perspectives."""
    _check(idx0, "feature_indices_0", torch.int32, 2)
    B, K = idx0.shape
    T, C = weight_grad.shape
    P = 1 if idx1 is None else 2
    if (grad1 is None) != (idx1 is None):
        raise ValueError("pass both or neither of feature_indices_1 / grad_output_1")
    if workspace is None:
        workspace = alloc_workspace(B, K, T, C, P, idx0.device)
    backward_prepare(idx0, idx1, T, C, workspace)
    backward_apply(grad0.contiguous(), None if grad1 is None else grad1.contiguous(), B, K, weight_grad, bias_grad,
                   accumulate, workspace)


def quantized_forward_pair(idx0, idx1, weight_q, psqt_q, bias_q, map_training: bool):
    """int16 accumulators + int32 PSQT for one or two perspectives."""
    _check(idx0, "feature_indices_0", torch.int32, 2)
    dev = idx0.device
    _check(weight_q, "weight_q", torch.int16, 2, dev)
    _check(psqt_q, "psqt_q", torch.int32, 2, dev)
    _check(bias_q, "bias_q", torch.int16, 1, dev)
    P = 1 if idx1 is None else 2
    if P == 2:
        _check(idx1, "feature_indices_1", torch.int32, 2, dev)
    B, K = idx0.shape
    Tq, L1 = weight_q.shape
    NP = psqt_q.shape[1]
    acc = [torch.empty(B, L1, dtype=torch.int16, device=dev) for _ in range(P)]
    ps = [torch.empty(B, NP, dtype=torch.int32, device=dev) for _ in range(P)]
    with torch.cuda.device(dev):
        _native.call("nnue_ft_quantized_forward_pair", idx0.data_ptr(), 0 if P == 1 else idx1.data_ptr(), P, B, K,
                     weight_q.data_ptr(), psqt_q.data_ptr(), Tq, L1, NP, bias_q.data_ptr(), int(bool(map_training)),
                     acc[0].data_ptr(), acc[-1].data_ptr(), ps[0].data_ptr(), ps[-1].data_ptr(), _stream_ptr(dev))
    return (acc[0], ps[0]) if P == 1 else (acc[0], acc[1], ps[0], ps[1])


def halfka_export_quantize(weight, virtual_weight, l1: int, w_scale: float = 255.0, psqt_scale: float = 9600.0):
    """HalfKA training table -> quantised export tables (int16 weights, int32 PSQT)."""
    _check(weight, "weight", torch.float32, 2)
    dev = weight.device
    if weight.shape[0] != 24576:
        raise ValueError("HalfKAv2_hm training table must have 24576 rows")
    C = weight.shape[1]
    if virtual_weight is not None:
        _check(virtual_weight, "virtual_weight", torch.float32, 2, dev)
        if tuple(virtual_weight.shape) != (768, C):
            raise ValueError("virtual_weight must be [768, C]")
    NP = C - l1
    wq = torch.empty(22528, l1, dtype=torch.int16, device=dev)
    pq = torch.empty(22528, NP, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _native.call("nnue_ft_halfka_export_quantize", weight.data_ptr(),
                     0 if virtual_weight is None else virtual_weight.data_ptr(), l1, NP, w_scale, psqt_scale,
                     wq.data_ptr(), pq.data_ptr(), _stream_ptr(dev))
    return wq, pq


def quantize_i16(x: torch.Tensor, scale: float) -> torch.Tensor:
    _check(x, "x", torch.float32, x.dim())
    q = torch.empty(x.shape, dtype=torch.int16, device=x.device)
    with torch.cuda.device(x.device):
        _native.call("nnue_ft_quantize_i16", x.data_ptr(), x.numel(), scale, q.data_ptr(), _stream_ptr(x.device))
    return q


def _ptr_array(tensors):
    import ctypes

    return (ctypes.c_void_p * len(tensors))(*[t.data_ptr() for t in tensors])


def _rows_array(tensors):
    import ctypes

    return (ctypes.c_int64 * len(tensors))(*[t.shape[0] for t in tensors])


def _check_tables(tables, dev, C, what):
    if not 1 <= len(tables) <= 4:
        raise ValueError(f"{what}: 1 to 4 tables supported, got {len(tables)}")
    for i, t in enumerate(tables):
        _check(t, f"{what}[{i}]", torch.float32, 2, dev)
        if t.shape[1] != C:
            raise ValueError(f"{what}[{i}] has {t.shape[1]} columns, expected {C}")


def forward_pair_tables_prepare(idx0, idx1, tables, bias, out0, out1, workspace: torch.Tensor) -> None:
    """forward_pair_prepare over a feature set whose rows are split over
    separate tables (composed.py:49-54 without the torch.cat copy)."""
    _check(idx0, "feature_indices_0", torch.int32, 2)
    dev = idx0.device
    _check(idx1, "feature_indices_1", torch.int32, 2, dev)
    _check(bias, "bias", torch.float32, 1, dev)
    C = bias.shape[0]
    _check_tables(tables, dev, C, "tables")
    _check(out0, "output_0", torch.float32, 2, dev)
    _check(out1, "output_1", torch.float32, 2, dev)
    if idx0.shape != idx1.shape:
        raise ValueError("both perspectives need the same [batch, max_active] shape")
    B, K = idx0.shape
    if tuple(out0.shape) != (B, C) or tuple(out1.shape) != (B, C):
        raise ValueError("output shapes do not match")
    with torch.cuda.device(dev):
        _native.call("nnue_ft_forward_pair_tables_prepare", idx0.data_ptr(), idx1.data_ptr(), B, K,
                     _ptr_array(tables), _rows_array(tables), len(tables), C, bias.data_ptr(), out0.data_ptr(),
                     out1.data_ptr(), workspace.data_ptr(), workspace.numel(), _stream_ptr(dev))


def backward_apply_tables(grad0, grad1, batch: int, max_active: int, weight_grads, bias_grad,
                          workspace: torch.Tensor) -> None:
    """Segment sums written straight into per-table gradients (every row)."""
    dev = bias_grad.device
    _check(bias_grad, "bias_grad", torch.float32, 1, dev)
    C = bias_grad.shape[0]
    _check_tables(weight_grads, dev, C, "weight_grads")
    _check(grad0, "grad_output_0", torch.float32, 2, dev)
    _check(grad1, "grad_output_1", torch.float32, 2, dev)
    if tuple(grad0.shape) != (batch, C) or tuple(grad1.shape) != (batch, C):
        raise ValueError("gradient shapes do not match")
    with torch.cuda.device(dev):
        _native.call("nnue_ft_backward_apply_tables", grad0.data_ptr(), grad1.data_ptr(), batch, max_active,
                     _ptr_array(weight_grads), _rows_array(weight_grads), len(weight_grads), C, bias_grad.data_ptr(),
                     0, workspace.data_ptr(), workspace.numel(), _stream_ptr(dev))


def merge_virtual(weight: torch.Tensor, virtual_weight: torch.Tensor) -> torch.Tensor:
    """weight + virtual_weight.repeat(weight.shape[0] // virtual rows, 1)
    (halfka_v2_hm.py:69-70) in one pass, without the repeated copy."""
    _check(weight, "weight", torch.float32, 2)
    dev = weight.device
    _check(virtual_weight, "virtual_weight", torch.float32, 2, dev)
    R, C = weight.shape
    Vr = virtual_weight.shape[0]
    if virtual_weight.shape[1] != C or Vr == 0 or R % Vr:
        raise ValueError("virtual_weight must have the weight's columns and a row count dividing its rows")
    out = torch.empty_like(weight)
    with torch.cuda.device(dev):
        _native.call("nnue_ft_merge_virtual", weight.data_ptr(), R, virtual_weight.data_ptr(), Vr, C, out.data_ptr(),
                     _stream_ptr(dev))
    return out
