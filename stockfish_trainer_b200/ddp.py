"""Data-parallel plumbing for the feature-transformer step (torchrun, one
process per GPU).

Reference behaviour (src/train/common.py:186-199, 256-263 and
src/train/distributed.py:47-77): the global batch is split evenly over
ranks, every rank holds the full table, and DDP averages the dense gradients
with an allreduce.  Here the FT weight and bias gradients live in ONE flat
fp32 buffer so the exchange is a single collective (or a few row chunks) that
NCCL runs over NVLink / NVSwitch, followed by the division by world size that
DDP applies.
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


@dataclass
class Runtime:
    rank: int = 0
    local_rank: int = 0
    world_size: int = 1

    @property
    def is_distributed(self) -> bool:
        return self.world_size > 1


def init_from_env(backend: str = "nccl", timeout_s: float = 120.0) -> Runtime:
    """torchrun environment -> process group (reference distributed.py:47-77)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if world <= 1:
        return Runtime()
    if backend == "nccl":
        torch.cuda.set_device(local)
    if not dist.is_initialized():
        kwargs = {}
        if backend == "nccl":
            kwargs["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend=backend, init_method="env://",
                                timeout=datetime.timedelta(seconds=timeout_s), **kwargs)
    return Runtime(rank=rank, local_rank=local, world_size=world)


def shard(global_batch: int, rank: int, world: int) -> tuple[int, int]:
    """(first position, count) of this rank's even share (common.py:256-263)."""
    if global_batch % world != 0:
        raise ValueError(f"global batch {global_batch} is not divisible by world size {world}")
    n = global_batch // world
    return rank * n, n


class GradientBuffer:
    """One flat fp32 buffer holding the FT weight gradient [T, C] and the bias
    gradient [C], so the data-parallel exchange is one collective."""

    def __init__(self, num_inputs: int, output_size: int, device: torch.device):
        self.flat = torch.empty(num_inputs * output_size + output_size, dtype=torch.float32, device=device)
        self.weight = self.flat[: num_inputs * output_size].view(num_inputs, output_size)
        self.bias = self.flat[num_inputs * output_size:]

    def allreduce_mean(self, world_size: int, group=None, chunks: int = 1) -> None:
        """Sum over ranks then divide by world size (DDP gradient averaging).

        ``chunks`` > 1 splits the buffer into row ranges, each its own
        collective, so a caller can start reducing finished rows early."""
        if world_size <= 1:
            return
        if chunks <= 1:
            dist.all_reduce(self.flat, group=group)
        else:
            for part in torch.tensor_split(self.flat, chunks):
                dist.all_reduce(part, group=group)
        self.flat.div_(world_size)


_comm_streams: dict[int, torch.cuda.Stream] = {}


def _comm_stream(device: torch.device) -> torch.cuda.Stream:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _comm_streams:
        _comm_streams[idx] = torch.cuda.Stream(device=idx)
    return _comm_streams[idx]


def backward_allreduce_overlapped(grad0, grad1, batch: int, max_active: int, buf: GradientBuffer,
                                  workspace: torch.Tensor, world_size: int, n_blocks: int = 4,
                                  group=None, comm_stream: Optional[torch.cuda.Stream] = None) -> None:
    """Dense FT gradients of this rank's shard, averaged over all ranks, with
    the exchange overlapped with the computation.

    The weight gradient is produced in ``n_blocks`` row blocks
    (nnue_ft_backward_apply_rows); as soon as a block is written, its rows are
    allreduced on a separate stream while the next block is computed, so only
    the last block's exchange is exposed.  The bias gradient travels with the
    last block (it sits after the weight in the flat buffer).  Requires
    ``backward_prepare`` (or ``forward_pair_prepare``) to have filled
    ``workspace`` on the current stream.  Without a process group (a single
    process) it is the plain backward; with one, even of a single rank, the
    row blocks and their collectives run."""
    from .feature_transformer import ops

    T, C = buf.weight.shape
    if world_size <= 1 and group is None and not (dist.is_available() and dist.is_initialized()):
        ops.backward_apply(grad0, grad1, batch, max_active, buf.weight, buf.bias, False, workspace)
        return
    compute = torch.cuda.current_stream(buf.flat.device)
    comm = comm_stream or _comm_stream(buf.flat.device)
    n_blocks = max(1, min(n_blocks, T))
    bounds = [T * i // n_blocks for i in range(n_blocks + 1)]
    avg = dist.get_backend(group) == "nccl"
    works = []
    for i in range(n_blocks):
        last = i == n_blocks - 1
        ops.backward_apply_rows(grad0, grad1, batch, max_active, buf.weight, buf.bias, False, workspace,
                                bounds[i], bounds[i + 1], with_bias=last)
        ready = torch.cuda.Event()
        ready.record(compute)
        part = buf.flat[bounds[i] * C:] if last else buf.flat[bounds[i] * C: bounds[i + 1] * C]
        with torch.cuda.stream(comm):
            comm.wait_event(ready)
            op = dist.ReduceOp.AVG if avg else dist.ReduceOp.SUM
            works.append(dist.all_reduce(part, op=op, group=group, async_op=True))
    for w in works:
        w.wait()  # the current stream waits for the collective
    if not avg:
        buf.flat.div_(world_size)



class SparseLinearPairAllreduce(torch.autograd.Function):
    """``SparseLinearPairFunction`` for data-parallel training.

    (idx_white, idx_black, weight, bias, world_size, n_blocks, group) ->
    (out_white, out_black).  The forward is the pair forward with the
    backward's index phase beside it; the backward returns the dense weight
    and bias gradients already averaged over the process group, with the
    exchange overlapped with the gradient computation row block by row block
    (``backward_allreduce_overlapped``).  This is the averaging the
    reference's DDP applies to the FT parameters (src/train/common.py:186-199,
    src/train/distributed.py:47-77), done inside the FT's own backward instead
    of a second pass over the finished gradient, so those two parameters must
    be left out of any other gradient averaging.  Every rank calls it with the
    same shapes; world_size 1 gives the plain backward."""

    @staticmethod
    def forward(ctx, feature_indices_0, feature_indices_1, weight, bias, world_size: int = 1, n_blocks: int = 4,
                group=None):
        from .feature_transformer import functions

        functions._check_inputs(feature_indices_0, weight, bias)
        functions._check_inputs(feature_indices_1, weight, bias)
        assert feature_indices_0.shape == feature_indices_1.shape
        out0, out1, ws = functions._forward_pair(feature_indices_0, feature_indices_1, weight, bias)
        ctx.workspace = ws
        ctx.shapes = (tuple(feature_indices_0.shape), tuple(weight.shape))
        ctx.world, ctx.blocks, ctx.group = int(world_size), int(n_blocks), group
        return out0, out1

    @staticmethod
    def backward(ctx, grad0, grad1):
        assert not ctx.needs_input_grad[0] and not ctx.needs_input_grad[1]
        (B, K), (T, C) = ctx.shapes
        ws, ctx.workspace = ctx.workspace, None
        dev = ws.device
        # a missing output gradient counts as zeros, so every rank runs the
        # same collectives
        g0 = grad0.contiguous() if grad0 is not None else torch.zeros(B, C, device=dev)
        g1 = grad1.contiguous() if grad1 is not None else torch.zeros(B, C, device=dev)
        buf = GradientBuffer(T, C, dev)
        backward_allreduce_overlapped(g0, g1, B, K, buf, ws, ctx.world, n_blocks=ctx.blocks, group=ctx.group)
        return None, None, buf.weight, buf.bias, None, None, None
