"""Data-parallel FT training step with the Ranger22 state sharded by table rows.

The reference trains data-parallel with DDP (src/train/common.py:186-199):
every rank averages the whole FT weight gradient with an allreduce and then
runs Ranger22 over the whole table (src/ranger22/optimizer.py:307-551).  In the
trainer's configuration Ranger22 updates a 2-D parameter row by row -- the norm
loss takes each row's norm (optimizer.py:79-107), everything else is
elementwise -- so rows are independent and the update splits over ranks:

1. the backward produces this rank's weight gradient in row blocks
   (``nnue_ft_backward_apply_rows``);
2. each finished block is reduce-scattered with the average, so rank r holds
   the averaged gradient of the r-th 1/N slice of every block;
3. rank r runs the fused Ranger22 update (``nnue_ft_ranger22_step``) on those
   rows only, so its optimizer state covers T/N rows;
4. the updated slices are all-gathered back into every rank's table.

Steps 2-4 of a block run on a communication stream while the next block's
gradient is computed.  The bias (1-D: its norm is over the whole vector) is
averaged with an allreduce and updated identically on every rank.  NVLink
carries the bytes of one allreduce (a reduce-scatter and an all-gather);
optimizer traffic and optimizer-state memory drop N-fold.  The result on every
rank is the table and bias the unsharded path (allreduce + Ranger22 over the
whole table on every rank) produces, bit for bit whenever the averaged
gradient is (with two ranks always: (a + b) / 2 is one rounding in any order).
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from . import optim


def row_block_bounds(num_rows: int, n_blocks: int, world_size: int) -> list[int]:
    """Row-block bounds [0 = b_0 < b_1 < ... < b_n = num_rows] whose lengths
    are multiples of ``world_size`` (so every block splits into N equal
    slices).  ``num_rows`` must be a multiple of ``world_size``."""
    if world_size < 1 or num_rows % world_size:
        raise ValueError(f"{num_rows} table rows do not split evenly over {world_size} ranks")
    units = num_rows // world_size
    n_blocks = max(1, min(n_blocks, units))
    return [world_size * (units * i // n_blocks) for i in range(n_blocks + 1)]


class _CudaKernels:
    """The native kernels the sharded step calls (tests on CPU substitute
    reference implementations with the same signatures)."""

    @staticmethod
    def block_gradient(grad0, grad1, batch, max_active, weight_grad, bias_grad, workspace, row_begin, row_end,
                       with_bias):
        from .feature_transformer import ops

        ops.backward_apply_rows(grad0, grad1, batch, max_active, weight_grad, bias_grad, False, workspace,
                                row_begin, row_end, with_bias)

    @staticmethod
    def update(p, grad, variance_ma, gma_cur, gma_prev, scalars, lookahead, merge, alpha):
        optim.ranger22_update_(p, grad, variance_ma, gma_cur, gma_prev, scalars, lookahead, merge, alpha)


class ShardedRanger22FT:
    """Ranger22 (the trainer's configuration, as ``optim.Ranger22FT``) for the
    FT table and bias of one data-parallel job, with the table's optimizer
    state sharded by rows over the ranks of ``group``.

    ``backward_step`` replaces [backward, gradient allreduce, optimizer step]
    for the two FT parameters: it consumes the workspace prepared by the
    forward (``forward_pair_prepare``) and the output gradients of this rank's
    shard of the batch, and leaves the updated ``weight`` and ``bias`` on every
    rank (stream-ordered: the current stream waits for the communication
    stream before returning).

    State layout: ``variance_ma``, ``grad_ma``, ``neg_grad_ma`` and
    ``lookahead`` hold this rank's rows packed block by block: block i's slice
    [b_i + r*s_i, b_i + (r+1)*s_i), s_i = (b_{i+1} - b_i) / N, sits at rows
    [sum_{j<i} s_j, ...) of the packed tensors.  ``step`` and the lookahead
    counter follow ``Ranger22FT`` (the two grad EMAs swap roles every step).
    """

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor, lr: float, betas=(0.9, 0.999), eps: float = 1e-7,
                 normloss_factor: float = 1e-4, lookahead_mergetime: int = 5, lookahead_alpha: float = 0.5,
                 n_blocks: int = 4, group=None, kernels=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        T, C = weight.shape
        self.weight, self.bias = weight, bias
        self.bounds = row_block_bounds(T, n_blocks, self.world)
        self.lr, self.betas, self.eps = lr, betas, eps
        self.normloss_factor = normloss_factor
        self.mergetime, self.alpha = lookahead_mergetime, lookahead_alpha
        self.kernels = kernels or _CudaKernels()
        dev = weight.device
        rows = T // self.world
        self.slices = []  # (row_begin, row_end) of this rank's rows of each block, and their packed offset
        off = 0
        for i in range(len(self.bounds) - 1):
            s = (self.bounds[i + 1] - self.bounds[i]) // self.world
            lo = self.bounds[i] + self.rank * s
            self.slices.append((lo, lo + s, off))
            off += s
        with torch.no_grad():
            self.variance_ma = torch.zeros(rows, C, device=dev)
            self.grad_ma = torch.zeros(rows, C, device=dev)
            self.neg_grad_ma = torch.zeros(rows, C, device=dev)
            self.lookahead = torch.empty(rows, C, device=dev)
            for lo, hi, o in self.slices:
                self.lookahead[o:o + hi - lo].copy_(weight[lo:hi])
            self.grad_shard = torch.empty(rows, C, device=dev)
            self.bias_state = {k: torch.zeros_like(bias) for k in ("variance_ma", "grad_ma", "neg_grad_ma")}
            self.bias_state["lookahead"] = bias.detach().clone()
            # this rank's un-averaged gradients, one flat buffer (weight rows, then bias)
            self.partial = torch.empty(T * C + C, device=dev)
        self.partial_weight = self.partial[: T * C].view(T, C)
        self.partial_bias = self.partial[T * C:]
        self.step = 0
        self.lookahead_step = 0
        self._comm = None

    # -- collectives (NCCL: average in the collective; others: sum, then scale)
    def _nccl(self) -> bool:
        return dist.is_initialized() and dist.get_backend(self.group) == "nccl"

    def _reduce_scatter_mean(self, out: torch.Tensor, inp: torch.Tensor):
        if self.world == 1:
            out.copy_(inp)
            return
        if self._nccl():
            dist.reduce_scatter_tensor(out, inp, op=dist.ReduceOp.AVG, group=self.group)
            return
        tmp = inp.clone()
        dist.all_reduce(tmp, group=self.group)
        n = out.shape[0]
        out.copy_(tmp[self.rank * n:(self.rank + 1) * n]).div_(self.world)

    def _all_reduce_mean(self, t: torch.Tensor):
        if self.world == 1:
            return
        if self._nccl():
            dist.all_reduce(t, op=dist.ReduceOp.AVG, group=self.group)
        else:
            dist.all_reduce(t, group=self.group)
            t.div_(self.world)

    def _all_gather_into(self, block: torch.Tensor, mine: torch.Tensor):
        if self.world == 1:
            return
        if self._nccl():
            dist.all_gather_into_tensor(block, mine, group=self.group)
        else:
            parts = [torch.empty_like(mine) for _ in range(self.world)]
            dist.all_gather(parts, mine.contiguous(), group=self.group)
            block.copy_(torch.cat(parts))

    # -- one step
    def _scalars_and_merge(self):
        self.step += 1
        merge = False
        self.lookahead_step += 1
        if self.lookahead_step >= self.mergetime:
            self.lookahead_step = 0
            merge = True
        sc = optim.ranger22_scalars(float(self.lr), self.step, self.betas, float(self.eps), self.normloss_factor,
                                    True)
        return sc, merge

    def _emas(self, state_cur, state_neg):
        # optim.Ranger22FT: grad_ma is the current EMA on odd steps, neg_grad_ma on even steps
        return (state_cur, state_neg) if self.step % 2 == 1 else (state_neg, state_cur)

    @torch.no_grad()
    def backward_step(self, grad0, grad1, batch: int, max_active: int, workspace,
                      comm_stream: Optional[torch.cuda.Stream] = None) -> None:
        sc, merge = self._scalars_and_merge()
        m_cur, m_prev = self._emas(self.grad_ma, self.neg_grad_ma)
        cuda = self.weight.is_cuda
        if cuda:
            compute = torch.cuda.current_stream(self.weight.device)
            if comm_stream is None:
                if self._comm is None:
                    # high priority: each block's update kernel is scheduled as
                    # soon as its reduce-scatter lands instead of queueing
                    # behind the gradient kernel's blocks, which would hold up
                    # the all-gather and the next block's reduce-scatter
                    # (2 x B200: 2.61 ms per training step against 2.98 ms)
                    self._comm = torch.cuda.Stream(device=self.weight.device, priority=-1)
                comm_stream = self._comm
        n_blocks = len(self.bounds) - 1
        for i in range(n_blocks):
            b0, b1 = self.bounds[i], self.bounds[i + 1]
            last = i == n_blocks - 1
            self.kernels.block_gradient(grad0, grad1, batch, max_active, self.partial_weight, self.partial_bias,
                                        workspace, b0, b1, last)
            lo, hi, o = self.slices[i]
            n = hi - lo
            if cuda:
                ready = torch.cuda.Event()
                ready.record(compute)
                ctx = torch.cuda.stream(comm_stream)
            else:
                ctx = _nullcontext()
            with ctx:
                if cuda:
                    comm_stream.wait_event(ready)
                g = self.grad_shard[o:o + n]
                self._reduce_scatter_mean(g, self.partial_weight[b0:b1])
                self.kernels.update(self.weight[lo:hi], g, self.variance_ma[o:o + n], m_cur[o:o + n],
                                    m_prev[o:o + n], sc, self.lookahead[o:o + n], merge, self.alpha)
                self._all_gather_into(self.weight[b0:b1], self.weight[lo:hi])
                if last:
                    self._all_reduce_mean(self.partial_bias)
                    bs = self.bias_state
                    bc, bp = self._emas(bs["grad_ma"], bs["neg_grad_ma"])
                    self.kernels.update(self.bias, self.partial_bias, bs["variance_ma"], bc, bp, sc,
                                        bs["lookahead"], merge, self.alpha)
        if cuda:
            compute.wait_stream(comm_stream)


class _nullcontext:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False
