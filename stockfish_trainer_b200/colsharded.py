"""Column-sharded feature transformer over the ranks of a process group.

The reference trains data-parallel (src/train/common.py:186-199, 256-263,
src/train/distributed.py:47-77): the global batch is split evenly over ranks,
every rank holds the whole table and DDP averages the dense FT weight
gradient -- T x C fp32, 357.6 MB at the headline size -- with an allreduce
every step.  That exchange does not shrink as ranks are added, while each
rank's share of the gathers does.

Here rank r owns a slice of the table's COLUMNS (``column_slices``): its
slice of the weight, of the bias and of any optimizer state, for all T rows.
Every position's output row is bias + a sum of table rows, column by column,
so a rank can produce its columns of every position's output, and the
gradient of its columns needs only its columns of every position's output
gradient.  One step:

1. ``gather_indices``: every rank receives all ranks' index rows (int32,
   B x K per perspective; they are inputs, known before the step);
2. ``forward``: the pair forward + the backward's index phase over the WHOLE
   batch on this rank's columns (the same kernels as one GPU), then an
   exchange: rank r sends rows [s*b, (s+1)*b) of its columns to rank s, and
   each rank joins the column blocks into its own positions' full rows
   [b, C] -- what the data-parallel forward returns;
3. ``backward``: the exchange the other way (rank r sends its positions'
   output gradients of rank s's columns to s, scaled by 1/N: DDP's
   averaging), then the segment sums over the whole batch on this rank's
   columns -> this rank's columns of the averaged weight and bias gradients.

Bytes over NVLink per rank and step, N ranks, global batch B, C columns,
both perspectives: indices (N-1)/N * 2BK*4 in, outputs and output gradients
(N-1)/N^2 * 2BC*4 each way, against an allreduce's 2(N-1)/N * TC*4 (ring).
At the headline (B = 65536, K = 160, C = 1048, T = 85296): 42 + 137 + 137 MB
at N = 2 against 358 MB; 73 + 60 + 60 MB at N = 8 against 626 MB.

Sums are taken in the single-GPU order (ascending position per row, each
perspective from zero, then added), so the gradient of rank r's columns is
the one-GPU full-batch gradient of those columns times 1/N -- bit for bit
when N is a power of two (the scale is exact), independent of the exchange.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

class _CudaArray:
    """A raw device allocation as a tensor (``__cuda_array_interface__``)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def _device_view(ptr: int, shape, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    typestr = {torch.float32: "<f4", torch.int32: "<i4"}[dtype]
    return torch.as_tensor(_CudaArray(ptr, shape, typestr), device=device)


def _copy_desc_type():
    import ctypes

    class CopyDesc(ctypes.Structure):  # nnue_ft_copy_desc
        _fields_ = [("src", ctypes.c_void_p), ("dst", ctypes.c_void_p), ("rows", ctypes.c_int64),
                    ("src_ld", ctypes.c_int64), ("dst_ld", ctypes.c_int64), ("width", ctypes.c_int32),
                    ("scale", ctypes.c_float)]

    return CopyDesc


_CopyDesc = _copy_desc_type()

VECTOR = 4  # floats per 16-byte vector: slices are whole vectors when C % 4 == 0
CHUNK = 32  # vectors per column chunk of the gather kernels (one per lane)
PACKED_TAILS = (2, 3, 4, 6, 8)  # narrow last chunks that run in the packed tail kernels


def _slice_cost(v: int) -> int:
    """Relative gather cost of a v-vector column slice, in 1/1000 of a full
    chunk: full 32-vector chunks cost one each; a narrow last chunk the
    packed tail kernels take costs little; any other narrow chunk runs with
    idle lanes in the main kernels at nearly a full chunk's instructions."""
    full, tail = divmod(v, CHUNK)
    if tail == 0:
        return 1000 * full
    if full and tail in PACKED_TAILS:
        return 1000 * full + 100 + 10 * tail
    return 1000 * full + 500 + (500 * tail) // CHUNK


def column_slices(output_size: int, world: int) -> list[tuple[int, int]]:
    """[(c0, c1)] per rank: contiguous column slices covering output_size.

    With output_size a multiple of 4 every slice is whole 16-byte vectors
    (the kernels' vector path), sized to minimise the slowest rank's gather
    cost (``_slice_cost``), then the total, then the widest slice; otherwise
    an even split of the columns.  Deterministic: every rank computes the
    same list."""
    if world < 1:
        raise ValueError("world size must be >= 1")
    if output_size < world:
        raise ValueError(f"{output_size} columns cannot be split over {world} ranks")
    if output_size % VECTOR:
        return [(output_size * r // world, output_size * (r + 1) // world) for r in range(world)]
    n = output_size // VECTOR
    if n < world:
        raise ValueError(f"{n} 16-byte column vectors cannot be split over {world} ranks")
    lo_w, hi_w = max(1, n // world - 2 * CHUNK), n // world + 2 * CHUNK
    # best[m] = (key, widths) over the ranks placed so far, m vectors used
    best: dict[int, tuple[tuple[int, int, int], tuple[int, ...]]] = {0: ((0, 0, 0), ())}
    for _ in range(world):
        nxt: dict[int, tuple[tuple[int, int, int], tuple[int, ...]]] = {}
        for m, ((mx, tot, wide), widths) in best.items():
            for v in range(lo_w, hi_w + 1):
                if m + v > n:
                    break
                c = _slice_cost(v)
                cand = ((max(mx, c), tot + c, max(wide, v)), widths + (v,))
                cur = nxt.get(m + v)
                if cur is None or cand[0] < cur[0]:
                    nxt[m + v] = cand
        best = nxt
    if n not in best:
        raise ValueError(f"no column split of {n} vectors over {world} ranks")
    widths = sorted(best[n][1], reverse=True)
    out, c = [], 0
    for v in widths:
        out.append((c * VECTOR, (c + v) * VECTOR))
        c += v
    return out


class _CudaKernels:
    """The native kernels the column-sharded step calls (CPU tests substitute
    reference implementations with the same signatures)."""

    @staticmethod
    def alloc_workspace(batch, max_active, num_inputs, width, device):
        from .feature_transformer import ops

        return ops.alloc_workspace(batch, max_active, num_inputs, width, 2, device)

    @staticmethod
    def forward_prepare(idx0, idx1, weight, bias, out0, out1, workspace):
        from .feature_transformer import ops

        ops.forward_pair_prepare(idx0, idx1, weight, bias, out0, out1, workspace)

    @staticmethod
    def forward(idx0, idx1, weight, bias, out0, out1):
        from .feature_transformer import ops

        ops.forward_pair_into(idx0, idx1, weight, bias, out0, out1)

    @staticmethod
    def prepare(idx0, idx1, num_inputs, width, workspace):
        from .feature_transformer import ops

        ops.backward_prepare(idx0, idx1, num_inputs, width, workspace)

    @staticmethod
    def backward_apply(grad0, grad1, batch, max_active, weight_grad, bias_grad, workspace):
        from .feature_transformer import ops

        ops.backward_apply(grad0, grad1, batch, max_active, weight_grad, bias_grad, False, workspace)


class ColumnShardedFT:
    """Buffers, column slices and collectives of the column-sharded FT step
    for one process group (every rank constructs it with the same sizes).

    ``batch`` is the GLOBAL batch (a multiple of the group size); each rank
    passes its own ``batch / N`` positions' index rows and output gradients,
    as in data-parallel training.  The rank's parameters are its column slice
    ``weight[:, c0:c1]`` / ``bias[c0:c1]`` as contiguous tensors
    (``shard_columns``).  One step in flight per object: ``forward`` fills the
    workspace ``backward`` consumes.

    ``exchange``: "peer" (the default on CUDA tensors in an NCCL group of at
    most 15 ranks with C and K multiples of 4) moves the data with this
    library's exchange kernel, which stores straight into the other GPUs'
    buffers (CUDA IPC) in the layout the receiver uses -- index rows at their
    global positions, output blocks at their column offsets, 1/N-scaled
    gradient blocks at their row offsets -- and ends with a bounded barrier
    (a rank that does not arrive within ``timeout_ms`` raises
    NNUE_DEVERR_EXCHANGE_TIMEOUT instead of hanging); "p2p" uses
    ``torch.distributed`` point-to-point operations (any backend) and joins
    the blocks with torch ops.  With "peer" the returned outputs live in the
    exchange buffer, two steps' worth: a step's outputs stay valid until the
    forward after the next one.  Call ``close`` on every rank (it is a
    collective) before the process group goes away.

    ``prepare``: "forward" runs the backward's index phase beside the forward
    on the library's high-priority side stream (as one GPU does); "overlap"
    (the default on CUDA) runs it on a normal-priority stream of its own, so
    the forward's gathers come first and the index phase continues through
    the exchanges (4 x B200: 1.76 ms per step against 2.03 ms)."""

    def __init__(self, num_inputs: int, output_size: int, batch: int, max_active: int, device=None, group=None,
                 kernels=None, exchange: Optional[str] = None, timeout_ms: int = 5000, prepare: Optional[str] = None):
        self.group = group
        self.timeout_ms = int(timeout_ms)
        dist_on = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if dist_on else 1
        self.rank = dist.get_rank(group) if dist_on else 0
        if batch % self.world:
            raise ValueError(f"global batch {batch} is not divisible by world size {self.world}")
        self.T, self.C, self.B, self.K = int(num_inputs), int(output_size), int(batch), int(max_active)
        self.b = self.B // self.world
        self.slices = column_slices(self.C, self.world)
        self.c0, self.c1 = self.slices[self.rank]
        self.width = self.c1 - self.c0
        self.widths = [c1 - c0 for c0, c1 in self.slices]
        self.kernels = kernels or _CudaKernels()
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        dev = self.device
        self.scale = 1.0 / self.world
        if prepare is None:  # overlap where there is a CUDA stream to put it on
            prepare = "overlap" if dev.type == "cuda" else "forward"
        if prepare not in ("forward", "overlap"):
            raise ValueError(f"prepare must be 'forward' or 'overlap', got {prepare!r}")
        self.prepare = prepare
        self._prep_stream = self._prep_done = None
        if prepare == "overlap" and dev.type == "cuda":
            self._prep_stream = torch.cuda.Stream(device=dev)  # normal priority
            self._prep_done = torch.cuda.Event()
        # this rank's columns of every position's output
        self.y = torch.empty(2, self.B, self.width, device=dev)
        self.workspace = self.kernels.alloc_workspace(self.B, self.K, self.T, self.width, dev)
        self._peer = None
        self._slot = 0
        self._pending = None
        self._pf_stream = None
        if exchange not in (None, "peer", "p2p"):
            raise ValueError(f"exchange must be 'peer' or 'p2p', got {exchange!r}")
        if exchange == "peer" and not self._peer_capable():
            raise ValueError("the peer exchange needs CUDA tensors in an NCCL group of at most 15 ranks with "
                             "output_size and max_active multiples of 4; use exchange='p2p'")
        if exchange == "peer" or (exchange is None and self._peer_capable()):
            err = self._setup_peer_exchange()
            if err is not None:  # every rank saw the same failure (a collective): all fall back or all raise
                if exchange == "peer":
                    raise RuntimeError(f"peer exchange unavailable: {err}")
                exchange = "p2p"
            else:
                exchange = "peer"
        exchange = exchange or "p2p"
        self.exchange = exchange
        if exchange == "p2p":
            # all positions' index rows, per perspective [B, K]
            self.idx = torch.empty(2, self.B, self.K, dtype=torch.int32, device=dev)
            # this rank's columns of every position's output gradient
            self.d = torch.empty(2, self.B, self.width, device=dev)
            # per peer s: its columns of this rank's positions (received
            # outputs, sent gradients), [2, b, w_s] blocks packed peer by peer
            self.blk_off = [0]
            for w in self.widths:
                self.blk_off.append(self.blk_off[-1] + 2 * self.b * w)
            self.recv = torch.empty(self.blk_off[-1], device=dev)
            self.send = torch.empty(self.blk_off[-1], device=dev)

    # -- peer exchange setup ---------------------------------------------------
    _FLAG_BYTES = 256
    # index-row slots: a step's rows stay in place until every rank is past
    # that step's backward (its index phase may still read them), the next
    # step's may be arriving (prefetch_indices), and one more is free
    _IDX_SLOTS = 3
    _CH_STEP, _CH_PREFETCH = 0, 1  # exchange channels

    def _peer_capable(self) -> bool:
        if self.device.type != "cuda" or self.world > 15 or self.C % VECTOR or self.K % VECTOR:
            return False
        if self.world == 1:
            return True
        return dist.get_backend(self.group) == "nccl"

    def _setup_peer_exchange(self) -> Optional[str]:
        """Allocate, share and map the exchange buffers; None on success, else
        the first rank's error (every rank returns the same, having undone
        its own allocations and mappings)."""
        import ctypes

        from . import _native

        def up(n):  # 256-byte aligned offsets
            return (n + 255) // 256 * 256

        f32 = 4
        off_idx = self._FLAG_BYTES
        idx_slot = up(2 * self.B * self.K * 4)
        off_out = off_idx + self._IDX_SLOTS * idx_slot
        off_d = off_out + up(2 * 2 * self.b * self.C * f32)  # two steps' outputs
        total = off_d + up(2 * self.B * max(self.widths) * f32)
        with torch.cuda.device(self.device):
            base = ctypes.c_void_p(0)
            handle = ctypes.create_string_buffer(64)
            _native.call("nnue_ft_exchange_alloc", total, ctypes.byref(base), handle)
            handles = [None] * self.world
            if self.world > 1:
                dist.all_gather_object(handles, handle.raw, group=self.group)
            else:
                handles[0] = handle.raw
            bases, err = [], None
            for s, h in enumerate(handles):
                if s == self.rank:
                    bases.append(base.value)
                    continue
                p = ctypes.c_void_p(0)
                try:
                    _native.call("nnue_ft_exchange_open", ctypes.create_string_buffer(h, 64), ctypes.byref(p))
                except _native.NativeError as e:
                    err = f"rank {self.rank} mapping rank {s}'s buffer: {e}"
                    break
                bases.append(p.value)
            errs = [err] * self.world
            if self.world > 1:
                dist.all_gather_object(errs, err, group=self.group)
            first = next((e for e in errs if e), None)
            if first is not None:
                for s, b in enumerate(bases):
                    if s != self.rank:
                        _native.call("nnue_ft_exchange_close", b)
                if self.world > 1:
                    dist.barrier(group=self.group)  # nobody maps this rank's buffer any more
                _native.call("nnue_ft_exchange_free", base.value)
                return first
        self._peer = {"base": bases, "own": base.value, "off_idx": off_idx, "idx_slot": idx_slot, "off_out": off_out,
                      "off_d": off_d,
                      "epoch": [0, 0, 0, 0], "flags": (ctypes.c_void_p * self.world)(*bases), "total": total}
        own = base.value
        self._idx_slots = [_device_view(own + off_idx + i * idx_slot, (2, self.B, self.K), torch.int32, self.device)
                           for i in range(self._IDX_SLOTS)]
        self._cur = 0
        self.idx = self._idx_slots[0]
        self._out = [_device_view(own + off_out + i * 2 * self.b * self.C * f32, (2, self.b, self.C), torch.float32,
                                  self.device) for i in range(2)]
        self.d = _device_view(own + off_d, (2, self.B, self.width), torch.float32, self.device)
        return None

    def close(self) -> None:
        """Unmap the other ranks' exchange buffers and free this rank's (a
        collective: every rank calls it once its exchanges are done)."""
        if self._peer is None:
            return
        from . import _native

        if self._pending is not None:  # a prefetch nobody consumed: let it land
            self._take_prefetched()
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)  # nobody writes into a buffer after this
        with torch.cuda.device(self.device):
            for s, b in enumerate(self._peer["base"]):
                if s != self.rank:
                    _native.call("nnue_ft_exchange_close", b)
            if self.world > 1:
                dist.barrier(group=self.group)  # every mapping of this rank's buffer is gone
            _native.call("nnue_ft_exchange_free", self._peer["own"])
        self._peer = None
        self.idx = self.d = self._out = self._idx_slots = None

    def _peer_exchange(self, copies, channel: int = 0) -> None:
        """copies: [(src_ptr, dst_ptr, rows, src_ld, dst_ld, width, scale)],
        strides and widths in 16-byte vectors; on the current stream."""
        import ctypes

        from . import _native

        arr = (_CopyDesc * max(len(copies), 1))()
        for i, (src, dst, rows, sld, dld, w, sc) in enumerate(copies):
            arr[i] = _CopyDesc(src, dst, rows, sld, dld, w, sc)
        ep = self._peer["epoch"]
        ep[channel] += 1
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device).cuda_stream
            _native.call("nnue_ft_exchange", arr, len(copies), self._peer["flags"], self.world, self.rank, channel,
                         ep[channel] & 0xFFFFFFFF, self.timeout_ms, stream)

    # -- parameters ---------------------------------------------------------
    def shard_columns(self, full: torch.Tensor) -> torch.Tensor:
        """This rank's columns of a [T, C] table or [C] vector, contiguous."""
        return full[..., self.c0:self.c1].contiguous()

    def gather_columns(self, cols: torch.Tensor) -> torch.Tensor:
        """The whole [T, C] table (or [C] vector) from every rank's columns
        (for checkpoints and export; a collective)."""
        if self.world == 1:
            return cols.clone()
        parts = []
        for s, w in enumerate(self.widths):
            shape = list(cols.shape)
            shape[-1] = w
            parts.append(cols.contiguous() if s == self.rank else torch.empty(shape, dtype=cols.dtype,
                                                                               device=cols.device))
        for s in range(self.world):
            dist.broadcast(parts[s], src=self._global(s), group=self.group)
        return torch.cat(parts, dim=-1)

    # -- collectives ----------------------------------------------------------
    def _global(self, s: int) -> int:
        return dist.get_global_rank(self.group, s) if self.group is not None else s

    def _block(self, buf: torch.Tensor, s: int, p: int) -> torch.Tensor:
        w = self.widths[s]
        o = self.blk_off[s] + p * self.b * w
        return buf[o:o + self.b * w].view(self.b, w)

    def _exchange(self, sends, recvs) -> None:
        """Point-to-point exchange: sends = [(peer, tensor)], recvs = [(peer,
        tensor)], in the same per-peer order on every rank (one NCCL group)."""
        ops = [dist.P2POp(dist.isend, t, self._global(s), self.group) for s, t in sends]
        ops += [dist.P2POp(dist.irecv, t, self._global(s), self.group) for s, t in recvs]
        if ops:
            for w in dist.batch_isend_irecv(ops):
                w.wait()

    def gather_indices(self, idx0: torch.Tensor, idx1: torch.Tensor):
        """Every rank's [b, K] index rows -> all positions' rows [B, K] per
        perspective (rank s's rows at [s*b, (s+1)*b))."""
        for x in (idx0, idx1):
            if tuple(x.shape) != (self.b, self.K):
                raise ValueError(f"index rows must be [{self.b}, {self.K}], got {tuple(x.shape)}")
        if self._peer is not None:
            if self._pending is not None:  # prefetched rows nobody used: let them land, then reuse their slot
                torch.cuda.current_stream(self.device).wait_event(self._pending[1])
                self._pending = None
            slot = (self._cur + 1) % self._IDX_SLOTS
            self._peer_exchange(self._index_copies(idx0, idx1, slot), self._CH_STEP)
            self._cur = slot
            self.idx = self._idx_slots[slot]
            return self.idx[0], self.idx[1]
        for p, x in enumerate((idx0, idx1)):
            if self.world == 1:
                self.idx[p].copy_(x)
            elif dist.get_backend(self.group) == "nccl":
                dist.all_gather_into_tensor(self.idx[p], x.contiguous(), group=self.group)
            else:
                parts = list(self.idx[p].view(self.world, self.b, self.K).unbind(0))
                tmp = [torch.empty_like(t) for t in parts]
                dist.all_gather(tmp, x.contiguous(), group=self.group)
                for t, u in zip(parts, tmp):
                    t.copy_(u)
        return self.idx[0], self.idx[1]

    def _index_copies(self, idx0, idx1, slot):
        xs = [x.contiguous() for x in (idx0, idx1)]
        kv = self.K // VECTOR
        copies = []
        for s in range(self.world):
            for p in range(2):
                dst = self._peer["base"][s] + self._peer["off_idx"] + slot * self._peer["idx_slot"] + \
                    (p * self.B + self.rank * self.b) * self.K * 4
                copies.append((xs[p].data_ptr(), dst, self.b, kv, kv, kv, 1.0))
        return copies

    def prefetch_indices(self, idx0: torch.Tensor, idx1: torch.Tensor) -> None:
        """Start moving the NEXT step's index rows (this rank's [b, K] per
        perspective) to every rank, on a stream of their own beside the
        current step's exchanges and backward; the next ``forward_local`` /
        ``forward`` uses them (without index arguments).  Peer exchange only."""
        if self._peer is None:
            raise RuntimeError("prefetch_indices needs the peer exchange")
        if self._pending is not None:
            raise RuntimeError("index rows already prefetched")
        for x in (idx0, idx1):
            if tuple(x.shape) != (self.b, self.K):
                raise ValueError(f"index rows must be [{self.b}, {self.K}], got {tuple(x.shape)}")
        if self._pf_stream is None:
            self._pf_stream = torch.cuda.Stream(device=self.device)
        slot = (self._cur + 1) % self._IDX_SLOTS
        # contiguous rows made on the current stream; the prefetch stream reads
        # them, so the caching allocator must not reuse them before it has
        xs = [x.contiguous() for x in (idx0, idx1)]
        self._pf_stream.wait_stream(torch.cuda.current_stream(self.device))  # the rows are ready
        with torch.cuda.stream(self._pf_stream):
            self._peer_exchange(self._index_copies(xs[0], xs[1], slot), self._CH_PREFETCH)
            ev = torch.cuda.Event()
            ev.record(self._pf_stream)
        for x in xs:
            x.record_stream(self._pf_stream)
        self._pending = (slot, ev)

    def _take_prefetched(self) -> bool:
        if self._pending is None:
            return False
        slot, ev = self._pending
        self._pending = None
        torch.cuda.current_stream(self.device).wait_event(ev)
        self._cur = slot
        self.idx = self._idx_slots[slot]
        return True

    # -- the step -------------------------------------------------------------
    def forward_local(self, weight_cols: torch.Tensor, bias_cols: torch.Tensor) -> None:
        """The pair forward + the backward's index phase over all positions
        (``gather_indices`` first) on this rank's columns."""
        if tuple(weight_cols.shape) != (self.T, self.width) or tuple(bias_cols.shape) != (self.width,):
            raise ValueError(f"this rank's parameters must be [{self.T}, {self.width}] and [{self.width}]")
        self._take_prefetched()
        if self._prep_stream is None:
            self.kernels.forward_prepare(self.idx[0], self.idx[1], weight_cols, bias_cols, self.y[0], self.y[1],
                                         self.workspace)
            return
        # the index phase on its own normal-priority stream: the forward's
        # gathers take the SMs first, the index phase fills what they leave
        # and runs on into the exchanges; backward_local waits for it
        cur = torch.cuda.current_stream(self.device)
        self._prep_stream.wait_stream(cur)
        with torch.cuda.stream(self._prep_stream):
            self.kernels.prepare(self.idx[0], self.idx[1], self.T, self.width, self.workspace)
            self._prep_done.record(self._prep_stream)
        self.kernels.forward(self.idx[0], self.idx[1], weight_cols, bias_cols, self.y[0], self.y[1])

    def exchange_outputs(self, out0: Optional[torch.Tensor] = None, out1: Optional[torch.Tensor] = None):
        """Rank s receives rows [s*b, (s+1)*b) of every rank's columns; each
        rank joins them into its positions' full output rows [b, C]."""
        r, b = self.rank, self.b
        if self._peer is not None:
            self._slot ^= 1
            wv, cv = self.width // VECTOR, self.C // VECTOR
            copies = []
            for s in range(self.world):
                for p in range(2):
                    src = self.y[p, s * b].data_ptr()
                    dst = self._peer["base"][s] + self._peer["off_out"] + \
                        ((self._slot * 2 + p) * b * self.C + self.c0) * 4
                    copies.append((src, dst, b, wv, cv, wv, 1.0))
            self._peer_exchange(copies)
            res = self._out[self._slot]
            if out0 is not None:
                out0.copy_(res[0])
            if out1 is not None:
                out1.copy_(res[1])
            return (res[0] if out0 is None else out0), (res[1] if out1 is None else out1)
        sends, recvs = [], []
        for s in range(self.world):
            if s == r:
                continue
            for p in range(2):
                sends.append((s, self.y[p, s * b:(s + 1) * b]))
                recvs.append((s, self._block(self.recv, s, p)))
        self._exchange(sends, recvs)
        outs = []
        for p, o in enumerate((out0, out1)):
            parts = [self.y[p, r * b:(r + 1) * b] if s == r else self._block(self.recv, s, p)
                     for s in range(self.world)]
            if o is None:
                o = torch.empty(b, self.C, device=self.y.device)
            torch.cat(parts, dim=1, out=o)
            outs.append(o)
        return outs[0], outs[1]

    def exchange_grads(self, grad0: torch.Tensor, grad1: torch.Tensor) -> None:
        """This rank's positions' output gradients [b, C] -> every rank
        receives its columns of them (scaled by 1/N), rows in position order."""
        r, b = self.rank, self.b
        for g in (grad0, grad1):
            if tuple(g.shape) != (b, self.C):
                raise ValueError(f"output gradients must be [{b}, {self.C}], got {tuple(g.shape)}")
        if self._peer is not None:
            gs = [g.contiguous() for g in (grad0, grad1)]
            cv = self.C // VECTOR
            copies = []
            for s, (c0, c1) in enumerate(self.slices):
                ws = c1 - c0
                for p in range(2):
                    src = gs[p].data_ptr() + c0 * 4
                    dst = self._peer["base"][s] + self._peer["off_d"] + (p * self.B + r * b) * ws * 4
                    copies.append((src, dst, b, cv, ws // VECTOR, ws // VECTOR, self.scale))
            self._peer_exchange(copies)
            return
        for p, g in enumerate((grad0, grad1)):
            for s, (c0, c1) in enumerate(self.slices):
                dst = self.d[p, r * b:(r + 1) * b] if s == r else self._block(self.send, s, p)
                torch.mul(g[:, c0:c1], self.scale, out=dst)
        sends, recvs = [], []
        for s in range(self.world):
            if s == r:
                continue
            for p in range(2):
                sends.append((s, self._block(self.send, s, p)))
                recvs.append((s, self.d[p, s * b:(s + 1) * b]))
        self._exchange(sends, recvs)

    def backward_local(self, weight_grad_cols: torch.Tensor, bias_grad_cols: torch.Tensor) -> None:
        """The segment sums over all positions on this rank's columns (after
        ``exchange_grads``; needs the workspace of ``forward_local``)."""
        if self._prep_done is not None:
            torch.cuda.current_stream(self.device).wait_event(self._prep_done)
        self.kernels.backward_apply(self.d[0], self.d[1], self.B, self.K, weight_grad_cols, bias_grad_cols,
                                    self.workspace)

    def forward(self, weight_cols: torch.Tensor, bias_cols: torch.Tensor, idx0: Optional[torch.Tensor],
                idx1: Optional[torch.Tensor], out0: Optional[torch.Tensor] = None,
                out1: Optional[torch.Tensor] = None):
        """This rank's positions' outputs [b, C] per perspective (the
        data-parallel forward's result) from its positions' index rows (None:
        the rows ``prefetch_indices`` sent; rows passed here take precedence
        over a pending prefetch); also runs the backward's index phase over
        the whole batch."""
        if (idx0 is None) != (idx1 is None):
            raise ValueError("pass both perspectives' index rows or neither")
        if idx0 is not None:
            self.gather_indices(idx0, idx1)  # lets a pending prefetch land first, then replaces it
        elif self._pending is None:
            raise ValueError("no index rows: pass them or prefetch_indices first")
        self.forward_local(weight_cols, bias_cols)
        return self.exchange_outputs(out0, out1)

    def backward(self, grad0: torch.Tensor, grad1: torch.Tensor, weight_grad_cols: torch.Tensor,
                 bias_grad_cols: torch.Tensor) -> None:
        """From this rank's positions' output gradients [b, C]: this rank's
        columns of the weight and bias gradients averaged over the group
        (written, not accumulated).  Needs the workspace of ``forward``."""
        self.exchange_grads(grad0, grad1)
        self.backward_local(weight_grad_cols, bias_grad_cols)


class SparseLinearPairColumnSharded(torch.autograd.Function):
    """``SparseLinearPairFunction`` for column-sharded training:
    (idx_white, idx_black, weight_cols, bias_cols, sharded) -> (out_white,
    out_black), the inputs and outputs this rank's ``batch / N`` positions,
    the parameters this rank's column slice; the backward returns the
    group-averaged gradients of that slice (what DDP's allreduce gives the
    data-parallel form, restricted to the rank's columns).  Leave the two
    parameters out of any other gradient averaging."""

    @staticmethod
    def forward(ctx, feature_indices_0, feature_indices_1, weight_cols, bias_cols, sharded: ColumnShardedFT):
        # None index rows: the rows sharded.prefetch_indices already sent
        out0, out1 = sharded.forward(weight_cols, bias_cols, feature_indices_0, feature_indices_1)
        ctx.sharded = sharded
        ctx.shapes = (tuple(weight_cols.shape), weight_cols.device)
        return out0, out1

    @staticmethod
    def backward(ctx, grad0, grad1):
        sh = ctx.sharded
        (T, w), dev = ctx.shapes
        # a missing output gradient counts as zeros, so every rank runs the same exchanges
        g0 = grad0.contiguous() if grad0 is not None else torch.zeros(sh.b, sh.C, device=dev)
        g1 = grad1.contiguous() if grad1 is not None else torch.zeros(sh.b, sh.C, device=dev)
        dW = torch.empty(T, w, device=dev)
        dB = torch.empty(w, device=dev)
        sh.backward(g0, g1, dW, dB)
        return None, None, dW, dB, None
