#!/usr/bin/env python
"""Benchmark: sparse NNUE feature transformer forward + backward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1)

Workload (the reference's headline configuration): Full_Threats+HalfKAv2_hm^
feature transformer, global batch 65536 positions, L1 = 1040 + 8 PSQT
columns (C = 1048), table 85296 x 1048 fp32, K = 160 padded int32 indices per
perspective.  One step = forward of both perspectives + backward (dense
weight gradient written once, bias gradient) and, for N > 1, the fp32
allreduce-mean of both gradients over NVLink.  The global batch is split
evenly over ranks (strong scaling, like the reference's DDP path,
src/train/common.py:256-263).

Inputs are synthetic: seeded random positions (stockfish_trainer_b200.positions)
encoded by the native restatement of the reference's feature functions,
W ~ N(0, 0.01), bias 0, dOut ~ N(0, 1).  All inputs (idx 84 MB, W 357 MB,
dOut 550 MB) are larger than the 126 MB L2, so no flush between steps.

Prints ONE JSON line on rank 0.  Beside this library's numbers the line
carries two baselines:
* ``tilelang``: the reference's own SparseLinearFunction (TileLang kernels,
  staged unmodified by oracle/build.py) timed on the same GPU and tensors in
  a separate process that does not load this library (oracle/tilelang_timing.py),
  with a bit-for-bit comparison of its outputs and weight gradient;
* ``cpu_baseline``: the C restatement of the reference path (oracle/) on this
  host's cores, the whole batch per step.
``--impl reference`` prints the reference arm: that same CPU measurement as
its own line, inputs built by the oracle's encoder (oracle/positions.py), so
that process loads none of this library's code.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "positions/s FT fwd+bwd @B=65536 L1=1040, 1/2/4/8 B200; % HBM roofline"
FEATURE_SET = "Full_Threats+HalfKAv2_hm^"
L1, NPSQT = 1040, 8
C = L1 + NPSQT
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the
# gather kernels come from a one-pass ncu capture of the default 1-GPU
# headline command, summarised in this file with a digest of the kernel
# sources it was taken on; a capture whose digest differs from the current
# sources is stale and is not reported.
TRAFFIC_FILE = os.path.join("profiles", "dram_traffic_headline_fullsize.md")
DATA = ("synthetic: seeded random positions (kings + U{0..30} pieces), indices from the native restatement "
        "of the reference feature functions; W~N(0,0.01), bias=0, dOut~N(0,1)")


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=["headline", "halfka", "quantized", "gather-probe", "ranger22", "epilogue",
                                          "composed", "train"],
                   default="headline",
                   help="headline: Full_Threats+HalfKAv2_hm^, B=65536 (the headline metric); halfka: HalfKAv2_hm^, "
                        "B=16384 (phases reported separately); quantized: int16 forward, HalfKAv2_hm^, "
                        "B=65536; gather-probe: random-row gather bandwidth versus table size (the ceiling "
                        "for the FT gathers); ranger22, epilogue, composed: the FT optimizer step, the FT "
                        "epilogue and the composed FT module; train: forward + backward + optimizer step "
                        "(row-sharded optimizer for N > 1)")
    p.add_argument("--batch", type=int, default=65536, help="global batch (positions)")
    p.add_argument("--seed", type=int, default=2024)
    p.add_argument("--feature-set", default=FEATURE_SET)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--serial-prepare", action="store_true",
                   help="run the backward's index phase after the forward instead of concurrently with it")
    p.add_argument("--parallel", choices=["auto", "cols", "dp"], default="auto",
                   help="N > 1: cols = each rank owns a column slice of the table and the ranks exchange "
                        "outputs and output gradients (stockfish_trainer_b200.colsharded); dp = every rank "
                        "holds the whole table and the weight gradient is allreduce-averaged (the reference's "
                        "DDP scheme); auto = dp below 4 GPUs, cols from 4 (on B200s: 2 GPUs dp 30.6 against "
                        "cols 25.0 M positions/s, 4 GPUs dp 37.5 against cols 42.8, 8 GPUs dp 39.1 against "
                        "cols 58.8)")
    p.add_argument("--exchange", choices=["peer", "p2p"], default=None,
                   help="--parallel cols: peer = this library's exchange kernel storing into the other GPUs' "
                        "buffers (the default), p2p = torch.distributed point-to-point operations")
    p.add_argument("--cols-prepare", choices=["forward", "overlap"], default="overlap",
                   help="--parallel cols: where the backward's index phase runs (colsharded.ColumnShardedFT)")
    p.add_argument("--cols-prefetch", type=int, choices=[0, 1, 2], default=2,
                   help="--parallel cols: move the next step's index rows during the current step "
                        "(ColumnShardedFT.prefetch_indices) -- 1: issued after the forward, 2: after the "
                        "gradient exchange (beside the backward) -- or 0: at the step's start")
    p.add_argument("--ddp-blocks", type=int, default=4,
                   help="N > 1: row blocks whose gradient allreduce overlaps the next block's backward "
                        "(0 = one allreduce after the whole backward)")
    p.add_argument("--param", action="append", default=[], metavar="NAME=VALUE",
                   help="native tuning knob (see include/nnue_ft.h nnue_ft_set_param)")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline time budget")
    p.add_argument("--no-tilelang", action="store_true",
                   help="skip the reference TileLang kernels timed on the same GPU (N = 1 only)")
    p.add_argument("--tilelang-timeout", type=float, default=900.0)
    return p.parse_args()


def kernel_sources_digest() -> str:
    """sha256 (16 hex digits) over the CUDA sources of the native library."""
    import hashlib

    csrc = os.path.join(ROOT, "stockfish_trainer_b200", "csrc")
    h = hashlib.sha256()
    for name in sorted(os.listdir(csrc)):
        if name.endswith((".cu", ".cuh", ".h", ".cpp")):
            h.update(name.encode())
            with open(os.path.join(csrc, name), "rb") as f:
                h.update(f.read())
    return h.hexdigest()[:16]


def captured_traffic():
    """The DRAM-traffic capture summarised in TRAFFIC_FILE: its JSON block
    (per-launch bytes per kernel, the git head and kernel-source digest it was
    taken on, the command), plus "current" = whether the digest matches the
    sources of this checkout.  None if absent."""
    try:
        with open(os.path.join(ROOT, TRAFFIC_FILE)) as f:
            text = f.read()
        block = text.split("```json", 1)[1].split("```", 1)[0]
        cap = json.loads(block)
    except (OSError, IndexError, ValueError):
        return None
    cap["current"] = cap.get("sources_digest") == kernel_sources_digest()
    return cap


def timed_kernel_columns(C: int, tail_knob: int, items: int, forward: bool) -> int:
    """Columns (floats) the timed main gather kernel covers.  The library
    packs a narrow last column chunk (2, 3, 4, 6 or 8 of the row's 16-byte
    vectors past full 32-vector chunks) into a kernel of its own when the
    tail knob is on (forward mode 3: only from 2^17 items); that kernel is
    not timed with the main one."""
    n_vec, tail = C // 4, (C // 4) % 32
    if C % 4 or n_vec < 32 or tail not in (2, 3, 4, 6, 8):
        return C
    mode = tail_knob
    if forward and mode == 3:
        mode = 2 if items >= (1 << 17) else 0
    return C if mode == 0 else (n_vec - tail) * 4


def hbm_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index: int):
        self.rows = []
        self.marks = []
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "-i", str(gpu_index), "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.time(), [x.strip() for x in line.split(",")]))

    def mark(self):
        self.marks.append(time.time())

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        t0, t1 = (self.marks + [0, 0])[:2] if len(self.marks) >= 2 else (0, float("inf"))
        inside = [r for t, r in self.rows if t0 - 0.15 <= t <= t1 + 0.15] or [r for _, r in self.rows]
        sm, smax, reasons = [], [], set()
        for r in inside:
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
            except (ValueError, IndexError):
                continue
            for name, val in zip(self.REASONS, r[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU baseline (oracle port of the reference path, all host threads)
# ---------------------------------------------------------------------------
def host_threads() -> int:
    """All cores this process may run on (torchrun sets OMP_NUM_THREADS=1,
    which must not throttle the CPU baseline)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_inputs(n: int, T: int, seed: int):
    """Table and output gradients for the CPU legs (numpy, seeded)."""
    rng = np.random.default_rng(seed + 99)
    W_np = (rng.standard_normal((T, C), dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    g0 = rng.standard_normal((n, C), dtype=np.float32)
    g1 = rng.standard_normal((n, C), dtype=np.float32)
    return W_np, g0, g1


def cpu_step(white, black, W_np, g0, g1, nthreads: int) -> float:
    """One step of the reference path restated on the CPU (oracle/ft_oracle.c,
    OpenMP): the forward of both perspectives (kernel.py:93-103), then each
    perspective's backward into its own zero-filled dense weight gradient in
    the reference's order (functions.py:62-65, kernel.py:108-188, bias
    :269), added once as autograd does.  Returns seconds."""
    import oracle

    bias = np.zeros(C, np.float32)
    t0 = time.perf_counter()
    oracle.ft_forward(white, W_np, bias, nthreads=nthreads)
    oracle.ft_forward(black, W_np, bias, nthreads=nthreads)
    oracle.ft_backward_pair(white, black, g0, g1, W_np.shape[0], nthreads=nthreads)
    return time.perf_counter() - t0


CPU_SAMPLE = ("every step: the whole batch ({n} positions), forward of both perspectives + the reference's "
              "backward (two zero-filled dense dW, one per perspective, added once) in the reference's "
              "summation order; C restatement of the reference kernels (oracle/ft_oracle.c) with OpenMP")


def cpu_baseline(white, black, T, seed, budget_s):
    """The reference arm's measurement, run inside this arm on rank 0: whole
    batch per step, median of up to 5 steps within ``budget_s`` (>= 2)."""
    nt = host_threads()
    n = white.shape[0]
    W_np, g0, g1 = cpu_inputs(n, T, seed)
    cpu_step(white, black, W_np, g0, g1, nt)  # first touch of the buffers
    times = []
    t_start = time.perf_counter()
    while len(times) < 2 or (time.perf_counter() - t_start < budget_s and len(times) < 5):
        times.append(cpu_step(white, black, W_np, g0, g1, nt))
    t_med = statistics.median(times)
    return {
        "value": n / t_med,
        "unit": "positions/s",
        "cores": nt,
        "kind": "port",
        "sample": CPU_SAMPLE.format(n=n) + f"; median of {len(times)} steps",
        "ms_per_step": t_med * 1e3,
    }


def base_config(args, world, b_rank, T, K, nnz=None):
    cols = world > 1 and getattr(args, "parallel", "dp") == "cols"
    exchange = ""
    if world > 1:
        exchange = (", column-sharded table: index rows all-gathered, outputs and 1/N-scaled output gradients "
                    "exchanged between ranks, each rank's columns of the averaged dW + dB") if cols else \
            ", fp32 allreduce-mean"
    cfg = {
        "workload": f"{args.feature_set} feature transformer fwd+bwd, both perspectives, dense dW + dB" + exchange,
        "feature_set": args.feature_set,
        "global_batch": args.batch,
        "batch_per_gpu": b_rank,
        "L1": L1,
        "psqt": NPSQT,
        "num_inputs": T,
        "max_active": K,
        "parallelism": f"cols{world}" if cols else f"dp{world}",
        "l2": "inputs larger than L2 (126 MB), no flush",
    }
    if nnz is not None:
        cfg["nnz_per_step"] = nnz
    return cfg


# ---------------------------------------------------------------------------
# the reference's TileLang kernels on the same GPU (separate process)
# ---------------------------------------------------------------------------
def row_checksums(x):
    """Per-row checksum of fp32 bit patterns: sum_c bits(x[r, c]) * (c + 1),
    int64 (the same function as oracle/tilelang_timing.py computes)."""
    import torch

    bits = x.contiguous().view(torch.int32).to(torch.int64)
    w = torch.arange(1, x.shape[1] + 1, dtype=torch.int64, device=x.device)
    return (bits * w).sum(dim=1).cpu().numpy()


def tilelang_baseline(args, white, black, T, ours: dict, ours_ms: float):
    """Runs oracle/tilelang_timing.py in a child process on the same GPU and
    tensors (indices passed in a temporary file, W / g0 / g1 regenerated from
    the same seeds) and compares its outputs and gradients with this arm's
    through per-row bit checksums."""
    import shutil
    import tempfile

    tmp = tempfile.mkdtemp(prefix="ft_tilelang_")
    try:
        idx_path = os.path.join(tmp, "indices.npz")
        np.savez(idx_path, white=white, black=black)
        out = os.path.join(tmp, "result.json")
        cmd = [sys.executable, "-m", "oracle.tilelang_timing", "--indices", idx_path, "--seed", str(args.seed),
               "--num-inputs", str(T), "--output-size", str(C), "--steps", str(max(args.steps, 20)),
               "--warmup", str(max(args.warmup, 3)), "--out", out]
        env = {k: v for k, v in os.environ.items()
               if k not in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT")}
        try:
            r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True,
                               timeout=args.tilelang_timeout)
        except subprocess.TimeoutExpired:
            return {"unavailable": f"the TileLang run did not finish within {args.tilelang_timeout:.0f} s"}
        if r.returncode != 0 or not os.path.exists(out):
            tail = ((r.stderr or "") + (r.stdout or "")).strip().splitlines()[-3:]
            return {"unavailable": f"the TileLang run exited {r.returncode}: {' | '.join(tail)}"}
        with open(out) as f:
            res = json.load(f)
        sums = dict(np.load(out + ".npz"))
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    same_inputs = bool(np.array_equal(sums["W"], ours["W"]) and np.array_equal(sums["g"], ours["g"]))
    bit_exact = {k: bool(np.array_equal(sums[k], ours[k])) for k in ("out0", "out1", "dW")}
    db_diff = float(np.max(np.abs(sums["dB"].astype(np.float64) - ours["dB"].astype(np.float64))))
    repo_so = [p for p in res["shared_objects"] if p.startswith(ROOT) or "torch_extensions" in p]
    B = white.shape[0]
    return {
        "impl": "the reference's SparseLinearFunction (TileLang kernels of src/model/modules/feature_transformer/"
                "kernel.py, staged unmodified), both perspectives on one table + autograd backward, as "
                "composed.py:52-53 drives it",
        "value": B / (res["ms_per_step"] / 1e3),
        "unit": "positions/s",
        "ms_per_step": res["ms_per_step"],
        "ms_per_step_mean": res["ms_per_step_mean"],
        "forward_ms": res["forward_ms"],
        "ours_ms_per_step": ours_ms,
        "speedup_ours_over_tilelang": res["ms_per_step"] / ours_ms,
        "target_speedup": 2.0,
        "same_inputs": same_inputs,
        "bit_exact_vs_ours": bit_exact,
        "bias_grad_max_abs_diff_vs_ours": db_diff,
        "first_call_s": res["first_call_s"],
        "steps": res["steps"],
        "warmup": res["warmup"],
        "timing": "CUDA events around each step on the current stream, median; the first call (TileLang "
                  "autotune + JIT) excluded and reported as first_call_s",
        "process": "child process (oracle/tilelang_timing.py) that does not import this library",
        "shared_objects_from_this_repo": repo_so,
        "gpu": res["gpu"],
    }


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------
def run_reference(args):
    """The reference arm: the reference path restated on the CPU, on this
    host's cores, over the whole workload of this arm's config every step.
    The reference has no CPU implementation of its own (functions.py:21-25
    asserts CUDA tensors), so the restatement in oracle/ is what runs.  Inputs
    come from the oracle's own position generator and feature encoder
    (oracle/positions.py), so this process loads none of this library's code.
    Under torchrun only rank 0 works."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    from oracle import features as oracle_features
    from oracle import positions as oracle_positions

    T, K = oracle_features.feature_set_sizes(args.feature_set)
    nt = host_threads()
    white, black, _ = oracle_positions.synthetic_batch(args.batch, args.feature_set, seed=args.seed, processes=nt)
    nnz = int((white >= 0).sum() + (black >= 0).sum())
    W_np, g0, g1 = cpu_inputs(args.batch, T, args.seed)
    for _ in range(max(args.warmup, 3)):
        cpu_step(white, black, W_np, g0, g1, nt)
    times = [cpu_step(white, black, W_np, g0, g1, nt) for _ in range(args.steps)]
    total = sum(times)
    value = args.batch * len(times) / total
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "positions/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": max(args.warmup, 3),
        "ms_per_step": total / len(times) * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": DATA,
        "config": base_config(args, world, args.batch // max(world, 1), T, K, nnz),
        "cpu_baseline": {"value": value, "unit": "positions/s", "cores": nt, "kind": "port",
                         "sample": CPU_SAMPLE.format(n=args.batch)},
        "e2e": {"value": value, "unit": "positions/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist

    from stockfish_trainer_b200 import SparseLinearPairFunction, _native, ddp, positions
    from stockfish_trainer_b200.feature_transformer import ops

    for kv in args.param:
        name, value = kv.split("=", 1)
        _native.set_param(name, int(value))
    rt = ddp.init_from_env("nccl", timeout_s=180.0)
    rank, world = rt.rank, rt.world_size
    dev = torch.device("cuda", rt.local_rank)
    torch.cuda.set_device(dev)
    if world != args.gpus and rank == 0:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)

    fid, T, K = positions.feature_set_info(args.feature_set)
    first, b_rank = ddp.shard(args.batch, rank, world)
    white, black, _ = positions.synthetic_batch(b_rank, args.feature_set, seed=args.seed, first=first)
    nnz_rank = int((white >= 0).sum() + (black >= 0).sum())
    nnz_all = nnz_rank
    if world > 1:
        t_nnz = torch.tensor([nnz_rank], dtype=torch.int64, device=dev)
        dist.all_reduce(t_nnz)
        nnz_all = int(t_nnz.item())

    gen = torch.Generator(device=dev).manual_seed(args.seed)
    W = torch.randn(T, C, device=dev, generator=gen) * 0.01
    bias = torch.zeros(C, device=dev)
    gen_r = torch.Generator(device=dev).manual_seed(args.seed + 1000 + rank)
    g0 = torch.randn(b_rank, C, device=dev, generator=gen_r)
    g1 = torch.randn(b_rank, C, device=dev, generator=gen_r)
    i0 = torch.from_numpy(white).to(dev)
    i1 = torch.from_numpy(black).to(dev)
    out0 = torch.empty(b_rank, C, device=dev)
    out1 = torch.empty_like(out0)
    cols = world > 1 and args.parallel == "cols"
    if cols:
        # this rank's kernels read its column slice of the table and run over
        # every position of the global batch
        from stockfish_trainer_b200 import colsharded

        if world >= 8 and not any(kv.startswith("bwd_heavy_first=") for kv in args.param):
            # light rows on an 8-way slice are short: start the heavy rows'
            # walks first on the side stream (one B200, the 136-column slice over
            # 65536 positions: backward 0.336 ms against 0.356; the 264-column
            # slice of 4 GPUs: 0.432 against 0.424, so only from 8)
            _native.set_param("bwd_heavy_first", 1)

        plan = colsharded.ColumnShardedFT(T, C, args.batch, K, device=dev, exchange=args.exchange,
                                          prepare=args.cols_prepare)
        Wk, bk, kc, kb = plan.shard_columns(W), plan.shard_columns(bias), plan.width, args.batch
        W = None  # this rank keeps its columns only
        ws = plan.workspace
        dist.barrier()  # every rank arrives at its first exchange together
        plan.gather_indices(i0, i1)
        # all positions' rows, a private copy for the forward-alone timing
        kidx = plan.idx.clone()
        if args.cols_prefetch:
            plan.prefetch_indices(i0, i1)
        ki0, ki1, ko0, ko1 = kidx[0], kidx[1], plan.y[0], plan.y[1]
        knnz = nnz_all
        kcounts = torch.bincount(kidx[kidx >= 0].long(), minlength=T).cpu().numpy()
    else:
        Wk, bk, kc, kb = W, bias, C, b_rank
        ws = ops.alloc_workspace(b_rank, K, T, C, 2, dev)
        ki0, ki1, ko0, ko1 = i0, i1, out0, out1
        knnz = nnz_rank
        kcounts = np.bincount(white[white >= 0], minlength=T) + np.bincount(black[black >= 0], minlength=T)
    grads = ddp.GradientBuffer(T, kc, dev)

    n_ev = 6 if cols else 5
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(n_ev)] for _ in range(max(args.steps, 1))]

    def step_cols(e=None):
        if e:
            e[0].record()
        if not args.cols_prefetch:
            plan.gather_indices(i0, i1)
        if e:
            e[1].record()
        plan.forward_local(Wk, bk)
        if args.cols_prefetch == 1:
            plan.prefetch_indices(i0, i1)  # the next step's rows (the same synthetic batch)
        if e:
            e[2].record()
        plan.exchange_outputs()
        if e:
            e[3].record()
        plan.exchange_grads(g0, g1)
        if args.cols_prefetch == 2:
            plan.prefetch_indices(i0, i1)
        if e:
            e[4].record()
        plan.backward_local(grads.weight, grads.bias)
        if e:
            e[5].record()

    def step(e=None):
        if cols:
            return step_cols(e)
        if e:
            e[0].record()
        if args.serial_prepare:
            ops.forward_pair_into(i0, i1, W, bias, out0, out1)
            if e:
                e[1].record()
            ops.backward_prepare(i0, i1, T, C, ws)
        else:
            # forward + the backward's index-only phase, concurrently
            ops.forward_pair_prepare(i0, i1, W, bias, out0, out1, ws)
            if e:
                e[1].record()
        if e:
            e[2].record()
        if world > 1 and args.ddp_blocks > 0:
            # segment sums in row blocks, each block's allreduce overlapped with the next block
            ddp.backward_allreduce_overlapped(g0, g1, b_rank, K, grads, ws, world, n_blocks=args.ddp_blocks)
            if e:
                e[3].record()
                e[4].record()
        else:
            ops.backward_apply(g0, g1, b_rank, K, grads.weight, grads.bias, False, ws)
            if e:
                e[3].record()
            grads.allreduce_mean(world)
            if e:
                e[4].record()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(max(args.warmup, 3)):
        step()
    barrier()

    clocks = ClockSampler(rt.local_rank) if rank == 0 else None
    time.sleep(0.3)  # let the sampler start
    barrier()
    # the timed region: K steps with nothing but the two bracketing events
    l0 = _native.launch_count()
    if clocks:
        clocks.mark()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for k in range(args.steps):
        step()
    end.record()
    barrier()
    if clocks:
        clocks.mark()
    launches = _native.launch_count() - l0
    ms_local = start.elapsed_time(end)
    ms = max_over_ranks(ms_local)
    flags = _native.device_errors(clear=True)
    if flags:
        raise RuntimeError(f"device error flags {flags:#x} during the bench")
    clock_info = clocks.stop() if clocks else None

    # The same K steps again, instrumented: every launch of the gather kernels
    # bracketed by a CUDA event pair on its own stream
    # (nnue_ft_kernel_timer_arm) and per-phase events on the compute stream.
    # The event records cost a few percent of the step, so this second region
    # gives the per-kernel and per-phase durations, not `value`.
    timed_kinds = (_native.TIMED_FORWARD, _native.TIMED_LIGHT_ROWS, _native.TIMED_HEAVY_ROWS)
    barrier()
    _native.kernel_timer_arm(timed_kinds, (2 + 2 * max(args.ddp_blocks, 1)) * args.steps + 16)
    start_i, end_i = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start_i.record()
    for k in range(args.steps):
        step(ev[k])
    end_i.record()
    barrier()
    live = {k: _native.kernel_timer_read(k) for k in timed_kinds}
    _native.kernel_timer_arm((), 0)
    ms_instrumented = max_over_ranks(start_i.elapsed_time(end_i)) / args.steps
    # with --ddp-blocks the "backward_apply" phase includes the overlapped allreduce
    names = ["gather_indices", "forward+prepare", "exchange_outputs", "exchange_grads", "backward_apply"] if cols \
        else ["forward" if args.serial_prepare else "forward+prepare", "backward_prepare", "backward_apply",
              "allreduce"]
    phases = {n: [e[i].elapsed_time(e[i + 1]) for e in ev[: args.steps]] for i, n in enumerate(names)}
    phase_ms = {k: max_over_ranks(float(np.mean(v))) for k, v in phases.items()}
    if _native.device_errors(clear=True):
        raise RuntimeError("device error flags raised during the instrumented steps")

    ms_per_step = ms / args.steps
    value = args.batch / (ms_per_step / 1e3)

    # ---- roofline: the gather kernels, timed live in the instrumented steps --
    # Durations come from the event pairs recorded around each launch on its
    # own stream (so they include the concurrent side-stream work of the real
    # step).  The roofline object describes the kernel with the largest time
    # per step; "kernels" lists all three.  Algorithmic bytes per launch:
    #   forward: every active row gathered once + outputs written + indices
    #            read + bias;
    #   light rows: the dOut rows of the light rows' entries gathered + their
    #            positions + segment bounds and row kinds of all rows + every
    #            light row of dW written once;
    #   heavy rows: the same for the heavy rows.
    peak, peak_src = hbm_peak()
    # With the narrow last column chunk packed into its own kernel on the side
    # stream, the timed forward / light-row kernels cover the other columns
    # only: count the bytes of the columns each timed kernel covers.
    # (column-sharded: the kernels cover every position on this rank's columns)
    c_fwd = timed_kernel_columns(kc, _native.get_param("fwd_tail"), 2 * kb, forward=True)
    c_light = timed_kernel_columns(kc, _native.get_param("bwd_tail"), 2 * kb, forward=False)
    heavy = np.sort(kcounts[kcounts > _native.get_param("heavy_threshold")])[::-1][:_native.get_param("heavy_cap")]
    n_heavy, nnz_heavy = int(heavy.size), int(heavy.sum())
    nnz_light = knnz - nnz_heavy
    a_fwd = knnz * c_fwd * 4 + 2 * kb * c_fwd * 4 + 2 * kb * K * 4 + c_fwd * 4
    a_light = nnz_light * (c_light * 4 + 4) + (2 * T + 1) * 4 + T + (T - n_heavy) * c_light * 4
    a_heavy = nnz_heavy * (kc * 4 + 4) + n_heavy * kc * 4
    a_step_survey = (knnz * kc * 4 + 2 * kb * kc * 4 + 2 * kb * K * 4) + \
                    (knnz * kc * 4 + 2 * kb * K * 4 + T * kc * 4)
    # DRAM bytes per launch from a one-pass ncu capture of this exact command
    # taken on the current kernel sources (other shapes: not captured)
    capture = captured_traffic()
    default_run = (args.workload == "headline" and b_rank == 65536 and not args.param and world == 1
                   and args.feature_set == FEATURE_SET)
    traffic_ref = capture["per_launch_bytes"] if (capture and capture["current"] and default_run) else {}
    kernels = {}
    for kind, name, a_bytes in ((_native.TIMED_FORWARD, "ft_forward_kernel", a_fwd),
                                (_native.TIMED_LIGHT_ROWS, "ft_segsum_light_kernel", a_light),
                                (_native.TIMED_HEAVY_ROWS, "ft_segsum_heavy_kernel", a_heavy)):
        durations = live[kind]
        # every rank takes part in the max, launched or not
        per_step_ms = max_over_ranks(float(np.sum(durations)) / args.steps if durations else 0.0)
        if per_step_ms <= 0.0:
            continue
        launches_per_step = len(durations) / args.steps
        achieved_k = a_bytes / (per_step_ms / 1e3) / 1e9
        traffic_k = traffic_ref.get(name)
        kernels[name] = {"ms_per_step": per_step_ms, "launches_per_step": launches_per_step,
                         "algorithmic_bytes": a_bytes, "achieved": achieved_k, "frac": achieved_k / peak,
                         "traffic": traffic_k,
                         "dram_frac": (traffic_k / launches_per_step / (per_step_ms / launches_per_step / 1e3)
                                       / 1e9 / peak) if traffic_k else None}
    # the forward alone, K launches with nothing beside it
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(max(args.steps, 1))]
    barrier()
    for a, b in kev:
        a.record()
        ops.forward_pair_into(ki0, ki1, Wk, bk, ko0, ko1)
        b.record()
    barrier()
    fwd_alone_ms = max_over_ranks(float(np.mean([a.elapsed_time(b) for a, b in kev])))
    if "ft_forward_kernel" in kernels:
        kernels["ft_forward_kernel"]["ms_alone"] = fwd_alone_ms
    # Most row gathers hit L2, so the ceiling that bounds these kernels is the
    # random 512-byte-row gather bandwidth from a table the size of one column
    # slice of W (T rows x 512 B), measured here on this GPU
    # (nnue_ft_gather_probe, 32 warps per SM, 8 rows in flight per warp).
    n_warps, per_warp = 148 * 32, 2048
    probe_rows = T
    probe_table = torch.zeros(probe_rows * 128, device=dev)
    probe_idx = torch.randint(0, probe_rows, (n_warps * per_warp,), dtype=torch.int32, device=dev,
                              generator=torch.Generator(device=dev).manual_seed(args.seed + 7))
    probe_out = torch.empty(n_warps * 128, device=dev)
    stream_ptr = torch.cuda.current_stream(dev).cuda_stream

    def probe():
        _native.call("nnue_ft_gather_probe", probe_table.data_ptr(), probe_rows, probe_idx.data_ptr(), per_warp,
                     n_warps, probe_out.data_ptr(), stream_ptr)

    for _ in range(3):
        probe()
    pa, pb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pa.record()
    for _ in range(5):
        probe()
    pb.record()
    torch.cuda.synchronize()
    gather_ceiling = n_warps * per_warp * 512 / (pa.elapsed_time(pb) / 5 / 1e3) / 1e9
    del probe_table, probe_idx, probe_out
    for k in kernels.values():
        k["frac_of_l2_gather_ceiling"] = k["achieved"] / gather_ceiling
    top = max(kernels, key=lambda k: kernels[k]["ms_per_step"]) if kernels else None
    roofline = {"bound": "hbm", "peak": peak, "unit": "GB/s", "peak_source": f"{peak_src} hbm_gbs",
                "l2_gather_ceiling": gather_ceiling,
                "l2_gather_ceiling_source": f"random 512-byte-row gathers from a {probe_rows * 512 / 1e6:.0f} MB "
                                            "table (one column slice of W), measured in this run",
                "step_frac": a_step_survey / (ms_per_step / 1e3) / 1e9 / peak}
    if top:
        k = kernels[top]
        roofline.update({"achieved": k["achieved"], "frac": k["frac"], "traffic": k["traffic"],
                         "kernel": f"{top} (largest device time per step, timed live in the instrumented "
                                   "copy of the timed steps)",
                         "kernel_ms": k["ms_per_step"], "algorithmic_bytes": k["algorithmic_bytes"],
                         "dram_frac": k["dram_frac"],
                         "frac_of_l2_gather_ceiling": k["frac_of_l2_gather_ceiling"]})
    # frac counts every gathered row as HBM bytes (the byte model of the
    # reference path); most gathers hit L2, so frac exceeds 1.  dram_frac is
    # the measured DRAM traffic over the same duration, and the L2 gather
    # ceiling is the bound these kernels actually meet.
    roofline["frac_note"] = ("frac = algorithmic bytes (every gathered row counted as HBM traffic) / duration / "
                             "HBM peak; it exceeds 1 because most row gathers hit L2. dram_frac = measured DRAM "
                             "bytes / duration / HBM peak. frac_of_l2_gather_ceiling = achieved / the random-row "
                             "gather bandwidth of a table the size of one column slice")
    if capture:
        roofline["traffic_source"] = {"file": TRAFFIC_FILE, "head": capture.get("head"),
                                      "sources_digest": capture.get("sources_digest"),
                                      "current_sources_digest": kernel_sources_digest(),
                                      "used": bool(traffic_ref)}
    roofline["kernels"] = kernels

    # ---- e2e through the reference-facing autograd API, host buffers -------
    e2e = None
    if not args.no_e2e:
        h0 = torch.from_numpy(white).pin_memory()
        h1 = torch.from_numpy(black).pin_memory()
        host_out = torch.empty(kc, dtype=torch.float32).pin_memory()
        Wp = Wk.detach().clone().requires_grad_()
        bp = bk.detach().clone().requires_grad_()

        def ft_pair(idx0, idx1):
            # one GPU: the reference-facing autograd function; N GPUs: its
            # column-sharded form (this rank's columns as the parameters, its
            # positions in and out) or its data-parallel form, whose backward
            # returns the averaged gradients with the exchange overlapped in
            # row blocks
            if cols:
                return colsharded.SparseLinearPairColumnSharded.apply(idx0, idx1, Wp, bp, plan)
            if world > 1:
                return ddp.SparseLinearPairAllreduce.apply(idx0, idx1, Wp, bp, world, max(args.ddp_blocks, 1))
            return SparseLinearPairFunction.apply(idx0, idx1, Wp, bp)

        # Inputs move on a copy stream one step ahead (double-buffered), as a
        # data loader feeding the GPU would: step k's copy overlaps step k-1's
        # compute, and step k waits only for its own copy.
        copy_stream = torch.cuda.Stream(dev)
        dbuf = [(torch.empty_like(i0), torch.empty_like(i1)) for _ in range(2)]
        copied = [torch.cuda.Event() for _ in range(2)]
        consumed = [torch.cuda.Event() for _ in range(2)]

        def enqueue_copy(k):
            s = k % 2
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(consumed[s])  # the step that last read this slot is done with it
                dbuf[s][0].copy_(h0, non_blocking=True)
                dbuf[s][1].copy_(h1, non_blocking=True)
                copied[s].record(copy_stream)

        def e2e_step(k):
            s = k % 2
            cur = torch.cuda.current_stream(dev)
            cur.wait_event(copied[s])
            enqueue_copy(k + 1)
            o0, o1 = ft_pair(dbuf[s][0], dbuf[s][1])
            consumed[s].record(cur)  # the indices are read by the forward and its index phase only
            torch.autograd.backward([o0, o1], [g0, g1])
            host_out.copy_(bp.grad, non_blocking=True)
            Wp.grad = None
            bp.grad = None

        enqueue_copy(0)
        n_warm = max(args.warmup, 3)
        for k in range(n_warm):
            e2e_step(k)
        barrier()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for k in range(n_warm, n_warm + args.steps):
            e2e_step(k)
        e2.record()
        barrier()
        ms_e2e = max_over_ranks(s2.elapsed_time(e2)) / args.steps

        # An unchanged caller: the reference's module code with only its
        # SparseLinearFunction import switched to this library's
        # (composed.py:52-53 calls it once per perspective on one table; each
        # call's backward writes its own dense weight gradient and autograd
        # adds the two).  Same host copies; N = 1 only.
        ms_unchanged = None
        if world == 1:
            from stockfish_trainer_b200 import SparseLinearFunction

            def unchanged_step(k):
                s = k % 2
                cur = torch.cuda.current_stream(dev)
                cur.wait_event(copied[s])
                enqueue_copy(k + 1)
                o0 = SparseLinearFunction.apply(dbuf[s][0], Wp, bp)
                o1 = SparseLinearFunction.apply(dbuf[s][1], Wp, bp)
                torch.autograd.backward([o0, o1], [g0, g1])
                consumed[s].record(cur)  # the backward reads the indices again
                host_out.copy_(bp.grad, non_blocking=True)
                Wp.grad = None
                bp.grad = None

            k0 = n_warm + args.steps
            for k in range(k0, k0 + n_warm):
                unchanged_step(k)
            barrier()
            s6, e6 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s6.record()
            for k in range(k0 + n_warm, k0 + n_warm + args.steps):
                unchanged_step(k)
            e6.record()
            barrier()
            ms_unchanged = s6.elapsed_time(e6) / args.steps
            torch.cuda.current_stream(dev).wait_stream(copy_stream)  # the last prefetch
            barrier()

        # the same step with each copy issued on the compute stream right before
        # its step (no overlap), for reference
        def serial_step():
            d0 = h0.to(dev, non_blocking=True)
            d1 = h1.to(dev, non_blocking=True)
            o0, o1 = ft_pair(d0, d1)
            torch.autograd.backward([o0, o1], [g0, g1])
            host_out.copy_(bp.grad, non_blocking=True)
            Wp.grad = None
            bp.grad = None

        for _ in range(n_warm):
            serial_step()
        barrier()
        s3, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s3.record()
        for _ in range(args.steps):
            serial_step()
        e3.record()
        barrier()
        ms_serial = max_over_ranks(s3.elapsed_time(e3)) / args.steps

        # Boards instead of index rows: the loader ships 64 bytes per position
        # (copied on the copy stream one step ahead, double-buffered) and the
        # device encoder (nnue_ft_encode_features, bit-identical to the host
        # encoder) builds both perspectives' index rows at the start of the
        # step.  (Encoding one step ahead on the copy stream instead measured
        # slower: its blocks take SM room the forward's gathers need.)
        board_np, _ = positions.generate_positions(b_rank, seed=args.seed, first=first)  # the same positions
        hboard = torch.from_numpy(board_np).pin_memory()
        bbuf = [torch.empty(b_rank, 64, dtype=torch.uint8, device=dev) for _ in range(2)]
        ibuf = (torch.empty_like(i0), torch.empty_like(i1))
        bcopied = [torch.cuda.Event() for _ in range(2)]
        bconsumed = [torch.cuda.Event() for _ in range(2)]

        def enqueue_board_copy(k):
            s = k % 2
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(bconsumed[s])
                bbuf[s].copy_(hboard, non_blocking=True)
                bcopied[s].record(copy_stream)

        def boards_step(k):
            s = k % 2
            cur = torch.cuda.current_stream(dev)
            cur.wait_event(bcopied[s])
            enqueue_board_copy(k + 1)
            positions.encode_device(bbuf[s], args.feature_set, out=ibuf)
            bconsumed[s].record(cur)
            o0, o1 = ft_pair(ibuf[0], ibuf[1])
            torch.autograd.backward([o0, o1], [g0, g1])
            host_out.copy_(bp.grad, non_blocking=True)
            Wp.grad = None
            bp.grad = None

        enqueue_board_copy(0)
        for k in range(n_warm):
            boards_step(k)
        barrier()
        s4, e4 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s4.record()
        for k in range(n_warm, n_warm + args.steps):
            boards_step(k)
        e4.record()
        barrier()
        ms_boards = max_over_ranks(s4.elapsed_time(e4)) / args.steps
        # the device encoder alone, boards resident
        s5, e5 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s5.record()
        for _ in range(args.steps):
            positions.encode_device(bbuf[0], args.feature_set)
        e5.record()
        barrier()
        ms_encode = max_over_ranks(s5.elapsed_time(e5)) / args.steps
        if _native.device_errors(clear=True):
            raise RuntimeError("device encoder rejected a synthetic position")
        host_enc = None
        if rank == 0:
            sample = board_np[: min(b_rank, 16384)]
            positions.encode(sample, args.feature_set)
            t0 = time.perf_counter()
            positions.encode(sample, args.feature_set)
            host_enc = sample.shape[0] / (time.perf_counter() - t0)
        e2e = {"value": args.batch / (ms_e2e / 1e3), "unit": "positions/s",
               "h2d_bytes_per_step": int(h0.numel() * 4 + h1.numel() * 4), "d2h_bytes_per_step": kc * 4,
               "ms_per_step": ms_e2e,
               "path": "SparseLinearPairFunction autograd fwd+bwd (N > 1: "
                       + ("colsharded.SparseLinearPairColumnSharded, this rank's columns of the averaged "
                          "gradients" if cols else "ddp.SparseLinearPairAllreduce, gradients averaged inside "
                                                   "the backward")
                       + "); each step's indices copied from pinned host memory on a copy stream one step "
                         "ahead (double-buffered); bias grad read back",
               "serial_copy_ms_per_step": ms_serial,
               "unchanged_caller": None if ms_unchanged is None else {
                   "value": args.batch / (ms_unchanged / 1e3), "unit": "positions/s", "ms_per_step": ms_unchanged,
                   "h2d_bytes_per_step": int(h0.numel() * 4 + h1.numel() * 4), "d2h_bytes_per_step": C * 4,
                   "path": "the reference's call pattern unchanged (composed.py:52-53): SparseLinearFunction once "
                           "per perspective on one table, each backward writing its own dense weight gradient, "
                           "autograd adding the two; same double-buffered host copies"},
               "boards": {"value": args.batch / (ms_boards / 1e3), "unit": "positions/s",
                          "ms_per_step": ms_boards, "h2d_bytes_per_step": int(hboard.numel()),
                          "d2h_bytes_per_step": kc * 4,
                          "path": "boards [B, 64] uint8 copied from pinned host memory on a copy stream one "
                                  "step ahead (double-buffered), encoded on the device at the start of the "
                                  "step (nnue_ft_encode_features), then the same autograd step",
                          "device_encode_ms": ms_encode,
                          "device_encode_positions_per_s": b_rank / (ms_encode / 1e3),
                          "host_encoder_positions_per_s": host_enc,
                          "host_encoder_threads": os.cpu_count()}}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(white, black, T, args.seed, args.cpu_seconds)

    tilelang = None
    if rank == 0 and world == 1 and not args.no_tilelang:
        # this arm's last timed step: outputs, dense dW and dB of the same tensors
        ours_sums = {"out0": row_checksums(out0), "out1": row_checksums(out1), "dW": row_checksums(grads.weight),
                     "dB": grads.bias.cpu().numpy(), "W": row_checksums(W),
                     "g": np.concatenate([row_checksums(g0), row_checksums(g1)])}
        tilelang = tilelang_baseline(args, white, black, T, ours_sums, ms_per_step)

    if rank == 0:
        metric = METRIC if args.workload == "headline" else \
            f"positions/s {args.feature_set} FT fwd+bwd @B={args.batch} L1={L1}"
        line = {
            "metric": metric,
            "value": value,
            "unit": "positions/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": max(args.warmup, 3),
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f32",
            "data": DATA,
            "config": base_config(args, world, b_rank, T, K, int(nnz_all)),
            "parallel": ({"scheme": "column-sharded", "exchange": plan.exchange, "column_slices": plan.slices,
                          "index_phase": plan.prepare, "index_prefetch": bool(args.cols_prefetch),
                          "bwd_heavy_first": _native.get_param("bwd_heavy_first")} if cols else
                         {"scheme": "data-parallel allreduce", "row_blocks": args.ddp_blocks} if world > 1
                         else None),
            "phases_ms": phase_ms,
            "instrumented_ms_per_step": ms_instrumented,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "tilelang": tilelang,
            "e2e": e2e,
            "gpu_launches": int(launches),
            "gpu_launches_per_step": launches / max(args.steps, 1),
            "clocks": clock_info,
            "gpu": torch.cuda.get_device_name(dev),
        }
        emit(line)
    if cols:
        plan.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_gather_probe(args):
    """Random 512-byte-row gather bandwidth versus table size."""
    import torch

    from stockfish_trainer_b200 import _native

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n_warps, per_warp = 148 * 32, 2048
    table = torch.zeros((512 << 20) // 4, device=dev)
    out = torch.empty(n_warps * 128, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    curve = {}
    for mb in (16, 32, 48, 64, 80, 96, 128, 192, 256, 512):
        rows = (mb << 20) // 512
        idx = torch.randint(0, rows, (n_warps * per_warp,), dtype=torch.int32, device=dev)
        run = lambda: _native.call("nnue_ft_gather_probe", table.data_ptr(), rows, idx.data_ptr(), per_warp, n_warps,
                                   out.data_ptr(), stream)
        for _ in range(3):
            run()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(max(args.steps, 5)):
            run()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / max(args.steps, 5)
        curve[f"{mb}MB"] = round(n_warps * per_warp * 512 / (ms / 1e3) / 1e9, 1)
    emit({"metric": "GB/s random 512-byte-row gather vs table size", "unit": "GB/s", "value": max(curve.values()),
          "curve": curve, "warps": n_warps, "rows_in_flight_per_warp": 8, "higher_is_better": True,
          "hbm_peak": hbm_peak()[0]})
    return 0


def run_quantized(args):
    """int16 quantised FT forward of both perspectives (B = 65536),
    HalfKAv2_hm^ export tables (22528 x 1040 int16 + 8 int32 PSQT) produced
    from random fp32 weights by the serializer's quantisation."""
    import torch

    from stockfish_trainer_b200 import _native, positions
    from stockfish_trainer_b200.feature_transformer import ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    fs = "HalfKAv2_hm^"
    B = args.batch
    white, black, _ = positions.synthetic_batch(B, fs, seed=args.seed)
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    W = torch.randn(24576, C, device=dev, generator=gen) * 0.01
    V = torch.randn(768, C, device=dev, generator=gen) * 0.002
    wq, pq = ops.halfka_export_quantize(W, V, L1)
    bq = ops.quantize_i16((torch.randn(L1, device=dev, generator=gen) * 0.05).contiguous(), 255.0)
    i0, i1 = torch.from_numpy(white).to(dev), torch.from_numpy(black).to(dev)
    step = lambda: ops.quantized_forward_pair(i0, i1, wq, pq, bq, True)
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    l0 = _native.launch_count()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        step()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.steps
    nnz = int((white >= 0).sum() + (black >= 0).sum())
    row_bytes = L1 * 2 + NPSQT * 4
    a_bytes = nnz * row_bytes + 2 * B * row_bytes + 2 * B * white.shape[1] * 4
    peak, src = hbm_peak()
    emit({
        "metric": "positions/s int16 FT forward (both perspectives) @B=65536 L1=1040, HalfKAv2_hm^",
        "value": B / (ms / 1e3), "unit": "positions/s", "n_gpus": 1, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "i16", "data": DATA,
        "config": {"workload": "int16 quantised FT forward, HalfKAv2_hm^ export tables, training indices mapped "
                               "in-kernel", "batch": B, "L1": L1, "psqt": NPSQT, "table_rows": 22528},
        "roofline": {"bound": "hbm", "achieved": a_bytes / (ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": a_bytes / (ms / 1e3) / 1e9 / peak, "traffic": None,
                     "kernel": "ft_qforward_kernel", "algorithmic_bytes": a_bytes,
                     "peak_source": f"{src} hbm_gbs"},
        "gpu_launches": int(_native.launch_count() - l0),
    })
    return 0


def run_ranger22(args):
    """Ranger22 step of the FT parameters (src/ranger22/optimizer.py): the merged
    85296 x 1048 table and the 1048 bias, each one fused update per step,
    the lookahead blend fused into every 5th step as in training.  One step =
    Ranger22FT.step() over both parameters."""
    import torch

    from oracle import ranger22 as oracle_r22
    from stockfish_trainer_b200 import _native, optim, positions

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    T = positions.feature_set_info(args.feature_set)[1]
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    w = torch.nn.Parameter(torch.randn(T, C, device=dev, generator=gen) * 0.01)
    b = torch.nn.Parameter(torch.zeros(C, device=dev))
    w.grad = torch.randn(T, C, device=dev, generator=gen) * 1e-3
    b.grad = torch.randn(C, device=dev, generator=gen) * 1e-3
    opt = optim.Ranger22FT([{"params": [w, b]}], lr=8.75e-4, betas=(0.9, 0.999), eps=1.0e-7)
    for _ in range(max(args.warmup, 3)):
        opt.step()
    torch.cuda.synchronize()
    l0 = _native.launch_count()
    steps = max(args.steps, 5)
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        opt.step()
    e.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(e) / steps
    n = w.numel() + b.numel()
    merges = sum(1 for k in range(steps) if (max(args.warmup, 3) + k + 1) % 5 == 0)
    a_bytes = (32 * n * steps + 8 * n * merges) / steps  # p, g, v, m, m_prev read; p, v, m written (+ lookahead)
    peak, src = hbm_peak()
    # CPU baseline: the numpy oracle on 2048 rows of the table, scaled to the full table
    rows = 2048
    rng = np.random.default_rng(args.seed)
    pc = (rng.standard_normal((rows, C)) * 0.01).astype(np.float32)
    gc = (rng.standard_normal((rows, C)) * 1e-3).astype(np.float32)
    vc, mc, mpc = (np.zeros_like(pc) for _ in range(3))
    sc = oracle_r22.scalars(8.75e-4, 5)
    t0 = time.perf_counter()
    reps = 3
    for _ in range(reps):
        oracle_r22.update(pc, gc, vc, mc, mpc, sc)
    cpu_s = (time.perf_counter() - t0) / reps * (T / rows)
    emit({
        "metric": "FT Ranger22 steps/s (85296x1048 table + bias, fused update, lookahead every 5th step)",
        "value": 1e3 / ms, "unit": "steps/s", "n_gpus": 1, "steps": steps, "warmup": max(args.warmup, 3),
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: W~N(0,0.01), grad~N(0,1e-3), zero-initialised optimizer state",
        "config": {"workload": "Ranger22 (trainer configuration) step of the FT table and bias, one fused kernel "
                               "per parameter", "rows": T, "cols": C, "lookahead_mergetime": 5,
                   "l2": "parameter and state larger than L2 (2.9 GB per step), no flush"},
        "roofline": {"bound": "hbm", "achieved": a_bytes / (ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": a_bytes / (ms / 1e3) / 1e9 / peak, "traffic": None,
                     "kernel": "ranger22_rows_kernel", "algorithmic_bytes": a_bytes,
                     "peak_source": f"{src} hbm_gbs"},
        "cpu_baseline": {"value": 1.0 / cpu_s, "unit": "steps/s", "cores": 1, "kind": "port",
                         "sample": f"numpy oracle update of {rows} table rows, scaled to {T} rows"},
        "gpu_launches": int(_native.launch_count() - l0),
    })
    return 0


def run_epilogue(args):
    """FT epilogue: NNUEModel._transform_inputs after the
    FT (model.py:93-115), forward + backward of both perspectives at the
    headline batch, one fused kernel each way."""
    import torch

    from stockfish_trainer_b200 import _native
    from stockfish_trainer_b200.feature_transformer import transform_inputs

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B = args.batch
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    wp = (torch.randn(B, C, device=dev, generator=gen) * 0.8 + 0.4).requires_grad_()
    bp = (torch.randn(B, C, device=dev, generator=gen) * 0.8 + 0.4).requires_grad_()
    us = (torch.rand(B, 1, device=dev, generator=gen) < 0.5).float()
    pidx = torch.randint(0, NPSQT, (B,), device=dev, generator=gen)
    d_l0 = torch.randn(B, L1, device=dev, generator=gen)
    d_psqt = torch.randn(B, 1, device=dev, generator=gen)

    def step():
        l0, psqt = transform_inputs(wp, bp, us, pidx, L1)
        torch.autograd.backward([l0, psqt], [d_l0, d_psqt])
        wp.grad = None
        bp.grad = None

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    l0c = _native.launch_count()
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        step()
    e.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(e) / args.steps
    launches = _native.launch_count() - l0c
    row = C * 4
    # forward: read wp, bp, us, index; write l0, psqt.  backward: read d_l0, d_psqt, wp, bp, us, index; write
    # d_wp, d_bp
    a_bytes = B * (2 * row + 4 + 8 + L1 * 4 + 4) + B * (L1 * 4 + 4 + 2 * row + 4 + 8 + 2 * row)
    peak, src = hbm_peak()
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import epilogue as oracle_epi

        n = 4096
        wc, bc = wp.detach()[:n].cpu(), bp.detach()[:n].cpu()
        uc, pc, gl, gp = us[:n].cpu(), pidx[:n].cpu(), d_l0[:n].cpu(), d_psqt[:n].cpu()
        oracle_epi.forward_backward(wc, bc, uc, pc, L1, gl, gp)
        t0 = time.perf_counter()
        reps = 5
        for _ in range(reps):
            oracle_epi.forward_backward(wc, bc, uc, pc, L1, gl, gp)
        cpu_ms = (time.perf_counter() - t0) / reps * 1e3
        cpu = {"value": n / (cpu_ms / 1e3), "unit": "positions/s", "cores": torch.get_num_threads(),
               "kind": "port", "sample": f"{n} positions, PyTorch CPU restatement of model.py:93-115 + autograd"}
    emit({
        "metric": "positions/s FT epilogue fwd+bwd (model.py _transform_inputs) @B=65536 L1=1040",
        "value": B / (ms / 1e3), "unit": "positions/s", "n_gpus": 1, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic: FT outputs ~N(0.4, 0.8), random us / PSQT buckets",
        "config": {"workload": "FT epilogue forward + backward, both perspectives", "batch": B, "L1": L1,
                   "psqt": NPSQT, "l2": "inputs larger than L2, no flush"},
        "roofline": {"bound": "hbm", "achieved": a_bytes / (ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": a_bytes / (ms / 1e3) / 1e9 / peak, "traffic": None,
                     "kernel": "ft_epilogue_forward_kernel + ft_epilogue_backward_kernel",
                     "algorithmic_bytes": a_bytes, "peak_source": f"{src} hbm_gbs"},
        "cpu_baseline": cpu,
        "gpu_launches": int(launches),
    })
    return 0


def run_composed(args):
    """Module-level composed FT (src/model/modules/features/composed.py): ComposedFeatureTransformer
    forward + backward through autograd at the headline size, the per-feature
    tables read in place (no merged copy), against the reference module's
    graph (torch.cat of the per-feature tables with the virtual rows repeated,
    then the FT op) run with this library's FT op on the same GPU."""
    import torch
    from torch import nn

    from stockfish_trainer_b200 import _native, positions
    from stockfish_trainer_b200.feature_transformer import SparseLinearFunction, SparseLinearPairFunction
    from stockfish_trainer_b200.feature_transformer.composed import ComposedFeatureTransformer

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B = args.batch
    white, black, _ = positions.synthetic_batch(B, "Full_Threats+HalfKAv2_hm^", seed=args.seed)

    class Feature(nn.Module):
        def __init__(self, rows, virtual_rows, name, h, max_active, real):
            super().__init__()
            self.num_outputs, self.NUM_INPUTS, self.FEATURE_NAME = C, rows, name
            self.INPUT_FEATURE_NAME, self.HASH, self.MAX_ACTIVE_FEATURES, self.NUM_REAL_FEATURES = name, h, max_active, real
            self.weight = nn.Parameter(torch.randn(rows, C, device=dev) * 0.01)
            if virtual_rows:
                self.NUM_BUCKETS = rows // virtual_rows
                self.virtual_weight = nn.Parameter(torch.randn(virtual_rows, C, device=dev) * 0.001)

        def merged_weight(self):
            if hasattr(self, "virtual_weight"):
                return self.weight + self.virtual_weight.repeat(self.NUM_BUCKETS, 1)
            return self.weight

    torch.manual_seed(args.seed)
    feats = [Feature(60720, 0, "Full_Threats", 0x8F234CB8, 128, 60720),
             Feature(24576, 768, "HalfKAv2_hm^", 0x7F234CB8, 32, 22528)]
    module = ComposedFeatureTransformer(feats).to(dev)
    i0, i1 = torch.from_numpy(white).to(dev), torch.from_numpy(black).to(dev)
    gen = torch.Generator(device=dev).manual_seed(args.seed + 1)
    d0 = torch.randn(B, C, device=dev, generator=gen)
    d1 = torch.randn(B, C, device=dev, generator=gen)

    def fused():
        o0, o1 = module(i0, i1)
        torch.autograd.backward([o0, o1], [d0, d1])
        for p in module.parameters():
            p.grad = None

    def cat_path():
        merged = torch.cat([f.merged_weight() for f in feats], dim=0)
        o0, o1 = SparseLinearPairFunction.apply(i0, i1, merged, module.bias)
        torch.autograd.backward([o0, o1], [d0, d1])
        for p in module.parameters():
            p.grad = None

    def dropin_graph():
        # the reference module's forward unchanged (composed.py:49-54), only
        # SparseLinearFunction taken from this library
        merged = torch.cat([f.merged_weight() for f in feats], dim=0)
        o0 = SparseLinearFunction.apply(i0, merged, module.bias)
        o1 = SparseLinearFunction.apply(i1, merged, module.bias)
        torch.autograd.backward([o0, o1], [d0, d1])
        for p in module.parameters():
            p.grad = None

    def timeit(fn):
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize()
        a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            fn()
        e.record()
        torch.cuda.synchronize()
        return a.elapsed_time(e) / args.steps

    ms_cat = timeit(cat_path)
    ms_dropin = timeit(dropin_graph)
    l0c = _native.launch_count()
    ms = timeit(fused)
    launches = _native.launch_count() - l0c
    # the two module-level passes the composed step still runs around the FT
    # kernels: the HalfKA table + virtual rows (one fp32 add per element) and
    # the virtual rows' gradient (the sum over the 32 buckets of the HalfKA
    # gradient, torch's repeat backward)
    halfka = feats[1]
    d_half = torch.randn(halfka.weight.shape, device=dev, generator=gen)
    from stockfish_trainer_b200.feature_transformer import ops as ft_ops

    ms_merge = timeit(lambda: ft_ops.merge_virtual(halfka.weight.detach(), halfka.virtual_weight.detach()))
    reps = halfka.weight.shape[0] // halfka.virtual_weight.shape[0]
    ms_vgrad = timeit(lambda: d_half.view(reps, -1, C).sum(0))
    nnz = int((white >= 0).sum() + (black >= 0).sum())
    T, K = 85296, white.shape[1]
    a_bytes = (nnz * C * 4 + 2 * B * C * 4 + 2 * B * K * 4) + (nnz * C * 4 + 2 * B * K * 4 + T * C * 4)
    peak, src = hbm_peak()
    emit({
        "metric": "positions/s composed FT module fwd+bwd (Full_Threats+HalfKAv2_hm^, autograd) @B=65536 L1=1040",
        "value": B / (ms / 1e3), "unit": "positions/s", "n_gpus": 1, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": DATA,
        "config": {"workload": "ComposedFeatureTransformer forward + backward (threat table, HalfKA table + 768 "
                               "virtual rows, bias) through autograd", "batch": B, "L1": L1, "psqt": NPSQT,
                   "l2": "inputs larger than L2, no flush"},
        "roofline": {"bound": "hbm", "achieved": a_bytes / (ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": a_bytes / (ms / 1e3) / 1e9 / peak, "traffic": None,
                     "kernel": "module step (forward + backward byte model of the FT op)", "algorithmic_bytes": a_bytes,
                     "peak_source": f"{src} hbm_gbs"},
        "module_passes_ms": {"halfka_virtual_merge": ms_merge, "virtual_grad_bucket_sum": ms_vgrad,
                             "what": "the two passes around the FT kernels in the composed step: weight + "
                                     "virtual rows (24576 x 1048, one add per element) and the virtual rows' "
                                     "gradient (sum of the 32 bucket blocks of the HalfKA gradient)"},
        "unchanged_module_same_gpu": {"ms_per_step": ms_dropin, "value": B / (ms_dropin / 1e3),
                                      "unit": "positions/s",
                                      "what": "the reference module's forward unchanged (torch.cat + repeat, "
                                              "SparseLinearFunction once per perspective, autograd adding the two "
                                              "dense weight gradients) with this library's SparseLinearFunction"},
        "cat_path_same_gpu": {"ms_per_step": ms_cat, "value": B / (ms_cat / 1e3), "unit": "positions/s",
                              "what": "reference module graph (torch.cat + repeat) with this library's FT op"},
        "gpu_launches": int(launches),
    })
    return 0


def run_train(args):
    """FT training step: forward of both perspectives (with the backward's
    index phase beside it), backward, and the Ranger22 update (the reference
    trainer's configuration) of the table and bias.  N = 1: dense gradients
    then the fused update over the whole table.  N > 1: the row-sharded step
    (reduce-scatter of each row block's averaged gradient, the update of this
    rank's rows, all-gather of the updated rows), with the unsharded path
    (allreduce of the whole gradient, then the update of the whole table on
    every rank, as the reference's DDP does) timed beside it."""
    import torch
    import torch.distributed as dist

    from stockfish_trainer_b200 import _native, ddp, optim, positions, sharded
    from stockfish_trainer_b200.feature_transformer import ops

    rt = ddp.init_from_env("nccl", timeout_s=180.0)
    rank, world = rt.rank, rt.world_size
    dev = torch.device("cuda", rt.local_rank)
    torch.cuda.set_device(dev)
    fid, T, K = positions.feature_set_info(args.feature_set)
    first, b_rank = ddp.shard(args.batch, rank, world)
    white, black, _ = positions.synthetic_batch(b_rank, args.feature_set, seed=args.seed, first=first)
    nnz = torch.tensor([int((white >= 0).sum() + (black >= 0).sum())], dtype=torch.int64, device=dev)
    if world > 1:
        dist.all_reduce(nnz)
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    W = torch.randn(T, C, device=dev, generator=gen) * 0.01
    bias = torch.zeros(C, device=dev)
    gen_r = torch.Generator(device=dev).manual_seed(args.seed + 1000 + rank)
    g0 = torch.randn(b_rank, C, device=dev, generator=gen_r)
    g1 = torch.randn(b_rank, C, device=dev, generator=gen_r)
    i0, i1 = torch.from_numpy(white).to(dev), torch.from_numpy(black).to(dev)
    o0, o1 = torch.empty(b_rank, C, device=dev), torch.empty(b_rank, C, device=dev)
    ws = ops.alloc_workspace(b_rank, K, T, C, 2, dev)
    lr = 8.75e-4
    n_blocks = max(args.ddp_blocks, 1)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def measure(step):
        """(ms per step, max over ranks; this library's launches in the timed steps)"""
        for _ in range(max(args.warmup, 3)):
            step()
        barrier()
        l0 = _native.launch_count()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            step()
        b.record()
        barrier()
        return max_over_ranks(a.elapsed_time(b) / args.steps), _native.launch_count() - l0

    # the unsharded step: whole gradient averaged, whole table updated on every rank
    Wp, bp = torch.nn.Parameter(W.clone()), torch.nn.Parameter(bias.clone())
    whole = optim.Ranger22FT([Wp, bp], lr=lr)
    buf = ddp.GradientBuffer(T, C, dev)

    def unsharded_step():
        ops.forward_pair_prepare(i0, i1, Wp.data, bp.data, o0, o1, ws)
        ddp.backward_allreduce_overlapped(g0, g1, b_rank, K, buf, ws, world, n_blocks=n_blocks) if world > 1 else \
            ops.backward_apply(g0, g1, b_rank, K, buf.weight, buf.bias, False, ws)
        Wp.grad, bp.grad = buf.weight, buf.bias
        whole.step()

    ms_whole, launches = measure(unsharded_step)
    del whole, buf, Wp, bp
    ms_sharded = None
    if world > 1:
        Ws, bs = W.clone(), bias.clone()
        opt = sharded.ShardedRanger22FT(Ws, bs, lr, n_blocks=n_blocks)

        def sharded_step():
            ops.forward_pair_prepare(i0, i1, Ws, bs, o0, o1, ws)
            opt.backward_step(g0, g1, b_rank, K, ws)

        ms_sharded, launches = measure(sharded_step)
    if _native.device_errors(clear=True):
        raise RuntimeError("device error flags raised during the training-step bench")
    ms = ms_sharded if ms_sharded is not None else ms_whole
    if rank == 0:
        emit({
            "metric": f"positions/s FT training step (fwd+bwd+Ranger22 update of the FT table and bias) "
                      f"{args.feature_set} @B={args.batch} L1={L1}",
            "value": args.batch / (ms / 1e3), "unit": "positions/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": DATA,
            "config": dict(base_config(args, world, b_rank, T, K, int(nnz.item())),
                           workload="FT training step: forward + backward + Ranger22 update (trainer "
                                    "configuration, lookahead every 5 steps)"
                                    + (", optimizer state sharded by table rows (reduce-scatter / update / "
                                       "all-gather per row block)" if world > 1 else "")),
            "unsharded": {"ms_per_step": ms_whole, "value": args.batch / (ms_whole / 1e3), "unit": "positions/s",
                          "what": "whole gradient allreduce-averaged (row blocks overlapped with the backward), "
                                  "whole table updated on every rank"},
            "gpu_launches": int(launches) if launches is not None else None,
        })
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


_JSON_FD = None


def emit(line: dict) -> None:
    """Writes the one JSON result line to the real stdout."""
    data = (json.dumps(line) + "\n").encode()
    if _JSON_FD is None:
        sys.stdout.write(data.decode())
        sys.stdout.flush()
    else:
        os.write(_JSON_FD, data)


def resolve_parallel(args, world: int) -> None:
    """--parallel auto -> the scheme measured faster at this many GPUs."""
    if args.parallel == "auto":
        args.parallel = "cols" if world >= 4 else "dp"


def main():
    global _JSON_FD
    args = parse_args()
    # Libraries (NCCL, torch) may print banners on stdout; route all of that
    # to stderr so stdout carries exactly one JSON line.
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    resolve_parallel(args, int(os.environ.get("WORLD_SIZE", "1")))
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "ranger22":
        return run_ranger22(args)
    if args.workload == "epilogue":
        return run_epilogue(args)
    if args.workload == "composed":
        return run_composed(args)
    if args.workload == "train":
        return run_train(args)
    if args.workload == "quantized":
        return run_quantized(args)
    if args.workload == "gather-probe":
        return run_gather_probe(args)
    if args.workload == "halfka":
        args.feature_set = "HalfKAv2_hm^"
        if args.batch == 65536:
            args.batch = 16384
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
