"""ORACLE -- TEST INFRASTRUCTURE ONLY: the GPU bar of the bench.

    python -m oracle.tilelang_timing --indices FILE.npz --seed S --steps K --warmup W --out RESULT.json

Times the reference's own ``SparseLinearFunction`` (its TileLang forward and
backward kernels, ``src/model/modules/feature_transformer/kernel.py``,
staged unmodified under ``oracle/_ref``) on one GPU, in a process that never
imports this repository's product package.  One step is what the reference's
composed module runs per training step for the feature transformer
(``src/model/modules/features/composed.py:52-53``): the op called once per
perspective on one shared table, then autograd's backward through both
calls (each call's backward allocates and fills a dense weight gradient,
``functions.py:64-72``; autograd adds the two).

Inputs: the two perspectives' index rows from ``--indices`` (``white``,
``black``); the table, bias and output gradients drawn on the device with the
same generator calls as ``bench.py`` (``torch.Generator(cuda).manual_seed``:
W = randn(T, C) * 0.01 from seed S, bias = 0, g0 and g1 = randn(B, C) from
seed S + 1000), so both processes hold the same tensors; a checksum of W and
of the gradients proves it.

The first call autotunes the TileLang kernels (compiles each thread
configuration and times it) and is reported separately; then W warm-up steps
and K timed steps, each bracketed by CUDA events on the current stream.
Writes a JSON result with the median and mean step time, the forward alone,
per-row checksums of both outputs and of the weight gradient (``--out`` +
``.npz``), the bias gradient, and the shared objects this process mapped.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def row_checksums(x):
    """Per-row checksum of the fp32 bit patterns: sum over columns of
    bits(x[r, c]) * (c + 1) in int64 (exact: |bits| < 2^31, C < 2^20)."""
    import torch

    bits = x.contiguous().view(torch.int32).to(torch.int64)
    w = torch.arange(1, x.shape[1] + 1, dtype=torch.int64, device=x.device)
    return (bits * w).sum(dim=1)


def mapped_shared_objects() -> list[str]:
    out = set()
    try:
        with open("/proc/self/maps") as f:
            for line in f:
                parts = line.split()
                if len(parts) >= 6 and ".so" in parts[-1]:
                    out.add(parts[-1])
    except OSError:
        pass
    return sorted(out)


def main(argv=None) -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--indices", required=True)
    p.add_argument("--seed", type=int, required=True)
    p.add_argument("--num-inputs", type=int, required=True)
    p.add_argument("--output-size", type=int, default=1048)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--out", required=True)
    args = p.parse_args(argv)

    import torch

    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    from oracle import tilelang_ref

    ref = tilelang_ref.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    data = np.load(args.indices)
    i0 = torch.from_numpy(data["white"]).to(dev)
    i1 = torch.from_numpy(data["black"]).to(dev)
    B, T, C = i0.shape[0], args.num_inputs, args.output_size
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    W = torch.randn(T, C, device=dev, generator=gen) * 0.01
    bias = torch.zeros(C, device=dev)
    gen_r = torch.Generator(device=dev).manual_seed(args.seed + 1000)
    g0 = torch.randn(B, C, device=dev, generator=gen_r)
    g1 = torch.randn(B, C, device=dev, generator=gen_r)
    Wp = W.clone().requires_grad_()
    bp = bias.clone().requires_grad_()

    def forward():
        o0 = ref.SparseLinearFunction.apply(i0, Wp, bp)
        o1 = ref.SparseLinearFunction.apply(i1, Wp, bp)
        return o0, o1

    def step():
        o0, o1 = forward()
        torch.autograd.backward([o0, o1], [g0, g1])
        return o0, o1

    t0 = time.perf_counter()
    o0, o1 = step()  # autotunes forward and backward kernels
    torch.cuda.synchronize()
    first_call_s = time.perf_counter() - t0
    for _ in range(max(args.warmup, 1)):
        Wp.grad = None
        bp.grad = None
        step()
    torch.cuda.synchronize()

    def timed(fn, n):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        for a, b in ev:
            Wp.grad = None
            bp.grad = None
            a.record()
            fn()
            b.record()
        torch.cuda.synchronize()
        return [a.elapsed_time(b) for a, b in ev]

    step_ms = timed(step, args.steps)
    with torch.no_grad():
        fwd_ms = timed(forward, args.steps)
    # outputs and gradients of one more step, for the bit-exact comparison
    Wp.grad = None
    bp.grad = None
    o0, o1 = step()
    torch.cuda.synchronize()
    sums = {
        "out0": row_checksums(o0.detach()).cpu().numpy(),
        "out1": row_checksums(o1.detach()).cpu().numpy(),
        "dW": row_checksums(Wp.grad).cpu().numpy(),
        "dB": bp.grad.detach().cpu().numpy(),
        "W": row_checksums(W).cpu().numpy(),
        "g": np.concatenate([row_checksums(g0).cpu().numpy(), row_checksums(g1).cpu().numpy()]),
    }
    np.savez(args.out + ".npz", **sums)
    res = {
        "ms_per_step": statistics.median(step_ms),
        "ms_per_step_mean": statistics.fmean(step_ms),
        "forward_ms": statistics.median(fwd_ms),
        "first_call_s": first_call_s,
        "steps": args.steps,
        "warmup": max(args.warmup, 1),
        "batch": B,
        "gpu": torch.cuda.get_device_name(dev),
        "shared_objects": mapped_shared_objects(),
    }
    with open(args.out, "w") as f:
        json.dump(res, f)
    return 0


if __name__ == "__main__":
    sys.exit(main())
