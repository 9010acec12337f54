"""Host-side rules of bench.py that decide what a bench line reports: the
multi-GPU scheme picked by GPU count, the columns the timed gather kernels
cover when the library packs the narrow last column chunk into its own
kernel, and the kernel-source digest that stamps DRAM-traffic captures."""

import argparse

import pytest

import bench


@pytest.mark.parametrize("world,want", [(1, "dp"), (2, "dp"), (3, "dp"), (4, "cols"), (8, "cols")])
def test_auto_scheme_by_gpu_count(world, want):
    args = argparse.Namespace(parallel="auto")
    bench.resolve_parallel(args, world)
    assert args.parallel == want
    for fixed in ("dp", "cols"):  # an explicit choice is kept
        args = argparse.Namespace(parallel=fixed)
        bench.resolve_parallel(args, world)
        assert args.parallel == fixed


def test_config_is_the_same_for_both_arms():
    """The reference arm and this arm build `config` from the same rule, so a
    multi-GPU line's config names the scheme the run used."""
    args = argparse.Namespace(parallel="cols", feature_set=bench.FEATURE_SET, batch=65536)
    cfg = bench.base_config(args, 8, 8192, 85296, 160, nnz=1)
    assert cfg["parallelism"] == "cols8" and "column-sharded" in cfg["workload"]
    args.parallel = "dp"
    cfg = bench.base_config(args, 8, 8192, 85296, 160)
    assert cfg["parallelism"] == "dp8" and "allreduce" in cfg["workload"]
    assert bench.base_config(args, 1, 65536, 85296, 160)["parallelism"] == "dp1"


@pytest.mark.parametrize("C,knob,items,forward,want", [
    (1048, 2, 2 * 65536, False, 1024),  # headline light rows: 6-vector tail packed on the side stream
    (1048, 3, 2 * 65536, True, 1024),   # forward mode 3: packed from 2^17 items
    (1048, 3, 2 * 8192, True, 1048),    # ... and not below
    (1048, 0, 2 * 65536, False, 1048),  # knob off
    (136, 2, 2 * 65536, False, 128),    # an 8-way column slice: one chunk + a 2-vector tail
    (128, 2, 2 * 65536, False, 128),    # whole chunks only
    (132, 2, 2 * 65536, False, 132),    # a 1-vector tail is not packed
    (120, 2, 2 * 65536, False, 120),    # narrower than one chunk
    (1050, 2, 2 * 65536, False, 1050),  # not whole vectors
])
def test_timed_kernel_columns(C, knob, items, forward, want):
    assert bench.timed_kernel_columns(C, knob, items, forward) == want


def test_kernel_sources_digest_is_stable():
    d = bench.kernel_sources_digest()
    assert len(d) == 16 and int(d, 16) >= 0
    assert bench.kernel_sources_digest() == d
