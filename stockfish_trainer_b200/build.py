"""Build the native library in-tree: ``stockfish_trainer_b200/libnnue_ft.so``.

    python -m stockfish_trainer_b200.build [--force] [--verbose]

One nvcc invocation compiles the CUDA kernels for sm_100a (nnue_ft.cu) and the
host-side position / feature-index code (features.cpp) into a single shared
library with a plain C ABI (include/nnue_ft.h).  ``-fmad=false`` keeps every
fp32 operation a separately rounded IEEE op, which the bit-exact parity with
the reference relies on.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB_NAME = "libnnue_ft.so"
LIB_PATH = os.path.join(PKG, LIB_NAME)

SOURCES = ["nnue_ft.cu", "features.cpp"]
DEPS = SOURCES + ["common.cuh", "ft_forward.cuh", "ft_backward.cuh", "ft_quant.cuh", "ft_epilogue.cuh",
                  "ft_optim.cuh", "ft_encode.cuh", "ft_exchange.cuh", "feature_tables.h", "feature_encode.h"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put CUDA's bin directory on PATH)")


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    deps = [os.path.join(CSRC, d) for d in DEPS] + [os.path.join(INCLUDE, "nnue_ft.h")]
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [
        nvcc(), *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-fmad=false",
        "-Xcompiler", "-fPIC,-O3,-pthread", "-shared",
        "-I", INCLUDE,
        *(os.path.join(CSRC, s) for s in SOURCES),
        "-o", tmp, "-lpthread",
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
