"""Build recipe for the oracle's C restatement (test infrastructure only).

    python oracle/build.py          # -> oracle/_build/liboracle_ft.so

The reference path itself cannot be compiled here: it is Python + TileLang
(JIT-compiled on a GPU at first call) and its native code is Rust (no rustc in
this image, and its ``sfbinpack`` dependency is not vendored).  So there is no
``oracle/_ref`` build; the oracle is this C restatement plus the Python one in
``oracle/features.py``.
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "ft_oracle.c")
OUT_DIR = os.path.join(HERE, "_build")
OUT = os.path.join(OUT_DIR, "liboracle_ft.so")


def build(force: bool = False) -> str:
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= os.path.getmtime(SRC):
        return OUT
    os.makedirs(OUT_DIR, exist_ok=True)
    # -ffp-contract=off: no fused multiply-add, so quantisation and the
    # summation order stay exactly IEEE single precision as written.
    cmd = ["gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-shared", "-fPIC",
           SRC, "-o", OUT + ".tmp", "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
