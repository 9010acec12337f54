"""Build recipes for the checkers (test infrastructure only).

    python oracle/build.py [--force] [--reference DIR]

1. ``oracle/_build/liboracle_ft.so``: the oracle's C restatement
   (``ft_oracle.c``), compiled with gcc.
2. ``oracle/_ref/ref_feature_transformer/``: the reference's own feature
   transformer package (``src/model/modules/feature_transformer/__init__.py``,
   ``functions.py``, ``kernel.py``: ``SparseLinearFunction`` and its TileLang
   kernels) staged UNMODIFIED from a checkout of the reference, byte for byte,
   with a manifest of sha256 sums.  TileLang compiles those kernels at their
   first call on a GPU, so the staged package is the GPU checker of the fp32
   math (``tests/test_gpu_tilelang.py``) and the GPU bar of the bench
   (``oracle/tilelang_timing.py``).  Only tests and the bench's baseline legs
   import it; ``oracle/_ref/`` is git-ignored, so the reference's sources never
   enter this repository's history, but it travels with the working tree.

The reference's Rust crate cannot be built here (no rustc, and its
``sfbinpack`` dependency is not vendored), so the feature-index functions
are checked against the Python restatement in ``oracle/features.py``.
"""

from __future__ import annotations

import hashlib
import json
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "ft_oracle.c")
OUT_DIR = os.path.join(HERE, "_build")
OUT = os.path.join(OUT_DIR, "liboracle_ft.so")

REF_DIR = os.path.join(HERE, "_ref")
REF_PKG = "ref_feature_transformer"
# the reference's feature-transformer package, relative to its checkout root
REF_FT_FILES = ("__init__.py", "functions.py", "kernel.py")
REF_FT_SUBDIR = os.path.join("src", "model", "modules", "feature_transformer")


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


def _sha256(path: str) -> str:
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def stage_reference(reference_root: str) -> str:
    """Copy the reference's feature-transformer package into
    ``oracle/_ref/ref_feature_transformer/`` without changing a byte.

    Returns the staged package directory.  Raises ``FileNotFoundError`` when
    ``reference_root`` does not hold the package."""
    src_dir = os.path.join(reference_root, REF_FT_SUBDIR)
    for name in REF_FT_FILES:
        if not os.path.isfile(os.path.join(src_dir, name)):
            raise FileNotFoundError(f"{os.path.join(src_dir, name)} not found")
    dst = os.path.join(REF_DIR, REF_PKG)
    tmp = dst + ".tmp"
    if os.path.isdir(tmp):
        shutil.rmtree(tmp)
    os.makedirs(tmp)
    manifest = {"source": REF_FT_SUBDIR, "files": {}}
    for name in REF_FT_FILES:
        shutil.copyfile(os.path.join(src_dir, name), os.path.join(tmp, name))
        manifest["files"][name] = _sha256(os.path.join(tmp, name))
    with open(os.path.join(tmp, "MANIFEST.json"), "w") as f:
        json.dump(manifest, f, indent=1)
    if os.path.isdir(dst):
        shutil.rmtree(dst)
    os.replace(tmp, dst)
    return dst


def staged_reference() -> str | None:
    """The staged package directory if it is present and unmodified, else None."""
    dst = os.path.join(REF_DIR, REF_PKG)
    try:
        with open(os.path.join(dst, "MANIFEST.json")) as f:
            manifest = json.load(f)
        for name, digest in manifest["files"].items():
            if _sha256(os.path.join(dst, name)) != digest:
                return None
    except (OSError, ValueError, KeyError):
        return None
    return dst


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
    if "--reference" in sys.argv:
        print(stage_reference(sys.argv[sys.argv.index("--reference") + 1]))
