"""Builds libtthrml_b200.so in-tree from csrc/*.cu with nvcc for sm_100a.

Run as ``python -m tt_thrml_b200.build``.  Objects go to ``_build/`` at the
repository root; the shared library lands next to this file so it travels with
the package.  Rebuilds only what changed (source or header newer than object).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = REPO_DIR / "_build" / "tthrml"
LIB_PATH = PKG_DIR / "libtthrml_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-Wall",
    "--expt-relaxed-constexpr",
    f"-I{REPO_DIR / 'include'}",
]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists() and shutil.which(cand) is None:
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libtthrml_b200.so")
    return cand


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((REPO_DIR / "include").glob("*.h"))


def build(verbose: bool = False, force: bool = False) -> Path:
    nvcc = _nvcc()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    objects = []
    for src in sources:
        obj = BUILD_DIR / (src.stem + ".o")
        objects.append(obj)
        if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, newest_header):
            continue
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    newest_obj = max(o.stat().st_mtime for o in objects)
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < newest_obj:
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objects)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    out = build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(out)
