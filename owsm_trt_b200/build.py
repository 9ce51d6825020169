"""Build ``libowsmdec.so`` in-tree with nvcc for sm_100a (``python -m owsm_trt_b200.build``)."""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
LIB = PKG / "libowsmdec.so"
SOURCES = [PKG / "csrc" / "decoder.cu"]
HEADERS = [PKG / "csrc" / "ptx.cuh", PKG / "csrc" / "cluster.cuh", ROOT / "include" / "owsm_dec.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found (CUDA 12.9 toolkit expected)")
    return path


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the shared library if a source is newer than it; returns its path."""
    if not force and not stale():
        return LIB
    cmd = [nvcc(), *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-shared",
           "-I", str(ROOT / "include"), "-o", str(LIB) + ".tmp", *map(str, SOURCES)]  # fmt: skip
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{res.stderr}")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
