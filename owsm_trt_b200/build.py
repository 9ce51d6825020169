"""Build ``libowsmdec.so`` in-tree with nvcc for sm_100a (``python -m owsm_trt_b200.build``).

Each ``csrc/*.cu`` translation unit is compiled to an object file in parallel (``_build/``), then linked."""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
LIB = PKG / "libowsmdec.so"
OBJ = PKG / "_build"
SOURCES = [PKG / "csrc" / "decoder.cu", PKG / "csrc" / "xkv.cu"]
HEADERS = sorted((PKG / "csrc").glob("*.cuh")) + [ROOT / "include" / "owsm_dec.h"]
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


def _compile(src: Path, verbose: bool) -> tuple[Path, subprocess.CompletedProcess]:
    obj = OBJ / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-c",
           "-I", str(ROOT / "include"), "-o", str(obj), str(src)]  # fmt: skip
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    return obj, subprocess.run(cmd, capture_output=True, text=True)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the shared library if a source is newer than it; returns its path."""
    if not force and not stale():
        return LIB
    OBJ.mkdir(exist_ok=True)
    with ThreadPoolExecutor(len(SOURCES)) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), SOURCES))
    for obj, res in results:
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {obj.stem}.cu:\n{res.stderr}")
        if verbose:
            sys.stderr.write(res.stderr)
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB) + ".tmp", *(str(o) for o, _ in results)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{res.stderr}")
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
