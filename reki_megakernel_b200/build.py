"""Build recipe for the in-tree CUDA library ``libmkx.so`` (sm_100a only).

    python -m reki_megakernel_b200.build

nvcc cross-compiles without a GPU; the library lands next to this file so it travels with the
source tree and is the one ``reki_megakernel_b200._lib`` loads.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
LIB = PKG / "libmkx.so"
SOURCES = [PKG / "csrc" / "mk_expert.cu", PKG / "csrc" / "mk_prepare.cu", PKG / "csrc" / "mk_mods.cu"]
HEADERS = [PKG / "csrc" / "mkx_device.cuh", ROOT / "include" / "mkx.h", ROOT / "include" / "mkx_prepare.h",
           ROOT / "include" / "mkx_mods.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libmkx.so")
    return cand


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    tmp = LIB.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           "-I", str(ROOT / "include"), "-I", str(PKG / "csrc"), "-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(r.stderr, file=sys.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
