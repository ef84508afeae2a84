"""Build recipe for the in-tree CUDA library ``libmkx.so`` (sm_100a only).

    python -m reki_megakernel_b200.build             # libmkx.so
    python -m reki_megakernel_b200.build --traced    # libmkx_trace.so (profiling variant)

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
# Profiling variant: the same sources with -DMKX_SUBSTAGE_TRACE (thread 0 of CTAs 0 and 100 stamps
# %globaltimer at numbered points inside each stage); loaded only after _lib.use_traced_build().
TRACE_LIB = PKG / "libmkx_trace.so"
SOURCES = [PKG / "csrc" / "mk_expert.cu", PKG / "csrc" / "mk_prepare.cu", PKG / "csrc" / "mk_mods.cu",
           PKG / "csrc" / "mk_batch.cu", PKG / "csrc" / "mk_copies.cu"]
HEADERS = [PKG / "csrc" / "mkx_device.cuh", PKG / "csrc" / "mkx_tma.cuh", ROOT / "include" / "mkx.h",
           ROOT / "include" / "mkx_prepare.h", ROOT / "include" / "mkx_mods.h", ROOT / "include" / "mkx_batch.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libmkx.so")
    return cand


def stale(lib: Path | None = None) -> bool:
    lib = lib or LIB
    if not lib.exists():
        return True
    t = lib.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False, traced: bool = False) -> Path:
    lib = TRACE_LIB if traced else LIB
    if not force and not stale(lib):
        return lib
    tmp = lib.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           *(["-DMKX_SUBSTAGE_TRACE"] if traced else []),
           "-I", str(ROOT / "include"), "-I", str(PKG / "csrc"), "-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(r.stderr, file=sys.stderr)
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv, traced="--traced" in sys.argv))
