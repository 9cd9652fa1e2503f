"""Build libgdn_b200.so (the sm_100a CUDA kernels + C ABI) in-tree with nvcc.

The library is one translation unit (csrc/gdn_b200.cu) compiled for
sm_100a only; it is written next to this file so that it travels with the
source tree and is the exact binary the Python mirror loads.

`build(debug=True)` writes libgdn_b200_debug.so instead: the same kernels
compiled with -DGDN_DEBUG_CHECKS, whose device-side index checks record
device status 4 on a violation instead of trapping (select it with the
environment variable GDN_B200_LIBRARY).
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
LIB = HERE / "libgdn_b200.so"
LIB_DEBUG = HERE / "libgdn_b200_debug.so"
INCLUDE = HERE.parent / "include"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: cannot build libgdn_b200.so")


def sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def is_stale(lib: Path = LIB) -> bool:
    if not lib.exists():
        return True
    mtime = lib.stat().st_mtime
    return any(p.stat().st_mtime > mtime for p in sources())


def build(force: bool = False, verbose: bool = False, debug: bool = False) -> Path:
    lib = LIB_DEBUG if debug else LIB
    if not force and not is_stale(lib):
        return lib
    tmp = lib.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [_nvcc(), *NVCC_FLAGS, *(["-DGDN_DEBUG_CHECKS"] if debug else []), "-I", str(INCLUDE),
           "-o", str(tmp), str(CSRC / "gdn_b200.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        print(res.stderr)
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    import sys

    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv, debug="--debug" in sys.argv))
