"""Build libfp4x.so in-tree with nvcc for sm_100a.

The library is one translation unit (csrc/fp4x_all.cu includes every kernel
file) compiled with ``-gencode arch=compute_100a,code=sm_100a``; the CUDA
runtime is linked statically so the .so does not depend on the runtime version
torch ships.  The driver API (tensor maps) is reached through
cudaGetDriverEntryPoint, so no -lcuda is needed.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent                      # rust-fp4-blackwell_b200/
REPO = ROOT.parent
CSRC = ROOT / "csrc"
INCLUDE = REPO / "include"
LIB = PKG / "libfp4x.so"
HOST = ROOT / "host"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: libfp4x.so cannot be built")


def _sources():
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
                  + list(HOST.glob("*.cpp")) + list(HOST.glob("*.h")))


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    tmp = PKG / f"libfp4x.{os.getpid()}.tmp.so"
    cmd = [nvcc(), *NVCC_FLAGS, "-shared", f"-I{INCLUDE}", f"-I{CSRC}",
           "-o", str(tmp), str(CSRC / "fp4x_all.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(r.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    import sys
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
