"""Build librxla_b200.so in-tree with nvcc for sm_100a.

    python -m rxla_b200.build            # or rxla_b200.build.build()

The library is one translation unit (csrc/librxla_b200.cu) compiled with
`-gencode arch=compute_100a,code=sm_100a`; the CUDA runtime is linked
statically, so the .so needs only the driver on the GPU box.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "librxla_b200.so"
INCLUDE = PKG.parent / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "rxla_b200.h"]


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(s.stat().st_mtime <= t for s in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
           "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared", "-I", str(INCLUDE),
           "-Xptxas", "-v" if verbose else "-O3",
           "-o", str(tmp), str(CSRC / "librxla_b200.cu"), "-ldl", "-lpthread"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed for librxla_b200")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
