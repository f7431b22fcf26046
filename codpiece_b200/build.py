"""Build libcpq.so (sm_100a) in-tree with nvcc.

The library is one CUDA translation unit (csrc/libcpq.cu) compiled straight
for ``sm_100a``; it links only the CUDA runtime (NCCL is dlopen'ed on first
use). The output lands next to this file so it travels with the repository
snapshot to the GPU box.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libcpq.so"
INCLUDE = PKG.parent / "include"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xptxas", "-v",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: libcpq needs the CUDA toolkit to build")


def _sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.inl"))
                  + [INCLUDE / "cpq.h"])


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile csrc/libcpq.cu into codpiece_b200/libcpq.so (skips when current)."""
    if not force and up_to_date():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", str(INCLUDE), "-o", str(tmp), str(CSRC / "libcpq.cu"), "-lcudart"]
    env = dict(os.environ)
    # nvcc drives the system gcc; a CC/CXX pointing elsewhere is not used here
    env.pop("CC", None)
    env.pop("CXX", None)
    res = subprocess.run(cmd, cwd=str(CSRC), env=env, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed ({res.returncode}) building {LIB.name}")
    if verbose:
        sys.stderr.write(res.stderr)
    (PKG / "ptxas_report.txt").write_text(res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
