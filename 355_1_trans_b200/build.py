"""Build the sm_100a shared library in-tree with nvcc.

    python 355_1_trans_b200/build.py        -> 355_1_trans_b200/_build/libbsgemm_b200.so

The library is one translation unit (csrc/bsgemm.cu) compiled for
``-gencode arch=compute_100a,code=sm_100a`` with the CUDA runtime linked
statically, so the .so has no dependency on the CUDA runtime that torch
bundles; the driver (libcuda) is reached through cudaGetDriverEntryPoint.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_build"
LIB = OUT_DIR / "libbsgemm_b200.so"
INCLUDE = PKG.parent / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources())


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    if not force and not needs_build():
        return LIB
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [
        nvcc(), *ARCH_FLAGS, "-O3", "-std=c++17", "-lineinfo", "-shared",
        "-Xcompiler", "-fPIC,-fvisibility=hidden", "-cudart", "static",
        "--expt-relaxed-constexpr", "-ccbin", shutil.which("g++") or "g++",
        "-I", str(INCLUDE), "-o", str(tmp), str(CSRC / "bsgemm.cu"),
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    if extra:
        cmd[1:1] = extra
    env = dict(os.environ)
    # a compiler wrapper in CC/CXX must not leak into nvcc's host compilation
    env.pop("CC", None)
    env.pop("CXX", None)
    res = subprocess.run(cmd, capture_output=True, text=True, env=env)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed ({res.returncode})")
    if verbose:
        sys.stderr.write(res.stdout + res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
