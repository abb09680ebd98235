"""Build ``libqf_b200.so`` (the C-ABI library) in-tree with nvcc for sm_100a.

``python -m qwen_a100_fastpath_b200.build`` (or ``build_library()``) compiles ``csrc/*.cu`` into
``qwen_a100_fastpath_b200/libqf_b200.so`` with the CUDA runtime linked statically, so the library needs no
toolkit at run time and loads on a machine without a GPU (no CUDA call happens at load).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB = PKG / "libqf_b200.so"
SOURCES = ["qf_w8a16.cu", "qf_allreduce.cu", "qf_quant.cu", "qf_w8a8.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists() and not shutil.which(cand):
        raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")
    return cand


def _inputs() -> list[Path]:
    return [CSRC / s for s in SOURCES] + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + \
        sorted(INCLUDE.glob("*.h"))


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _inputs())


def build_library(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           "-cudart", "static", f"-I{INCLUDE}", "-o", str(tmp), *[str(CSRC / s) for s in SOURCES]]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose or ptxas_info:
        print(res.stderr, file=sys.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build_library(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas-info" in sys.argv))
