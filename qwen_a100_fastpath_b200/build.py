"""Build ``libqf_b200.so`` (the C-ABI library) in-tree with nvcc for sm_100a, and the thin PyTorch operator over it.

``python -m qwen_a100_fastpath_b200.build`` (or ``build_library()``) compiles ``csrc/*.cu`` into
``qwen_a100_fastpath_b200/libqf_b200.so`` with the CUDA runtime linked statically, so the library needs no
toolkit at run time and loads on a machine without a GPU (no CUDA call happens at load).  It then compiles
``csrc/qf_torch_ops.cpp`` with the host C++ compiler against the installed PyTorch into ``_qf_torch_ops.so``
(``torch.ops.qf_b200.int8_linear``), linked to ``libqf_b200.so`` next to it.
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
TORCH_OPS = PKG / "_qf_torch_ops.so"
TORCH_OPS_SOURCE = "qf_torch_ops.cpp"
SOURCES = ["qf_w8a16.cu", "qf_allreduce.cu", "qf_quant.cu", "qf_w8a8.cu", "qf_spec_attn.cu"]
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
    if not LIB.exists() or not TORCH_OPS.exists():
        return True
    t = min(LIB.stat().st_mtime, TORCH_OPS.stat().st_mtime)
    return any(p.stat().st_mtime > t for p in _inputs() + [CSRC / TORCH_OPS_SOURCE])


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
    build_torch_ops(verbose=verbose)
    return LIB


def build_torch_ops(verbose: bool = False) -> Path:
    """Compile the PyTorch operator layer (host C++ only, no device code) against the installed torch."""
    import torch
    from torch.utils.cpp_extension import include_paths
    tdir = Path(torch.__file__).resolve().parent
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cxx = os.environ.get("CXX") or shutil.which("g++") or "g++"
    incs = [f"-I{p}" for p in include_paths()] + [f"-I{Path(nvcc_path()).resolve().parent.parent / 'include'}",
                                                   f"-I{INCLUDE}"]
    tmp = TORCH_OPS.with_suffix(".so.tmp")
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}", *incs,
           str(CSRC / TORCH_OPS_SOURCE), "-o", str(tmp), f"-L{PKG}", "-lqf_b200", f"-L{tdir / 'lib'}", "-lc10",
           "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"{cxx} failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, TORCH_OPS)
    return TORCH_OPS


if __name__ == "__main__":
    print(build_library(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas-info" in sys.argv))
