"""ctypes binding of ``libqf_b200.so`` (declarations in include/qf_b200.h).

The library is the only compute path: if it is missing or fails to load, importing this module raises, and
nothing falls back to a CPU or framework implementation.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libqf_b200.so"

QF_OK = 0
QF_ERR_TIMEOUT = -9
QF_DTYPE_BF16 = 0
QF_DTYPE_F32 = 1
QF_MAX_M = 16
QF_MAX_N = 1048576
QF_FLAG_PDL = 1
QF_NOALLOC_MAX_N = 262144
QF_AR_MAX_RANKS = 8
QF_AR_MAX_CHUNKS = 256
QF_IPC_HANDLE_BYTES = 64
ABI_VERSION = 1

# (name, restype, argtypes) -- one entry per function declared in include/qf_b200.h
_c = ctypes
SIGNATURES = [
    ("qf_w8a16_workspace_bytes", _c.c_size_t, [_c.c_int, _c.c_int, _c.c_int]),
    ("qf_w8a16_gemm", _c.c_int,
     [_c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_int64,
      _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_void_p, _c.c_size_t, _c.c_uint, _c.c_void_p]),
    ("qf_w8a16_head", _c.c_int,
     [_c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_void_p, _c.c_int64, _c.c_int,
      _c.c_int, _c.c_int, _c.c_int, _c.c_int64, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_void_p,
      _c.c_size_t, _c.c_uint, _c.c_void_p]),
    ("qf_w8a16_head_sample", _c.c_int,
     [_c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_void_p, _c.c_int64, _c.c_int,
      _c.c_int, _c.c_int, _c.c_int, _c.c_int64, _c.c_float, _c.c_uint64, _c.c_uint64, _c.c_void_p, _c.c_void_p,
      _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_size_t, _c.c_uint, _c.c_void_p]),
    ("qf_w8a16_gemm_noalloc", _c.c_int,
     [_c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_int64,
      _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_uint, _c.c_void_p]),
    ("qf_workspace_status", _c.c_int, [_c.c_void_p, _c.c_void_p, _c.POINTER(_c.c_int)]),
    ("qf_w8a16_noalloc_status", _c.c_int, [_c.c_void_p, _c.POINTER(_c.c_int)]),
    ("qf_w8a16_gemm_silu_mul", _c.c_int,
     [_c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_void_p, _c.c_int64, _c.c_int, _c.c_int,
      _c.c_int, _c.c_void_p, _c.c_size_t, _c.c_uint, _c.c_void_p]),
    ("qf_w8a16_gemm_rmsnorm", _c.c_int,
     [_c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_float, _c.c_void_p, _c.c_int64, _c.c_void_p,
      _c.c_int64, _c.c_void_p, _c.c_void_p, _c.c_int64, _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_void_p,
      _c.c_size_t, _c.c_uint, _c.c_void_p]),
    ("qf_w8a8_workspace_bytes", _c.c_size_t, [_c.c_int, _c.c_int]),
    ("qf_w8a8_gemm", _c.c_int,
     [_c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_int64, _c.c_int,
      _c.c_int, _c.c_int, _c.c_void_p, _c.c_size_t, _c.c_uint, _c.c_void_p]),
    ("qf_spec_attn_workspace_bytes", _c.c_size_t, [_c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_int]),
    ("qf_spec_attn", _c.c_int,
     [_c.c_void_p, _c.c_int64, _c.c_int64, _c.c_void_p, _c.c_int64, _c.c_int64, _c.c_int64, _c.c_void_p, _c.c_int64,
      _c.c_int64, _c.c_int64, _c.c_int, _c.c_int, _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_void_p, _c.c_int64,
      _c.c_int64, _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_float, _c.c_void_p, _c.c_size_t, _c.c_uint,
      _c.c_void_p]),
    ("qf_quantize_rows_int8", _c.c_int,
     [_c.c_void_p, _c.c_int64, _c.c_int, _c.c_int, _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_void_p]),
    ("qf_allreduce_buffer_bytes", _c.c_size_t, [_c.c_int]),
    ("qf_symm_alloc", _c.c_int, [_c.c_size_t, _c.POINTER(_c.c_void_p)]),
    ("qf_symm_free", _c.c_int, [_c.c_void_p]),
    ("qf_ipc_handle", _c.c_int, [_c.c_void_p, _c.c_void_p]),
    ("qf_ipc_open", _c.c_int, [_c.c_void_p, _c.POINTER(_c.c_void_p)]),
    ("qf_ipc_close", _c.c_int, [_c.c_void_p]),
    ("qf_allreduce_bf16", _c.c_int,
     [_c.c_void_p, _c.c_void_p, _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.POINTER(_c.c_void_p), _c.c_uint,
      _c.c_void_p]),
    ("qf_allreduce_status", _c.c_int, [_c.c_void_p, _c.c_void_p, _c.POINTER(_c.c_int)]),
    ("qf_allreduce_set_wait", _c.c_int, [_c.c_void_p, _c.c_uint, _c.c_void_p]),
    ("qf_w8a16_gemm_allreduce", _c.c_int,
     [_c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_void_p, _c.c_int64, _c.c_int, _c.c_int,
      _c.c_int, _c.c_void_p, _c.c_size_t, _c.c_int, _c.c_int, _c.POINTER(_c.c_void_p), _c.c_int, _c.c_uint,
      _c.c_void_p]),
    ("qf_strerror", _c.c_char_p, [_c.c_int]),
    ("qf_last_error_detail", _c.c_char_p, []),
    ("qf_abi_version", _c.c_int, []),
]


class QFError(RuntimeError):
    """A libqf_b200 entry point returned a QF_ERR_* code."""

    def __init__(self, fn: str, code: int):
        self.code = code
        detail = LIB.qf_last_error_detail().decode(errors="replace")
        super().__init__(f"{fn}: {LIB.qf_strerror(code).decode()} ({code}): {detail}")


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH.name} is not built; run `python -m qwen_a100_fastpath_b200.build` "
                          "(nvcc, sm_100a)")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.qf_abi_version() != ABI_VERSION:
        raise ImportError(f"{LIB_PATH.name} ABI {lib.qf_abi_version()} != expected {ABI_VERSION}; rebuild it")
    return lib


LIB = _load()


def check(fn: str, code: int) -> None:
    if code != QF_OK:
        raise QFError(fn, code)


TORCH_OPS_PATH = Path(__file__).resolve().parent / "_qf_torch_ops.so"
_torch_ops_loaded = False


def load_torch_ops():
    """Registers ``torch.ops.qf_b200.int8_linear`` (the PyTorch operator over this C ABI, csrc/qf_torch_ops.cpp);
    raises if it is not built.  Returns the op."""
    global _torch_ops_loaded
    import torch
    if not _torch_ops_loaded:
        if not TORCH_OPS_PATH.exists():
            raise ImportError(f"{TORCH_OPS_PATH.name} is not built; run `python -m qwen_a100_fastpath_b200.build`")
        torch.ops.load_library(str(TORCH_OPS_PATH))
        _torch_ops_loaded = True
    return torch.ops.qf_b200.int8_linear
