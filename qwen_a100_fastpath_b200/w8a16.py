"""Small-M W8A16 GEMM over the int8 weights vLLM's W8A8 linear method already holds -- B200 host side.

Mirrors ``qwen_fastpath.w8a16`` (plugin/qwen_fastpath/w8a16.py) of EurekaZang/qwen-a100-fastpath: the same
``SMALL_M``, ``pick_config(N, K)`` and ``w8a16_mm(x, w_t, w_scale, cfg, out_dtype)`` surface, with the
Triton kernel replaced by the sm_100a CUDA library ``libqf_b200.so`` (C ABI in include/qf_b200.h):

* the weight tensor is read in place: vLLM's ``w_q`` is the checkpoint's int8 ``[N, K]`` row-major viewed as
  ``[K, N]`` with stride ``(1, K)`` (no repacking, no extra weight memory, w8a16.py:7);
* ``y = (x @ w) * scale`` with exact bf16 x int8 products, fp32 accumulation, one rounding to ``out_dtype``
  (w8a16.py:28-38); split-K runs inside one launch (no ``torch.zeros`` + cast, w8a16.py:78-83);
* ``w8a16_head`` adds the fused per-row (max, argmax, logsumexp) of the int8 draft LM head.

All tensors must be CUDA tensors; there is no CPU path.
"""
from __future__ import annotations

import os
import threading

import torch

from . import _lib
from ._lib import LIB, check

SMALL_M = 16  # rows handled by the small-M path (w8a16.py:12); larger M keeps vLLM's int8 tensor-core GEMM

# The reference's ``pick_config`` returns a Triton launch tuple (BLOCK_M, BLOCK_N, BLOCK_K, SPLIT_K, num_warps,
# num_stages) or None.  The B200 library chooses its tile shape, grid and split per call in C++ (pick_tiles in
# csrc/qf_w8a16.cu: 128x256, 64x512 or 32x1024 output rows x k bytes per stage, data-parallel or stream-K over the
# SMs, 10 warps); the tuple below only marks a shape as eligible and keeps the reference's return type.  Its
# entries are BLOCK_M = 16 rows, BLOCK_N = 128 (largest tile height), BLOCK_K = 256, SPLIT_K = 0 ("chosen per
# launch"), 10 warps, 0 (ring depth chosen per tile shape).
B200_CONFIG = (16, 128, 256, 0, 10, 0)
_PDL_DEFAULT = os.environ.get("QF_PDL", "0") == "1"


def pick_config(N: int, K: int):
    """Launch configuration for an ``[N, K]`` weight, or ``None`` if the small-M path cannot take it.

    The reference's ``pick_config`` (w8a16.py:58-68) returns ``None`` unless ``K`` divides its block sizes;
    the B200 kernel handles any ``K >= 1`` (TMA zero-fills the ragged edge), so ``None`` is returned only for
    empty or oversized shapes.
    """
    if N < 1 or K < 1 or N > _lib.QF_MAX_N:
        return None
    return B200_CONFIG


# ----------------------------------------------------------------------------------------------
# workspace: one zero-initialised buffer per (device, stream); calls on a stream are ordered, so they
# can share it.  Kernels leave its counters at zero.
# ----------------------------------------------------------------------------------------------
_ws_lock = threading.Lock()
_ws: dict[tuple[int, int], torch.Tensor] = {}
_MIN_WS = 8 << 20


def workspace(device: torch.device, stream: torch.cuda.Stream, nbytes: int) -> torch.Tensor:
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream.cuda_stream)
    with _ws_lock:
        buf = _ws.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(max(nbytes, _MIN_WS), dtype=torch.uint8, device=device)
            _ws[key] = buf
        return buf


def workspace_status(device=None, stream=None) -> int:
    """Read and clear the sticky device error flag of the current stream's workspace (synchronises)."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    stream = torch.cuda.current_stream(device) if stream is None else stream
    key = (device.index, stream.cuda_stream)
    buf = _ws.get(key)
    if buf is None:
        return _lib.QF_OK
    import ctypes
    st = ctypes.c_int(0)
    check("qf_workspace_status", LIB.qf_workspace_status(buf.data_ptr(), stream.cuda_stream, ctypes.byref(st)))
    return st.value


def _aligned_rows(x: torch.Tensor) -> torch.Tensor:
    """x [M, K] bf16 with unit column stride, 16-byte aligned base and row stride % 8 == 0 (TMA rules)."""
    if x.stride(-1) != 1:
        x = x.contiguous()
    if x.data_ptr() % 16 or (x.shape[0] > 1 and x.stride(0) % 8):
        x = x.clone(memory_format=torch.contiguous_format)
    return x


def _check_weight(w_t: torch.Tensor, K: int) -> int:
    if w_t.dtype != torch.int8 or w_t.dim() != 2:
        raise ValueError("w_t must be int8 [K, N]")
    if K == 0:
        return 16
    if w_t.stride(0) != 1:
        raise ValueError("w_t must be int8 [K, N] with stride (1, ldw) (vLLM's transposed w_q view)")
    ldw = w_t.stride(1) if w_t.shape[1] > 1 else (K + 15) // 16 * 16
    if w_t.data_ptr() % 16 or ldw % 16:
        raise ValueError("w_t must be 16-byte aligned with a row stride that is a multiple of 16 bytes")
    return ldw


def weight_supported(w_t: torch.Tensor) -> bool:
    """True if the int8 weight view satisfies the kernel's layout and alignment rules."""
    if w_t.dtype != torch.int8 or w_t.dim() != 2 or w_t.stride(0) != 1 or not w_t.is_cuda:
        return False
    ldw = w_t.stride(1) if w_t.shape[1] > 1 else 16
    return w_t.data_ptr() % 16 == 0 and ldw % 16 == 0


def w8a16_mm(x: torch.Tensor, w_t: torch.Tensor, w_scale: torch.Tensor, cfg=None, out_dtype=torch.bfloat16,
             bias: torch.Tensor | None = None, out: torch.Tensor | None = None, pdl: bool | None = None):
    """``x [M, K]`` bf16 (any row stride, unit column stride) @ ``w_t [K, N]`` int8 (stride ``(1, K)``), times
    ``w_scale [N]`` fp32 -> ``[M, N]`` in ``out_dtype`` (bf16 or fp32).  Same contract as the reference's
    ``w8a16_mm`` (w8a16.py:71-83).  ``bias`` (bf16 ``[N]``) is added as the reference's ``y + bias``
    (patches.py:96-97): a second bf16 rounding.  ``out`` may supply the output tensor.  ``pdl`` launches with
    programmatic dependent launch (weights must not be written by the previous kernel on the stream).
    """
    if x.dim() != 2:
        raise ValueError("x must be 2-D [M, K]")
    M, K = x.shape
    N = w_t.shape[1]
    if w_t.shape[0] != K:
        raise ValueError(f"shape mismatch: x {tuple(x.shape)} vs w_t {tuple(w_t.shape)}")
    if M > SMALL_M:
        raise ValueError(f"M={M} > {SMALL_M}: the small-M path handles at most {SMALL_M} rows")
    if not (x.is_cuda and w_t.is_cuda and w_scale.is_cuda):
        raise ValueError("libqf_b200 needs CUDA tensors (there is no CPU path)")
    if x.dtype != torch.bfloat16:
        raise ValueError("x must be bfloat16")
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("out_dtype must be torch.bfloat16 or torch.float32")
    scale = w_scale.reshape(-1)
    if scale.numel() != N or scale.dtype != torch.float32:
        raise ValueError("w_scale must hold N fp32 per-channel scales")
    scale = scale.contiguous()
    if bias is not None:
        if bias.numel() != N or bias.dtype != torch.bfloat16:
            raise ValueError("bias must be bf16 [N]")
        bias = bias.reshape(-1).contiguous()
    ldw = _check_weight(w_t, K)
    x = _aligned_rows(x)
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=x.device)
    elif out.shape != (M, N) or out.dtype != out_dtype or out.stride(-1) != 1:
        raise ValueError("out must be [M, N] of out_dtype with unit column stride")
    if M == 0 or N == 0:
        return out
    stream = torch.cuda.current_stream(x.device)
    nbytes = LIB.qf_w8a16_workspace_bytes(M, N, K)
    ws = workspace(x.device, stream, nbytes)
    flags = _lib.QF_FLAG_PDL if (_PDL_DEFAULT if pdl is None else pdl) else 0
    rc = LIB.qf_w8a16_gemm(x.data_ptr(), x.stride(0), w_t.data_ptr(), ldw, scale.data_ptr(),
                           bias.data_ptr() if bias is not None else None, out.data_ptr(), out.stride(0),
                           _lib.QF_DTYPE_F32 if out_dtype == torch.float32 else _lib.QF_DTYPE_BF16,
                           M, N, K, ws.data_ptr(), ws.numel(), flags, stream.cuda_stream)
    check("qf_w8a16_gemm", rc)
    return out


def w8a16_mm_silu_mul(x: torch.Tensor, w_t: torch.Tensor, w_scale: torch.Tensor, out: torch.Tensor | None = None,
                      pdl: bool | None = None) -> torch.Tensor:
    """gate_up projection with vLLM's SiluAndMul fused (``qf_w8a16_gemm_silu_mul``): ``w_t [K, 2I]`` holds the merged
    gate (columns ``[0, I)``) and up (``[I, 2I)``) weights, ``w_scale [2I]``; returns ``[M, I]`` bf16
    ``bf16(bf16(silu(g)) * u)`` with ``g``, ``u`` the bf16 GEMM outputs -- the same as ``F.silu(y[:, :I]) * y[:, I:]``
    on ``y = w8a16_mm(x, w_t, w_scale)``."""
    if x.dim() != 2 or w_t.shape[0] != x.shape[1]:
        raise ValueError("x must be [M, K] matching w_t [K, N]")
    M, K = x.shape
    N = w_t.shape[1]
    if N % 2 or M > SMALL_M or K < 1:
        raise ValueError(f"need an even N, K >= 1 and M <= {SMALL_M}")
    if not (x.is_cuda and w_t.is_cuda and w_scale.is_cuda) or x.dtype != torch.bfloat16:
        raise ValueError("libqf_b200 needs CUDA tensors and bf16 activations (there is no CPU path)")
    scale = w_scale.reshape(-1).contiguous()
    if scale.numel() != N or scale.dtype != torch.float32:
        raise ValueError("w_scale must hold N fp32 per-channel scales")
    ldw = _check_weight(w_t, K)
    x = _aligned_rows(x)
    if out is None:
        out = torch.empty((M, N // 2), dtype=torch.bfloat16, device=x.device)
    elif out.shape != (M, N // 2) or out.dtype != torch.bfloat16 or out.stride(-1) != 1:
        raise ValueError("out must be bf16 [M, N/2] with unit column stride")
    stream = torch.cuda.current_stream(x.device)
    ws = workspace(x.device, stream, LIB.qf_w8a16_workspace_bytes(M, N, K))
    flags = _lib.QF_FLAG_PDL if (_PDL_DEFAULT if pdl is None else pdl) else 0
    rc = LIB.qf_w8a16_gemm_silu_mul(x.data_ptr(), x.stride(0), w_t.data_ptr(), ldw, scale.data_ptr(), out.data_ptr(),
                                    out.stride(0), M, N, K, ws.data_ptr(), ws.numel(), flags, stream.cuda_stream)
    check("qf_w8a16_gemm_silu_mul", rc)
    return out


def w8a16_mm_allreduce(x: torch.Tensor, w_t: torch.Tensor, w_scale: torch.Tensor, comm, out: torch.Tensor | None = None,
                       pdl: bool | None = None) -> torch.Tensor:
    """Row-parallel layer with its all-reduce fused into the GEMM (``qf_w8a16_gemm_allreduce``): this rank holds the
    K-shard ``x [M, K_r]`` / ``w_t [K_r, N]``; the result ``[M, N]`` bf16 is the rank-order fp32 sum of every rank's
    bf16 partial, identical on all ranks (vLLM's RowParallelLinear + all-reduce).  ``comm`` is the
    ``tp.NVLinkAllReduce`` that owns the ranks' symmetric buffers.  Collective: every rank calls it with the same
    shapes."""
    if x.dim() != 2 or w_t.shape[0] != x.shape[1]:
        raise ValueError("x must be [M, K] matching w_t [K, N]")
    M, K = x.shape
    N = w_t.shape[1]
    if M > SMALL_M or K < 1:
        raise ValueError(f"need 1 <= K and M <= {SMALL_M}")
    if not (x.is_cuda and w_t.is_cuda and w_scale.is_cuda) or x.dtype != torch.bfloat16:
        raise ValueError("libqf_b200 needs CUDA tensors and bf16 activations (there is no CPU path)")
    scale = w_scale.reshape(-1).contiguous()
    if scale.numel() != N or scale.dtype != torch.float32:
        raise ValueError("w_scale must hold N fp32 per-channel scales")
    ldw = _check_weight(w_t, K)
    x = _aligned_rows(x)
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    elif out.shape != (M, N) or out.dtype != torch.bfloat16 or out.stride(-1) != 1:
        raise ValueError("out must be bf16 [M, N] with unit column stride")
    stream = torch.cuda.current_stream(x.device)
    ws = workspace(x.device, stream, LIB.qf_w8a16_workspace_bytes(M, N, K))
    flags = _lib.QF_FLAG_PDL if (_PDL_DEFAULT if pdl is None else pdl) else 0
    rc = LIB.qf_w8a16_gemm_allreduce(x.data_ptr(), x.stride(0), w_t.data_ptr(), ldw, scale.data_ptr(), out.data_ptr(),
                                     out.stride(0), M, N, K, ws.data_ptr(), ws.numel(), comm.rank, comm.world,
                                     comm.buffer_list, comm.max_count, flags, stream.cuda_stream)
    check("qf_w8a16_gemm_allreduce", rc)
    return out


def w8a16_head(x: torch.Tensor, w_t: torch.Tensor, w_scale: torch.Tensor, n_valid: int | None = None,
               vocab_offset: int = 0, want_logits: bool = True, pdl: bool | None = None, out=None):
    """Int8 draft LM head: bf16 logits ``[M, N]`` (or ``None``) and per-row statistics over columns
    ``[0, n_valid)`` of those logits: ``(row_max fp32 [M], row_argmax int64 [M] (+ vocab_offset, first index on
    ties), row_lse fp32 [M])``.  Same contraction as ``w8a16_mm``; replaces ``int8_logits`` /
    ``get_top_tokens`` (plugin/qwen_fastpath/patches.py:157-185) without a second pass over the logits.
    ``out`` may supply the four output tensors (logits may be None).
    """
    if x.dim() != 2:
        raise ValueError("hidden states must be 2-D [M, K]")
    M, K = x.shape
    N = w_t.shape[1]
    if w_t.shape[0] != K or M > SMALL_M or M < 1:
        raise ValueError("bad head shapes")
    if not (x.is_cuda and w_t.is_cuda and w_scale.is_cuda) or x.dtype != torch.bfloat16:
        raise ValueError("head needs CUDA tensors and bf16 hidden states")
    n_valid = N if n_valid is None else int(n_valid)
    scale = w_scale.reshape(-1).contiguous()
    if scale.numel() != N or scale.dtype != torch.float32:
        raise ValueError("w_scale must hold N fp32 scales")
    ldw = _check_weight(w_t, K)
    x = _aligned_rows(x)
    dev = x.device
    if out is not None:
        logits, row_max, row_arg, row_lse = out
        if logits is not None and (logits.shape != (M, N) or logits.dtype != torch.bfloat16 or logits.stride(-1) != 1):
            raise ValueError("logits must be bf16 [M, N] with unit column stride")
    else:
        logits = torch.empty((M, N), dtype=torch.bfloat16, device=dev) if want_logits else None
        row_max = torch.empty((M,), dtype=torch.float32, device=dev)
        row_arg = torch.empty((M,), dtype=torch.int64, device=dev)
        row_lse = torch.empty((M,), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    ws = workspace(dev, stream, LIB.qf_w8a16_workspace_bytes(M, N, K))
    flags = _lib.QF_FLAG_PDL if (_PDL_DEFAULT if pdl is None else pdl) else 0
    rc = LIB.qf_w8a16_head(x.data_ptr(), x.stride(0), w_t.data_ptr(), ldw, scale.data_ptr(),
                           logits.data_ptr() if logits is not None else None,
                           logits.stride(0) if logits is not None else N, M, N, K, n_valid,
                           int(vocab_offset), row_max.data_ptr(), row_arg.data_ptr(), row_lse.data_ptr(),
                           ws.data_ptr(), ws.numel(), flags, stream.cuda_stream)
    check("qf_w8a16_head", rc)
    return logits, row_max, row_arg, row_lse


def w8a16_head_sample(x: torch.Tensor, w_t: torch.Tensor, w_scale: torch.Tensor, temperature: float, seed: int,
                      offset: int = 0, n_valid: int | None = None, vocab_offset: int = 0, want_logits: bool = True,
                      pdl: bool | None = None):
    """Int8 draft head with one temperature draw per row, for probabilistic drafting (the reference's draft head
    is greedy only, plugin/qwen_fastpath/patches.py:176-185).  The logits are those of ``w8a16_head``; the
    statistics are of the scaled logits ``s = logits / temperature``; each row also gets a Gumbel-max draw from
    ``softmax(s)`` whose noise is Philox4x32-10 of ``(seed, offset, global column, row)`` (see
    ``qf_w8a16_head_sample`` in ``include/qf_b200.h``), fused into the same pass over the logits.

    Returns ``(logits, row_max, row_argmax, row_lse, sample, sample_score, sample_logit)``; the draft probability
    of ``sample`` is ``exp(sample_logit - row_lse)``.  Vocab shards combine with ``tp.combine_head_samples``.
    """
    if not (temperature > 0.0) or temperature != temperature:
        raise ValueError("temperature must be > 0 (use w8a16_head for greedy drafting)")
    if x.dim() != 2:
        raise ValueError("hidden states must be 2-D [M, K]")
    M, K = x.shape
    N = w_t.shape[1]
    if w_t.shape[0] != K or M > SMALL_M or M < 1:
        raise ValueError("bad head shapes")
    if not (x.is_cuda and w_t.is_cuda and w_scale.is_cuda) or x.dtype != torch.bfloat16:
        raise ValueError("head needs CUDA tensors and bf16 hidden states")
    n_valid = N if n_valid is None else int(n_valid)
    scale = w_scale.reshape(-1).contiguous()
    if scale.numel() != N or scale.dtype != torch.float32:
        raise ValueError("w_scale must hold N fp32 scales")
    ldw = _check_weight(w_t, K)
    x = _aligned_rows(x)
    dev = x.device
    logits = torch.empty((M, N), dtype=torch.bfloat16, device=dev) if want_logits else None
    row_max = torch.empty((M,), dtype=torch.float32, device=dev)
    row_arg = torch.empty((M,), dtype=torch.int64, device=dev)
    row_lse = torch.empty((M,), dtype=torch.float32, device=dev)
    sample = torch.empty((M,), dtype=torch.int64, device=dev)
    score = torch.empty((M,), dtype=torch.float32, device=dev)
    slogit = torch.empty((M,), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    ws = workspace(dev, stream, LIB.qf_w8a16_workspace_bytes(M, N, K))
    flags = _lib.QF_FLAG_PDL if (_PDL_DEFAULT if pdl is None else pdl) else 0
    rc = LIB.qf_w8a16_head_sample(x.data_ptr(), x.stride(0), w_t.data_ptr(), ldw, scale.data_ptr(),
                                  logits.data_ptr() if logits is not None else None,
                                  logits.stride(0) if logits is not None else N, M, N, K, n_valid,
                                  int(vocab_offset), float(1.0 / temperature), int(seed) & (2**64 - 1),
                                  int(offset) & (2**64 - 1), row_max.data_ptr(), row_arg.data_ptr(),
                                  row_lse.data_ptr(), sample.data_ptr(), score.data_ptr(), slogit.data_ptr(),
                                  ws.data_ptr(), ws.numel(), flags, stream.cuda_stream)
    check("qf_w8a16_head_sample", rc)
    return logits, row_max, row_arg, row_lse, sample, score, slogit


# ----------------------------------------------------------------------------------------------
# prefill (M > 16): per-token int8 activations x int8 weights on tcgen05 (qf_w8a8_gemm)
# ----------------------------------------------------------------------------------------------
_pf_ws: dict[tuple[int, int], torch.Tensor] = {}


def _prefill_workspace(device: torch.device, stream: torch.cuda.Stream, nbytes: int) -> torch.Tensor:
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream.cuda_stream)
    with _ws_lock:
        buf = _pf_ws.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _pf_ws[key] = buf
        return buf


def w8a8_mm(x: torch.Tensor, w_t: torch.Tensor, w_scale: torch.Tensor, bias: torch.Tensor | None = None,
            out: torch.Tensor | None = None, pdl: bool | None = None) -> torch.Tensor:
    """``x [M, K]`` bf16 (any M) quantized per token to int8 and multiplied with ``w_t [K, N]`` int8 (stride
    ``(1, ldw)``) on the tensor cores: ``y = bf16(s_x[m] * (w_scale[n] * acc[m, n]) (+ bias))`` -- what the reference's
    ``qf_int8_linear`` gets from vLLM's ``scaled_int8_quant`` + ``cutlass_scaled_mm`` for the rows its small-M
    kernel does not take (plugin/qwen_fastpath/patches.py:99-100)."""
    if x.dim() != 2:
        raise ValueError("x must be 2-D [M, K]")
    M, K = x.shape
    N = w_t.shape[1]
    if w_t.shape[0] != K or K < 1:
        raise ValueError(f"shape mismatch: x {tuple(x.shape)} vs w_t {tuple(w_t.shape)}")
    if not (x.is_cuda and w_t.is_cuda and w_scale.is_cuda) or x.dtype != torch.bfloat16:
        raise ValueError("libqf_b200 needs CUDA tensors and bf16 activations (there is no CPU path)")
    scale = w_scale.reshape(-1)
    if scale.numel() != N or scale.dtype != torch.float32:
        raise ValueError("w_scale must hold N fp32 per-channel scales")
    scale = scale.contiguous()
    if bias is not None:
        if bias.numel() != N or bias.dtype != torch.bfloat16:
            raise ValueError("bias must be bf16 [N]")
        bias = bias.reshape(-1).contiguous()
    ldw = _check_weight(w_t, K)
    if x.stride(-1) != 1:
        x = x.contiguous()
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    elif out.shape != (M, N) or out.dtype != torch.bfloat16 or out.stride(-1) != 1:
        raise ValueError("out must be bf16 [M, N] with unit column stride")
    if M == 0 or N == 0:
        return out
    stream = torch.cuda.current_stream(x.device)
    ws = _prefill_workspace(x.device, stream, LIB.qf_w8a8_workspace_bytes(M, K))
    flags = _lib.QF_FLAG_PDL if (_PDL_DEFAULT if pdl is None else pdl) else 0
    rc = LIB.qf_w8a8_gemm(x.data_ptr(), x.stride(0), w_t.data_ptr(), ldw, scale.data_ptr(),
                          bias.data_ptr() if bias is not None else None, out.data_ptr(), out.stride(0), M, N, K,
                          ws.data_ptr(), ws.numel(), flags, stream.cuda_stream)
    check("qf_w8a8_gemm", rc)
    return out


def prefill_workspace_status(device=None, stream=None) -> int:
    """Read and clear the sticky device error flag of the current stream's prefill workspace (synchronises)."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    stream = torch.cuda.current_stream(device) if stream is None else stream
    buf = _pf_ws.get((device.index, stream.cuda_stream))
    if buf is None:
        return _lib.QF_OK
    import ctypes
    st = ctypes.c_int(0)
    check("qf_workspace_status", LIB.qf_workspace_status(buf.data_ptr(), stream.cuda_stream, ctypes.byref(st)))
    return st.value


def w8a16_mm_rmsnorm(x: torch.Tensor, gamma: torch.Tensor, eps: float, w_t: torch.Tensor, w_scale: torch.Tensor,
                     residual: torch.Tensor | None = None, silu_mul: bool = False,
                     residual_out: torch.Tensor | None = None, want_residual: bool = True, out: torch.Tensor | None = None,
                     pdl: bool | None = None):
    """The RMSNorm before qkv / gate_up fused into the W8A16 GEMM (``qf_w8a16_gemm_rmsnorm``): with
    ``z = x (+ residual)``, returns ``(y, bf16(z))`` where ``y`` is the GEMM of the normalized activations (vLLM's
    ``RMSNorm(x, residual)`` followed by the linear), ``[M, N]`` bf16, or with ``silu_mul`` the gate_up activation
    ``[M, N/2]``.  The activation fed to the contraction is ``bf16(bf16(z) * gamma)`` and each token's accumulators
    are scaled by ``rsqrt(mean(z^2) + eps)``: the same result up to the rounding of the normalized activation."""
    if x.dim() != 2 or w_t.shape[0] != x.shape[1]:
        raise ValueError("x must be [M, K] matching w_t [K, N]")
    M, K = x.shape
    N = w_t.shape[1]
    if M > SMALL_M or K < 8 or K % 8 or K > 8192 or (silu_mul and N % 2):
        raise ValueError(f"need M <= {SMALL_M}, K % 8 == 0, 8 <= K <= 8192 (and an even N with silu_mul)")
    tensors = [x, w_t, w_scale, gamma] + ([residual] if residual is not None else [])
    if not all(t.is_cuda for t in tensors) or x.dtype != torch.bfloat16 or gamma.dtype != torch.bfloat16:
        raise ValueError("libqf_b200 needs CUDA tensors, bf16 activations and a bf16 gamma (there is no CPU path)")
    if residual is not None and (residual.shape != x.shape or residual.dtype != torch.bfloat16):
        raise ValueError("residual must be bf16 [M, K]")
    scale = w_scale.reshape(-1).contiguous()
    if scale.numel() != N or scale.dtype != torch.float32:
        raise ValueError("w_scale must hold N fp32 per-channel scales")
    gamma = gamma.reshape(-1).contiguous()
    if gamma.numel() != K:
        raise ValueError("gamma must hold K values")
    ldw = _check_weight(w_t, K)
    x = _aligned_rows(x)
    if residual is not None:
        residual = _aligned_rows(residual)
    if want_residual and residual_out is None:
        residual_out = torch.empty((M, K), dtype=torch.bfloat16, device=x.device)
    n_out = N // 2 if silu_mul else N
    if out is None:
        out = torch.empty((M, n_out), dtype=torch.bfloat16, device=x.device)
    stream = torch.cuda.current_stream(x.device)
    ws = workspace(x.device, stream, LIB.qf_w8a16_workspace_bytes(M, N, K))
    flags = _lib.QF_FLAG_PDL if (_PDL_DEFAULT if pdl is None else pdl) else 0
    rc = LIB.qf_w8a16_gemm_rmsnorm(
        x.data_ptr(), x.stride(0), residual.data_ptr() if residual is not None else None,
        residual.stride(0) if residual is not None else K, gamma.data_ptr(), float(eps),
        residual_out.data_ptr() if residual_out is not None else None,
        residual_out.stride(0) if residual_out is not None else K, w_t.data_ptr(), ldw, scale.data_ptr(),
        out.data_ptr(), out.stride(0), M, N, K, 1 if silu_mul else 0, ws.data_ptr(), ws.numel(), flags,
        stream.cuda_stream)
    check("qf_w8a16_gemm_rmsnorm", rc)
    return out, residual_out
