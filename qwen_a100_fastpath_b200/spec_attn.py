"""Split-KV, GQA-packed attention for uniform speculative-verification batches on the B200 (``qf_spec_attn`` in
``libqf_b200``).

Drop-in for ``gqa_packed_spec_attention`` of the reference plugin (plugin/qwen_fastpath/spec_attn.py:139-173): same
arguments, same semantics -- ``num_reqs`` requests x ``Q`` query tokens each (token ``b * Q + qi``), query ``qi`` of
request ``b`` attends the cached keys ``[0, seq_lens[b] - Q + qi]`` of a paged cache, GQA with ``H / num_kv_heads``
query heads per KV head, rows with no key give zeros.  The reference's tuning arguments (``num_splits``,
``min_chunk``, ``block_n``, ``num_warps``, ``num_stages``, ``combine_warps``) are accepted for signature
compatibility; the CUDA kernel derives its split count from the SM count and the batch (one wave of CTAs), its tiles
are fixed.  There is no fallback: a call the kernel cannot take raises.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib
from ._lib import LIB, check

_ws_lock = threading.Lock()
_ws: dict[tuple[int, int], torch.Tensor] = {}


def _workspace(device: torch.device, stream: torch.cuda.Stream, nbytes: int) -> torch.Tensor:
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream.cuda_stream)
    with _ws_lock:
        buf = _ws.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _ws[key] = buf
        return buf


def workspace_status(device=None, stream=None) -> int:
    """Read and clear the sticky device error flag of the attention workspace of ``stream`` (synchronises)."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    stream = torch.cuda.current_stream(device) if stream is None else stream
    buf = _ws.get((device.index, stream.cuda_stream))
    if buf is None:
        return _lib.QF_OK
    st = ctypes.c_int(0)
    check("qf_workspace_status", LIB.qf_workspace_status(buf.data_ptr(), stream.cuda_stream, ctypes.byref(st)))
    return st.value


def supported(num_heads: int, num_kv_heads: int, head_size: int, q_len: int, page_size: int) -> bool:
    """Whether ``qf_spec_attn`` takes this attention layer and batch shape (the host-side checks of the C ABI)."""
    return (num_kv_heads >= 1 and num_heads % num_kv_heads == 0 and head_size in (64, 128, 256) and q_len >= 1
            and q_len * (num_heads // num_kv_heads) <= 64 and page_size >= 16 and page_size % 16 == 0)


def gqa_packed_spec_attention(query, key_cache, value_cache, out, seq_lens, block_table, num_reqs, Q, num_kv_heads,
                              scale, num_splits=64, min_chunk=128, block_n=32, num_warps=4, num_stages=2,
                              combine_warps=2, pdl: bool = True):
    """Causal attention for a uniform decode batch (spec_attn.py:139-146 of the reference).

    ``query`` / ``out``: bf16 ``[>= num_reqs * Q, H, D]`` (unit stride over D); ``key_cache`` / ``value_cache``: bf16
    ``[num_blocks, page, num_kv_heads, D]`` views (strided views such as the reference's ``kv_cache.transpose(1, 2)
    .split(D, -1)`` or vLLM's ``kv_cache.unbind(0)`` are fine); ``seq_lens`` int32 ``[num_reqs]``; ``block_table``
    int32 ``[num_reqs, max_pages]``.  This step's keys and values must already be in the cache.  Returns ``out``.
    """
    del num_splits, min_chunk, block_n, num_warps, num_stages, combine_warps  # the reference's Triton tuning knobs
    H, D = query.shape[1], query.shape[2]
    B = int(num_reqs)
    if B == 0:
        return out
    for name, t in (("query", query), ("key_cache", key_cache), ("value_cache", value_cache), ("out", out)):
        if t.dtype != torch.bfloat16 or not t.is_cuda or t.stride(-1) != 1:
            raise ValueError(f"{name} must be a bf16 CUDA tensor with unit stride over the head dimension")
    if key_cache.shape[2] != num_kv_heads or key_cache.shape[3] != D or value_cache.shape != key_cache.shape:
        raise ValueError("key_cache / value_cache must be [num_blocks, page, num_kv_heads, head_size] like query")
    if seq_lens.dtype != torch.int32 or block_table.dtype != torch.int32:
        raise ValueError("seq_lens and block_table must be int32")
    if block_table.stride(-1) != 1:
        raise ValueError("block_table rows must be contiguous")
    if seq_lens.stride(0) != 1:
        seq_lens = seq_lens.contiguous()
    dev = query.device
    stream = torch.cuda.current_stream(dev)
    nbytes = LIB.qf_spec_attn_workspace_bytes(B, int(Q), H, int(num_kv_heads), D)
    ws = _workspace(dev, stream, nbytes)
    kc, vc = key_cache, value_cache
    rc = LIB.qf_spec_attn(query.data_ptr(), query.stride(0), query.stride(1),
                          kc.data_ptr(), kc.stride(0), kc.stride(1), kc.stride(2),
                          vc.data_ptr(), vc.stride(0), vc.stride(1), vc.stride(2),
                          kc.shape[0], kc.shape[1], block_table.data_ptr(), block_table.stride(0),
                          seq_lens.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1),
                          B, int(Q), H, int(num_kv_heads), D, float(scale), ws.data_ptr(), ws.numel(),
                          _lib.QF_FLAG_PDL if pdl else 0, stream.cuda_stream)
    check("qf_spec_attn", rc)
    return out
