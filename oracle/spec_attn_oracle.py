"""CPU oracle for the speculative-verification attention (test infrastructure only).

This module is the checker, never the product: only ``tests/`` and ``bench.py``'s CPU legs may import it.

The reference's ``gqa_packed_spec_attention`` (plugin/qwen_fastpath/spec_attn.py:139-173) computes, for a uniform
batch of ``num_reqs`` requests x ``Q`` query tokens (token ``b * Q + qi``), "the same semantics as FA2 varlen causal
with seqused_k=seq_lens and the block table" (:141-146): query ``qi`` of request ``b`` attends the cached keys
``[0, seq_lens[b] - Q + qi]``, key ``pos`` living in page ``block_table[b, pos // page]`` at slot ``pos % page``, KV
head ``h // G`` for query head ``h`` (G = H / HKV), softmax of ``scale * q . k``; a row with no key at all gives zeros
(:129-130, ``l > 0 ? l : 1`` with a zero accumulator).  The reference evaluates it as a split prefix (:17-67) plus a
causal suffix merged by log-sum-exp (:70-136); both are exact rewritings of the definition restated here,
``attention``, in float64.

Pinned: ``tests/golden/spec_attn_reference.npz`` holds outputs of the reference's own two Triton kernels, run by
``tests/golden/make_spec_attn_fixtures.py`` under Triton's CPU interpreter on bf16-valued inputs held in fp32 (the
interpreter mishandles bf16 tensors), over empty prefixes, a request shorter than Q, several requests of different
lengths, shuffled pages and several splits; ``tests/test_oracle_spec_attn.py`` checks ``attention`` against them.
"""
from __future__ import annotations

import numpy as np

from oracle.w8a16_oracle import bf16_to_f32


def gather_kv(cache, block_table_row, n: int):
    """Keys (or values) of positions 0 .. n-1 of one request: ``cache[page, slot]`` -> ``[n, HKV, D]``."""
    pos = np.arange(n)
    page = cache.shape[1]
    return cache[np.asarray(block_table_row)[pos // page], pos % page]


def attention(q, k_cache, v_cache, block_table, seq_lens, num_reqs: int, Q: int, num_kv_heads: int, scale: float):
    """The definition in float64.  ``q`` ``[num_reqs * Q, H, D]``; ``k_cache`` / ``v_cache``
    ``[num_blocks, page, HKV, D]`` (float arrays, or uint16 bf16 bit patterns); returns float64 ``[num_reqs * Q, H, D]``.
    """
    def f64(a):
        a = np.asarray(a)
        return (bf16_to_f32(a) if a.dtype == np.uint16 else a).astype(np.float64)

    qf = f64(q)
    H, D = qf.shape[1], qf.shape[2]
    G = H // num_kv_heads
    out = np.zeros((num_reqs * Q, H, D), np.float64)
    for b in range(num_reqs):
        L = max(int(seq_lens[b]), 0)
        K = f64(gather_kv(k_cache, block_table[b], L))  # [L, HKV, D]
        V = f64(gather_kv(v_cache, block_table[b], L))
        for qi in range(Q):
            n = min(L - Q + qi + 1, L)  # keys 0 .. seq_len - Q + qi
            if n <= 0:
                continue
            for h in range(H):
                s = K[:n, h // G] @ qf[b * Q + qi, h] * scale
                p = np.exp(s - s.max())
                out[b * Q + qi, h] = (p / p.sum()) @ V[:n, h // G]
    return out


def make_case(seed: int, num_reqs: int, Q: int, H: int, HKV: int, D: int, page: int, lens, spare_pages: int = 1):
    """Seeded inputs of one case, as bf16 bit patterns: q [B*Q, H, D], kv [num_blocks, HKV, page, 2D] (the reference
    test's cache layout, bench/test_spec_attn.py:13-14: K = kv[..., :D], V = kv[..., D:] after transpose(1, 2)),
    shuffled block table [B, max_pages] int32, seq_lens [B] int32."""
    from oracle.w8a16_oracle import f32_to_bf16
    rs = np.random.RandomState(seed)
    max_pages = max((max(lens) + page - 1) // page, 1)
    nblk = num_reqs * max_pages + spare_pages
    kv = f32_to_bf16(rs.standard_normal((nblk, HKV, page, 2 * D)).astype(np.float32))
    q = f32_to_bf16(rs.standard_normal((num_reqs * Q, H, D)).astype(np.float32))
    bt = rs.permutation(nblk)[: num_reqs * max_pages].astype(np.int32).reshape(num_reqs, max_pages)
    return q, kv, bt, np.asarray(lens, np.int32)


def split_kv(kv):
    """``kv [num_blocks, HKV, page, 2D]`` -> (K, V) views ``[num_blocks, page, HKV, D]`` (transpose(1, 2).split(D))."""
    D = kv.shape[-1] // 2
    t = np.swapaxes(kv, 1, 2)
    return t[..., :D], t[..., D:]
