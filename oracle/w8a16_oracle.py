"""CPU oracle for the W8A16 decode-GEMM path (test infrastructure only).

This module is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.  The CUDA library in
``qwen_a100_fastpath_b200`` never calls into it and fails loudly when its extension is missing.

It restates, in numpy, the arithmetic of EurekaZang/qwen-a100-fastpath's ``qwen_fastpath`` plugin:

* ``dequant_matmul_f32``  -- the reference's exact-product oracle
  ``F.linear(x.float(), W.float() * ws[:, None])`` chunked over 8192 output rows
  (bench/test_w8a16.py:15; same expression in bench/kernels/linear_kernels.py:91).
* ``w8a16_mm``            -- the kernel's contract (plugin/qwen_fastpath/w8a16.py:15-44, :71-83):
  ``y[m, n] = s[n] * sum_k x[m, k] * W[n, k]`` with exact bf16 x int8 products, fp32 accumulation,
  the per-channel scale applied to the accumulator, then one round to the output dtype.
* ``qf_int8_linear``      -- the op wrapper (plugin/qwen_fastpath/patches.py:84-101): leading dims
  flattened, bias added *after* the bf16 round as a separate bf16 op (two roundings).
* ``quantize_rows``       -- the draft lm_head int8 quantizer (plugin/qwen_fastpath/patches.py:143-147).
* ``top_tokens`` / ``head_stats`` -- ``get_top_tokens`` (patches.py:182-185: padding columns to -inf,
  first-index argmax, + vocab start offset) and the fused per-row (max, argmax, logsumexp) over the
  same bf16 logits.
* ``head_sample``         -- the fused temperature draw for probabilistic drafting (no reference
  counterpart: the reference drafts greedily): Gumbel-max over the scaled bf16 logits with
  Philox4x32-10 noise (``philox4x32_10``, pinned by the generator's published known-answer vectors).

Parity is pinned: ``tests/golden/make_fixtures.py`` ran the reference's own ``w8a16_mm``,
``qf_int8_linear`` and draft-head patches (Triton interpreter, with two interpreter bf16 bugs fixed) and
stored their outputs; ``tests/test_oracle_golden.py`` checks this module against them.

bf16 tensors are carried as ``uint16`` bit patterns (numpy has no bfloat16).
"""
from __future__ import annotations

import numpy as np

CHUNK_ROWS = 8192  # bench/test_w8a16.py:15 chunks the fp32 weight copy over 8192 output rows


# ----------------------------------------------------------------------------------------------
# bf16 helpers (round-to-nearest-even, as torch's float -> bfloat16 conversion)
# ----------------------------------------------------------------------------------------------
def f32_to_bf16(a) -> np.ndarray:
    """fp32 -> bf16 bits (uint16), round to nearest, ties to even; NaN stays NaN."""
    a = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        rounded = rounded.copy()
        rounded[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return rounded


def bf16_to_f32(b) -> np.ndarray:
    """bf16 bits (uint16) -> exact fp32 values."""
    b = np.ascontiguousarray(np.asarray(b, dtype=np.uint16))
    return (b.astype(np.uint32) << 16).view(np.float32)


# ----------------------------------------------------------------------------------------------
# seeded inputs with the distributions the reference benchmarks on
# ----------------------------------------------------------------------------------------------
def make_inputs(seed: int, M: int, N: int, K: int, *, scale_lo: float = 1e-3, scale_hi: float = 1e-2,
                x_row_stride: int | None = None):
    """Seeded (x_bf16_bits [M, ldx], W int8 [N, K], scale fp32 [N]).

    W ~ uniform int in [-127, 127] (bench/test_w8a16.py:10), per-output-channel scale ~ U(scale_lo,
    scale_hi) (bench/test_w8a16.py:11 uses U(1e-3, 1.1e-2); the benchmark configuration uses
    U(1e-3, 1e-2)), x ~ N(0, 1) rounded to bf16 (bench/test_w8a16.py:13).  ``x_row_stride`` > K pads each
    activation row (the reference accepts any row stride, plugin/qwen_fastpath/w8a16.py:72); the pad is
    filled with NaN so that reading it would poison the result.  ``np.random.RandomState`` is used
    because its streams are frozen across numpy versions.
    """
    rs = np.random.RandomState(seed)
    W = rs.randint(-127, 128, size=(N, K)).astype(np.int8)
    s = (rs.random_sample(N) * (scale_hi - scale_lo) + scale_lo).astype(np.float32)
    x = f32_to_bf16(rs.standard_normal((M, K)).astype(np.float32))
    ldx = K if x_row_stride is None else int(x_row_stride)
    if ldx != K:
        xp = np.full((M, ldx), 0x7FC0, dtype=np.uint16)  # bf16 NaN in the pad
        xp[:, :K] = x
        x = xp
    return x, W, s


def make_bias(seed: int, N: int) -> np.ndarray:
    rs = np.random.RandomState(seed)
    return f32_to_bf16(rs.standard_normal(N).astype(np.float32) * 0.5)


# ----------------------------------------------------------------------------------------------
# the contraction
# ----------------------------------------------------------------------------------------------
def dequant_matmul_f32(x_bits, W, s, K: int | None = None) -> np.ndarray:
    """``F.linear(x.float(), W.float() * ws[:, None])`` chunked over 8192 rows (bench/test_w8a16.py:15).

    fp32 arithmetic throughout, as the reference's oracle.  Returns fp32 [M, N].
    """
    K = W.shape[1] if K is None else K
    x = bf16_to_f32(np.asarray(x_bits)[:, :K])
    out = []
    for i in range(0, W.shape[0], CHUNK_ROWS):
        wd = W[i:i + CHUNK_ROWS].astype(np.float32) * s[i:i + CHUNK_ROWS, None]
        out.append(x @ wd.T)
    return np.concatenate(out, axis=1).astype(np.float32) if out else np.zeros((x.shape[0], 0), np.float32)


def dequant_matmul_f64(x_bits, W, s, K: int | None = None) -> np.ndarray:
    """Exact-product reference in fp64: ``s[n] * sum_k x[m,k] W[n,k]`` (the kernel's math, w8a16.py:28-38)."""
    K = W.shape[1] if K is None else K
    x = bf16_to_f32(np.asarray(x_bits)[:, :K]).astype(np.float64)
    out = []
    for i in range(0, W.shape[0], CHUNK_ROWS):
        acc = x @ W[i:i + CHUNK_ROWS].astype(np.float64).T
        out.append(acc * s[i:i + CHUNK_ROWS].astype(np.float64)[None, :])
    return np.concatenate(out, axis=1) if out else np.zeros((x.shape[0], 0), np.float64)


def w8a16_mm(x_bits, W, s, out_dtype: str = "bf16", K: int | None = None) -> np.ndarray:
    """The kernel contract of ``w8a16_mm`` (plugin/qwen_fastpath/w8a16.py:71-83).

    fp32 accumulator (computed here in fp64, then rounded to fp32 -- the closest fp32 a summation can
    give), scale applied to the accumulator (w8a16.py:37-38), one rounding to ``out_dtype``.
    Returns bf16 bits (uint16) or fp32.
    """
    y = dequant_matmul_f64(x_bits, W, s, K).astype(np.float32)
    if out_dtype == "bf16":
        return f32_to_bf16(y)
    if out_dtype == "f32":
        return y
    raise ValueError(out_dtype)


def add_bias_bf16(y_bits, bias_bits) -> np.ndarray:
    """``y + bias`` on bf16 tensors (plugin/qwen_fastpath/patches.py:96-97): fp32 add, one bf16 round."""
    return f32_to_bf16(bf16_to_f32(y_bits) + bf16_to_f32(bias_bits)[None, :])


def qf_int8_linear(x_bits, W, s, bias_bits=None) -> np.ndarray:
    """``qf_int8_linear`` small-M branch (plugin/qwen_fastpath/patches.py:84-98) on a [..., K] input.

    ``x_bits`` may carry leading dims; returns bf16 bits [..., N].
    """
    x_bits = np.asarray(x_bits)
    lead = x_bits.shape[:-1]
    x2 = x_bits.reshape(-1, x_bits.shape[-1])
    y = w8a16_mm(x2, W, s, "bf16")
    if bias_bits is not None:
        y = add_bias_bf16(y, bias_bits)
    return y.reshape(*lead, W.shape[0])


# ----------------------------------------------------------------------------------------------
# draft LM head
# ----------------------------------------------------------------------------------------------
def quantize_rows(weight_bits, block_rows: int = 16384):
    """Per-row symmetric int8 quantizer of the draft lm_head (plugin/qwen_fastpath/patches.py:143-147).

    ``s = max(|w|, 1e-8) / 127`` in fp32, ``q = clamp(round_half_even(w / s), -127, 127)``.
    Returns (int8 [V, H], fp32 [V]).
    """
    w = bf16_to_f32(weight_bits)
    V = w.shape[0]
    q = np.empty(w.shape, dtype=np.int8)
    sc = np.empty((V,), dtype=np.float32)
    for i in range(0, V, block_rows):
        blk = w[i:i + block_rows]
        s = np.maximum(np.abs(blk).max(axis=1), np.float32(1e-8)).astype(np.float32) / np.float32(127.0)
        s = s.astype(np.float32)
        q[i:i + block_rows] = np.clip(np.rint(blk / s[:, None]), -127, 127).astype(np.int8)
        sc[i:i + block_rows] = s
    return q, sc


def silu_mul(y_bits, I: int):
    """vLLM's SiluAndMul on the bf16 gate_up output ``y [M, 2I]`` (vllm/model_executor/layers/activation.py,
    ``SiluAndMul.forward_native``: ``F.silu(x[..., :d]) * x[..., d:]`` on bf16 tensors): ``act = bf16(g / (1 +
    exp(-g)))`` in fp32, ``out = bf16(act * u)``.  Returns bf16 bits ``[M, I]``."""
    y = bf16_to_f32(y_bits)
    g = y[:, :I].astype(np.float32)
    u = y[:, I:2 * I].astype(np.float32)
    with np.errstate(over="ignore"):
        act = f32_to_bf16((g / (np.float32(1.0) + np.exp(-g))).astype(np.float32))
    return f32_to_bf16((bf16_to_f32(act) * u).astype(np.float32))


def top_tokens(logits_bits, num_pad: int, vocab_start: int = 0) -> np.ndarray:
    """``get_top_tokens`` (plugin/qwen_fastpath/patches.py:182-185) on bf16 logits [M, V]."""
    v = bf16_to_f32(logits_bits).astype(np.float64)
    if num_pad > 0:
        v[..., -num_pad:] = -np.inf
    return np.argmax(v, axis=-1).astype(np.int64) + int(vocab_start)


def head_stats(logits_bits, n_valid: int, vocab_offset: int = 0):
    """Per-row (max, argmax, logsumexp) over the first ``n_valid`` bf16 logits of each row.

    max/argmax follow ``torch.argmax`` on the bf16 tensor (first index on ties), with columns
    ``>= n_valid`` masked as ``get_top_tokens`` masks vocab padding (patches.py:182-184); argmax gets
    ``vocab_offset`` added (patches.py:185).  logsumexp (the normaliser probabilistic drafting needs) is
    computed in fp64 over the same bf16 values.  Returns (fp32 [M], int64 [M], fp64 [M]).
    """
    v = bf16_to_f32(logits_bits)[:, :n_valid].astype(np.float64)
    mx = v.max(axis=1)
    am = np.argmax(v, axis=1).astype(np.int64) + int(vocab_offset)
    lse = mx + np.log(np.exp(v - mx[:, None]).sum(axis=1))
    return mx.astype(np.float32), am, lse


_PHILOX_M = (0xD2511F53, 0xCD9E8D57)
_PHILOX_W = (0x9E3779B9, 0xBB67AE85)


def philox4x32_10(ctr, key):
    """Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC 2011).

    ``ctr``: uint32 array [..., 4]; ``key``: two uint32.  Ten rounds of
    ``(c0, c1, c2, c3) -> (hi(M1*c2) ^ c1 ^ k0, lo(M1*c2), hi(M0*c0) ^ c3 ^ k1, lo(M0*c0))`` with the key advanced
    by the Weyl constants between rounds.  Checked against the generator's published known-answer vectors in
    ``tests/test_oracle_golden.py``.  Returns uint32 [..., 4].
    """
    c = np.asarray(ctr, dtype=np.uint64) & np.uint64(0xFFFFFFFF)
    c0, c1, c2, c3 = (c[..., i].copy() for i in range(4))
    k0, k1 = np.uint64(key[0] & 0xFFFFFFFF), np.uint64(key[1] & 0xFFFFFFFF)
    mask = np.uint64(0xFFFFFFFF)
    for r in range(10):
        p0 = np.uint64(_PHILOX_M[0]) * c0
        p1 = np.uint64(_PHILOX_M[1]) * c2
        c0, c1, c2, c3 = ((p1 >> np.uint64(32)) ^ c1 ^ k0) & mask, p1 & mask, \
            ((p0 >> np.uint64(32)) ^ c3 ^ k1) & mask, p0 & mask
        if r < 9:
            k0 = (k0 + np.uint64(_PHILOX_W[0])) & mask
            k1 = (k1 + np.uint64(_PHILOX_W[1])) & mask
    return np.stack([c0, c1, c2, c3], axis=-1).astype(np.uint32)


def gumbel_noise(M: int, cols, seed: int, offset: int) -> np.ndarray:
    """Gumbel noise g[m, j] (fp64) of the fused draft draw for rows m < M and global columns ``cols``: the word
    ``m % 4`` of Philox4x32-10 with counter (column, m // 4, offset low, offset high) and key (seed low, seed high),
    u = ((word >> 9) + 1/2) * 2^-23 (exact in fp32), g = -log(-log u)."""
    cols = np.asarray(cols, dtype=np.uint64)
    q = np.arange((M + 3) // 4, dtype=np.uint64)
    ctr = np.zeros((len(q), len(cols), 4), dtype=np.uint64)
    ctr[..., 0] = cols[None, :]
    ctr[..., 1] = q[:, None]
    ctr[..., 2] = offset & 0xFFFFFFFF
    ctr[..., 3] = (offset >> 32) & 0xFFFFFFFF
    words = philox4x32_10(ctr, (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF))  # [quads, cols, 4]
    words = np.transpose(words, (0, 2, 1)).reshape(-1, len(cols))[:M]             # row m = 4 q + e
    u = ((words >> np.uint32(9)).astype(np.float64) + 0.5) * 2.0 ** -23
    return -np.log(-np.log(u))


def head_sample(logits_bits, n_valid: int, inv_temp: float, seed: int, offset: int, vocab_offset: int = 0):
    """Fused temperature draw of the draft head (``qf_w8a16_head_sample``) on bf16 logits [M, V].

    s = fp32(logit) * fp32(inv_temp) (one fp32 rounding, as the kernel); statistics (max, argmax + offset,
    logsumexp in fp64) of s over columns < n_valid; Gumbel-max draw argmax_j s_j + g[m, j + vocab_offset] (first
    column on ties).  Returns (max fp32, argmax int64, lse fp64, sample int64, score fp64, sample logit fp32,
    margin fp64 = best minus second-best perturbed score, for tolerance decisions)."""
    l = bf16_to_f32(logits_bits)[:, :n_valid]
    sv = (l * np.float32(inv_temp)).astype(np.float32)
    M = sv.shape[0]
    mx = sv.max(axis=1)
    am = np.argmax(sv, axis=1).astype(np.int64) + int(vocab_offset)
    s64 = sv.astype(np.float64)
    lse = s64.max(axis=1) + np.log(np.exp(s64 - s64.max(axis=1, keepdims=True)).sum(axis=1))
    z = s64 + gumbel_noise(M, np.arange(n_valid, dtype=np.int64) + int(vocab_offset), seed, offset)
    smp = np.argmax(z, axis=1)
    zs = np.sort(z, axis=1)
    margin = zs[:, -1] - zs[:, -2] if n_valid > 1 else np.full(M, np.inf)
    return (mx, am, lse, smp.astype(np.int64) + int(vocab_offset), z[np.arange(M), smp],
            sv[np.arange(M), smp], margin)


def combine_head_samples(parts):
    """Merge per-shard draws (score [M], global column [M], logit [M]) of a vocab-sharded head: the largest score
    wins, lowest column on ties -- equal to the unsharded draw because the noise is keyed by the global column."""
    sc = np.stack([np.asarray(p[0], np.float64) for p in parts])
    col = np.stack([np.asarray(p[1], np.int64) for p in parts])
    lg = np.stack([np.asarray(p[2], np.float64) for p in parts])
    best = sc.max(axis=0)
    cand = np.where(sc == best[None, :], col, np.iinfo(np.int64).max)
    pick = cand.min(axis=0)
    which = np.argmax((col == pick[None, :]) & (sc == best[None, :]), axis=0)
    return pick, lg[which, np.arange(sc.shape[1])]


def top2_gap(logits_bits, n_valid: int) -> np.ndarray:
    """Gap between the largest and second-largest bf16 logit per row (0 means a tie in bf16)."""
    v = np.sort(bf16_to_f32(logits_bits)[:, :n_valid].astype(np.float64), axis=1)
    return v[:, -1] - v[:, -2]


# ----------------------------------------------------------------------------------------------
# tensor-parallel restatement (the reference runs TP=1 only; vLLM's row-parallel linear sums the
# per-rank partial outputs, model_executor/layers/linear.py:1556-1559 in the vLLM host)
# ----------------------------------------------------------------------------------------------
def shard_columns(W, s, rank: int, world: int):
    """Column-parallel shard: output rows [rank*N/t, (rank+1)*N/t)."""
    N = W.shape[0]
    assert N % world == 0
    n = N // world
    return W[rank * n:(rank + 1) * n], s[rank * n:(rank + 1) * n]


def shard_rows(W, x_bits, rank: int, world: int):
    """Row-parallel shard: input columns [rank*K/t, (rank+1)*K/t) of W and of x."""
    K = W.shape[1]
    assert K % world == 0
    k = K // world
    return W[:, rank * k:(rank + 1) * k], np.ascontiguousarray(np.asarray(x_bits)[:, rank * k:(rank + 1) * k])


def combine_head_stats(parts):
    """Merge per-shard (max, argmax, lse) of a vocab-sharded head, in rank order.

    Global max/argmax: largest max, lowest global index on ties.  lse = m* + log(sum_r exp(lse_r - m*)).
    ``parts`` is a list of (max [M], argmax [M] (global indices), lse [M]).
    """
    mx = np.stack([np.asarray(p[0], np.float64) for p in parts])
    am = np.stack([np.asarray(p[1], np.int64) for p in parts])
    ls = np.stack([np.asarray(p[2], np.float64) for p in parts])
    best = mx.max(axis=0)
    cand = np.where(mx == best[None, :], am, np.iinfo(np.int64).max)
    arg = cand.min(axis=0)
    m_star = ls.max(axis=0)
    lse = m_star + np.log(np.exp(ls - m_star[None, :]).sum(axis=0))
    return best.astype(np.float32), arg, lse


# ----------------------------------------------------------------------------------------------
# fused RMSNorm before qkv / gate_up (survey row (f)1; vLLM's RMSNorm, not the reference plugin)
# ----------------------------------------------------------------------------------------------
def rms_norm_ref(x_bits, res_bits, gamma_bits, eps: float):
    """vLLM's RMSNorm on bf16 tensors (vllm/ir/ops/layernorm.py, ``rms_norm`` / ``fused_add_rms_norm``):
    ``z = float(x) (+ float(residual))``, new residual ``bf16(z)``, ``r = rsqrt(mean(z^2) + eps)`` in fp32,
    output ``bf16(float(bf16(z * r)) * float(gamma))``.  Returns (normalized bf16 bits [M, K], new residual bits)."""
    z = bf16_to_f32(x_bits).astype(np.float32)
    if res_bits is not None:
        z = (z + bf16_to_f32(res_bits)).astype(np.float32)
    var = (z.astype(np.float64) ** 2).mean(axis=1, keepdims=True).astype(np.float32)
    r = (np.float32(1.0) / np.sqrt((var + np.float32(eps)).astype(np.float32))).astype(np.float32)
    zr = f32_to_bf16((z * r).astype(np.float32))
    out = f32_to_bf16((bf16_to_f32(zr) * bf16_to_f32(gamma_bits)[None, :]).astype(np.float32))
    return out, f32_to_bf16(z)


def rmsnorm_w8a16_mm(x_bits, res_bits, gamma_bits, eps: float, W, s, silu: bool = False):
    """The unfused sequence the fused kernel replaces: vLLM's RMSNorm, then the W8A16 GEMM (``w8a16_mm``) on its bf16
    output, then (``silu``) vLLM's SiluAndMul on the merged gate_up output.  Returns (y bits, new residual bits)."""
    a, res_out = rms_norm_ref(x_bits, res_bits, gamma_bits, eps)
    y = w8a16_mm(a, W, s, "bf16")
    if silu:
        y = silu_mul(y, W.shape[0] // 2)
    return y, res_out
