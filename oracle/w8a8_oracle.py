"""CPU oracle for the prefill (M > 16) int8 path (test infrastructure only).

This module is the checker, never the product: only ``tests/`` and ``bench.py``'s CPU legs may import it.

For the rows its small-M kernel does not take, the reference plugin's ``qf_int8_linear`` falls back to vLLM's W8A8
path (plugin/qwen_fastpath/patches.py:99-100)::

    x_q, x_s, _ = ops.scaled_int8_quant(x2.contiguous(), None, None, symmetric=True)
    y = ops.cutlass_scaled_mm(x_q, w_q, scale_a=x_s, scale_b=w_s, out_dtype=x.dtype, bias=bias)

Both functions live in vLLM's compiled extension (vllm==0.31.0 pinned by the reference's server/requirements.lock;
the container has vLLM 0.22, whose compiled kernels cannot run without a GPU), not in the reference source.  This
module restates their published arithmetic:

* ``quantize_tokens`` -- dynamic symmetric per-token int8: ``a = max_k |x[m, k]|`` (fp32 of the bf16 values),
  ``s_x[m] = a / 127``, ``q[m, k] = round_half_even(x[m, k] * (127 / a))`` saturated to [-128, 127]; a zero row
  gives ``q = 0`` (its product is NaN, which the conversion sends to 0) and ``s_x = 0``.  Every step is one IEEE
  fp32 operation.
* ``w8a8_mm`` -- the scaled GEMM epilogue: exact int32 ``acc = sum_k q[m, k] * W[n, k]``, then
  ``t = w_scale[n] * float(acc)`` and ``y = x_scale[m] * t`` in fp32 (with a bias, ``fma(x_scale[m], t, bias[n])``),
  one rounding to bf16.

Parity unpinned against the reference itself: the reference runs this path in vLLM's CUDA kernels, which cannot
run here and ship no test vectors.  The GPU tests compare the CUDA path with this oracle (bit-exact int32
accumulation, identical fp32 scaling) and, where vLLM's compiled ops load on the GPU box, with vLLM's own
``scaled_int8_quant`` and ``cutlass_scaled_mm``.
"""
from __future__ import annotations

import numpy as np

from oracle.w8a16_oracle import bf16_to_f32, f32_to_bf16


def quantize_tokens(x_bits, K: int | None = None):
    """Per-token int8 of bf16 activations ``[M, >= K]``: returns (q int8 [M, K], s_x fp32 [M])."""
    x = np.asarray(x_bits)
    K = x.shape[1] if K is None else K
    xf = bf16_to_f32(x[:, :K])
    a = np.abs(xf).max(axis=1) if K else np.zeros(x.shape[0], np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        inv = np.float32(127.0) / a                       # +inf for a zero row
        prod = (xf * inv[:, None]).astype(np.float32)     # NaN for 0 * inf
    q = np.where(np.isnan(prod), 0.0, np.clip(np.rint(prod), -128, 127)).astype(np.int8)
    sx = (a / np.float32(127.0)).astype(np.float32)
    return q, sx


def int_acc(q, W, cols=None) -> np.ndarray:
    """Exact ``sum_k q[m, k] * W[n, k]`` as int64 (fp64 BLAS: every partial sum stays below 2^53)."""
    Wc = W if cols is None else W[cols]
    acc = q.astype(np.float64) @ Wc.astype(np.float64).T
    return acc.astype(np.int64)


def w8a8_mm(x_bits, W, w_scale, bias_bits=None, cols=None):
    """The prefill path on bf16 activations ``[M, K]`` and int8 ``W [N, K]``: returns bf16 bits ``[M, N]`` (or
    ``[M, len(cols)]`` for the output columns ``cols``)."""
    K = W.shape[1]
    q, sx = quantize_tokens(x_bits, K)
    acc = int_acc(q, W, cols)
    ws = np.asarray(w_scale, np.float32) if cols is None else np.asarray(w_scale, np.float32)[cols]
    t = (acc.astype(np.float32) * ws[None, :]).astype(np.float32)
    if bias_bits is None:
        y = (sx[:, None] * t).astype(np.float32)
    else:
        b = bf16_to_f32(np.asarray(bias_bits) if cols is None else np.asarray(bias_bits)[cols]).astype(np.float64)
        # fma: the fp64 product of two fp32 values is exact; one rounding of the sum (to fp64, then fp32)
        y = (sx[:, None].astype(np.float64) * t.astype(np.float64) + b[None, :]).astype(np.float32)
    return f32_to_bf16(y)
