"""The RMSNorm before qkv / gate_up fused into the W8A16 GEMM (qf_w8a16_gemm_rmsnorm) against the unfused sequence
on the CPU oracle: vLLM's RMSNorm (vllm/ir/ops/layernorm.py, restated in oracle.rms_norm_ref and pinned to vLLM's own
function in tests/test_oracle_golden.py), then the W8A16 GEMM contract, then (gate_up) SiluAndMul.

Bars: the new residual bf16(x + residual) is bit-identical; the GEMM output, whose only difference from the unfused
sequence is the rounding of the normalized activation (the fused kernel rounds bf16(z) * gamma once and scales the
fp32 accumulators by rsqrt(mean z^2 + eps); vLLM rounds z * r and then times gamma), is within the north-star bound
(max abs error <= 2e-2 * max|y|) and within 5e-3 relative in Frobenius norm (1e-2 with the SiLU gate, whose product
silu(g) * u carries the rounding difference of both g and u); also against the library's own unfused pair (the
oracle's normalized activations through qf_w8a16_gemm).
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import w8a16_oracle as orc
from tests.conftest import from_dev_bf16, to_dev_bf16

pytestmark = pytest.mark.gpu


def close(got_bits, ref_bits, frob=5e-3):
    a = orc.bf16_to_f32(got_bits).astype(np.float64)
    b = orc.bf16_to_f32(ref_bits).astype(np.float64)
    assert np.all(np.isfinite(a))
    assert np.abs(a - b).max() <= 2e-2 * np.abs(b).max()
    assert np.linalg.norm(a - b) <= frob * np.linalg.norm(b)


def inputs(M, N, K, seed, with_res=True):
    rs = np.random.RandomState(seed)
    x = orc.f32_to_bf16(rs.standard_normal((M, K)).astype(np.float32) * 3.0)
    res = orc.f32_to_bf16(rs.standard_normal((M, K)).astype(np.float32) * 2.0) if with_res else None
    gamma = orc.f32_to_bf16((rs.random_sample(K) * 1.5 + 0.25).astype(np.float32))
    W = rs.randint(-127, 128, size=(N, K)).astype(np.int8)
    s = (rs.random_sample(N) * 0.009 + 0.001).astype(np.float32)
    return x, res, gamma, W, s


@pytest.mark.parametrize("M,N,K,silu,with_res", [
    (5, 10240, 5120, False, True),     # qkv after input_layernorm
    (5, 34816, 5120, True, True),      # gate_up + SiLU after post_attention_layernorm
    (1, 10240, 5120, False, False),    # first layer: no residual yet
    (16, 10240, 5120, False, True),    # two token tiles (NT = 2, half-depth stages)
    (12, 34816, 5120, True, True),
    (3, 1000, 2048, False, True),      # ragged N
    (8, 4352, 4096, True, True),       # gate_up shard at TP = 8 (data-parallel grid)
])
def test_fused_rmsnorm_gemm(dev, M, N, K, silu, with_res):
    import torch
    from qwen_a100_fastpath_b200.w8a16 import w8a16_mm, w8a16_mm_rmsnorm
    x, res, gamma, W, s = inputs(M, N, K, M * 7 + N, with_res)
    eps = 1e-6
    wt = torch.from_numpy(W).to(dev).t()
    st = torch.from_numpy(s).to(dev)
    y, res_out = w8a16_mm_rmsnorm(to_dev_bf16(x, dev), to_dev_bf16(gamma, dev), eps, wt, st,
                                  residual=to_dev_bf16(res, dev) if with_res else None, silu_mul=silu)
    torch.cuda.synchronize()
    y_ref, res_ref = orc.rmsnorm_w8a16_mm(x, res, gamma, eps, W, s, silu=silu)
    assert np.array_equal(from_dev_bf16(res_out), res_ref)
    close(from_dev_bf16(y), y_ref, frob=1e-2 if silu else 5e-3)
    if not silu:  # against the library's own unfused pair: oracle norm, then the GEMM kernel
        a_ref, _ = orc.rms_norm_ref(x, res, gamma, eps)
        y2 = w8a16_mm(to_dev_bf16(a_ref, dev), wt, st, None, torch.bfloat16)
        torch.cuda.synchronize()
        close(from_dev_bf16(y), from_dev_bf16(y2))


def test_fused_rmsnorm_rejects_bad_arguments(dev):
    import torch
    from qwen_a100_fastpath_b200 import _lib
    from qwen_a100_fastpath_b200.w8a16 import w8a16_mm_rmsnorm
    x, res, gamma, W, s = inputs(2, 256, 512, 3)
    xd, rd = to_dev_bf16(x, dev), to_dev_bf16(res, dev)
    wt, st = torch.from_numpy(W).to(dev).t(), torch.from_numpy(s).to(dev)
    with pytest.raises(_lib.QFError):  # residual_out may not overlap the activations every CTA reads
        w8a16_mm_rmsnorm(xd, to_dev_bf16(gamma, dev), 1e-6, wt, st, residual=rd, residual_out=rd)
    with pytest.raises(ValueError):
        w8a16_mm_rmsnorm(xd[:, :500], to_dev_bf16(gamma[:500], dev), 1e-6, wt[:500], st)  # K % 8 != 0
