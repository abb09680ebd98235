"""The oracle's RMSNorm (oracle.rms_norm_ref) against vLLM's own implementation in this image
(vllm/ir/ops/layernorm.py: rms_norm and fused_add_rms_norm, run with torch on CPU): bit-identical normalized output
and new residual, with and without a residual.  This pins the reference side of tests/test_gpu_rmsnorm.py."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import w8a16_oracle as orc

pytestmark = pytest.mark.slow


def t(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def bits(tensor):
    return tensor.contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("M,K,with_res", [(5, 5120, True), (1, 5120, False), (16, 2048, True)])
def test_rms_norm_ref_matches_vllm(M, K, with_res):
    layernorm = pytest.importorskip("vllm.ir.ops.layernorm")
    rs = np.random.RandomState(M + K)
    x = orc.f32_to_bf16(rs.standard_normal((M, K)).astype(np.float32) * 3.0)
    res = orc.f32_to_bf16(rs.standard_normal((M, K)).astype(np.float32) * 2.0) if with_res else None
    gamma = orc.f32_to_bf16((rs.random_sample(K) * 1.5 + 0.25).astype(np.float32))
    eps = 1e-6
    a, res_out = orc.rms_norm_ref(x, res, gamma, eps)
    fn_add = getattr(layernorm.fused_add_rms_norm, "impl", layernorm.fused_add_rms_norm)
    fn = getattr(layernorm.rms_norm, "impl", layernorm.rms_norm)
    if with_res:
        out_v, res_v = fn_add(t(x), t(res), t(gamma), eps)
        assert np.array_equal(bits(res_v), res_out)
    else:
        out_v = fn(t(x), t(gamma), eps)
        assert np.array_equal(res_out, x)
    got, ref = orc.bf16_to_f32(a), orc.bf16_to_f32(bits(out_v))
    # fp32 reductions may order the mean's sum differently: allow one bf16 ulp on at most 0.5 % of elements
    ulp = np.spacing(np.maximum(np.abs(got), np.abs(ref))) * 2.0 ** 16
    assert np.all(np.abs(got - ref) <= ulp)
    assert np.mean(a != bits(out_v)) <= 5e-3
