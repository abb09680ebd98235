"""The drop-in surface on the GPU: the ``qf_int8_linear`` op body (plugin/qwen_fastpath/patches.py:84-101 of the
reference) and the patched draft-head hooks ``compute_logits`` / ``get_top_tokens`` (patches.py:157-185), run with
CUDA tensors and checked against the oracle.

Covered: 3-D ``[B, T, K]`` input flattened to rows, a bias rounded like the reference's ``y + bias``, activation rows
with a stride, M = 1, 5 and 16 on the BASELINE config-2 shapes, and the gate: M = 17 rows take the prefill kernel,
fp16 activations and a weight view the tensor maps cannot take go to vLLM's W8A8 path (replaced here by a sentinel,
so the routing is checked without vLLM's compiled kernels).  The hooks are driven with a fake drafter on the GPU:
vocab padding, a nonzero ``org_vocab_start_index``, the ``org_vocab_size`` slice, and the fallbacks to the original
methods.  Tolerances as the GEMM tests (one bf16 ulp plus 2^-16 max|y|, at most 1 % of outputs differing; with a bias, plus one ulp of the pre-bias
value); argmax exact.
"""
from __future__ import annotations

import types

import numpy as np
import pytest

from oracle import w8a16_oracle as orc
from tests.conftest import from_dev_bf16, to_dev_bf16
from tests.test_gpu_gemm import bf16_close, bias_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def op():
    from qwen_a100_fastpath_b200.patches import make_int8_linear_op
    return make_int8_linear_op()[0]


@pytest.fixture()
def fallback(monkeypatch):
    """Replace vLLM's W8A8 fallback by a sentinel that records its calls and returns zeros of the right shape."""
    from qwen_a100_fastpath_b200 import patches
    calls = []

    def sentinel(x2, w_q, w_s, bias, out_dtype):
        calls.append((tuple(x2.shape), x2.dtype, out_dtype))
        return x2.new_zeros((x2.shape[0], w_q.shape[1]), dtype=out_dtype)

    monkeypatch.setattr(patches, "w8a8_fallback", sentinel)
    return calls


_WEIGHTS = {}


def weights(dev, N, K, seed):
    """Seeded 16-row activations and an int8 weight in vLLM's layout, cached per (N, K, seed)."""
    import torch
    key = (N, K, seed)
    if key not in _WEIGHTS:
        _WEIGHTS.clear()
        x_bits, W, s = orc.make_inputs(seed, 16, N, K)
        w_q = torch.from_numpy(W).to(dev).t()             # vLLM's w_q: [K, N] view with stride (1, K)
        w_s = torch.from_numpy(s).to(dev).reshape(N, 1)   # vLLM's w_s: fp32 [N, 1]
        _WEIGHTS[key] = (x_bits, W, s, w_q, w_s)
    return _WEIGHTS[key]


@pytest.mark.parametrize("name,N,K", [("qkv", 10240, 5120), ("o_proj", 5120, 8192), ("gate_up", 34816, 5120),
                                      ("down", 5120, 17408)])
@pytest.mark.parametrize("M", [1, 5, 16])
def test_op_config2_shapes(dev, op, fallback, name, N, K, M):
    import torch
    x_bits, W, s, w_q, w_s = weights(dev, N, K, N + K)
    y = op(to_dev_bf16(x_bits[:M], dev), w_q, w_s, None)
    torch.cuda.synchronize()
    assert not fallback and y.shape == (M, N) and y.dtype == torch.bfloat16
    bf16_close(from_dev_bf16(y), orc.qf_int8_linear(x_bits[:M], W, s))


def test_op_3d_input_with_bias(dev, op, fallback):
    import torch
    N, K = 10240, 5120
    x_bits, W, s, w_q, w_s = weights(dev, N, K, 21)
    b_bits = orc.make_bias(22, N)
    x3 = to_dev_bf16(x_bits[:6], dev).view(2, 3, K)       # [B, T, K]: six decode rows
    y = op(x3, w_q, w_s, to_dev_bf16(b_bits, dev))
    torch.cuda.synchronize()
    assert not fallback and y.shape == (2, 3, N)
    bias_close(from_dev_bf16(y).reshape(6, N), x_bits[:6], W, s, b_bits)


def test_op_strided_rows(dev, op, fallback):
    """Activation rows taken out of a wider buffer (row stride 5184 elements, unit column stride), and rows with a
    non-unit column stride, which are made contiguous first (patches.py:93-94 of the reference)."""
    import torch
    N, K = 5120, 5120
    x_bits, W, s, w_q, w_s = weights(dev, N, K, 23)
    wide = torch.zeros((5, K + 64), dtype=torch.bfloat16, device=dev)
    wide[:, :K] = to_dev_bf16(x_bits[:5], dev)
    y = op(wide[:, :K], w_q, w_s, None)
    torch.cuda.synchronize()
    assert not fallback
    bf16_close(from_dev_bf16(y), orc.qf_int8_linear(x_bits[:5], W, s))
    xt = to_dev_bf16(x_bits[:3], dev).t().contiguous().t()
    assert xt.stride(-1) != 1
    y2 = op(xt, w_q, w_s, None)
    torch.cuda.synchronize()
    bf16_close(from_dev_bf16(y2), orc.qf_int8_linear(x_bits[:3], W, s))


def test_op_gate(dev, op, fallback):
    """M = 17 bf16 rows take the prefill kernel; fp16 activations and a weight the tensor maps cannot take go to
    vLLM's W8A8 path; eligible small-M calls stay on the decode kernel."""
    import torch
    from oracle import w8a8_oracle as pre
    N, K = 1024, 512
    x_bits, W, s, w_q, w_s = weights(dev, N, K, 24)
    x17_bits = orc.make_inputs(25, 17, 8, K)[0]
    y17 = op(to_dev_bf16(x17_bits, dev), w_q, w_s, None)              # M > SMALL_M: the prefill kernel
    torch.cuda.synchronize()
    assert not fallback
    assert np.array_equal(from_dev_bf16(y17), pre.w8a8_mm(x17_bits, W, s))
    x16 = to_dev_bf16(x_bits, dev)
    assert op(x16.half(), w_q, w_s, None).dtype == torch.float16      # fp16 activations
    raw = torch.zeros(N * K + 8, dtype=torch.int8, device=dev)
    w_mis = raw[8:].view(N, K).t()                                    # base 8 bytes off a 16-byte boundary
    assert w_mis.stride(0) == 1 and w_mis.data_ptr() % 16 != 0
    op(x16[:4], w_mis, w_s, None)
    op(to_dev_bf16(x17_bits, dev), w_mis, w_s, None)                  # also above 16 rows
    assert [c[0] for c in fallback] == [(16, K), (4, K), (17, K)]
    assert fallback[0][2] == torch.float16
    y = op(x16[:4], w_q, w_s, None)                                   # and the eligible call stays on the kernel
    torch.cuda.synchronize()
    assert len(fallback) == 3
    bf16_close(from_dev_bf16(y), orc.qf_int8_linear(x_bits[:4], W, s))


# ---------------------------------------------------------------------------------------------------- draft head
def fake_drafter(dev, V, H, pad, start, seed):
    """A ``Qwen3_5MTP``-like drafter on the GPU whose lm_head was quantized by ``attach_int8_head``."""
    import torch
    from qwen_a100_fastpath_b200 import patches
    rs = np.random.RandomState(seed)
    wb = orc.f32_to_bf16(rs.standard_normal((V, H)).astype(np.float32) * 0.05)
    weight = torch.from_numpy(wb.view(np.int16)).view(torch.bfloat16).to(dev)
    lm_head = types.SimpleNamespace(weight=weight, tp_size=1,
                                    shard_indices=types.SimpleNamespace(num_org_vocab_padding=pad,
                                                                        org_vocab_start_index=start))
    lp = types.SimpleNamespace(logits_as_input=False, soft_cap=None, scale=1.0, org_vocab_size=V - pad)
    m = types.SimpleNamespace(lm_head=lm_head, logits_processor=lp)
    assert patches.attach_int8_head(m)
    q, sc = orc.quantize_rows(wb)
    return m, q, sc


@pytest.mark.parametrize("V,H,M,pad,start", [(4160, 1024, 4, 64, 0), (2112, 512, 3, 40, 1000), (1088, 256, 16, 0, 7)])
def test_draft_hooks(dev, V, H, M, pad, start):
    import torch
    from qwen_a100_fastpath_b200 import patches
    m, q, sc = fake_drafter(dev, V, H, pad, start, V + M)
    x_bits = orc.make_inputs(V + H, M, 8, H)[0]
    h = to_dev_bf16(x_bits, dev)

    def never(*a, **k):
        pytest.fail("original method called although the int8 head applies")

    logits = patches.draft_compute_logits(m, h, 0, never)
    top = patches.draft_get_top_tokens(m, h, never, never)
    torch.cuda.synchronize()
    ref = orc.w8a16_mm(x_bits, q, sc, "bf16")                          # the int8 head's logits [M, V]
    assert logits.shape == (M, V - pad)                                # cut to org_vocab_size
    bf16_close(from_dev_bf16(logits), ref[:, : V - pad])
    want = orc.top_tokens(from_dev_bf16(patches.int8_head(m, h)[0]), pad, start)
    assert np.array_equal(top.cpu().numpy(), want)                     # get_top_tokens semantics on its logits
    ok = orc.top2_gap(ref, V - pad) > 0
    assert np.array_equal(top.cpu().numpy()[ok], orc.top_tokens(ref, pad, start)[ok])


def test_draft_hooks_fall_back(dev):
    import torch
    from qwen_a100_fastpath_b200 import patches
    m, _, _ = fake_drafter(dev, 1088, 256, 0, 0, 5)
    h = torch.randn(2, 256, device=dev).to(torch.bfloat16)
    m.logits_processor.soft_cap = 30.0                                 # soft-capped logits: the original path
    seen = []

    def orig_logits(model, hs, idx=0):
        seen.append("logits")
        out = torch.zeros((hs.shape[0], 1088), device=dev)
        out[:, 1000] = 1.0
        return out

    assert patches.draft_compute_logits(m, h, 0, orig_logits).shape == (2, 1088)
    assert patches.draft_get_top_tokens(m, h, orig_logits, lambda model, hs: torch.full((2,), 3)).tolist() == [3, 3]
    assert patches.draft_get_top_tokens(m, h, orig_logits, None).tolist() == [1000, 1000]
    assert seen == ["logits", "logits"]
