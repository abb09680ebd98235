"""CUDA int8 draft LM head: bf16 logits + fused per-row (max, argmax, logsumexp) against the oracle."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import w8a16_oracle as orc
from tests.conftest import from_dev_bf16, to_dev_bf16

pytestmark = pytest.mark.gpu


def head(dev, x_bits, W, s, n_valid, offset, want_logits=True):
    import torch
    from qwen_a100_fastpath_b200.w8a16 import w8a16_head
    xt = to_dev_bf16(x_bits, dev)
    wt = torch.from_numpy(W).to(dev).t()
    st = torch.from_numpy(s).to(dev)
    out = w8a16_head(xt, wt, st, n_valid=n_valid, vocab_offset=offset, want_logits=want_logits)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("V,H,M,pad,offset", [(1000, 256, 1, 0, 0), (4100, 512, 4, 36, 0), (3000, 1024, 3, 0, 12345),
                                              (16384 + 640, 256, 16, 64, 0), (130, 128, 8, 2, 7)])
def test_head_matches_oracle(dev, V, H, M, pad, offset):
    x, W, s = orc.make_inputs(V + H + M, M, V, H)
    logits, mx, am, lse = head(dev, x, W, s, V - pad, offset)
    lg = from_dev_bf16(logits)
    ref = orc.w8a16_mm(x, W, s, "bf16")
    frac = np.mean(lg != ref)
    assert frac < 0.01
    # statistics are over the kernel's own bf16 logits: exact against numpy on them
    mx_own, am_own, lse_own = orc.head_stats(lg, V - pad, offset)
    assert np.array_equal(mx.cpu().numpy(), mx_own)
    assert np.array_equal(am.cpu().numpy(), am_own)
    np.testing.assert_allclose(lse.cpu().numpy(), lse_own, rtol=2e-6)
    # and against the oracle's logits wherever the oracle's top-2 gap exceeds rounding noise
    mx_r, am_r, lse_r = orc.head_stats(ref, V - pad, offset)
    gap = orc.top2_gap(ref, V - pad)
    ok = gap > 0
    assert np.array_equal(am.cpu().numpy()[ok], am_r[ok])
    np.testing.assert_allclose(lse.cpu().numpy(), lse_r, rtol=1e-5)


def test_head_first_index_on_ties_and_padding(dev):
    V, H, M = 2048, 256, 2
    x, W, s = orc.make_inputs(5, M, V, H)
    xf = orc.bf16_to_f32(x)
    s[:] = np.float32(0.005)
    hot = np.where(xf[0] >= 0, 127, -127).astype(np.int8)
    for r in (700, 1500, 2040):        # identical top rows: first index wins; 2040 lies in the padding
        W[r] = hot
    logits, mx, am, lse = head(dev, x, W, s, n_valid=2000, offset=100)
    assert am[0].item() == 700 + 100
    lg = from_dev_bf16(logits)
    assert lg[0, 700] == lg[0, 1500] == lg[0, 2040]
    mx_own, am_own, lse_own = orc.head_stats(lg, 2000, 100)
    assert np.array_equal(am.cpu().numpy(), am_own)
    np.testing.assert_allclose(lse.cpu().numpy(), lse_own, rtol=2e-6)
    assert np.array_equal(orc.top_tokens(lg, V - 2000, 100), am.cpu().numpy())  # get_top_tokens semantics


def test_head_without_logits_store(dev):
    V, H, M = 5000, 384, 4
    x, W, s = orc.make_inputs(8, M, V, H)
    full = head(dev, x, W, s, V, 0)
    part = head(dev, x, W, s, V, 0, want_logits=False)
    assert part[0] is None
    for a, b in zip(full[1:], part[1:]):
        assert np.array_equal(a.cpu().numpy(), b.cpu().numpy())


@pytest.mark.parametrize("M", [1, 2, 3, 4])
def test_full_vocab_config3(dev, M):
    """Config 3 (vocab 151936 x 5120): statistics agree exactly with torch ops on the returned logits and the
    logits with the reference's fp32 dequant-matmul."""
    import torch
    import torch.nn.functional as F
    from qwen_a100_fastpath_b200.w8a16 import w8a16_head
    V, H = 151936, 5120
    g = torch.Generator(device=dev).manual_seed(M)
    W = torch.randint(-127, 128, (V, H), dtype=torch.int8, device=dev, generator=g)
    s = torch.rand(V, device=dev, generator=g) * 0.009 + 0.001
    x = torch.randn(M, H, device=dev, generator=g).to(torch.bfloat16)
    logits, mx, am, lse = w8a16_head(x, W.t(), s)
    lf = logits.float()
    assert torch.equal(am, lf.argmax(-1))
    assert torch.equal(mx, lf.max(-1).values)
    torch.testing.assert_close(lse, torch.logsumexp(lf.double(), -1).float(), rtol=2e-6, atol=0)
    torch.backends.cuda.matmul.allow_tf32 = False
    ref = torch.cat([F.linear(x.float(), W[i:i + 8192].float() * s[i:i + 8192, None]) for i in range(0, V, 8192)], 1)
    assert ((lf - ref).norm() / ref.norm()).item() < 3e-3
    # the draft argmax is the reference's: the argmax of the fp32 dequant-matmul logits rounded to bf16, wherever
    # their top-2 gap exceeds one bf16 ulp of the top logit (closer pairs are decided by fp32 summation order)
    rb = ref.to(torch.bfloat16).float()
    top2 = rb.topk(2, dim=-1).values
    ulp = (top2[:, 0].abs() * 2.0 ** -7).clamp_min(2.0 ** -133)
    clear = (top2[:, 0] - top2[:, 1]) > ulp
    assert clear.any()
    assert torch.equal(am[clear], rb.argmax(-1)[clear])


def test_head_deterministic(dev):
    V, H, M = 151936 // 8, 5120, 4
    x, W, s = orc.make_inputs(31, M, V, H)
    a = head(dev, x, W, s, V, 0)
    b = head(dev, x, W, s, V, 0)
    import torch
    for u, v in zip(a, b):
        assert torch.equal(u.view(torch.uint8) if u.dtype != torch.bfloat16 else u.view(torch.int16),
                           v.view(torch.uint8) if v.dtype != torch.bfloat16 else v.view(torch.int16))


def test_device_quantizer_bit_exact(dev):
    """qf_quantize_rows_int8 (via patches.quantize_head_rows on a CUDA weight) == the reference quantizer
    (patches.py:143-147, oracle.quantize_rows), bit for bit: the golden head weight (zero row, large outlier) and a
    random Qwen-width block."""
    import json
    from pathlib import Path

    import torch

    from qwen_a100_fastpath_b200.patches import quantize_head_rows
    meta = json.loads((Path(__file__).resolve().parent / "golden" / "reference_outputs.json").read_text())["head"]
    rs = np.random.RandomState(meta["weight_seed"])
    wf = rs.standard_normal((meta["V"], meta["H"])).astype(np.float32) * 0.05
    wf[7] = 0.0
    wf[11, 3] = 40.0
    cases = [orc.f32_to_bf16(wf),
             orc.f32_to_bf16(np.random.RandomState(5).standard_normal((3000, 5120)).astype(np.float32) * 0.02)]
    for wb in cases:
        q, s = quantize_head_rows(to_dev_bf16(wb, dev))
        torch.cuda.synchronize()
        q_ref, s_ref = orc.quantize_rows(wb)
        assert np.array_equal(q.cpu().numpy(), q_ref)
        assert np.array_equal(s.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


# ---- fused temperature draw (qf_w8a16_head_sample) -----------------------------------------------------------------
def head_sample(dev, x_bits, W, s, T, seed, offset, n_valid, vocab_offset):
    import torch
    from qwen_a100_fastpath_b200.w8a16 import w8a16_head_sample
    out = w8a16_head_sample(to_dev_bf16(x_bits, dev), torch.from_numpy(W).to(dev).t(), torch.from_numpy(s).to(dev),
                            temperature=T, seed=seed, offset=offset, n_valid=n_valid, vocab_offset=vocab_offset)
    torch.cuda.synchronize()
    return [o if o is None else o.cpu() for o in out]


def check_draw(lg, n_valid, T, seed, offset, vocab_offset, out):
    """The kernel's statistics and draw against the oracle on the kernel's own bf16 logits: statistics of the
    scaled logits exact (lse within 2e-6); the draw identical wherever the oracle's best perturbed score leads the
    second by more than fp32 noise (1e-4), else within 1e-4 of the best; the draw's logit exactly s there."""
    _, mx, am, lse, smp, score, slog = out
    o_mx, o_am, o_lse, o_smp, o_score, o_slog, margin = orc.head_sample(lg, n_valid, np.float32(1.0 / T), seed,
                                                                        offset, vocab_offset)
    assert np.array_equal(mx.numpy(), o_mx)
    assert np.array_equal(am.numpy(), o_am)
    np.testing.assert_allclose(lse.numpy(), o_lse, rtol=2e-6)
    smp = smp.numpy()
    clear = margin > 1e-4
    assert np.array_equal(smp[clear], o_smp[clear])
    sv = (orc.bf16_to_f32(lg)[:, :n_valid] * np.float32(1.0 / T)).astype(np.float32)
    cols = smp - vocab_offset
    assert np.all((cols >= 0) & (cols < n_valid))
    z = sv.astype(np.float64) + orc.gumbel_noise(lg.shape[0], np.arange(n_valid) + vocab_offset, seed, offset)
    rows = np.arange(lg.shape[0])
    assert np.all(z[rows, cols] >= o_score - 1e-4)
    np.testing.assert_allclose(score.numpy(), z[rows, cols], atol=1e-4, rtol=0)
    assert np.array_equal(slog.numpy(), sv[rows, cols])


@pytest.mark.parametrize("V,H,M,pad,T,vocab_offset", [(151936, 5120, 4, 0, 0.8, 0), (4100, 2048, 16, 36, 1.3, 0),
                                                       (1000, 512, 5, 8, 0.5, 3000), (130, 128, 9, 2, 2.0, 7),
                                                       (18992, 1024, 12, 0, 1.0, 18992 * 3)])
def test_head_draw_matches_oracle(dev, V, H, M, pad, T, vocab_offset):
    x, W, s = orc.make_inputs(V + H + M + 1, M, V, H)
    for seed, offset in ((1234, 0), (2**40 + 5, 2**33 + 17)):
        out = head_sample(dev, x, W, s, T, seed, offset, V - pad, vocab_offset)
        lg = from_dev_bf16(out[0])
        assert np.mean(lg != orc.w8a16_mm(x, W, s, "bf16")) < 0.01
        check_draw(lg, V - pad, T, seed, offset, vocab_offset, out)


def test_head_draw_unit_temperature_statistics_equal_greedy_head(dev):
    V, H, M = 8192, 1024, 6
    x, W, s = orc.make_inputs(21, M, V, H)
    g_logits, g_mx, g_am, g_lse = [o.cpu() for o in head(dev, x, W, s, V - 10, 40)]
    out = head_sample(dev, x, W, s, 1.0, 5, 6, V - 10, 40)
    assert np.array_equal(from_dev_bf16(out[0]), from_dev_bf16(g_logits))
    assert np.array_equal(out[1].numpy(), g_mx.numpy()) and np.array_equal(out[2].numpy(), g_am.numpy())
    assert np.array_equal(out[3].numpy(), g_lse.numpy())


def test_head_draw_vocab_shards_equal_unsharded(dev):
    """Two vocab shards (the tensor-parallel head) draw exactly what the unsharded head draws."""
    import torch
    from qwen_a100_fastpath_b200 import tp
    V, H, M = 4096, 1024, 5
    x, W, s = orc.make_inputs(33, M, V, H)
    full = head_sample(dev, x, W, s, 0.9, 11, 3, V, 0)
    parts = []
    for r in range(2):
        n0, n1 = r * V // 2, (r + 1) * V // 2
        o = head_sample(dev, x, np.ascontiguousarray(W[n0:n1]), s[n0:n1].copy(), 0.9, 11, 3, n1 - n0, n0)
        parts.append(torch.stack([o[5].double(), o[4].double(), o[6].double()], dim=1))
    col, logit = tp.combine_head_samples(torch.stack(parts))
    assert np.array_equal(col.numpy(), full[4].numpy())
    assert np.array_equal(logit.numpy(), full[6].numpy())
