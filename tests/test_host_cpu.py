"""Host logic on CPU: plugin registration and patch surface against the installed vLLM, the int8 draft-head
quantizer against the oracle (bit-exact), the draft-head gates, and the no-CPU-fallback rule."""
from __future__ import annotations

import json
import types
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import w8a16_oracle as orc

GOLD = Path(__file__).resolve().parent / "golden"


def test_pick_config_and_small_m():
    from qwen_a100_fastpath_b200.w8a16 import B200_CONFIG, SMALL_M, pick_config
    assert SMALL_M == 16
    for N, K in [(10240, 5120), (5120, 8192), (34816, 5120), (5120, 17408), (151936, 5120), (5120, 2176), (64, 100)]:
        assert pick_config(N, K) == B200_CONFIG
    assert pick_config(0, 128) is None and pick_config(128, 0) is None and pick_config(2 ** 21, 128) is None


def test_quantize_head_rows_matches_reference_quantizer():
    """patches.quantize_head_rows restates plugin/qwen_fastpath/patches.py:143-147; pinned by the golden hash."""
    from qwen_a100_fastpath_b200.patches import quantize_head_rows
    meta = json.loads((GOLD / "reference_outputs.json").read_text())["head"]
    rs = np.random.RandomState(meta["weight_seed"])
    wf = rs.standard_normal((meta["V"], meta["H"])).astype(np.float32) * 0.05
    wf[7] = 0.0
    wf[11, 3] = 40.0
    wb = orc.f32_to_bf16(wf)
    w = torch.from_numpy(wb.view(np.int16)).view(torch.bfloat16)
    q, s = quantize_head_rows(w)
    q_ref, s_ref = orc.quantize_rows(wb)
    assert np.array_equal(q.numpy(), q_ref)
    assert np.array_equal(s.numpy().view(np.uint32), s_ref.view(np.uint32))


def fake_model(V=512, H=128, pad=12, tp_size=1):
    lm_head = types.SimpleNamespace(weight=torch.randn(V, H).to(torch.bfloat16), tp_size=tp_size,
                                    shard_indices=types.SimpleNamespace(num_org_vocab_padding=pad,
                                                                        org_vocab_start_index=0))
    lp = types.SimpleNamespace(logits_as_input=False, soft_cap=None, scale=1.0, org_vocab_size=V - pad)
    return types.SimpleNamespace(lm_head=lm_head, logits_processor=lp)


def test_attach_int8_head_and_gates():
    from qwen_a100_fastpath_b200 import patches
    m = fake_model()
    assert patches.attach_int8_head(m)
    w_t, scale, num_pad, cfg = m._qf_head_i8
    assert w_t.shape == (128, 512) and w_t.stride() == (1, 128) and num_pad == 12 and cfg is not None
    m2 = fake_model(tp_size=2)                                         # a vocab shard: accepted (the reference is
    assert patches.attach_int8_head(m2) and m2._qf_head_tp == 2       # tp_size == 1 only, patches.py:138)
    m3 = fake_model()
    m3.lm_head.shard_indices.num_added_elements = 8                    # added (LoRA) vocabulary: original path
    assert not patches.attach_int8_head(m3)
    h = torch.zeros(3, 128, dtype=torch.bfloat16)
    assert patches.int8_head(m, h.float()) is None                     # dtype gate
    assert patches.int8_head(m, torch.zeros(17, 128, dtype=torch.bfloat16)) is None   # M > 16
    m.logits_processor.soft_cap = 30.0
    assert patches.int8_head(m, h) is None                             # soft-capped logits keep the original path
    m.logits_processor.soft_cap = None
    with pytest.raises(ValueError):                                    # eligible, but CPU tensors: no CPU fallback
        patches.int8_head(m, h)


def test_w8a16_mm_refuses_cpu_tensors():
    from qwen_a100_fastpath_b200.w8a16 import w8a16_mm
    with pytest.raises(ValueError):
        w8a16_mm(torch.zeros((1, 128), dtype=torch.bfloat16), torch.zeros((64, 128), dtype=torch.int8).t(),
                 torch.ones(64), None, torch.bfloat16)


@pytest.mark.slow
def test_register_patches_installed_vllm(monkeypatch):
    """register() against the vLLM in this image: the int8 linear patch lands on CutlassInt8ScaledMMLinearKernel
    with the custom op and its fake, is idempotent, and the draft-head patch degrades gracefully where the
    speculator hook is missing."""
    vllm_cutlass = pytest.importorskip("vllm.model_executor.kernels.linear.scaled_mm.cutlass")
    import qwen_a100_fastpath_b200 as plugin
    from qwen_a100_fastpath_b200 import patches
    cls = vllm_cutlass.CutlassInt8ScaledMMLinearKernel
    orig = cls.apply_weights
    from vllm.model_executor.layers.linear import RowParallelLinear
    from vllm.v1.attention.backends import flash_attn as fa
    orig_row = RowParallelLinear.forward
    orig_attn = fa.FlashAttentionImpl.forward
    try:
        monkeypatch.setenv("QWEN_FAST_ATTN", "1")
        monkeypatch.setenv("QWEN_FAST_LINEAR", "1")
        monkeypatch.setenv("QWEN_FAST_DRAFT_HEAD", "1")
        monkeypatch.setattr(plugin, "_registered", False)
        plugin.register()
        assert getattr(cls.apply_weights, "_qwen_fastpath", False)
        assert hasattr(torch.ops.vllm, "qf_int8_linear")
        assert patches.patch_int8_linear() is False                      # second patch is a no-op
        plugin.register()                                                # idempotent
        # the fake (meta) implementation gives the output shape without running a kernel
        x = torch.empty((2, 3, 256), dtype=torch.bfloat16, device="meta")
        w = torch.empty((256, 640), dtype=torch.int8, device="meta")
        s = torch.empty((640, 1), dtype=torch.float32, device="meta")
        y = torch.ops.vllm.qf_int8_linear(x, w, s, None)
        assert y.shape == (2, 3, 640)
        from vllm.model_executor.models import qwen3_5_mtp
        assert getattr(qwen3_5_mtp.Qwen3_5MTP.compute_logits, "_qwen_fastpath", False)
        assert getattr(RowParallelLinear.forward, "_qwen_fastpath", False)
        assert patches.patch_row_parallel() is False                     # idempotent
        assert getattr(fa.FlashAttentionImpl.forward, "_qwen_fastpath", False)
        assert patches.patch_flash_attention() is False                  # idempotent
    finally:
        cls.apply_weights = getattr(cls.apply_weights, "_qf_orig", orig)
        RowParallelLinear.forward = orig_row
        fa.FlashAttentionImpl.forward = orig_attn


def test_switches_off(monkeypatch):
    import qwen_a100_fastpath_b200 as plugin
    from qwen_a100_fastpath_b200 import patches
    called = []
    monkeypatch.setattr(patches, "patch_int8_linear", lambda: called.append("linear"))
    monkeypatch.setattr(patches, "patch_row_parallel", lambda: called.append("row"))
    monkeypatch.setattr(patches, "patch_draft_lm_head", lambda: called.append("head"))
    monkeypatch.setattr(patches, "patch_flash_attention", lambda: called.append("attn"))
    monkeypatch.setattr(plugin, "_registered", False)
    monkeypatch.setenv("QWEN_FAST_ATTN", "0")
    monkeypatch.setenv("QWEN_FAST_LINEAR", "0")
    monkeypatch.setenv("QWEN_FAST_DRAFT_HEAD", "1")
    plugin.register()
    assert called == ["head"]
    monkeypatch.setattr(plugin, "_registered", False)
    monkeypatch.setenv("QWEN_FAST_ATTN", "1")
    monkeypatch.setenv("QWEN_FAST_LINEAR", "1")
    monkeypatch.setenv("QWEN_FAST_DRAFT_HEAD", "0")
    plugin.register()
    assert called == ["head", "attn", "linear", "row"]


# ---------------------------------------------------------------------------------------------- QWEN_FAST_ATTN
def fake_attn_impl(**kw):
    import types
    from vllm.v1.attention.backends import flash_attn as fa
    d = dict(attn_type=fa.AttentionType.DECODER, dcp_world_size=1, sliding_window=(-1, -1), alibi_slopes=None,
             logits_soft_cap=None, sinks=None, kv_cache_dtype="auto", num_heads=24, num_kv_heads=4, head_size=256,
             kv_sharing_target_layer_name=None, scale=256 ** -0.5)
    d.update(kw)
    return types.SimpleNamespace(**d)


def fake_md(num_reqs, q_len, num_tokens=None, **kw):
    import types
    d = dict(max_query_len=q_len, use_cascade=False, causal=True,
             query_start_loc=torch.arange(num_reqs + 1, dtype=torch.int32) * q_len,
             num_actual_tokens=num_reqs * q_len if num_tokens is None else num_tokens,
             seq_lens=torch.full((num_reqs,), 100, dtype=torch.int32),
             block_table=torch.zeros((num_reqs, 4), dtype=torch.int32))
    d.update(kw)
    return types.SimpleNamespace(**d)


@pytest.mark.slow
def test_spec_attn_routing(monkeypatch):
    """patches.spec_attn_forward (the body of the patched FlashAttentionImpl.forward, patches.py:44-66 of the
    reference): uniform batches with 1 < Q <= 8 go to the kernel with the right cache views for both layouts;
    everything else returns None (FlashAttention)."""
    pytest.importorskip("vllm.v1.attention.backends.flash_attn")
    from qwen_a100_fastpath_b200 import patches, spec_attn
    calls = []

    def record(q3, kc, vc, o3, seq_lens, bt, num_reqs, Q, hkv, scale):
        calls.append((tuple(q3.shape), tuple(kc.shape), kc.stride(), tuple(vc.shape), num_reqs, Q, hkv, scale))
        return o3

    monkeypatch.setattr(spec_attn, "gqa_packed_spec_attention", record)
    H, HKV, D, page, nb = 24, 4, 256, 800, 6
    vllm_cache = torch.zeros((2, nb, page, HKV, D), dtype=torch.bfloat16)   # vLLM FlashAttention layout
    ref_cache = torch.zeros((nb, HKV, page, 2 * D), dtype=torch.bfloat16)   # the reference's interleaved layout
    q = torch.zeros((8, H, D), dtype=torch.bfloat16)
    out = torch.zeros((8, H * D), dtype=torch.bfloat16)
    impl = fake_attn_impl()
    assert patches.spec_attn_forward(impl, q[:6], vllm_cache, fake_md(2, 3), out[:6]) is not None
    assert calls[-1][:2] == ((6, H, D), (nb, page, HKV, D)) and calls[-1][4:7] == (2, 3, HKV)
    assert calls[-1][2] == vllm_cache[0].stride()
    assert patches.spec_attn_forward(impl, q[:8], ref_cache, fake_md(2, 4), out[:8]) is not None
    assert calls[-1][1] == (nb, page, HKV, D) and calls[-1][2] == ref_cache.transpose(1, 2).stride()
    n = len(calls)
    for md in (fake_md(3, 1), fake_md(1, 9), fake_md(2, 3, num_tokens=5), fake_md(2, 3, use_cascade=True),
               fake_md(2, 3, causal=False), None):
        assert patches.spec_attn_forward(impl, q[:6], vllm_cache, md, out[:6]) is None
    assert patches.spec_attn_forward(impl, q[:6].half(), vllm_cache, fake_md(2, 3), out[:6]) is None
    assert patches.spec_attn_forward(impl, q[:6], vllm_cache, fake_md(2, 3), out[:6],
                                     output_scale=torch.ones(1)) is None
    assert patches.spec_attn_forward(impl, q[:6], vllm_cache.half(), fake_md(2, 3), out[:6]) is None
    for bad in (dict(sliding_window=(127, 0)), dict(logits_soft_cap=30.0), dict(head_size=96),
                dict(num_heads=66, num_kv_heads=1), dict(kv_sharing_target_layer_name="x")):
        assert patches.spec_attn_forward(fake_attn_impl(**bad), q[:6], vllm_cache, fake_md(2, 3), out[:6]) is None
    g8 = fake_attn_impl(num_heads=32, num_kv_heads=4, head_size=128)             # G = 8, Q = 8: 64 packed rows
    q8, o8 = torch.zeros((8, 32, 128), dtype=torch.bfloat16), torch.zeros((8, 32 * 128), dtype=torch.bfloat16)
    assert patches.spec_attn_forward(g8, q8, torch.zeros((2, nb, 32, 4, 128), dtype=torch.bfloat16),
                                     fake_md(1, 8), o8) is not None
    g16 = fake_attn_impl(num_heads=64, num_kv_heads=4, head_size=128)            # G = 16, Q = 5: 80 rows, not taken
    q16, o16 = torch.zeros((5, 64, 128), dtype=torch.bfloat16), torch.zeros((5, 64 * 128), dtype=torch.bfloat16)
    assert patches.spec_attn_forward(g16, q16, torch.zeros((2, nb, 32, 4, 128), dtype=torch.bfloat16),
                                     fake_md(1, 5), o16) is None
    assert len(calls) == n + 1
