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
    orig_row = RowParallelLinear.forward
    try:
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
    finally:
        cls.apply_weights = getattr(cls.apply_weights, "_qf_orig", orig)
        RowParallelLinear.forward = orig_row


def test_switches_off(monkeypatch):
    import qwen_a100_fastpath_b200 as plugin
    from qwen_a100_fastpath_b200 import patches
    called = []
    monkeypatch.setattr(patches, "patch_int8_linear", lambda: called.append("linear"))
    monkeypatch.setattr(patches, "patch_row_parallel", lambda: called.append("row"))
    monkeypatch.setattr(patches, "patch_draft_lm_head", lambda: called.append("head"))
    monkeypatch.setattr(plugin, "_registered", False)
    monkeypatch.setenv("QWEN_FAST_LINEAR", "0")
    monkeypatch.setenv("QWEN_FAST_DRAFT_HEAD", "1")
    plugin.register()
    assert called == ["head"]
    monkeypatch.setattr(plugin, "_registered", False)
    monkeypatch.setenv("QWEN_FAST_LINEAR", "1")
    monkeypatch.setenv("QWEN_FAST_DRAFT_HEAD", "0")
    plugin.register()
    assert called == ["head", "linear", "row"]
