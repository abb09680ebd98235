"""Run as ``python -m tests._grid_cap_case`` with QF_TEST_OVERRIDES=1 and QF_GRID_CAP, QF_TILES, QF_SK_SKEW,
QF_PEER_WAIT_NS or QF_F16_PATH set: GEMM and head shapes whose tiles are split between CTAs in ways the full grid
never produces (one CTA, a few CTAs, stream-K shares of many stages, even or skewed shares where every tile is split),
run on a forced tile shape, or on the all-bf16 activation path, checked against the oracle.  Exits non-zero on a
mismatch.  Used by test_gpu_schedule.py."""
from __future__ import annotations

import sys

import numpy as np


def main() -> int:
    import torch
    from oracle import w8a16_oracle as orc
    from qwen_a100_fastpath_b200.w8a16 import pick_config, w8a16_head, w8a16_mm
    from tests.conftest import from_dev_bf16, to_dev_bf16
    from tests.test_gpu_gemm import bf16_close, silu_close
    dev = torch.device("cuda", 0)
    for (N, K, M) in [(1000, 1024, 5), (10240, 1024, 3), (4100, 2048, 12), (19072, 512, 1), (2048, 8192, 7)]:
        x, W, s = orc.make_inputs(N + K + M, M, N, K)
        y = w8a16_mm(to_dev_bf16(x, dev), torch.from_numpy(W).to(dev).t(), torch.from_numpy(s).to(dev),
                     pick_config(N, K), torch.bfloat16)
        torch.cuda.synchronize()
        bf16_close(from_dev_bf16(y), orc.w8a16_mm(x, W, s, "bf16"))
    from qwen_a100_fastpath_b200.w8a16 import w8a16_mm_silu_mul
    for (I, K, M) in [(1000, 1024, 5), (4100, 2048, 12)]:  # fused gate_up activation on the same schedules
        x, W, s = orc.make_inputs(I + K, M, 2 * I, K)
        out = w8a16_mm_silu_mul(to_dev_bf16(x, dev), torch.from_numpy(W).to(dev).t(), torch.from_numpy(s).to(dev))
        torch.cuda.synchronize()
        y_orc = orc.w8a16_mm(x, W, s, "bf16")
        silu_close(from_dev_bf16(out), orc.silu_mul(y_orc, I), y_orc, I)
    for (V, H, M, pad) in [(4100, 2048, 4, 36), (16384 + 640, 1024, 16, 64), (3000, 8192, 3, 8)]:
        x, W, s = orc.make_inputs(V + H, M, V, H)
        logits, mx, am, lse = w8a16_head(to_dev_bf16(x, dev), torch.from_numpy(W).to(dev).t(),
                                         torch.from_numpy(s).to(dev), n_valid=V - pad, vocab_offset=0)
        torch.cuda.synchronize()
        lg = from_dev_bf16(logits)
        assert np.mean(lg != orc.w8a16_mm(x, W, s, "bf16")) < 0.01
        mx_own, am_own, lse_own = orc.head_stats(lg, V - pad, 0)
        assert np.array_equal(mx.cpu().numpy(), mx_own)
        assert np.array_equal(am.cpu().numpy(), am_own)
        np.testing.assert_allclose(lse.cpu().numpy(), lse_own, rtol=2e-6)
    from qwen_a100_fastpath_b200.w8a16 import w8a16_head_sample
    for (V, H, M) in [(4100, 2048, 5), (3000, 8192, 13)]:  # the fused draw on the same schedules
        x, W, s = orc.make_inputs(V + H + 7, M, V, H)
        out = w8a16_head_sample(to_dev_bf16(x, dev), torch.from_numpy(W).to(dev).t(), torch.from_numpy(s).to(dev),
                                temperature=0.7, seed=5, offset=9, n_valid=V - 3, vocab_offset=100)
        torch.cuda.synchronize()
        from tests.test_gpu_head import check_draw
        lg = from_dev_bf16(out[0])
        check_draw(lg, V - 3, 0.7, 5, 9, 100, [o.cpu() if o is not None else None for o in out])
    from qwen_a100_fastpath_b200.w8a16 import w8a16_mm_rmsnorm
    from tests.test_gpu_rmsnorm import close as norm_close
    for (N, K, M, silu) in [(2048, 8192, 7, False), (4100, 2048, 12, False), (2000, 1024, 5, True)]:
        rs = np.random.RandomState(N + M)  # fused RMSNorm on the same schedules (sums of squares handed off too)
        xb = orc.f32_to_bf16(rs.standard_normal((M, K)).astype(np.float32) * 3.0)
        rb = orc.f32_to_bf16(rs.standard_normal((M, K)).astype(np.float32))
        gb = orc.f32_to_bf16((rs.random_sample(K) + 0.5).astype(np.float32))
        W = rs.randint(-127, 128, size=(N, K)).astype(np.int8)
        sc = (rs.random_sample(N) * 0.009 + 0.001).astype(np.float32)
        y, res_out = w8a16_mm_rmsnorm(to_dev_bf16(xb, dev), to_dev_bf16(gb, dev), 1e-6, torch.from_numpy(W).to(dev).t(),
                                      torch.from_numpy(sc).to(dev), residual=to_dev_bf16(rb, dev), silu_mul=silu)
        torch.cuda.synchronize()
        y_ref, r_ref = orc.rmsnorm_w8a16_mm(xb, rb, gb, 1e-6, W, sc, silu=silu)
        assert np.array_equal(from_dev_bf16(res_out), r_ref)
        norm_close(from_dev_bf16(y), y_ref, frob=1e-2 if silu else 5e-3)
    from qwen_a100_fastpath_b200.w8a16 import workspace_status
    assert workspace_status() == 0
    print("ok")
    return 0


if __name__ == "__main__":
    sys.exit(main())
