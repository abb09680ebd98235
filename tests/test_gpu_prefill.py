"""The prefill (M > 16) int8 path on tcgen05 (qf_w8a8_gemm, through the C ABI and through ``qf_int8_linear``)
against the CPU oracle of the reference's vLLM W8A8 fallback (plugin/qwen_fastpath/patches.py:99-100).

Bars: the per-token quantization (int8 rows and fp32 scales, read back from the documented workspace layout) is
bit-identical to the oracle; the int32 accumulation is exact and the fp32 scaling follows the same operations, so the
bf16 outputs are bit-identical to the oracle except where the bias's fused multiply-add and the oracle's fp64
emulation of it round differently (at most one bf16 ulp, in at most 0.1 % of outputs).  Shapes: the BASELINE config-2
GEMMs at M = 17 and 64 (every column) and at M = 300, 1024 and 4096 (a seeded sample of 512 columns), ragged M, N
and K, strided and misaligned activation rows, zero and outlier rows, and a bias.  Where vLLM's compiled
``scaled_int8_quant`` / ``cutlass_scaled_mm`` run on the GPU box they are compared too.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import w8a8_oracle as pre
from oracle import w8a16_oracle as orc
from tests.conftest import from_dev_bf16, to_dev_bf16

pytestmark = pytest.mark.gpu


def call(dev, x, w, s, bias=None, M=None, K=None):
    """qf_w8a8_gemm through the C ABI; returns (y, workspace)."""
    import torch
    from qwen_a100_fastpath_b200 import _lib
    lib = _lib.LIB
    M = x.shape[0] if M is None else M
    K = w.shape[1] if K is None else K
    N = w.shape[0]
    ws_bytes = lib.qf_w8a8_workspace_bytes(M, K)
    ws = torch.zeros(ws_bytes + 256, dtype=torch.uint8, device=dev)
    y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)
    rc = lib.qf_w8a8_gemm(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), s.data_ptr(),
                          bias.data_ptr() if bias is not None else None, y.data_ptr(), N, M, N, K, ws.data_ptr(),
                          ws.numel(), 0, torch.cuda.current_stream(dev).cuda_stream)
    assert rc == 0, lib.qf_last_error_detail()
    torch.cuda.synchronize(dev)
    return y, ws


def workspace_quant(ws, M, K):
    """(q int8 [M, K], s_x fp32 [M]) from the workspace layout of include/qf_b200.h."""
    ldq = (K + 15) // 16 * 16
    raw = ws.cpu().numpy()
    qb = (M * ldq + 255) // 256 * 256
    q = raw[256:256 + M * ldq].view(np.int8).reshape(M, ldq)
    sx = raw[256 + qb:256 + qb + 4 * M].view(np.float32)
    assert not q[:, K:].any()                      # the row padding is zero
    return q[:, :K], sx


def assert_out(got_bits, ref_bits, bias):
    if not bias:
        assert np.array_equal(got_bits, ref_bits), f"{np.mean(got_bits != ref_bits):.4%} of outputs differ"
        return
    a = orc.bf16_to_f32(got_bits).astype(np.float64)
    b = orc.bf16_to_f32(ref_bits).astype(np.float64)
    ulp = np.spacing(np.maximum(np.abs(a), np.abs(b)).astype(np.float32)).astype(np.float64) * 2.0 ** 16
    assert np.all(np.abs(a - b) <= ulp)
    assert np.mean(got_bits != ref_bits) <= 1e-3


_W = {}


def weight(dev, N, K):
    """Seeded int8 weight [N, K] and scales, host and device copies, cached for the last shape."""
    import torch
    if (N, K) not in _W:
        _W.clear()
        rs = np.random.RandomState(N + K)
        W = rs.randint(-127, 128, size=(N, K)).astype(np.int8)
        s = (rs.random_sample(N) * 0.009 + 0.001).astype(np.float32)
        _W[(N, K)] = (W, s, torch.from_numpy(W).to(dev), torch.from_numpy(s).to(dev))
    return _W[(N, K)]


@pytest.mark.parametrize("M", [17, 64, 300, 1024, 4096])
@pytest.mark.parametrize("name,N,K", [("qkv", 10240, 5120), ("o_proj", 5120, 8192), ("gate_up", 34816, 5120),
                                      ("down", 5120, 17408)])
def test_prefill_config2(dev, name, N, K, M):
    W, s, Wd, sd = weight(dev, N, K)
    x_bits = orc.f32_to_bf16(np.random.RandomState(M).standard_normal((M, K)).astype(np.float32))
    y, ws = call(dev, to_dev_bf16(x_bits, dev), Wd, sd)
    q, sx = workspace_quant(ws, M, K)
    q_o, sx_o = pre.quantize_tokens(x_bits)
    assert np.array_equal(q, q_o) and np.array_equal(sx.view(np.uint32), sx_o.view(np.uint32))
    cols = None if M <= 64 else np.sort(np.random.RandomState(M).choice(N, 512, replace=False))
    got = from_dev_bf16(y)
    assert_out(got if cols is None else got[:, cols], pre.w8a8_mm(x_bits, W, s, cols=cols), bias=False)


@pytest.mark.parametrize("M,N,K,ldx,off,bias", [
    (17, 1000, 200, None, 0, False),     # ragged N, K % 16 != 0
    (129, 384, 1000, 1032, 0, True),     # a second token tile, strided rows, bias
    (33, 640, 520, None, 1, False),      # rows 2-byte aligned only: the scalar quantization path
    (200, 4352, 4096, None, 0, True),    # gate_up shard at TP = 8, bias
])
def test_prefill_edges(dev, M, N, K, ldx, off, bias):
    import torch
    rs = np.random.RandomState(M * N + K)
    W = rs.randint(-127, 128, size=(N, K)).astype(np.int8)
    s = (rs.random_sample(N) * 0.009 + 0.001).astype(np.float32)
    xf = rs.standard_normal((M, K)).astype(np.float32)
    xf[3] = 0.0                              # a zero row: q = 0, s_x = 0
    xf[5, 7] = 300.0                         # an outlier that sets its row's scale
    x_bits = orc.f32_to_bf16(xf)
    ld = ldx or K
    buf = torch.zeros(M * ld + off + 8, dtype=torch.bfloat16, device=dev)
    x = buf[off:off + M * ld].view(M, ld)[:, :K]
    x.copy_(to_dev_bf16(x_bits, dev))
    b_bits = orc.make_bias(M + N, N) if bias else None
    ldw = (K + 15) // 16 * 16                  # TMA: weight rows padded to a 16-byte stride
    Wp = np.zeros((N, ldw), np.int8)
    Wp[:, :K] = W
    Wd = torch.from_numpy(Wp).to(dev)[:, :K]
    y, ws = call(dev, x, Wd, torch.from_numpy(s).to(dev), bias=to_dev_bf16(b_bits, dev) if bias else None)
    q, sx = workspace_quant(ws, M, K)
    q_o, sx_o = pre.quantize_tokens(x_bits)
    assert np.array_equal(q, q_o) and np.array_equal(sx.view(np.uint32), sx_o.view(np.uint32))
    assert sx[3] == 0 and not q[3].any()
    assert_out(from_dev_bf16(y), pre.w8a8_mm(x_bits, W, s, b_bits), bias)
    from qwen_a100_fastpath_b200 import _lib
    import ctypes
    st = ctypes.c_int(-1)
    assert _lib.LIB.qf_workspace_status(ws.data_ptr(), torch.cuda.current_stream(dev).cuda_stream,
                                        ctypes.byref(st)) == 0 and st.value == 0


def test_prefill_through_op(dev, monkeypatch):
    """qf_int8_linear routes bf16 rows above 16 to the prefill kernel (3-D input, bias), not to vLLM's fallback."""
    import torch
    from qwen_a100_fastpath_b200 import patches
    monkeypatch.setattr(patches, "w8a8_fallback", lambda *a: pytest.fail("vLLM fallback called"))
    op = patches.make_int8_linear_op()[0]
    N, K = 2048, 1024
    rs = np.random.RandomState(3)
    W = rs.randint(-127, 128, size=(N, K)).astype(np.int8)
    s = (rs.random_sample(N) * 0.009 + 0.001).astype(np.float32)
    x_bits = orc.f32_to_bf16(rs.standard_normal((32, K)).astype(np.float32))
    b_bits = orc.make_bias(4, N)
    y = op(to_dev_bf16(x_bits, dev).view(4, 8, K), torch.from_numpy(W).to(dev).t(),
           torch.from_numpy(s).to(dev).view(N, 1), to_dev_bf16(b_bits, dev))
    torch.cuda.synchronize(dev)
    assert y.shape == (4, 8, N)
    assert_out(from_dev_bf16(y).reshape(32, N), pre.w8a8_mm(x_bits, W, s, b_bits), bias=True)


def test_prefill_matches_vllm_ops_when_available(dev):
    """vLLM's own compiled scaled_int8_quant / cutlass_scaled_mm, where they run on this GPU."""
    import torch
    try:
        from vllm import _custom_ops as ops
        N, K, M = 1024, 2048, 48
        rs = np.random.RandomState(11)
        W = rs.randint(-127, 128, size=(N, K)).astype(np.int8)
        s = (rs.random_sample(N) * 0.009 + 0.001).astype(np.float32)
        x = to_dev_bf16(orc.f32_to_bf16(rs.standard_normal((M, K)).astype(np.float32)), dev)
        wq = torch.from_numpy(W).to(dev).t()
        ws_ = torch.from_numpy(s).to(dev).view(N, 1)
        x_q, x_s, _ = ops.scaled_int8_quant(x.contiguous(), None, None, symmetric=True)
        y_v = ops.cutlass_scaled_mm(x_q, wq, scale_a=x_s, scale_b=ws_, out_dtype=torch.bfloat16)
        torch.cuda.synchronize(dev)
    except Exception as e:  # noqa: BLE001 -- vLLM's compiled kernels are optional on the test box
        pytest.skip(f"vLLM ops unavailable on this box: {type(e).__name__}: {str(e)[:200]}")
    y, wsb = call(dev, x, torch.from_numpy(W).to(dev), torch.from_numpy(s).to(dev))
    q, sx = workspace_quant(wsb, M, K)
    assert np.array_equal(q, x_q.cpu().numpy())
    assert np.array_equal(sx.view(np.uint32), x_s.reshape(-1).float().cpu().numpy().view(np.uint32))
    a = y.float().cpu().numpy().astype(np.float64)
    b = y_v.float().cpu().numpy().astype(np.float64)
    ulp = np.spacing(np.maximum(np.abs(a), np.abs(b)).astype(np.float32)).astype(np.float64) * 2.0 ** 16
    assert np.all(np.abs(a - b) <= ulp)
