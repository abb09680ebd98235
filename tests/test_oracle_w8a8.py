"""The prefill oracle (oracle/w8a8_oracle.py) on CPU: the restated per-token quantization and scaled int8 GEMM."""
from __future__ import annotations

import numpy as np

from oracle import w8a8_oracle as pre
from oracle import w8a16_oracle as orc


def test_quantize_tokens_properties():
    rs = np.random.RandomState(0)
    xf = rs.standard_normal((6, 300)).astype(np.float32)
    xf[1] = 0.0
    xf[2, 5] = -1000.0
    x = orc.f32_to_bf16(xf)
    q, sx = pre.quantize_tokens(x)
    xb = orc.bf16_to_f32(x)
    a = np.abs(xb).max(axis=1)
    assert np.array_equal(sx, (a / np.float32(127)).astype(np.float32))
    assert not q[1].any() and sx[1] == 0                      # zero row
    assert q[2, 5] == -127                                    # the row maximum maps to +-127
    big = np.abs(xb).argmax(axis=1)
    for m in (0, 3, 4, 5):
        assert abs(int(q[m, big[m]])) == 127
    rec = q.astype(np.float64) * sx[:, None]
    assert np.all(np.abs(rec - xb) <= 0.5 * sx[:, None] * (1 + 1e-6) + 1e-30)


def test_quantize_tokens_rounds_half_to_even():
    # row maximum 127 gives the factor 1: values k + 0.5 round to the even neighbour
    xf = np.array([[127.0, 2.5, 3.5, -2.5, -0.5, 0.5, 1.5, 126.5]], np.float32)
    q, sx = pre.quantize_tokens(orc.f32_to_bf16(xf))
    assert q.tolist() == [[127, 2, 4, -2, 0, 0, 2, 126]] and sx[0] == 1.0


def test_w8a8_mm_matches_float_reference():
    rs = np.random.RandomState(1)
    M, N, K = 20, 96, 200
    x = orc.f32_to_bf16(rs.standard_normal((M, K)).astype(np.float32))
    W = rs.randint(-127, 128, size=(N, K)).astype(np.int8)
    s = (rs.random_sample(N) * 0.009 + 0.001).astype(np.float32)
    b = orc.make_bias(2, N)
    q, sx = pre.quantize_tokens(x)
    ref = (q.astype(np.float64) @ W.astype(np.float64).T) * s[None, :].astype(np.float64) * sx[:, None]
    y = orc.bf16_to_f32(pre.w8a8_mm(x, W, s)).astype(np.float64)
    assert np.all(np.abs(y - ref) <= np.abs(ref) * 2.0 ** -8 + 1e-30)
    cols = np.array([3, 50, 95])
    assert np.array_equal(pre.w8a8_mm(x, W, s, b, cols=cols), pre.w8a8_mm(x, W, s, b)[:, cols])
    # the product approximates the bf16 x int8 GEMM within the activation quantization error
    exact = orc.dequant_matmul_f64(x, W, s)
    assert np.linalg.norm(y - exact) / np.linalg.norm(exact) < 1e-2
