"""The allocation-free entry point qf_w8a16_gemm_noalloc, called through the C ABI.

Callers that cannot allocate device memory (a host binding with no device allocator of its own, or a path that
must not call cudaMalloc) use this entry point; its scratch is a fixed array inside the library.  Here its output
is checked against the workspace entry point qf_w8a16_gemm on the same inputs, for two calls in a row of
different shapes (the second call reuses the array the first one left behind).  Tolerance as the other GEMM
tests: within one bf16 ulp plus 2^-16 * max|y|, at most 1 % of outputs differing.  This file is collected last
so that a run stopping at the first failure has already run every other test.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import w8a16_oracle as orc
from tests.conftest import from_dev_bf16, to_dev_bf16

pytestmark = pytest.mark.gpu


def close(a_bits, b_bits):
    a = orc.bf16_to_f32(a_bits).astype(np.float64)
    b = orc.bf16_to_f32(b_bits).astype(np.float64)
    ulp = np.spacing(np.maximum(np.abs(a), np.abs(b)).astype(np.float32)).astype(np.float64) * 2.0 ** 16
    assert np.all(np.abs(a - b) <= ulp + 2.0 ** -16 * np.abs(b).max())
    assert np.mean(a_bits != b_bits) <= 0.01


def test_noalloc_matches_workspace_entry_point(dev):
    import torch
    from qwen_a100_fastpath_b200 import _lib
    lib = _lib.LIB
    stream = torch.cuda.current_stream(dev)
    for (N, K, M, seed) in [(5120, 8192, 5, 11), (1000, 1024, 3, 12)]:
        x_bits, W, s = orc.make_inputs(seed, M, N, K)
        x = to_dev_bf16(x_bits, dev)
        w = torch.from_numpy(W).to(dev)                   # [N, K] row-major, row stride K bytes
        sc = torch.from_numpy(s).to(dev)
        ws_bytes = lib.qf_w8a16_workspace_bytes(M, N, K)
        ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
        y_ref = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        y_new = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)
        rc = lib.qf_w8a16_gemm(x.data_ptr(), K, w.data_ptr(), K, sc.data_ptr(), None, y_ref.data_ptr(), N,
                               _lib.QF_DTYPE_BF16, M, N, K, ws.data_ptr(), ws_bytes, 0, stream.cuda_stream)
        assert rc == 0, lib.qf_last_error_detail()
        rc = lib.qf_w8a16_gemm_noalloc(x.data_ptr(), K, w.data_ptr(), K, sc.data_ptr(), None, y_new.data_ptr(), N,
                                       _lib.QF_DTYPE_BF16, M, N, K, 0, stream.cuda_stream)
        assert rc == 0, lib.qf_last_error_detail()
        torch.cuda.synchronize(dev)
        close(from_dev_bf16(y_new), from_dev_bf16(y_ref))
        close(from_dev_bf16(y_new), orc.w8a16_mm(x_bits, W, s, "bf16"))


def test_noalloc_rejects_oversized_n():
    from qwen_a100_fastpath_b200 import _lib
    rc = _lib.LIB.qf_w8a16_gemm_noalloc(1 << 20, 128, 1 << 20, 128, 1 << 20, None, 1 << 20, 65537, 0, 1,
                                        _lib.QF_NOALLOC_MAX_N + 1, 128, 0, None)
    assert rc == -2
    assert b"QF_NOALLOC_MAX_N" in _lib.LIB.qf_last_error_detail()
