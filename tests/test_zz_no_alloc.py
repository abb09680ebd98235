"""The allocation-free entry point qf_w8a16_gemm_noalloc, called through the C ABI.

Some callers cannot allocate device memory: a host that embeds only this library through the C ABI (a Go, Java or C
binding with no device allocator of its own), or a latency-critical path that must not call cudaMalloc, which can
synchronise the device.  They use this entry point; its scratch is a fixed array inside the library.  Here its output
is checked against the workspace entry point qf_w8a16_gemm on the same inputs, for two calls in a row of different
shapes (the second call reuses the array the first one left behind), over bf16 and fp32 outputs, with and without
bias, with and without programmatic dependent launch, and -- in a child process -- with stream-K reducers that hand
off at once (QF_PEER_WAIT_NS=0 under QF_TEST_OVERRIDES=1), the path that re-arms the array's tile counters from the
last contributor.  After each pair of calls the array's error word must read zero.  Tolerance as the other GEMM
tests: bf16 within one bf16 ulp plus 2^-16 * max|y| with at most 1 % of outputs differing; fp32 within 1e-6
relative of max|y| (both entry points run the same kernel).  This file is collected last so that a run stopping at
the first failure has already run every other test.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from oracle import w8a16_oracle as orc
from tests.conftest import from_dev_bf16, to_dev_bf16

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parent.parent
# two calls in a row: an every-tile-split shape (o_proj), then a ragged one
CASES = [(5120, 8192, 5, 11), (1000, 1024, 3, 12)]


def close_bf16(a_bits, b_bits):
    a = orc.bf16_to_f32(a_bits).astype(np.float64)
    b = orc.bf16_to_f32(b_bits).astype(np.float64)
    ulp = np.spacing(np.maximum(np.abs(a), np.abs(b)).astype(np.float32)).astype(np.float64) * 2.0 ** 16
    assert np.all(np.abs(a - b) <= ulp + 2.0 ** -16 * np.abs(b).max())
    assert np.mean(a_bits != b_bits) <= 0.01


def compare_pair(dev, y_dtype: str, bias: bool, flags: int) -> None:
    """Both entry points on CASES in order; the allocation-free one's outputs against the workspace one's."""
    import torch
    from qwen_a100_fastpath_b200 import _lib
    lib = _lib.LIB
    stream = torch.cuda.current_stream(dev)
    dt = _lib.QF_DTYPE_F32 if y_dtype == "f32" else _lib.QF_DTYPE_BF16
    tdt = torch.float32 if y_dtype == "f32" else torch.bfloat16
    for (N, K, M, seed) in CASES:
        x_bits, W, s = orc.make_inputs(seed, M, N, K)
        x = to_dev_bf16(x_bits, dev)
        w = torch.from_numpy(W).to(dev)                   # [N, K] row-major, row stride K bytes
        sc = torch.from_numpy(s).to(dev)
        b = to_dev_bf16(orc.make_bias(seed + 3, N), dev) if bias else None
        ws_bytes = lib.qf_w8a16_workspace_bytes(M, N, K)
        ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
        y_ref = torch.empty((M, N), dtype=tdt, device=dev)
        y_new = torch.full((M, N), float("nan"), dtype=tdt, device=dev)
        bp = b.data_ptr() if b is not None else None
        rc = lib.qf_w8a16_gemm(x.data_ptr(), K, w.data_ptr(), K, sc.data_ptr(), bp, y_ref.data_ptr(), N, dt, M, N, K,
                               ws.data_ptr(), ws_bytes, flags, stream.cuda_stream)
        assert rc == 0, lib.qf_last_error_detail()
        rc = lib.qf_w8a16_gemm_noalloc(x.data_ptr(), K, w.data_ptr(), K, sc.data_ptr(), bp, y_new.data_ptr(), N, dt,
                                       M, N, K, flags, stream.cuda_stream)
        assert rc == 0, lib.qf_last_error_detail()
        torch.cuda.synchronize(dev)
        if y_dtype == "f32":
            a, r = y_new.cpu().numpy().astype(np.float64), y_ref.cpu().numpy().astype(np.float64)
            assert np.all(np.isfinite(a))
            assert np.abs(a - r).max() <= 1e-6 * np.abs(r).max()
        else:
            close_bf16(from_dev_bf16(y_new), from_dev_bf16(y_ref))
            if not bias:
                close_bf16(from_dev_bf16(y_new), orc.w8a16_mm(x_bits, W, s, "bf16"))
    st = ctypes.c_int(-1)
    assert lib.qf_w8a16_noalloc_status(stream.cuda_stream, ctypes.byref(st)) == 0, lib.qf_last_error_detail()
    assert st.value == 0, f"device error flag {st.value}"


@pytest.mark.parametrize("y_dtype", ["bf16", "f32"])
@pytest.mark.parametrize("bias", [False, True], ids=["nobias", "bias"])
@pytest.mark.parametrize("pdl", [False, True], ids=["plain", "pdl"])
def test_noalloc_matches_workspace_entry_point(dev, y_dtype, bias, pdl):
    from qwen_a100_fastpath_b200 import _lib
    compare_pair(dev, y_dtype, bias, _lib.QF_FLAG_PDL if pdl else 0)


def test_noalloc_last_arriver_reduction(dev):
    """Child process with QF_PEER_WAIT_NS=0: every split tile is reduced by the last share to finish."""
    env = dict(os.environ)
    env["QF_TEST_OVERRIDES"] = "1"
    env["QF_PEER_WAIT_NS"] = "0"
    r = subprocess.run([sys.executable, "-m", "tests.test_zz_no_alloc"], cwd=REPO, env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]


def test_noalloc_rejects_oversized_n():
    from qwen_a100_fastpath_b200 import _lib
    rc = _lib.LIB.qf_w8a16_gemm_noalloc(1 << 20, 128, 1 << 20, 128, 1 << 20, None, 1 << 20, _lib.QF_NOALLOC_MAX_N + 1,
                                        0, 1, _lib.QF_NOALLOC_MAX_N + 1, 128, 0, None)
    assert rc == -2
    assert b"QF_NOALLOC_MAX_N" in _lib.LIB.qf_last_error_detail()


if __name__ == "__main__":
    import torch
    d = torch.device("cuda", 0)
    for dt in ("bf16", "f32"):
        compare_pair(d, dt, bias=(dt == "bf16"), flags=0)
    print("ok")
