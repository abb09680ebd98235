"""Bounded cross-GPU waits running out, on one GPU and without a fault.

Rank 0 of a two-rank all-reduce is launched with the "other rank's" buffer being a second buffer of the same GPU
that no kernel ever writes into this rank's slot, so the lines rank 0 waits for never arrive.  The wait bound is set
to 50 ms through the buffer header (qf_allreduce_set_wait).  The kernel must finish by itself, the buffer's error word
must then read QF_ERR_TIMEOUT exactly once (qf_allreduce_status clears it), and the next call on the same buffer --
a one-rank call, which waits for nobody -- must succeed and be exact.  Both the standalone one-shot all-reduce
(qf_allreduce_bf16) and the row-parallel GEMM with the all-reduce in its epilogue (qf_w8a16_gemm_allreduce) are
covered.  All memory touched lies inside the two buffers, which are allocated with the full slot capacity.
"""
from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest

from oracle import w8a16_oracle as orc
from tests.conftest import from_dev_bf16, to_dev_bf16

pytestmark = pytest.mark.gpu
WAIT_US = 50_000
MAX_COUNT = 8192


@pytest.fixture()
def two_buffers(dev):
    import torch
    from qwen_a100_fastpath_b200 import _lib
    lib = _lib.LIB
    torch.cuda.synchronize(dev)
    nbytes = lib.qf_allreduce_buffer_bytes(MAX_COUNT)
    ptrs = []
    for _ in range(2):
        p = ctypes.c_void_p()
        assert lib.qf_symm_alloc(nbytes, ctypes.byref(p)) == 0, lib.qf_last_error_detail()
        ptrs.append(p.value)
    stream = torch.cuda.current_stream(dev).cuda_stream
    assert lib.qf_allreduce_set_wait(ptrs[0], WAIT_US, stream) == 0
    yield ptrs
    torch.cuda.synchronize(dev)
    for p in ptrs:
        lib.qf_symm_free(p)


def status(buf, stream):
    from qwen_a100_fastpath_b200 import _lib
    st = ctypes.c_int(-1)
    assert _lib.LIB.qf_allreduce_status(buf, stream, ctypes.byref(st)) == 0
    return st.value


def test_allreduce_wait_runs_out(dev, two_buffers):
    import torch
    from qwen_a100_fastpath_b200 import _lib
    lib = _lib.LIB
    stream = torch.cuda.current_stream(dev).cuda_stream
    x = torch.randn(MAX_COUNT, device=dev).to(torch.bfloat16)
    out = torch.empty_like(x)
    bufs2 = (ctypes.c_void_p * 2)(*two_buffers)
    t0 = time.perf_counter()
    assert lib.qf_allreduce_bf16(x.data_ptr(), out.data_ptr(), MAX_COUNT, MAX_COUNT, 0, 2, bufs2, 0, stream) == 0
    torch.cuda.synchronize(dev)
    elapsed = time.perf_counter() - t0
    assert 0.04 <= elapsed < 1.5, elapsed                     # the 50 ms bound, not the 2 s default
    assert status(two_buffers[0], stream) == _lib.QF_ERR_TIMEOUT
    assert status(two_buffers[0], stream) == 0                # read and cleared
    # the next call on the same buffer (one rank: nothing to wait for) succeeds and is exact
    bufs1 = (ctypes.c_void_p * 1)(two_buffers[0])
    assert lib.qf_allreduce_bf16(x.data_ptr(), out.data_ptr(), MAX_COUNT, MAX_COUNT, 0, 1, bufs1, 0, stream) == 0
    torch.cuda.synchronize(dev)
    assert torch.equal(out.view(torch.int16), x.view(torch.int16))
    assert status(two_buffers[0], stream) == 0


def test_fused_gemm_allreduce_wait_runs_out(dev, two_buffers):
    import torch
    from qwen_a100_fastpath_b200 import _lib
    lib = _lib.LIB
    stream = torch.cuda.current_stream(dev).cuda_stream
    M, N, K = 4, 1024, 512
    x_bits, W, s = orc.make_inputs(9, M, N, K)
    x = to_dev_bf16(x_bits, dev)
    w = torch.from_numpy(W).to(dev)
    sc = torch.from_numpy(s).to(dev)
    y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    ws_bytes = lib.qf_w8a16_workspace_bytes(M, N, K)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
    bufs2 = (ctypes.c_void_p * 2)(*two_buffers)
    t0 = time.perf_counter()
    rc = lib.qf_w8a16_gemm_allreduce(x.data_ptr(), K, w.data_ptr(), K, sc.data_ptr(), y.data_ptr(), N, M, N, K,
                                     ws.data_ptr(), ws_bytes, 0, 2, bufs2, MAX_COUNT, 0, stream)
    assert rc == 0, lib.qf_last_error_detail()
    torch.cuda.synchronize(dev)
    assert time.perf_counter() - t0 < 1.5
    assert status(two_buffers[0], stream) == _lib.QF_ERR_TIMEOUT
    st = ctypes.c_int(-1)
    assert lib.qf_workspace_status(ws.data_ptr(), stream, ctypes.byref(st)) == 0 and st.value == 0
    # one rank: the fused all-reduce is the plain GEMM's output, bit for bit
    bufs1 = (ctypes.c_void_p * 1)(two_buffers[0])
    rc = lib.qf_w8a16_gemm_allreduce(x.data_ptr(), K, w.data_ptr(), K, sc.data_ptr(), y.data_ptr(), N, M, N, K,
                                     ws.data_ptr(), ws_bytes, 0, 1, bufs1, MAX_COUNT, 0, stream)
    assert rc == 0, lib.qf_last_error_detail()
    y_plain = torch.empty_like(y)
    rc = lib.qf_w8a16_gemm(x.data_ptr(), K, w.data_ptr(), K, sc.data_ptr(), None, y_plain.data_ptr(), N,
                           _lib.QF_DTYPE_BF16, M, N, K, ws.data_ptr(), ws_bytes, 0, stream)
    assert rc == 0
    torch.cuda.synchronize(dev)
    assert np.array_equal(from_dev_bf16(y), from_dev_bf16(y_plain))
    assert status(two_buffers[0], stream) == 0
