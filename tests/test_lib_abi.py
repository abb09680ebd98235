"""The C-ABI library loads without a GPU, exports every entry point include/qf_b200.h declares, and rejects bad
arguments with the documented codes before any CUDA call is made."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from qwen_a100_fastpath_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "qf_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(qf_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for n in ("qf_w8a16_gemm", "qf_w8a16_head", "qf_w8a16_workspace_bytes", "qf_workspace_status"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    bound = {name for name, _, _ in _lib.SIGNATURES}
    assert set(declared_functions()) <= bound, "every declared entry point has a ctypes signature"


def test_abi_version_and_strerror():
    assert _lib.LIB.qf_abi_version() == _lib.ABI_VERSION
    assert _lib.LIB.qf_strerror(0) == b"ok"
    assert _lib.LIB.qf_strerror(-4).startswith(b"alignment")
    assert _lib.LIB.qf_strerror(12345) == b"unknown error"


def test_workspace_bytes_layout():
    small = _lib.LIB.qf_w8a16_workspace_bytes(1, 128, 128)
    big = _lib.LIB.qf_w8a16_workspace_bytes(16, 151936, 5120)
    assert 0 < small == big  # fixed size: tile counters, stream-K partial slots, per-CTA head statistics
    assert big < 8 << 20


FAKE = 1 << 20  # a 16-byte-aligned non-null address; validation rejects before dereferencing anything


def gemm(**kw):
    a = dict(x=FAKE, ldx=5120, w=FAKE, ldw=5120, scale=FAKE, bias=None, y=FAKE, ldy=5120, y_dtype=0, M=4, N=5120,
             K=5120, ws=FAKE, ws_bytes=1 << 30, flags=0, stream=None)
    a.update(kw)
    return _lib.LIB.qf_w8a16_gemm(*a.values())


@pytest.mark.parametrize("kw,code", [
    (dict(M=17), -2),                        # beyond the small-M path
    (dict(M=-1), -2),
    (dict(N=_lib.QF_MAX_N + 1), -2),
    (dict(scale=None), -1),
    (dict(ws=None), -1),
    (dict(ws_bytes=1024), -6),
    (dict(ldw=5000), -3),                    # ldw < K
    (dict(ldx=100), -3),
    (dict(ldw=5136 + 8), -4),                # ldw % 16 != 0
    (dict(w=FAKE + 8), -4),
    (dict(x=FAKE + 2), -4),
    (dict(ldx=5124), -4),                    # ldx % 8 != 0
    (dict(ws=FAKE + 16), -4),
    (dict(y_dtype=7), -8),
    (dict(y=None), -1),
    (dict(ldy=10), -3),
])
def test_gemm_argument_validation(kw, code):
    assert gemm(**kw) == code
    assert len(_lib.LIB.qf_last_error_detail()) > 0


def test_empty_problem_is_a_noop_without_cuda():
    assert gemm(M=0) == 0
    assert gemm(N=0) == 0


def test_head_argument_validation():
    f = _lib.LIB.qf_w8a16_head
    args = [FAKE, 5120, FAKE, 5120, FAKE, FAKE, 151936, 4, 151936, 5120, 151936, 0, FAKE, FAKE, FAKE, FAKE,
            1 << 30, 0, None]
    bad_nvalid = list(args)
    bad_nvalid[10] = 151937
    assert f(*bad_nvalid) == -2
    bad_stats = list(args)
    bad_stats[13] = None
    assert f(*bad_stats) == -1
    k0 = list(args)
    k0[9] = 0
    assert f(*k0) == -2


def allreduce(**kw):
    bufs = (ctypes.c_void_p * 8)(*([FAKE] * 8))
    a = dict(inp=FAKE, out=FAKE, count=5 * 5120, max_count=16 * 5120, rank=0, world=2, bufs=bufs, flags=0,
             stream=None)
    a.update(kw)
    return _lib.LIB.qf_allreduce_bf16(*a.values())


@pytest.mark.parametrize("kw,code", [
    (dict(world=0), -1),
    (dict(world=9), -1),
    (dict(rank=2), -1),
    (dict(count=16 * 5120 + 8), -2),           # above max_count
    (dict(count=12), -2),                      # not a multiple of 8
    (dict(max_count=256 * 1024 + 8), -2),      # above QF_AR_MAX_CHUNKS * 1024
    (dict(inp=FAKE + 8), -4),
    (dict(out=None), -1),
])
def test_allreduce_argument_validation(kw, code):
    assert allreduce(**kw) == code
    assert len(_lib.LIB.qf_last_error_detail()) > 0


def test_allreduce_empty_and_buffer_size():
    assert allreduce(count=0) == 0
    assert _lib.LIB.qf_allreduce_buffer_bytes(0) == 0
    small = _lib.LIB.qf_allreduce_buffer_bytes(8)
    big = _lib.LIB.qf_allreduce_buffer_bytes(16 * 5120)
    # one 16-byte line per 4 elements, 2 parities, 8 source slots
    assert big - small == (16 * 5120 - 8) * 4 * 2 * _lib.QF_AR_MAX_RANKS


@pytest.mark.parametrize("args,code", [
    ((FAKE, 5120, -1, 5120, FAKE, 5120, FAKE, None), -2),
    ((FAKE, 9000, 4, 9000, FAKE, 9000, FAKE, None), -2),      # rows wider than 8192
    ((None, 5120, 4, 5120, FAKE, 5120, FAKE, None), -1),
    ((FAKE, 100, 4, 5120, FAKE, 5120, FAKE, None), -3),      # ldw < H
])
def test_quantizer_argument_validation(args, code):
    assert _lib.LIB.qf_quantize_rows_int8(*args) == code
    assert _lib.LIB.qf_quantize_rows_int8(FAKE, 64, 0, 64, FAKE, 64, FAKE, None) == 0   # V == 0: no-op


def head_sample(**kw):
    a = dict(x=FAKE, ldx=5120, w=FAKE, ldw=5120, scale=FAKE, logits=FAKE, ldl=151936, M=4, N=151936, K=5120,
             n_valid=151936, vocab_offset=0, inv_temperature=1.0, seed=1, offset=0, row_max=FAKE, row_argmax=FAKE,
             row_lse=FAKE, row_sample=FAKE, row_sample_score=FAKE, row_sample_logit=FAKE, ws=FAKE,
             ws_bytes=1 << 30, flags=0, stream=None)
    a.update(kw)
    return _lib.LIB.qf_w8a16_head_sample(*a.values())


@pytest.mark.parametrize("kw,code", [
    (dict(inv_temperature=0.0), -1),
    (dict(inv_temperature=-2.0), -1),
    (dict(inv_temperature=float("inf")), -1),
    (dict(inv_temperature=float("nan")), -1),
    (dict(row_sample=None), -1),
    (dict(row_sample_logit=None), -1),
    (dict(n_valid=0), -2),
    (dict(vocab_offset=(1 << 32) - 100), -2),  # global columns must fit the generator's 32-bit counter word
])
def test_head_sample_argument_validation(kw, code):
    assert head_sample(**kw) == code


def spec_attn(**kw):
    a = dict(q=FAKE, sq_t=24 * 256, sq_h=256, k=FAKE, sk_b=800 * 4 * 512, sk_t=512, sk_h=800 * 512, v=FAKE + 512,
             sv_b=800 * 4 * 512, sv_t=512, sv_h=800 * 512, num_blocks=8, page=800, bt=FAKE, s_bt=8, lens=FAKE,
             out=FAKE, so_t=24 * 256, so_h=256, num_reqs=1, q_len=3, num_heads=24, num_kv_heads=4, head_size=256,
             scale=0.0625, ws=FAKE, ws_bytes=1 << 30, flags=0, stream=None)
    a.update(kw)
    return _lib.LIB.qf_spec_attn(*a.values())


@pytest.mark.parametrize("kw,code", [
    (dict(q_len=0), -2),
    (dict(num_heads=25), -2),                  # not a multiple of num_kv_heads
    (dict(head_size=96), -2),
    (dict(q_len=11), -2),                      # Q * G = 66 > 64
    (dict(page=8), -2),
    (dict(page=40), -2),                       # not a multiple of 16
    (dict(num_blocks=0), -2),
    (dict(scale=0.0), -1),
    (dict(scale=float("nan")), -1),
    (dict(lens=None), -1),
    (dict(ws=None), -1),
    (dict(q=FAKE + 8), -4),
    (dict(k=FAKE + 2), -4),
    (dict(sq_h=260), -3),                      # not a multiple of 8 elements
    (dict(sk_t=0), -3),
    (dict(sv_t=800 * 512 * 4, sv_h=512), -3),  # V's slot / head order differs from K's
    (dict(s_bt=0), -3),
    (dict(ws=FAKE + 64), -4),
])
def test_spec_attn_argument_validation(kw, code):
    assert spec_attn(**kw) == code
    assert len(_lib.LIB.qf_last_error_detail()) > 0


def test_spec_attn_empty_batch_and_workspace():
    assert spec_attn(num_reqs=0) == 0
    lib = _lib.LIB
    assert lib.qf_spec_attn_workspace_bytes(0, 3, 24, 4, 256) == 256
    # no GPU here: sized for 160 SMs, i.e. 160 / (num_reqs * HKV) = 40 splits of the 4 heads x 18 packed rows
    rows = 1 * 4 * 40 * 18
    assert lib.qf_spec_attn_workspace_bytes(1, 3, 24, 4, 256) == 256 + (rows * 256 * 4 + 255) // 256 * 256 + rows * 4
