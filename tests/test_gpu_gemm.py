"""CUDA W8A16 GEMM (libqf_b200 via the C ABI) against the CPU oracle and the reference's golden outputs.

Tolerances (north star): every bf16 output within one bf16 ulp of the oracle's correctly rounded result plus
2^-16 * max|y| (the fp32 accumulation noise of cancelling partial sums), >= 99 % of outputs bit-identical,
max relative error <= 2e-2 (observed ~1e-3, i.e. one ulp); the fp32 export (accumulator x scale before
rounding) within 1e-3 relative of the fp64 exact product (observed 2e-7 .. 9e-7).
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from oracle import w8a16_oracle as orc
from tests.conftest import from_dev_bf16, to_dev_bf16

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden"


def bf16_close(a_bits, b_bits, max_mismatch_frac=0.01):
    a = orc.bf16_to_f32(a_bits).astype(np.float64)
    b = orc.bf16_to_f32(b_bits).astype(np.float64)
    big = np.maximum(np.abs(a), np.abs(b)).astype(np.float32)
    ulp = np.spacing(big).astype(np.float64) * 2.0 ** 16
    # one bf16 ulp, plus the fp32 accumulation noise of the partial sums (outputs near zero come from
    # cancelling sums ~|y|max; their absolute error is set by those sums, not by their own ulp)
    atol = 2.0 ** -16 * np.abs(b).max()
    diff = np.abs(a - b)
    bad = diff > ulp + atol
    assert not bad.any(), f"{int(bad.sum())} outputs beyond 1 ulp + {atol:.3g}; worst diff {diff[bad].max()}"
    frac = float(np.mean(np.asarray(a_bits) != np.asarray(b_bits)))
    assert frac <= max_mismatch_frac, f"{frac:.4%} of outputs differ from the oracle"
    rel = diff.max() / max(np.abs(b).max(), 1e-30)
    assert rel <= 2e-2
    return frac


def bias_close(got_bits, x_bits, W, s, b_bits, max_mismatch_frac=0.01):
    """bf16(bf16(acc * s) + bias), the reference's two roundings (patches.py:96-97): a one-ulp difference of the
    pre-bias value (fp32 summation order) is carried into the sum unchanged, so the tolerance is one ulp of the
    pre-bias value plus one ulp of the result (plus the accumulation noise of bf16_close)."""
    pre_bits = orc.w8a16_mm(x_bits, W, s, "bf16")
    pre = orc.bf16_to_f32(pre_bits).astype(np.float64)
    ref_bits = orc.add_bias_bf16(pre_bits, b_bits)
    a = orc.bf16_to_f32(got_bits).astype(np.float64)
    b = orc.bf16_to_f32(ref_bits).astype(np.float64)
    ulp = lambda v: np.spacing(np.abs(v).astype(np.float32)).astype(np.float64) * 2.0 ** 16  # noqa: E731
    tol = ulp(pre) + ulp(np.maximum(np.abs(a), np.abs(b))) + 2.0 ** -16 * np.abs(pre).max()
    diff = np.abs(a - b)
    assert not (diff > tol).any(), f"{int((diff > tol).sum())} outputs beyond tolerance; worst {diff.max()}"
    assert float(np.mean(np.asarray(got_bits) != ref_bits)) <= max_mismatch_frac
    assert diff.max() / max(np.abs(b).max(), 1e-30) <= 2e-2


def run_case(dev, M, N, K, seed, ldx=None, ldw=None, out_dtype="bf16", bias=False, x_bits=None, W=None, s=None):
    import torch
    from qwen_a100_fastpath_b200.w8a16 import pick_config, w8a16_mm
    if x_bits is None:
        x_bits, W, s = orc.make_inputs(seed, M, N, K, x_row_stride=ldx)
    xt = to_dev_bf16(x_bits, dev)[:, :K]
    if ldw is None or ldw == K:
        wt = torch.from_numpy(W).to(dev).t()
    else:  # padded weight rows: [N, ldw] storage, [K, N] view with stride (1, ldw)
        Wp = np.zeros((N, ldw), np.int8)
        Wp[:, :K] = W
        wt = torch.from_numpy(Wp).to(dev)[:, :K].t()
    st = torch.from_numpy(s).to(dev)
    b_bits = orc.make_bias(seed + 7, N) if bias else None
    bt = to_dev_bf16(b_bits, dev) if bias else None
    y = w8a16_mm(xt, wt, st, pick_config(N, K), torch.float32 if out_dtype == "f32" else torch.bfloat16, bias=bt)
    torch.cuda.synchronize()
    return x_bits, W, s, b_bits, y


SHAPES = [
    # (N, K, M, ldx, ldw)
    (5120, 5120, 1, None, None),       # config 1
    (10240, 5120, 5, None, None),      # qkv at verification M
    (5120, 8192, 5, None, None),       # o_proj
    (5120, 2176, 16, None, None),      # down shard at TP=8 (K = 17 * 128)
    (1000, 1024, 5, 1040, None),       # ragged N, strided activation rows
    (100, 512, 3, None, None),
    (64, 256, 1, None, None),          # two CTAs share one tile
    (300, 200, 9, None, 208),          # K % 16 != 0, padded weight rows
    (384, 1000, 16, 1008, 1008),
    (1, 4096, 7, None, None),          # single output channel
    (4352, 128, 4, None, None),        # one k stage per tile
    (19072, 1024, 5, None, None),      # 149 tiles of 128 rows: one stream-K tile shared by 8 CTAs
    (37984, 512, 12, None, None),      # two token tiles, 2 whole tiles per CTA + 1 stream-K tile
    (17024, 256, 3, None, None),       # 64-row tiles
    (4352, 5120, 5, None, None),       # gate_up shard at TP=8: data-parallel grid, 136 CTAs of one 32-row tile
    (8704, 5120, 16, None, None),      # gate_up shard at TP=4: data-parallel grid, 136 CTAs of one 64-row tile
]


@pytest.mark.parametrize("N,K,M,ldx,ldw", SHAPES, ids=lambda v: str(v))
def test_gemm_matches_oracle(dev, N, K, M, ldx, ldw):
    x, W, s, _, y = run_case(dev, M, N, K, seed=N * 7 + K + M, ldx=ldx, ldw=ldw)
    bf16_close(from_dev_bf16(y), orc.w8a16_mm(x, W, s, "bf16", K=K))


@pytest.mark.parametrize("M", list(range(1, 17)))
def test_every_m(dev, M):
    N, K = 2304, 1536
    x, W, s, _, y = run_case(dev, M, N, K, seed=100 + M)
    bf16_close(from_dev_bf16(y), orc.w8a16_mm(x, W, s, "bf16"))


@pytest.mark.parametrize("N,K,M", [(5120, 5120, 1), (5120, 17408, 16), (1000, 1024, 5), (64, 256, 3)])
def test_fp32_accumulator_parity(dev, N, K, M):
    x, W, s, _, y = run_case(dev, M, N, K, seed=11 + M, out_dtype="f32")
    ref = orc.dequant_matmul_f64(x, W, s)
    got = y.cpu().numpy().astype(np.float64)
    rel_inf = np.abs(got - ref).max() / np.abs(ref).max()
    rel_fro = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert rel_inf <= 1e-3 and rel_fro <= 1e-4, (rel_inf, rel_fro)


@pytest.mark.parametrize("N,K,M", [(384, 512, 6), (5120, 5120, 5)])
def test_bias_rounds_like_reference(dev, N, K, M):
    x, W, s, b, y = run_case(dev, M, N, K, seed=77, bias=True)
    bias_close(from_dev_bf16(y), x, W, s, b)


def test_golden_reference_outputs(dev):
    """The CUDA kernel reproduces the reference Triton kernel's own outputs (tests/golden)."""
    meta = json.loads((GOLD / "reference_outputs.json").read_text())
    arr = np.load(GOLD / "reference_outputs.npz")
    for c in meta["gemm"]:
        ldx = c["ldx"] if c["ldx"] != c["K"] else None
        *_, y = run_case(dev, c["M"], c["N"], c["K"], c["seed"], ldx=ldx)
        bf16_close(from_dev_bf16(y), arr[f"gemm{c['case']}_y"])


def test_deterministic_and_workspace_reuse(dev):
    """Same inputs -> bit-identical outputs; interleaving shapes on one workspace leaves it consistent."""
    import torch
    a = run_case(dev, 5, 5120, 8192, seed=3)
    b = run_case(dev, 3, 100, 512, seed=4)
    c = run_case(dev, 5, 5120, 8192, seed=3)
    assert torch.equal(a[-1], c[-1])
    bf16_close(from_dev_bf16(b[-1]), orc.w8a16_mm(b[0], b[1], b[2], "bf16"))
    from qwen_a100_fastpath_b200.w8a16 import workspace_status
    assert workspace_status() == 0


def test_k_zero_and_empty(dev):
    import torch
    from qwen_a100_fastpath_b200.w8a16 import w8a16_mm
    x = torch.zeros((3, 0), dtype=torch.bfloat16, device=dev)
    w = torch.zeros((0, 64), dtype=torch.int8, device=dev)
    s = torch.ones(64, dtype=torch.float32, device=dev)
    bias = torch.full((64,), 0.5, dtype=torch.bfloat16, device=dev)
    y = w8a16_mm(x, w, s, None, torch.bfloat16, bias=bias)
    assert torch.equal(y, torch.full((3, 64), 0.5, dtype=torch.bfloat16, device=dev))
    e = w8a16_mm(torch.zeros((0, 128), dtype=torch.bfloat16, device=dev),
                 torch.zeros((64, 128), dtype=torch.int8, device=dev).t(), s, None, torch.bfloat16)
    assert e.shape == (0, 64)


def test_cpu_tensors_are_rejected():
    """No CPU fallback: the op refuses host tensors."""
    import torch
    from qwen_a100_fastpath_b200.w8a16 import w8a16_mm
    with pytest.raises(ValueError):
        w8a16_mm(torch.zeros((1, 128), dtype=torch.bfloat16), torch.zeros((64, 128), dtype=torch.int8).t(),
                 torch.ones(64), None, torch.bfloat16)


def test_cuda_graph_and_pdl_chain(dev):
    """A captured chain of launches (with programmatic dependent launch) replays correctly on new inputs."""
    import torch
    from qwen_a100_fastpath_b200.w8a16 import w8a16_mm
    N1, K1, N2 = 2048, 1024, 768
    x_bits, W1, s1 = orc.make_inputs(21, 4, N1, K1)
    _, W2, s2 = orc.make_inputs(22, 4, N2, N1)
    w1 = torch.from_numpy(W1).to(dev).t()
    w2 = torch.from_numpy(W2).to(dev).t()
    t1, t2 = torch.from_numpy(s1).to(dev), torch.from_numpy(s2).to(dev)
    x = to_dev_bf16(x_bits, dev)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        y2 = w8a16_mm(w8a16_mm(x, w1, t1, None, torch.bfloat16, pdl=True), w2, t2, None, torch.bfloat16, pdl=True)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            y1g = w8a16_mm(x, w1, t1, None, torch.bfloat16, pdl=True)
            y2g = w8a16_mm(y1g, w2, t2, None, torch.bfloat16, pdl=True)
    stream.synchronize()
    ref1 = orc.w8a16_mm(x_bits, W1, s1, "bf16")
    bf16_close(from_dev_bf16(y2), orc.w8a16_mm(ref1, W2, s2, "bf16"), max_mismatch_frac=0.02)
    x_bits2, _, _ = orc.make_inputs(23, 4, N1, K1)
    x.copy_(to_dev_bf16(x_bits2, dev))
    g.replay()
    torch.cuda.synchronize()
    r1 = orc.w8a16_mm(x_bits2, W1, s1, "bf16")
    bf16_close(from_dev_bf16(y1g), r1)
    bf16_close(from_dev_bf16(y2g), orc.w8a16_mm(from_dev_bf16(y1g), W2, s2, "bf16"))


@pytest.mark.parametrize("name,N,K", [("qkv", 10240, 5120), ("o_proj", 5120, 8192), ("gate_up", 34816, 5120),
                                      ("down", 5120, 17408)])
def test_full_size_config2_against_torch_fp32(dev, name, N, K):
    """Full BASELINE config-2 shapes at M=5 against the reference's fp32 dequant-matmul run on the GPU
    (bench/test_w8a16.py:15, torch fp32 without TF32)."""
    import torch
    import torch.nn.functional as F
    from qwen_a100_fastpath_b200.w8a16 import w8a16_mm
    g = torch.Generator(device=dev).manual_seed(N + K)
    W = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
    s = torch.rand(N, device=dev, generator=g) * 0.009 + 0.001
    x = torch.randn(5, K, device=dev, generator=g).to(torch.bfloat16)
    torch.backends.cuda.matmul.allow_tf32 = False
    ref = torch.cat([F.linear(x.float(), W[i:i + 8192].float() * s[i:i + 8192, None]) for i in range(0, N, 8192)], 1)
    y32 = w8a16_mm(x, W.t(), s, None, torch.float32)
    y16 = w8a16_mm(x, W.t(), s, None, torch.bfloat16)
    rel32 = ((y32 - ref).norm() / ref.norm()).item()
    rel16 = ((y16.float() - ref).norm() / ref.norm()).item()
    assert rel32 < 1e-5, rel32
    assert rel16 < 3e-3, rel16                      # bf16 output rounding (reference reports 0.0016-0.0017)
    assert torch.equal(y16, y32.to(torch.bfloat16)) or (y16 != y32.to(torch.bfloat16)).float().mean() < 1e-3


@pytest.mark.parametrize("M", [1, 5, 12])
def test_activation_range_fallback(dev, M):
    """Stages whose activations fall outside the fp16 range (|x| >= 65536, here up to 3e5) take the exact bf16
    path; tiny activations (fp16 subnormal range) stay within the tolerance; results match the oracle."""
    N, K = 1536, 3072
    x, W, s = orc.make_inputs(900 + M, M, N, K)
    xf = orc.bf16_to_f32(x).copy()
    xf[0, 130] = 3.0e5          # k-stage 1 of row 0 falls back
    xf[M - 1, 2900] = -7.0e4    # last stage
    xf[:, 1024:1100] *= 1e-6    # tiny values on the fp16 path
    x2 = orc.f32_to_bf16(xf)
    *_, y = run_case(dev, M, N, K, seed=0, x_bits=x2, W=W, s=s)
    bf16_close(from_dev_bf16(y), orc.w8a16_mm(x2, W, s, "bf16"))
    *_, y32 = run_case(dev, M, N, K, seed=0, x_bits=x2, W=W, s=s, out_dtype="f32")
    ref = orc.dequant_matmul_f64(x2, W, s)
    got = y32.cpu().numpy().astype(np.float64)
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= 1e-5


def test_nan_activation_propagates(dev):
    N, K, M = 512, 1024, 3
    x, W, s = orc.make_inputs(77, M, N, K)
    x = x.copy()
    x[1, 500] = 0x7FC0  # NaN in row 1 only
    *_, y = run_case(dev, M, N, K, seed=0, x_bits=x, W=W, s=s)
    yf = y.float().cpu().numpy()
    assert np.isnan(yf[1]).all() and np.isfinite(yf[[0, 2]]).all()


@pytest.mark.parametrize("I,K,M", [(17408, 5120, 5), (17408, 5120, 16), (1000, 1024, 3), (4352, 5120, 1),
                                   (8704, 2048, 12)])
def test_fused_silu_mul_gate_up(dev, I, K, M):
    """qf_w8a16_gemm_silu_mul == vLLM's SiluAndMul (oracle.silu_mul) on the gate_up GEMM output: against the oracle's
    own GEMM, and against torch's F.silu(y[:, :I]) * y[:, I:] on this library's plain GEMM output (the fused kernel
    splits tiles differently, so a few outputs may differ by the bf16 ulp their inputs differ by)."""
    import torch
    import torch.nn.functional as F
    from qwen_a100_fastpath_b200.w8a16 import w8a16_mm, w8a16_mm_silu_mul
    x_bits, W, s = orc.make_inputs(3 * I + K + M, M, 2 * I, K)
    x = to_dev_bf16(x_bits, dev)
    wt = torch.from_numpy(W).to(dev).t()
    st = torch.from_numpy(s).to(dev)
    out = w8a16_mm_silu_mul(x, wt, st)
    y = w8a16_mm(x, wt, st, None, torch.bfloat16)
    ref_gpu = F.silu(y[:, :I]) * y[:, I:]
    torch.cuda.synchronize()
    silu_close(from_dev_bf16(out), from_dev_bf16(ref_gpu), from_dev_bf16(y), I)
    y_orc = orc.w8a16_mm(x_bits, W, s, "bf16")
    silu_close(from_dev_bf16(out), orc.silu_mul(y_orc, I), y_orc, I)


def silu_close(out_bits, ref_bits, y_bits, I, max_mismatch_frac=0.02):
    """The fused activation against a reference built from gate/up values ``y`` that may each differ from the
    kernel's by one bf16 ulp (fp32 summation order): the tolerance propagates those ulps through
    ``silu(g) * u`` (|d/du| = |silu(g)|, |d/dg| <= 1.1 |u|) plus one ulp of the output and 2^-16 max|ref|."""
    def ulp(v):
        return np.spacing(np.abs(v).astype(np.float32)).astype(np.float64) * 2.0 ** 16
    out = orc.bf16_to_f32(out_bits).astype(np.float64)
    ref = orc.bf16_to_f32(ref_bits).astype(np.float64)
    y = orc.bf16_to_f32(y_bits).astype(np.float64)
    g, u = y[:, :I], y[:, I:2 * I]
    silu = g / (1.0 + np.exp(-np.clip(g, -80, 80)))
    tol = ulp(np.maximum(np.abs(out), np.abs(ref))) + np.abs(silu) * ulp(u) + 1.1 * np.abs(u) * ulp(g) + \
        2.0 ** -16 * np.abs(ref).max()
    bad = np.abs(out - ref) > tol
    assert not bad.any(), f"{int(bad.sum())} outputs beyond the propagated tolerance"
    assert np.mean(np.asarray(out_bits) != np.asarray(ref_bits)) <= max_mismatch_frac
