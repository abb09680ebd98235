"""CPU baseline of the W8A16 decode-GEMM path (test/benchmark infrastructure only).

Times the reference's CPU expression of the path -- ``F.linear(x.float(), W.float() * ws[:, None])`` chunked
over 8192 output rows (bench/test_w8a16.py:15 of EurekaZang/qwen-a100-fastpath) -- on the host cores with
every available thread.  Only ``bench.py``'s ``cpu_baseline`` field and ``--impl reference`` arm use it; it is
never part of the product path.
"""
from __future__ import annotations

import os
import platform
import time

import torch
import torch.nn.functional as F

CHUNK_ROWS = 8192


def dequant_linear_f32(x: torch.Tensor, W: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """The reference's exact-product oracle on CPU tensors (bench/test_w8a16.py:15)."""
    return torch.cat([F.linear(x.float(), W[i:i + CHUNK_ROWS].float() * s[i:i + CHUNK_ROWS, None])
                      for i in range(0, W.shape[0], CHUNK_ROWS)], dim=1)


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


def make_layer(shapes, M: int, seed: int = 0):
    """Seeded int8 weights U[-127, 127], scales U(1e-3, 1e-2), bf16 activations N(0, 1) for each (N, K)."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for (N, K) in shapes:
        W = torch.randint(-127, 128, (N, K), dtype=torch.int8, generator=g)
        s = torch.rand(N, generator=g) * 0.009 + 0.001
        x = torch.randn(M, K, generator=g).to(torch.bfloat16)
        out.append((x, W, s))
    return out


def time_layer(layer, reps: int, threads: int | None = None):
    """Seconds per pass over ``layer`` (median of ``reps`` after one warm-up), and the thread count used."""
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    for x, W, s in layer:
        dequant_linear_f32(x, W, s)
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        for x, W, s in layer:
            dequant_linear_f32(x, W, s)
        times.append(time.perf_counter() - t0)
    times.sort()
    return times[len(times) // 2], threads
