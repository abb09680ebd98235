#!/usr/bin/env python
"""Benchmark of the B200 W8A16 decode-GEMM path (one JSON line on rank 0).

Workload: one speculative-verification decode step of a 64-layer Qwen3-style dense model at M = 5 rows:
per layer qkv 10240x5120, o_proj 5120x8192, gate_up 34816x5120, down 5120x17408, plus the int8 MTP draft
LM head 151936x5120 with fused (max, argmax, logsumexp): 23.93 GB of int8 weights, synthetic (seeded int8
U[-127,127], per-channel scales U(1e-3,1e-2), bf16 N(0,1) activations, random-init; no checkpoint).
With --gpus N the step is tensor-parallel: column-parallel qkv / gate_up / head (vocab shards), row-parallel
o_proj / down with an NCCL all-reduce of the bf16 [5, 5120] partial sums, and an all-gather of the per-shard
(max, argmax, lse) of the head.

``value`` is the whole-job rate: algorithmic bytes of the step (int8 weights + fp32 scales + bf16 inputs and
outputs, summed over ranks) / device time per step, with everything resident in HBM.  ``e2e`` is the same
metric through the public plugin op (``qf_int8_linear``) with the step's activations copied in from pinned
host memory and the head's statistics copied back, inside the timed region.  ``--impl reference`` times the
reference's CPU path (torch fp32 dequant-matmul, bench/test_w8a16.py:15 of the reference) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "W8A16 decode GEMM µs & HBM GB/s (% of peak) at M=1–16; 64-layer step µs @1/2/4/8"
# (name, N, K, parallel style)
LAYER = [("qkv", 10240, 5120, "col"), ("o_proj", 5120, 8192, "row"), ("gate_up", 34816, 5120, "col"),
         ("down", 5120, 17408, "row")]
HEAD = ("lm_head", 151936, 5120, "vocab")
NOMINAL_HBM_GBS = 8000.0


def alg_bytes(N: int, K: int, M: int, head: bool = False) -> int:
    """Algorithmic bytes of one GEMM: int8 weights + fp32 scales + bf16 x + bf16 y (+ 12 B/row statistics)."""
    return N * K + 4 * N + 2 * M * K + 2 * M * N + (12 * M if head else 0)


def shard(N: int, K: int, style: str, world: int):
    if style in ("col", "vocab"):
        assert N % world == 0
        return N // world, K
    assert K % world == 0
    return N, K // world


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=64)
    ap.add_argument("--m", type=int, default=5)
    ap.add_argument("--no-pdl", action="store_true")
    ap.add_argument("--allreduce", choices=["fused", "nvlink", "nccl"], default="fused",
                    help="row-parallel partial-sum all-reduce with TP > 1: fused into the GEMM epilogue over NVLink, "
                         "the standalone NVLink one-shot kernel, or NCCL")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-attn", action="store_true", help="skip the verification-attention figure added to the line")
    ap.add_argument("--sweep", action="store_true", help="per-shape table (config 4) instead of the step")
    ap.add_argument("--sweep-out", default="")
    ap.add_argument("--ref-triton", action="store_true", help="with --sweep: also time the reference's own Triton "
                    "kernel (w8a16_mm with its pick_config, from the reference installed in baseline/_ref)")
    ap.add_argument("--prefill-sweep", action="store_true", help="the M > 16 int8 path (qf_w8a8_gemm: per-token "
                    "quantization + tcgen05 GEMM) on every config-2 GEMM at M = 32..4096, beside torch._int_mm")
    ap.add_argument("--fused-sweep", action="store_true", help="RMSNorm fused into qkv and RMSNorm + SiLU fused into "
                    "gate_up (qf_w8a16_gemm_rmsnorm) against vLLM's RMSNorm in torch followed by the GEMM, at M = 1..16")
    ap.add_argument("--host-overhead", action="store_true", help="eager host time per call of the public entry "
                    "points (enqueue only) against the kernel's device time, o_proj at --m")
    ap.add_argument("--attn-sweep", action="store_true", help="verification attention (qf_spec_attn) on the reference's "
                    "attention shapes at context 0..100K beside FlashAttention-2 (and, with --ref-triton, the "
                    "reference's own Triton kernels)")
    ap.add_argument("--profile-attn", type=int, default=-1, help="a few launches of the verification attention at this "
                    "context (Q = 3, one request; the small case for an ncu capture), then exit")
    ap.add_argument("--profile-gemm", default="", help="comma list of qkv,o_proj,gate_up,down,lm_head,lm_head_sample "
                    "(or pf_qkv, pf_o_proj, pf_gate_up, pf_down: the prefill path): a few launches of each at --m (the "
                    "small case for an ncu capture), then exit")
    return ap.parse_args()


# ---------------------------------------------------------------------------------------------------------
# clocks during the timed region (NVML reads only)
# ---------------------------------------------------------------------------------------------------------
class ClockSampler:
    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, index: int, period_s: float = 0.02):
        self.index, self.period = index, period_s
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001
            self._nv = None
            return self
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def __exit__(self, *exc):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}


# ---------------------------------------------------------------------------------------------------------
def cpu_sample(M: int, reps: int = 3):
    """Reference CPU path (torch fp32 dequant-matmul) on one decoder layer's four GEMMs: bounded sample."""
    from oracle import cpu_baseline as cb
    layer = cb.make_layer([(N, K) for _, N, K, _ in LAYER], M, seed=0)
    sec, threads = cb.time_layer(layer, reps)
    nbytes = sum(alg_bytes(N, K, M) for _, N, K, _ in LAYER)
    return {"value": nbytes / sec / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"one decoder layer (qkv, o_proj, gate_up, down) at M={M}: {nbytes / 1e6:.1f} MB of "
                      f"algorithmic bytes per pass, median of {reps} passes after 1 warm-up, torch "
                      f"F.linear(x.float(), W.float()*s) chunked over 8192 rows",
            "cpu": cb.cpu_model(), "sec_per_layer": sec}


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return
    M = args.m
    from oracle import cpu_baseline as cb
    layer = cb.make_layer([(N, K) for _, N, K, _ in LAYER], M, seed=0)
    nbytes = sum(alg_bytes(N, K, M) for _, N, K, _ in LAYER)
    steps, warmup = max(1, min(args.steps, 5)), max(0, min(args.warmup, 1))
    torch_threads = os.cpu_count() or 1
    import torch
    torch.set_num_threads(torch_threads)
    for _ in range(warmup):
        for x, W, s in layer:
            cb.dequant_linear_f32(x, W, s)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        for x, W, s in layer:
            cb.dequant_linear_f32(x, W, s)
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    v = nbytes / sec / 1e9
    line = {"metric": METRIC, "value": round(v, 3), "unit": "GB/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": "64-layer dense decode step, M=5 (config 5); CPU sample: one layer's "
                                   "4 GEMMs per step", "m": M, "layers_sampled": 1},
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": torch_threads, "kind": "port",
                             "sample": "one decoder layer (qkv, o_proj, gate_up, down) at M=5 per step, "
                                       "torch fp32 dequant-matmul", "cpu": cb.cpu_model()},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------------------
class Step:
    """Weights, activation buffers and the launch sequence of one tensor-parallel decode step."""

    def __init__(self, layers: int, M: int, rank: int, world: int, dev, pdl: bool, allreduce: str = "nvlink"):
        import torch
        self.torch = torch
        self.M, self.rank, self.world, self.dev, self.pdl = M, rank, world, dev, pdl
        self.ar = None
        self.ar_off = False  # tensor-parallel breakdown only: row-parallel shards without their all-reduce
        self.fused = world > 1 and allreduce == "fused"
        if world > 1 and allreduce in ("nvlink", "fused"):
            from qwen_a100_fastpath_b200.tp import NVLinkAllReduce
            self.ar = NVLinkAllReduce(M * max(N for _, N, _, st in LAYER if st == "row"))
        g = torch.Generator(device=dev).manual_seed(1234 + rank)
        self.layers = []
        for _ in range(layers):
            ws = {}
            for name, N, K, style in LAYER:
                n, k = shard(N, K, style, world)
                W = torch.randint(-127, 128, (n, k), dtype=torch.int8, device=dev, generator=g)
                s = torch.rand(n, device=dev, generator=g) * 0.009 + 0.001
                ws[name] = (W.t(), s)
            self.layers.append(ws)
        n, k = shard(HEAD[1], HEAD[2], HEAD[3], world)
        self.head_w = (torch.randint(-127, 128, (n, k), dtype=torch.int8, device=dev, generator=g).t(),
                       torch.rand(n, device=dev, generator=g) * 0.009 + 0.001)
        self.head_n = n
        self.x, self.y = {}, {}
        for name, N, K, style in LAYER:
            n, k = shard(N, K, style, world)
            self.x[name] = torch.randn(M, k, device=dev, generator=g).to(torch.bfloat16)
            self.y[name] = torch.empty(M, n, device=dev, dtype=torch.bfloat16)
        self.hidden = torch.randn(M, HEAD[2], device=dev, generator=g).to(torch.bfloat16)
        self.logits = torch.empty(M, self.head_n, device=dev, dtype=torch.bfloat16)
        self.row_max = torch.empty(M, device=dev, dtype=torch.float32)
        self.row_arg = torch.empty(M, device=dev, dtype=torch.int64)
        self.row_lse = torch.empty(M, device=dev, dtype=torch.float32)
        self.gathered = torch.empty(world, M, 3, device=dev, dtype=torch.float64)
        self.launches_per_step = layers * len(LAYER) + 1
        self.bytes_rank = layers * sum(alg_bytes(*shard(N, K, st, world), M) for _, N, K, st in LAYER) + \
            alg_bytes(self.head_n, HEAD[2], M, head=True)

    def gemm_bytes(self, name: str) -> int:
        for nm, N, K, st in LAYER:
            if nm == name:
                return alg_bytes(*shard(N, K, st, self.world), self.M)
        raise KeyError(name)

    def run(self, linear=None, events=None, phase_events=None):
        """Enqueue the step.  ``linear(x, w_t, s) -> y`` replaces the GEMM call (the public op allocates its
        output); ``events`` records a CUDA event after every launch (instrumented pass, PDL off);
        ``phase_events`` records three events: step start, after the last decoder GEMM, after the head."""
        torch = self.torch
        from qwen_a100_fastpath_b200 import tp
        from qwen_a100_fastpath_b200.w8a16 import w8a16_head, w8a16_mm, w8a16_mm_allreduce
        if events is not None:
            events[0].record()
        if phase_events is not None:
            phase_events[0].record()
        e = 1
        for ws in self.layers:
            for name, _, _, style in LAYER:
                w, s = ws[name]
                fused_row = self.fused and style == "row" and not self.ar_off
                if fused_row:  # row-parallel GEMM with the all-reduce in its epilogue
                    y = w8a16_mm_allreduce(self.x[name], w, s, self.ar, out=None if linear else self.y[name],
                                           pdl=self.pdl)
                elif linear is None:
                    y = w8a16_mm(self.x[name], w, s, None, torch.bfloat16, out=self.y[name], pdl=self.pdl)
                else:
                    y = linear(self.x[name], w, s)
                if events is not None:
                    events[e].record()
                    e += 1
                if style == "row" and self.world > 1 and not fused_row and not self.ar_off:
                    if self.ar is not None:
                        self.ar(y, pdl=self.pdl)
                    else:
                        tp.all_reduce_partial(y)
        if phase_events is not None:
            phase_events[1].record()
        w, s = self.head_w
        w8a16_head(self.hidden, w, s, n_valid=self.head_n, vocab_offset=self.rank * self.head_n, pdl=self.pdl,
                   out=(self.logits, self.row_max, self.row_arg, self.row_lse))
        if events is not None:
            events[e].record()
        if phase_events is not None:
            phase_events[2].record()
        if self.world > 1:
            mx, am, lse = tp.gather_head_stats(self.row_max, self.row_arg, self.row_lse, out=self.gathered)
            self.row_max.copy_(mx)
            self.row_arg.copy_(am)
            self.row_lse.copy_(lse)


def time_graph(graph, stream, steps, warmup, sampler=None):
    import torch
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            graph.replay()
    torch.cuda.synchronize()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if sampler:
        sampler.__enter__()
    with torch.cuda.stream(stream):
        ev0.record()
        for _ in range(steps):
            graph.replay()
        ev1.record()
    torch.cuda.synchronize()
    if sampler:
        sampler.__exit__(None, None, None)
    barrier()
    return ev0.elapsed_time(ev1) / steps


def barrier():
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        dist.barrier()


def max_over_ranks(v: float) -> float:
    import torch
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return v


def traffic_from_profiles():
    """DRAM bytes per launch of the dominant kernel, read from the committed ncu summary of the M = 5 step (not
    measured by this run: ncu cannot run inside a timed bench).  Returns (bytes, source file)."""
    p = REPO / "profiles" / "w8a16_gemm_step_m5_ncu.md"
    if not p.exists():
        return None, None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1].split()[0]), p.name
    return None, None


def peak_hbm():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, copy)"
    return 6650.0, "fallback (6.65 TB/s)"


def run_ours(args, rank: int, world: int, local: int):
    import torch
    import torch.distributed as dist
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=180))
    torch.backends.cuda.matmul.allow_tf32 = False
    pdl = not args.no_pdl
    st = Step(args.layers, args.m, rank, world, dev, pdl, args.allreduce)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        st.run()                       # eager warm-up: workspace for this stream, NCCL communicators
        st.run()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        st.run()
    torch.cuda.synchronize()

    sampler = ClockSampler(local) if rank == 0 else None
    ms = time_graph(graph, stream, args.steps, args.warmup, sampler)
    ms = max_over_ranks(ms)
    total_bytes = st.bytes_rank * world
    value = total_bytes / (ms * 1e-3) / 1e9

    # ---- per-launch durations of the dominant kernel
    # (1) the step as timed (PDL on), with events only at the step start, after the last decoder GEMM and after
    #     the head: the decoder-GEMM phase / its launch count is the kernel's average launch duration in the
    #     running workload (world == 1; with TP the phase also holds the all-reduces)
    phase = None
    if True:  # with TP the decoder-GEMM phase also holds the all-reduces (reported apart below)
        try:
            pev = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(3)]
            gp = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gp, stream=stream):
                st.run(phase_events=pev)
            with torch.cuda.stream(stream):
                for _ in range(3):
                    gp.replay()
            torch.cuda.synchronize()
            g_ms, h_ms = [], []
            for _ in range(max(5, min(args.steps, 40))):
                with torch.cuda.stream(stream):
                    gp.replay()
                torch.cuda.synchronize()
                g_ms.append(pev[0].elapsed_time(pev[1]))
                h_ms.append(pev[1].elapsed_time(pev[2]))
            del gp
            phase = (statistics.median(g_ms), statistics.median(h_ms))
        except Exception as e:  # noqa: BLE001
            phase = None
            print(f"phase timing failed: {e!r}", file=sys.stderr)
    # (2) instrumented replay (events between launches, PDL off): per-GEMM breakdown, and the headline with TP
    roofline = None
    try:
        n_ev = st.launches_per_step + 1
        events = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(n_ev)]
        g2 = torch.cuda.CUDAGraph()
        saved_pdl = st.pdl
        st.pdl = False
        with torch.cuda.graph(g2, stream=stream):
            st.run(events=events)
        st.pdl = saved_pdl
        reps = 5
        gemm_ms, head_ms = [], []
        with torch.cuda.stream(stream):
            g2.replay()
        torch.cuda.synchronize()
        for _ in range(reps):
            with torch.cuda.stream(stream):
                g2.replay()
            torch.cuda.synchronize()
            d = [events[i].elapsed_time(events[i + 1]) for i in range(n_ev - 1)]
            gemm_ms.append(sum(d[:-1]))
            head_ms.append(d[-1])
        del g2
        n_gemm = st.launches_per_step - 1
        iso_launch_ms = statistics.median(gemm_ms) / n_gemm
        per_launch_ms = phase[0] / n_gemm if (phase and world == 1) else iso_launch_ms
        gemm_bytes = sum(st.gemm_bytes(nm) for nm, *_ in LAYER) * args.layers / n_gemm
        peak, peak_src = peak_hbm()
        achieved = gemm_bytes / (per_launch_ms * 1e-3) / 1e9
        traffic, tsrc = traffic_from_profiles()
        head_launch_ms = phase[1] if (phase and world == 1) else statistics.median(head_ms)
        head_bytes = alg_bytes(st.head_n, HEAD[2], args.m, head=True)
        roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(achieved / peak, 4), "traffic": traffic,
                    "kernel": "w8a16_kernel<BN, NT=1> (qkv/o_proj/gate_up/down launches of the step)",
                    "bytes_per_launch": round(gemm_bytes), "us_per_launch": round(per_launch_ms * 1e3, 3),
                    "peak_source": peak_src + ", 'of measured'", "frac_of_nominal_8TBs": round(achieved / NOMINAL_HBM_GBS, 4),
                    "traffic_source": (f"profiles/{tsrc}: ncu dram__bytes_read.sum + dram__bytes_write.sum per "
                                       "launch of the decoder GEMMs of a committed M=5 step capture, not measured "
                                       "by this run" if tsrc else None),
                    "timing": ("decoder-GEMM phase of the step graph (PDL on) between CUDA events at the step start "
                               "and after the last GEMM, / 256 launches, median over replays" if (phase and world == 1)
                               else
                               "CUDA events around every launch of a replay of the same step (PDL off), median of 5"),
                    "us_per_launch_isolated": round(iso_launch_ms * 1e3, 3),
                    "head": {"us": round(head_launch_ms * 1e3, 2),
                             "GBps": round(head_bytes / (head_launch_ms * 1e-3) / 1e9, 1),
                             "frac": round(head_bytes / (head_launch_ms * 1e-3) / 1e9 / peak, 4)},
                    "per_gemm_us": {}}
        # per-GEMM-kind medians from the last replay
        d = [events[i].elapsed_time(events[i + 1]) for i in range(n_ev - 1)]
        for j, (nm, *_r) in enumerate(LAYER):
            vals = d[j:n_gemm:len(LAYER)]
            us = statistics.median(vals) * 1e3
            roofline["per_gemm_us"][nm] = {"us_isolated": round(us, 2),
                                           "GBps": round(st.gemm_bytes(nm) / (us * 1e-6) / 1e9, 1)}
        if world > 1:
            # where the time goes with TP: the same instrumented replay with the row-parallel shards run as plain
            # GEMMs (no all-reduce); every rank runs it, so the collectives stay in step
            st.ar_off = True
            g3 = torch.cuda.CUDAGraph()
            st.pdl = False
            with torch.cuda.graph(g3, stream=stream):
                st.run(events=events)
            st.pdl = saved_pdl
            st.ar_off = False
            with torch.cuda.stream(stream):
                g3.replay()
            torch.cuda.synchronize()
            plain = {nm: [] for nm, *_r in LAYER}
            for _ in range(reps):
                with torch.cuda.stream(stream):
                    g3.replay()
                torch.cuda.synchronize()
                d3 = [events[i].elapsed_time(events[i + 1]) for i in range(n_ev - 1)]
                for j, (nm, *_r) in enumerate(LAYER):
                    plain[nm].append(statistics.median(d3[j:n_gemm:len(LAYER)]))
            del g3
            tpb = {"decoder_phase_us_per_layer": round(phase[0] * 1e3 / args.layers, 2) if phase else None,
                   "row_parallel_us": {}, "timing": "CUDA events around every launch (PDL off), median"}
            extra_ms = 0.0
            for nm, _n, _k, style in LAYER:
                if style != "row":
                    continue
                with_ar = roofline["per_gemm_us"][nm]["us_isolated"]
                gemm_only = statistics.median(plain[nm]) * 1e3
                tpb["row_parallel_us"][nm] = {"with_allreduce": with_ar, "gemm_only": round(gemm_only, 2),
                                              "allreduce": round(with_ar - gemm_only, 2)}
                extra_ms += (with_ar - gemm_only) * 1e-3 * args.layers
            tpb["allreduce_ms_per_step"] = round(extra_ms, 3)
            tpb["allreduce_share_of_step"] = round(extra_ms / ms, 4)
            roofline["tp"] = tpb
    except Exception as e:  # noqa: BLE001
        roofline = {"error": f"instrumented replay failed: {e!r}"}

    # ---- e2e through the public plugin op with host copies in the timed region
    e2e = None
    if not args.no_e2e:
        from qwen_a100_fastpath_b200.patches import make_int8_linear_op
        op, _ = make_int8_linear_op()
        host_in = {k: v.cpu().pin_memory() for k, v in st.x.items()}
        host_hidden = st.hidden.cpu().pin_memory()
        host_out = [torch.empty_like(t, device="cpu").pin_memory() for t in (st.row_max, st.row_arg, st.row_lse)]

        def linear(x, w, s):
            return op(x, w, s, None)

        g3 = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            st.run(linear=linear)
        torch.cuda.synchronize()
        with torch.cuda.graph(g3, stream=stream):
            for k, v in st.x.items():
                v.copy_(host_in[k], non_blocking=True)
            st.hidden.copy_(host_hidden, non_blocking=True)
            st.run(linear=linear)
            for h, d_ in zip(host_out, (st.row_max, st.row_arg, st.row_lse)):
                h.copy_(d_, non_blocking=True)
        torch.cuda.synchronize()
        ms_e2e = max_over_ranks(time_graph(g3, stream, args.steps, args.warmup))
        h2d = sum(v.numel() * v.element_size() for v in host_in.values()) + host_hidden.numel() * 2
        d2h = sum(h.numel() * h.element_size() for h in host_out)
        e2e = {"value": round(total_bytes / (ms_e2e * 1e-3) / 1e9, 1), "unit": "GB/s",
               "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
               "ms_per_step": round(ms_e2e, 4),
               "path": "torch.ops.vllm.qf_int8_linear implementation (patches.make_int8_linear_op) + "
                       "w8a16_head, CUDA graph with pinned-host H2D inputs and D2H head statistics"}
        del g3

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_sample(args.m)
    attn = None
    if rank == 0 and world == 1 and not args.no_attn:
        attn = measure_spec_attn(dev, stream)

    from qwen_a100_fastpath_b200.w8a16 import workspace_status
    status = workspace_status(dev, stream)
    del graph
    if world > 1:
        if st.ar is not None:
            st.ar.close()
        barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    clocks = sampler.summary() if sampler else None
    line = {"metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "step_us": round(ms * 1e3, 1),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded int8 U[-127,127] weights, U(1e-3,1e-2) scales, N(0,1) bf16 activations)",
            "config": {"workload": "64-layer dense decode step at M=5 (BASELINE config 5): per layer qkv "
                                   "10240x5120, o_proj 5120x8192, gate_up 34816x5120, down 5120x17408, "
                                   "+ int8 draft head 151936x5120 with fused max/argmax/lse",
                       "m": args.m, "layers": args.layers, "tp": world, "parallelism": f"tp{world}",
                       "int8_weight_bytes": sum(N * K for _, N, K, _ in LAYER) * args.layers + HEAD[1] * HEAD[2],
                       "alg_bytes_per_step": total_bytes, "cuda_graph": True, "pdl": pdl,
                       "allreduce": ("none" if world == 1 else
                                     "fused into the row-parallel GEMM epilogue over NVLink (qf_w8a16_gemm_allreduce)"
                                     if st.fused else "nvlink one-shot kernel (qf_allreduce_bf16)"
                                     if st.ar is not None else "nccl"),
                       "l2": "no flush: each step streams 23.9 GB of weights through the 126 MB L2"},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks,
            "gpu_launches": st.launches_per_step * args.steps,
            "step_floor_ms_at_measured_peak": round(st.bytes_rank / (peak_hbm()[0] * 1e9) * 1e3, 4),
            "device_error_flag": status,
            "spec_attn": attn}
    print(json.dumps(line), flush=True)


def measure_spec_attn(dev, stream, ctx: int = 38000):
    """The verification attention (QWEN_FAST_ATTN row) on the reference's attention shape at one context: one request,
    Q = 3, 24 query / 4 KV heads, head size 256, 800-slot pages; a CUDA graph of launches over three distinct KV caches
    (together above L2).  Reported beside the step, not part of it."""
    import torch
    from qwen_a100_fastpath_b200.spec_attn import gqa_packed_spec_attention, workspace_status
    H, HKV, D, page, Q = 24, 4, 256, 800, 3
    L = ctx + Q
    pages = (L + page - 1) // page
    g = torch.Generator(device=dev).manual_seed(17)
    caches = []
    for _ in range(3):
        kv = torch.randn(pages + 1, HKV, page, 2 * D, device=dev, generator=g).to(torch.bfloat16)
        bt = torch.randperm(pages + 1, device=dev, generator=g)[:pages].to(torch.int32).view(1, pages)
        caches.append((kv, *kv.transpose(1, 2).split(D, dim=-1), bt))
    q = torch.randn(Q, H, D, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty_like(q)
    lens = torch.tensor([L], dtype=torch.int32, device=dev)
    with torch.cuda.stream(stream):
        for c in caches:
            gqa_packed_spec_attention(q, c[1], c[2], out, lens, c[3], 1, Q, HKV, D ** -0.5)
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=stream):
        for _ in range(8):
            for c in caches:
                gqa_packed_spec_attention(q, c[1], c[2], out, lens, c[3], 1, Q, HKV, D ** -0.5)
    us = time_graph(gr, stream, 5, 3) / 24 * 1e3
    del gr
    kv_bytes = L * HKV * 2 * D * 2
    peak, _ = peak_hbm()
    res = {"ctx": ctx, "q_len": Q, "heads": H, "kv_heads": HKV, "head_size": D, "page": page, "us": round(us, 2),
           "kv_GBps": round(kv_bytes / us / 1e3, 1), "frac_of_measured_hbm": round(kv_bytes / us / 1e3 / peak, 3),
           "kernel": "spec_attn_tc_kernel<256, 32> + spec_attn_merge_kernel (tcgen05)",
           "status": workspace_status(dev)}
    del caches
    torch.cuda.empty_cache()
    return res


def load_reference_triton():
    """The reference plugin's Triton kernel module (plugin/qwen_fastpath/w8a16.py), installed into baseline/_ref by
    ``pip install --no-deps --target baseline/_ref <reference>/plugin``; None if it is not installed."""
    ref_dir = REPO / "baseline" / "_ref"
    if not (ref_dir / "qwen_fastpath" / "w8a16.py").exists():
        return None
    sys.path.insert(0, str(ref_dir))
    import qwen_fastpath.w8a16 as ref
    return ref


def run_sweep(args, local: int):
    """Config 4: every config-2 GEMM and the head at M in {1,2,3,4,5,8,12,16}, timed alone (CUDA graph of 64
    launches over distinct weights, so every launch streams from HBM).  With --ref-triton, the reference's own Triton
    kernel on the same launches (its w8a16_mm with pick_config; for the head its int8 logits followed by the
    masked argmax of get_top_tokens, plugin/qwen_fastpath/patches.py:157-185)."""
    import torch
    from qwen_a100_fastpath_b200.w8a16 import w8a16_head, w8a16_head_sample, w8a16_mm
    ref = load_reference_triton() if args.ref_triton else None
    if ref is not None:
        import triton
        print(json.dumps({"reference_triton": triton.__version__, "module": ref.__file__}), flush=True)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    peak, _ = peak_hbm()
    g = torch.Generator(device=dev).manual_seed(7)
    rows = []
    stream = torch.cuda.Stream(dev)
    for name, N, K, _ in LAYER + [HEAD, ("lm_head_sample",) + tuple(HEAD[1:])]:
        head = name.startswith("lm_head")
        copies = 64 if not head else 4
        Ws = [torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g) for _ in range(copies)]
        Ss = [torch.rand(N, device=dev, generator=g) * 0.009 + 0.001 for _ in range(copies)]
        for M in (1, 2, 3, 4, 5, 8, 12, 16):
            x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
            y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            outs = (y, torch.empty(M, device=dev), torch.empty(M, device=dev, dtype=torch.int64),
                    torch.empty(M, device=dev))

            def call(i):
                if name == "lm_head":
                    w8a16_head(x, Ws[i].t(), Ss[i], pdl=True, out=outs)
                elif name == "lm_head_sample":  # the fused temperature draw (probabilistic drafting)
                    w8a16_head_sample(x, Ws[i].t(), Ss[i], temperature=0.8, seed=1, offset=i, pdl=True)
                else:
                    w8a16_mm(x, Ws[i].t(), Ss[i], None, torch.bfloat16, out=y, pdl=True)

            with torch.cuda.stream(stream):
                for i in range(copies):
                    call(i)
            torch.cuda.synchronize()
            gr = torch.cuda.CUDAGraph()
            reps = 64 if not head else 16
            with torch.cuda.graph(gr, stream=stream):
                for i in range(reps):
                    call(i % copies)
            ms = time_graph(gr, stream, 5, 2) / reps
            b = alg_bytes(N, K, M, head=head)
            gbs = b / (ms * 1e-3) / 1e9
            rows.append({"gemm": name, "N": N, "K": K, "M": M, "us": round(ms * 1e3, 2), "GBps": round(gbs, 1),
                         "frac_measured": round(gbs / peak, 4), "frac_nominal": round(gbs / NOMINAL_HBM_GBS, 4)})
            del gr
            if ref is not None and name != "lm_head_sample":
                cfg = ref.pick_config(N, K)

                def ref_call(i):
                    lg = ref.w8a16_mm(x, Ws[i].t(), Ss[i], cfg, torch.bfloat16)
                    if head:  # get_top_tokens: the argmax over the logits (no padding here)
                        lg.argmax(dim=-1)

                try:
                    with torch.cuda.stream(stream):
                        for i in range(copies):
                            ref_call(i)
                    torch.cuda.synchronize()
                    gr = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(gr, stream=stream):
                        for i in range(reps):
                            ref_call(i % copies)
                    rms = time_graph(gr, stream, 5, 2) / reps
                    rows[-1]["ref_triton_us"] = round(rms * 1e3, 2)
                    rows[-1]["ref_triton_GBps"] = round(b / (rms * 1e-3) / 1e9, 1)
                    rows[-1]["ref_triton_cfg"] = list(cfg) if cfg else None
                except Exception as e:  # noqa: BLE001 -- the reference kernel may not compile for this GPU
                    rows[-1]["ref_triton_us"] = None
                    rows[-1]["ref_triton_error"] = f"{type(e).__name__}: {str(e)[:160]}"
            print(json.dumps(rows[-1]), flush=True)
        del Ws, Ss
        torch.cuda.empty_cache()
    if args.sweep_out:
        Path(args.sweep_out).write_text(json.dumps(rows, indent=1))


def run_profile_gemm(args, local: int):
    """Two launches of each named GEMM (int8 weights U[-127,127], distinct per launch) at M = --m."""
    import torch
    from qwen_a100_fastpath_b200.w8a16 import w8a16_head, w8a16_head_sample, w8a16_mm
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    shapes = {nm: (N, K) for nm, N, K, _ in LAYER + [HEAD]}
    shapes["lm_head_sample"] = shapes["lm_head"]
    g = torch.Generator(device=dev).manual_seed(3)
    from qwen_a100_fastpath_b200.w8a16 import w8a8_mm
    for nm, N, K, _ in LAYER:
        shapes["pf_" + nm] = (N, K)
    for name in args.profile_gemm.split(","):
        N, K = shapes[name]
        x = torch.randn(args.m, K, device=dev, generator=g).to(torch.bfloat16)
        for _ in range(2):
            W = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
            s = torch.rand(N, device=dev, generator=g) * 0.009 + 0.001
            torch.cuda.synchronize()
            if name == "lm_head":
                w8a16_head(x, W.t(), s)
            elif name == "lm_head_sample":
                w8a16_head_sample(x, W.t(), s, temperature=0.8, seed=1, offset=0)
            elif name.startswith("pf_"):
                w8a8_mm(x, W.t(), s)
            else:
                w8a16_mm(x, W.t(), s, None, torch.bfloat16)
            torch.cuda.synchronize()
            del W
    print("profile-gemm done:", args.profile_gemm)


def run_prefill_sweep(args, local: int):
    """Prefill path (M > 16): qf_w8a8_gemm (per-token int8 quantization of the bf16 activations, then the tcgen05
    int8 GEMM with the scaled bf16 epilogue) on every config-2 GEMM at M in {32, ..., 4096}; beside it torch._int_mm
    (cuBLASLt int8 x int8 -> int32, on already-quantized activations, no scaling: a plain library GEMM of the same
    contraction).  CUDA graph of launches over distinct weight copies (more than 2x L2 per pass); tera-ops/s =
    2 M N K / time, % of the nominal 4.5 dense int8 POPS (no measured int8 peak on this pool) and GB/s of the weight
    + activation + output bytes."""
    import torch
    from qwen_a100_fastpath_b200.w8a16 import w8a8_mm
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(11)
    stream = torch.cuda.Stream(dev)
    rows = []
    for name, N, K, _ in LAYER:
        copies = max(2, int(2 * 126e6 // (N * K)) + 1)
        Ws = [torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g) for _ in range(copies)]
        Ss = [torch.rand(N, device=dev, generator=g) * 0.009 + 0.001 for _ in range(copies)]
        for M in (32, 64, 128, 256, 512, 1024, 2048, 4096):
            x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
            xq = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev, generator=g)
            y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            res = {}
            for impl in ("ours", "torch_int_mm"):
                def call(i, impl=impl):
                    if impl == "ours":
                        w8a8_mm(x, Ws[i].t(), Ss[i], out=y, pdl=True)
                    else:
                        torch._int_mm(xq, Ws[i].t())
                try:
                    with torch.cuda.stream(stream):
                        for i in range(copies):
                            call(i)
                    torch.cuda.synchronize()
                    reps = max(copies, 8)
                    gr = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(gr, stream=stream):
                        for i in range(reps):
                            call(i % copies)
                    ms = time_graph(gr, stream, 5, 2) / reps
                    del gr
                    res[impl] = ms
                except Exception as e:  # noqa: BLE001 -- the library comparator may reject a shape
                    res[impl] = None
                    print(f"{impl} {name} M={M}: {type(e).__name__}: {str(e)[:120]}", file=sys.stderr)
            flops = 2.0 * M * N * K
            nbytes = N * K + 4 * N + 2 * M * K + 2 * M * N
            row = {"gemm": name, "N": N, "K": K, "M": M}
            for impl, ms in res.items():
                if ms is None:
                    row[impl] = None
                    continue
                row[impl] = {"us": round(ms * 1e3, 2), "TOPS": round(flops / (ms * 1e-3) / 1e12, 1),
                             "frac_int8_nominal": round(flops / (ms * 1e-3) / 4.5e15, 4),
                             "GBps": round(nbytes / (ms * 1e-3) / 1e9, 1)}
            rows.append(row)
            print(json.dumps(row), flush=True)
        del Ws, Ss
        torch.cuda.empty_cache()
    if args.sweep_out:
        Path(args.sweep_out).write_text(json.dumps(rows, indent=1))


def run_fused_sweep(args, local: int):
    """qkv with the preceding RMSNorm (input_layernorm, with residual) and gate_up with RMSNorm + SiLU fused
    (qf_w8a16_gemm_rmsnorm), against the unfused sequence: vLLM's fused_add_rms_norm as its torch expression
    (vllm/ir/ops/layernorm.py), then w8a16_mm (and, for gate_up, the GEMM with the SiLU gate fused).  CUDA graphs of
    launches over distinct weight copies; mean us per layer-norm + GEMM."""
    import torch
    from qwen_a100_fastpath_b200.w8a16 import w8a16_mm, w8a16_mm_rmsnorm, w8a16_mm_silu_mul
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(13)
    stream = torch.cuda.Stream(dev)
    K = 5120
    gamma = (torch.rand(K, device=dev, generator=g) + 0.5).to(torch.bfloat16)
    for name, N, silu in (("qkv", 10240, False), ("gate_up", 34816, True)):
        copies = 8
        Ws = [torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g) for _ in range(copies)]
        Ss = [torch.rand(N, device=dev, generator=g) * 0.009 + 0.001 for _ in range(copies)]
        for M in (1, 5, 8, 16):
            x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
            res = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
            res_out = torch.empty_like(res)
            y = torch.empty(M, N // 2 if silu else N, device=dev, dtype=torch.bfloat16)

            def unfused(i):
                z = x.float() + res.float()
                r = z.to(torch.bfloat16)
                a = (z * torch.rsqrt(z.pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16) * gamma
                if silu:
                    w8a16_mm_silu_mul(a, Ws[i].t(), Ss[i], out=y, pdl=True)
                else:
                    w8a16_mm(a, Ws[i].t(), Ss[i], None, torch.bfloat16, out=y, pdl=True)
                return r

            def fused(i):
                w8a16_mm_rmsnorm(x, gamma, 1e-6, Ws[i].t(), Ss[i], residual=res, silu_mul=silu,
                                 residual_out=res_out, out=y, pdl=True)

            row = {"gemm": name, "N": N, "K": K, "M": M}
            for tag, fn in (("unfused_torch_norm_then_gemm", unfused), ("fused", fused)):
                with torch.cuda.stream(stream):
                    for i in range(copies):
                        fn(i)
                torch.cuda.synchronize()
                reps = 32
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=stream):
                    for i in range(reps):
                        fn(i % copies)
                row[tag + "_us"] = round(time_graph(gr, stream, 5, 2) / reps * 1e3, 2)
                del gr
            print(json.dumps(row), flush=True)
        del Ws, Ss
        torch.cuda.empty_cache()


def load_reference_spec_attn():
    """The reference plugin's split-KV attention (plugin/qwen_fastpath/spec_attn.py) from baseline/_ref, or None."""
    ref_dir = REPO / "baseline" / "_ref"
    if not (ref_dir / "qwen_fastpath" / "spec_attn.py").exists():
        return None
    sys.path.insert(0, str(ref_dir))
    from qwen_fastpath.spec_attn import gqa_packed_spec_attention as ref
    return ref


def run_attn_sweep(args, local: int):
    """Verification attention through spec_attn.gqa_packed_spec_attention (qf_spec_attn) on the reference's attention
    shapes (H = 24, HKV = 4, D = 256, 800-slot pages: bench/test_spec_attn.py of the reference) at context 0..100K
    and (Q, requests) = (3, 1), (4, 1), (3, 2), (5, 1), beside FlashAttention-2 (vLLM's flash_attn_varlen_func, the
    path the reference replaces) and, with --ref-triton, the reference's own Triton kernels.  Each time is a CUDA
    graph of one launch per layer over `n` distinct KV caches (enough layers that together they exceed L2 where memory
    allows), us per layer; kv_GBps = the KV bytes a layer must read once (sum over requests of seq_len x HKV x 2 x D x
    2 bytes) / that time, frac = kv_GBps / the measured HBM copy bandwidth."""
    import torch
    from qwen_a100_fastpath_b200.spec_attn import gqa_packed_spec_attention, workspace_status
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    peak, peak_src = peak_hbm()
    H, HKV, D, page = 24, 4, 256, 800
    scale = D ** -0.5
    stream = torch.cuda.Stream(dev)
    g = torch.Generator(device=dev).manual_seed(11)
    fa2 = None
    try:
        from vllm.vllm_flash_attn import flash_attn_varlen_func as fa2
    except Exception as e:  # noqa: BLE001 -- FlashAttention-2 from vLLM is a comparator only
        print(json.dumps({"fa2": f"unavailable: {type(e).__name__}: {str(e)[:120]}"}), flush=True)
    ref = load_reference_spec_attn() if args.ref_triton else None
    if ref is not None:
        import triton
        print(json.dumps({"reference_triton": triton.__version__, "module": ref.__module__}), flush=True)
    if args.profile_attn >= 0:
        cases = [(args.profile_attn, 3, 1)]
    else:
        cases = [(c, q, b) for c in (0, 50, 1000, 8000, 38000, 100000) for q, b in ((3, 1), (4, 1), (3, 2), (5, 1))]
    print(json.dumps({"peak_hbm_GBps": peak, "peak_source": peak_src}), flush=True)
    for ctx, Q, B in cases:
        L = ctx + Q
        lens = [max(L - 7 * i, 1) for i in range(B)]
        pages = (L + page - 1) // page
        nblk = B * pages + 1
        layer_bytes = nblk * HKV * page * 2 * D * 2
        n = int(min(16, max(1, (4 * 126e6) // layer_bytes)))
        caches = []
        for _ in range(n):
            kv = torch.randn(nblk, HKV, page, 2 * D, device=dev, generator=g).to(torch.bfloat16)
            bt = torch.randperm(nblk, device=dev, generator=g)[: B * pages].to(torch.int32).view(B, pages)
            caches.append((kv, *kv.transpose(1, 2).split(D, dim=-1), bt))
        q = torch.randn(B * Q, H, D, device=dev, generator=g).to(torch.bfloat16)
        out = torch.empty_like(q)
        seq_lens = torch.tensor(lens, dtype=torch.int32, device=dev)
        cu_q = torch.arange(0, B + 1, device=dev, dtype=torch.int32) * Q
        kv_bytes = sum(lens) * HKV * 2 * D * 2
        if args.profile_attn >= 0:
            for i in range(3):
                gqa_packed_spec_attention(q, caches[i % n][1], caches[i % n][2], out, seq_lens, caches[i % n][3], B, Q,
                                          HKV, scale)
            torch.cuda.synchronize()
            print(json.dumps({"profile_attn": ctx, "launches": 3, "status": workspace_status(dev)}), flush=True)
            return

        def ours(i):
            gqa_packed_spec_attention(q, caches[i][1], caches[i][2], out, seq_lens, caches[i][3], B, Q, HKV, scale)

        def fa(i):
            fa2(q=q, k=caches[i][1], v=caches[i][2], out=out, cu_seqlens_q=cu_q, max_seqlen_q=Q, seqused_k=seq_lens,
                max_seqlen_k=131072, softmax_scale=scale, causal=True, block_table=caches[i][3], fa_version=2)

        def reference(i):
            ref(q, caches[i][1], caches[i][2], out, seq_lens, caches[i][3], B, Q, HKV, scale)

        row = {"ctx": ctx, "Q": Q, "reqs": B, "layers_in_graph": n, "kv_bytes": kv_bytes}
        for tag, fn in (("ours", ours), ("fa2", fa if fa2 else None), ("ref_triton", reference if ref else None)):
            if fn is None:
                continue
            try:
                with torch.cuda.stream(stream):
                    for i in range(n):
                        fn(i)
                torch.cuda.synchronize()
                reps = max(1, 32 // n)
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=stream):
                    for _ in range(reps):
                        for i in range(n):
                            fn(i)
                us = time_graph(gr, stream, 5, 2) / (reps * n) * 1e3
                del gr
                row[tag + "_us"] = round(us, 2)
                row[tag + "_kv_GBps"] = round(kv_bytes / us / 1e3, 1)
            except Exception as e:  # noqa: BLE001 -- a comparator that cannot run on this box is reported, not fatal
                row[tag] = f"unavailable: {type(e).__name__}: {str(e)[:120]}"
        if "ours_us" in row:
            row["ours_frac_of_measured"] = round(row["ours_kv_GBps"] / peak, 3)
        row["status"] = workspace_status(dev)
        print(json.dumps(row), flush=True)
        del caches
        torch.cuda.empty_cache()


def run_host_overhead(args, local: int):
    """Host cost of one eager call (argument checks, ctypes, tensor-map encoding, launch) of the C-ABI entry point,
    of ``w8a16_mm`` and of the ``qf_int8_linear`` op body, against the device time of the same launch, for o_proj at
    M = --m.  The host loop enqueues only (no synchronisation inside the timed loop)."""
    import torch
    from qwen_a100_fastpath_b200 import _lib
    from qwen_a100_fastpath_b200.patches import make_int8_linear_op
    from qwen_a100_fastpath_b200.w8a16 import w8a16_mm, workspace
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    N, K, M = 5120, 8192, args.m
    g = torch.Generator(device=dev).manual_seed(5)
    W = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
    s = torch.rand(N, device=dev, generator=g) * 0.009 + 0.001
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    op, _ = make_int8_linear_op()
    stream = torch.cuda.current_stream(dev)
    ws = workspace(dev, stream, _lib.LIB.qf_w8a16_workspace_bytes(M, N, K))

    def c_abi():
        _lib.LIB.qf_w8a16_gemm(x.data_ptr(), K, W.data_ptr(), K, s.data_ptr(), None, y.data_ptr(), N,
                               _lib.QF_DTYPE_BF16, M, N, K, ws.data_ptr(), ws.numel(), 0, stream.cuda_stream)

    calls = {"c_abi_ctypes": c_abi,
             "w8a16_mm": lambda: w8a16_mm(x, W.t(), s, None, torch.bfloat16, out=y, pdl=False),
             "qf_int8_linear_op": lambda: op(x, W.t(), s.view(N, 1), None)}
    res = {}
    n = 2000
    for name, fn in calls.items():
        for _ in range(50):
            fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(n):
            fn()
        host_us = (time.perf_counter() - t0) / n * 1e6
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(200):
            fn()
        e1.record()
        torch.cuda.synchronize()
        res[name] = {"host_us_per_call": round(host_us, 2), "device_us_per_call": round(e0.elapsed_time(e1) * 5, 2)}
    print(json.dumps({"host_overhead": res, "gemm": f"o_proj {N}x{K}", "m": M,
                      "note": "host_us: enqueue cost per eager call (no sync in the loop); device_us: back-to-back "
                              "launches on one weight (L2-resident, so shorter than the HBM-bound step)"}),
          flush=True)


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and world > 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.sweep:
        if rank == 0:
            run_sweep(args, local)
        return
    if args.profile_gemm:
        if rank == 0:
            run_profile_gemm(args, local)
        return
    if args.host_overhead:
        if rank == 0:
            run_host_overhead(args, local)
        return
    if args.prefill_sweep:
        if rank == 0:
            run_prefill_sweep(args, local)
        return
    if args.fused_sweep:
        if rank == 0:
            run_fused_sweep(args, local)
        return
    if args.attn_sweep or args.profile_attn >= 0:
        if rank == 0:
            run_attn_sweep(args, local)
        return
    run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
