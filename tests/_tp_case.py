"""Run under torchrun (one process per GPU, NCCL for the plumbing) or as one process with world size 1:
NVLinkAllReduce (qf_allreduce_bf16) against the fp32 rank-order sum of every rank's input, eager and inside a
CUDA graph, for the decode sizes M x 5120 (M = 1, 5, 16); and the row-parallel GEMM with the fused all-reduce
(qf_w8a16_gemm_allreduce) against the rank-order sum of every rank's partial computed by the plain GEMM kernel
(the same accumulation, so the comparison is bit-exact); with two ranks also the plugin's patched RowParallelLinear
body (patches.row_parallel_forward) with its own buffers.  Exits non-zero on a mismatch.  Used by test_gpu_tp.py."""
from __future__ import annotations

import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist


def inputs(seed: int, world: int, count: int, dev) -> list[torch.Tensor]:
    g = torch.Generator(device=dev).manual_seed(seed)
    return [(torch.randn(count, device=dev, generator=g) * (1 + r)).to(torch.bfloat16) for r in range(world)]


def reference(xs: list[torch.Tensor]) -> torch.Tensor:
    acc = torch.zeros_like(xs[0], dtype=torch.float32)
    for x in xs:  # rank order, fp32
        acc += x.float()
    return acc.to(torch.bfloat16)


def shard(seed: int, M: int, N: int, K: int, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    w = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
    return x, w


def fused_cases(ar, rank: int, world: int, dev, stream) -> int:
    from qwen_a100_fastpath_b200.w8a16 import w8a16_mm, w8a16_mm_allreduce
    bad = 0
    N = 5120
    scale = torch.rand(N, device=dev, generator=torch.Generator(device=dev).manual_seed(9)) * 0.009 + 0.001
    for (K, M) in [(1024, 1), (2176, 5), (4352, 16), (8192, 5)]:
        shards = [shard(1000 * K + 10 * M + r, M, N, K, dev) for r in range(world)]
        partials = [w8a16_mm(x, w.t(), scale, None, torch.bfloat16) for x, w in shards]
        want = reference(partials)
        x, w = shards[rank]
        y = w8a16_mm_allreduce(x, w.t(), scale, ar)
        torch.cuda.synchronize()
        if not torch.equal(y, want):
            bad += 1
            print(f"rank {rank}: fused mismatch K={K} M={M}: {(y != want).sum().item()} elements", flush=True)
    # graph: fused GEMM, standalone all-reduce and fused GEMM again on the same buffers (one epoch sequence)
    K, M = 2176, 5
    shards = [shard(77 + r, M, N, K, dev) for r in range(world)]
    x, w = shards[rank]
    xs = x.clone()
    y1 = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    y2 = torch.empty_like(y1)
    with torch.cuda.stream(stream):
        w8a16_mm_allreduce(xs, w.t(), scale, ar, out=y1, pdl=True)
        ar(y1.view(-1), out=y2.view(-1), pdl=True)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        w8a16_mm_allreduce(xs, w.t(), scale, ar, out=y1, pdl=True)
        ar(y1.view(-1), out=y2.view(-1), pdl=True)
        w8a16_mm_allreduce(xs, w.t(), scale, ar, out=y1, pdl=True)
    for rep in range(2):
        shards = [shard(300 + 10 * rep + r, M, N, K, dev) for r in range(world)]
        xs.copy_(shards[rank][0])
        # every rank's weights stay those captured; only the activations change
        partials = [w8a16_mm(shards[r][0], shard(77 + r, M, N, K, dev)[1].t(), scale, None, torch.bfloat16)
                    for r in range(world)]
        first = reference(partials)
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            graph.replay()
        torch.cuda.synchronize()
        if not torch.equal(y1, first) or not torch.equal(y2, reference([first] * world)):
            bad += 1
            print(f"rank {rank}: fused graph mismatch rep={rep}", flush=True)
    del graph
    return bad


def plugin_row_case(rank: int, world: int, dev) -> int:
    """The plugin's patched RowParallelLinear body (patches.row_parallel_forward) on a stand-in layer holding this
    rank's K-shard of an int8 weight: its own NVLink buffers (made by patches.row_comm over the default group) and the
    fused GEMM + all-reduce, against the rank-order sum of every shard's plain-GEMM partial plus the bias."""
    import types
    from qwen_a100_fastpath_b200 import patches
    from qwen_a100_fastpath_b200.w8a16 import w8a16_mm
    patches._tp_group = lambda: types.SimpleNamespace(cpu_group=None, device_group=None)

    class Kernel:
        def apply_weights(self, layer, x, bias=None):
            raise AssertionError("the fused path replaces apply_weights + all-reduce")
        apply_weights._qwen_fastpath = True

        def _get_layer_params(self, layer):
            return layer.w_q, layer.w_s, None, None, None

    bad = 0
    N = 5120
    scale = torch.rand(N, device=dev, generator=torch.Generator(device=dev).manual_seed(19)) * 0.009 + 0.001
    bias = (torch.randn(N, device=dev, generator=torch.Generator(device=dev).manual_seed(20)) * 0.5).to(torch.bfloat16)
    for (K, M) in [(2176, 5), (4352, 16)]:
        shards = [shard(5000 + K + M + r, M, N, K, dev) for r in range(world)]
        x, w = shards[rank]
        layer = types.SimpleNamespace(reduce_results=True, tp_size=world, tp_rank=rank, input_is_parallel=True,
                                      bias=bias, skip_bias_add=False, return_bias=False,
                                      scheme=types.SimpleNamespace(kernel=Kernel()), w_q=w.t(), w_s=scale.view(N, 1))
        y = patches.row_parallel_forward(layer, x.view(1, M, K))
        want = reference([w8a16_mm(xr, wr.t(), scale, None, torch.bfloat16) for xr, wr in shards]) + bias
        torch.cuda.synchronize()
        if y is None or y.shape != (1, M, N) or not torch.equal(y.view(M, N), want):
            bad += 1
            print(f"rank {rank}: plugin row-parallel mismatch K={K} M={M}", flush=True)
    for comm in patches._ROW_COMMS.values():
        if comm.status() != 0:
            bad += 1
        comm.close()
    patches._ROW_COMMS.clear()
    return bad


def main() -> int:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world == 1:
        dist.init_process_group("gloo", store=dist.HashStore(), rank=0, world_size=1)
    else:
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=60))
    from qwen_a100_fastpath_b200.tp import NVLinkAllReduce
    ar = NVLinkAllReduce(16 * 5120)
    bad = 0
    for it in range(4):
        for m in (1, 5, 16):
            xs = inputs(100 * it + m, world, m * 5120, dev)
            y = xs[rank].clone()
            ar(y)
            torch.cuda.synchronize()
            if not torch.equal(y, reference(xs)):
                bad += 1
                print(f"rank {rank}: eager mismatch it={it} m={m}", flush=True)
    # CUDA graph: two calls on static buffers (out of place, then in place), replayed with new inputs
    count = 5 * 5120
    a = torch.empty(count, device=dev, dtype=torch.bfloat16)
    b = torch.empty_like(a)
    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        a.copy_(inputs(7, world, count, dev)[rank])
        ar(a, out=b)
        ar(b)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        ar(a, out=b, pdl=True)
        ar(b, pdl=True)
    for rep in range(3):
        xs = inputs(500 + rep, world, count, dev)
        a.copy_(xs[rank])
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            graph.replay()
        torch.cuda.synchronize()
        first = reference(xs)
        want = reference([first] * world)
        if not torch.equal(b, want):
            bad += 1
            print(f"rank {rank}: graph mismatch rep={rep}", flush=True)
    del graph
    bad += fused_cases(ar, rank, world, dev, stream)
    if world > 1:
        bad += plugin_row_case(rank, world, dev)
    status = ar.status()
    if status != 0:
        bad += 1
        print(f"rank {rank}: device error word {status}", flush=True)
    ar.close()
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print("ok" if bad == 0 else f"{bad} mismatches", flush=True)
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())
