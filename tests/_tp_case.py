"""Run under torchrun (one process per GPU, NCCL for the plumbing) or as one process with world size 1:
NVLinkAllReduce (qf_allreduce_bf16) against the fp32 rank-order sum of every rank's input, eager and inside a
CUDA graph, for the decode sizes M x 5120 (M = 1, 5, 16).  Exits non-zero on a mismatch.  Used by
test_gpu_tp.py."""
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
