"""Tensor parallelism for the W8A16 decode path (one process per GPU, torch.distributed for the plumbing).

The reference runs on one GPU (its draft head even requires ``tp_size == 1``, plugin/qwen_fastpath/patches.py:138).
Under vLLM's tensor parallelism the same linear method runs on each rank's shard:

* column-parallel layers (qkv, gate_up, the vocab-sharded head) own output channels ``[r*N/t, (r+1)*N/t)``;
* row-parallel layers (o_proj, down) own input channels ``[r*K/t, (r+1)*K/t)`` and their bf16 partial outputs are
  summed across ranks (vLLM: ``tensor_model_parallel_all_reduce`` after ``RowParallelLinear``'s ``apply``);
* the vocab-sharded head keeps its logits sharded: each rank reduces its shard to per-row (max, argmax, logsumexp)
  and only those ``3*M`` values are gathered and combined.

Weights are vLLM's int8 ``w_q`` ``[K, N]`` views with stride ``(1, ldw)``; shards are views (no copies).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    if total % world:
        raise ValueError(f"{total} is not divisible by the tensor-parallel size {world}")
    n = total // world
    return rank * n, (rank + 1) * n


def shard_weight(w_q: torch.Tensor, w_s: torch.Tensor, style: str, rank: int, world: int):
    """Rank ``rank``'s view of a ``[K, N]`` int8 weight and its fp32 scales.

    ``style`` is ``"col"`` (output channels, also the vocab shard of the head) or ``"row"`` (input channels; the
    scales stay whole because every output channel is present on every rank)."""
    K, N = w_q.shape
    s = w_s.reshape(-1)
    if style in ("col", "vocab"):
        n0, n1 = shard_range(N, rank, world)
        return w_q[:, n0:n1], s[n0:n1]
    if style == "row":
        k0, k1 = shard_range(K, rank, world)
        return w_q[k0:k1, :], s
    raise ValueError(style)


def shard_activations(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Input columns of a row-parallel layer owned by ``rank``."""
    k0, k1 = shard_range(x.shape[-1], rank, world)
    return x[..., k0:k1]


def all_reduce_partial(y: torch.Tensor, group=None) -> torch.Tensor:
    """Sum the row-parallel partial outputs of all ranks in place (NCCL on GPUs, gloo on CPU)."""
    dist.all_reduce(y, group=group)
    return y


def pack_head_stats(row_max: torch.Tensor, row_argmax: torch.Tensor, row_lse: torch.Tensor) -> torch.Tensor:
    """``[M, 3]`` fp64 (max, global argmax, lse); fp64 holds every vocab index exactly."""
    return torch.stack([row_max.double(), row_argmax.double(), row_lse.double()], dim=1)


def combine_head_stats(gathered: torch.Tensor):
    """Fold per-shard ``[world, M, 3]`` (max, argmax, lse) in rank order into the full-vocab statistics.

    max = largest shard max; argmax = lowest global index among shards holding it (``torch.argmax`` on the full
    row returns the first maximal column); lse = m* + log sum_r exp(lse_r - m*), m* = max_r lse_r.
    Returns (row_max fp32, row_argmax int64, row_lse fp32)."""
    mx = gathered[:, :, 0].max(dim=0).values
    cand = torch.where(gathered[:, :, 0] == mx, gathered[:, :, 1], torch.full_like(gathered[:, :, 1], float("inf")))
    arg = cand.min(dim=0).values.to(torch.int64)
    lse = torch.logsumexp(gathered[:, :, 2], dim=0)
    return mx.float(), arg, lse.float()


def gather_head_stats(row_max, row_argmax, row_lse, group=None, out: torch.Tensor | None = None):
    """All-gather every rank's shard statistics and combine them (same result on every rank)."""
    world = dist.get_world_size(group)
    local = pack_head_stats(row_max, row_argmax, row_lse)
    if out is None:
        out = torch.empty((world, *local.shape), dtype=local.dtype, device=local.device)
    if local.is_cuda:
        dist.all_gather_into_tensor(out, local, group=group)
    else:  # gloo: list form
        parts = list(out.unbind(0))
        dist.all_gather(parts, local, group=group)
        out = torch.stack(parts)
    return combine_head_stats(out)
