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
    """Sum the row-parallel partial outputs of all ranks in place with torch.distributed (NCCL on GPUs, gloo on
    CPU): the collective vLLM issues after RowParallelLinear, kept as the comparison path."""
    dist.all_reduce(y, group=group)
    return y


class NVLinkAllReduce:
    """One-shot all-reduce of bf16 tensors between the ranks of one node over NVLink peer memory
    (``qf_allreduce_bf16``): the replacement for the NCCL all-reduce after the row-parallel layers.

    Collective construction: every rank allocates a symmetric buffer for vectors of up to ``max_count`` elements,
    the CUDA IPC handles are exchanged with ``all_gather_object`` and every rank opens the others' buffers. Calls
    are collective too (same sequence and sizes on every rank); the result is bit-identical on all ranks (fp32 sums
    in rank order, one bf16 rounding) and the call can be captured in a CUDA graph."""

    def __init__(self, max_count: int, group=None):
        import ctypes

        from ._lib import LIB, QF_AR_MAX_RANKS, QF_IPC_HANDLE_BYTES, check
        self._lib, self._check, self._ct = LIB, check, ctypes
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > QF_AR_MAX_RANKS:
            raise ValueError(f"at most {QF_AR_MAX_RANKS} ranks")
        self.max_count = (int(max_count) + 7) // 8 * 8
        ptr = ctypes.c_void_p()
        check("qf_symm_alloc", LIB.qf_symm_alloc(LIB.qf_allreduce_buffer_bytes(self.max_count), ctypes.byref(ptr)))
        self.own = ptr.value
        handle = (ctypes.c_char * QF_IPC_HANDLE_BYTES)()
        check("qf_ipc_handle", LIB.qf_ipc_handle(self.own, handle))
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened = []
        bufs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                bufs.append(self.own)
                continue
            pp = ctypes.c_void_p()
            check("qf_ipc_open", LIB.qf_ipc_open(h, ctypes.byref(pp)))
            self._opened.append(pp.value)
            bufs.append(pp.value)
        self._bufs = (ctypes.c_void_p * self.world)(*bufs)
        dist.barrier(group)

    @property
    def buffer_list(self):
        """ctypes array of every rank's buffer pointer (this rank's own at [rank]), for the C ABI."""
        return self._bufs

    def __call__(self, t: torch.Tensor, out: torch.Tensor | None = None, pdl: bool = False) -> torch.Tensor:
        """Sum ``t`` over the ranks into ``out`` (default: in place) on the current stream."""
        from ._lib import QF_FLAG_PDL
        if t.dtype != torch.bfloat16 or not t.is_cuda or not t.is_contiguous():
            raise ValueError("NVLinkAllReduce needs a contiguous bf16 CUDA tensor")
        if t.numel() > self.max_count or t.numel() % 8:
            raise ValueError(f"numel {t.numel()} must be a multiple of 8 and <= {self.max_count}")
        out = t if out is None else out
        stream = torch.cuda.current_stream(t.device).cuda_stream
        self._check("qf_allreduce_bf16", self._lib.qf_allreduce_bf16(
            t.data_ptr(), out.data_ptr(), t.numel(), self.max_count, self.rank, self.world, self._bufs,
            QF_FLAG_PDL if pdl else 0, stream))
        return out

    def status(self) -> int:
        """Sticky device error word of this rank's buffer (0 or QF_ERR_TIMEOUT), cleared on read; synchronises."""
        st = self._ct.c_int(0)
        self._check("qf_allreduce_status", self._lib.qf_allreduce_status(
            self.own, torch.cuda.current_stream().cuda_stream, self._ct.byref(st)))
        return st.value

    def set_wait(self, wait_us: int) -> None:
        """Bound of this rank's waits on the other ranks, in microseconds (0: the default 2 s); synchronises."""
        self._check("qf_allreduce_set_wait", self._lib.qf_allreduce_set_wait(
            self.own, int(wait_us), torch.cuda.current_stream().cuda_stream))

    def close(self) -> None:
        """Collective: unmap the other ranks' buffers, wait for every rank, free this rank's buffer."""
        if self.own is None:
            return
        torch.cuda.synchronize()
        for pp in self._opened:
            self._check("qf_ipc_close", self._lib.qf_ipc_close(pp))
        self._opened = []
        dist.barrier(self.group)
        self._check("qf_symm_free", self._lib.qf_symm_free(self.own))
        self.own = None


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


def combine_head_samples(gathered: torch.Tensor):
    """Fold per-shard ``[world, M, 3]`` (sample score, global sample column, sample logit) of
    ``w8a16_head_sample`` into the draw of the full vocabulary: the shard with the largest score wins (lowest
    global column on ties) -- the Gumbel-max draw of the unsharded head, since every shard's noise is keyed by the
    global column.  Returns (sample int64, sample_logit fp32); its draft probability is
    ``exp(sample_logit - lse)`` with the lse from ``combine_head_stats``."""
    best = gathered[:, :, 0].max(dim=0).values
    cand = torch.where(gathered[:, :, 0] == best, gathered[:, :, 1], torch.full_like(gathered[:, :, 1], float("inf")))
    col = cand.min(dim=0).values
    pick = (gathered[:, :, 1] == col) & (gathered[:, :, 0] == best)
    logit = torch.where(pick, gathered[:, :, 2], torch.zeros_like(gathered[:, :, 2])).sum(dim=0)
    return col.to(torch.int64), logit.float()


def gather_head_samples(sample, sample_score, sample_logit, group=None):
    """All-gather every rank's draw and combine them (same result on every rank)."""
    world = dist.get_world_size(group)
    local = torch.stack([sample_score.double(), sample.double(), sample_logit.double()], dim=1)
    out = torch.empty((world, *local.shape), dtype=local.dtype, device=local.device)
    if local.is_cuda:
        dist.all_gather_into_tensor(out, local, group=group)
    else:  # gloo: list form
        parts = list(out.unbind(0))
        dist.all_gather(parts, local, group=group)
        out = torch.stack(parts)
    return combine_head_samples(out)
