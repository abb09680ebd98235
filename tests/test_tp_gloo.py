"""Tensor-parallel host logic on CPU ranks (gloo, world size 2): row-parallel partial sums, the vocab-sharded
head's (max, argmax, lse) gather and its temperature draw match the unsharded oracle, ties resolved to the lowest
global index."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import w8a16_oracle as orc


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def worker(rank: int, world: int, port: int, result_dir: str):
    import torch.distributed as dist
    from qwen_a100_fastpath_b200 import tp
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        # row-parallel: partial sums of the rank's input columns, summed across ranks
        x_bits, W, s = orc.make_inputs(5, 4, 96, 512)
        w_q = torch.from_numpy(W).t()                          # [K, N] view, stride (1, K)
        w_r, s_r = tp.shard_weight(w_q, torch.from_numpy(s), "row", rank, world)
        x_r = tp.shard_activations(torch.from_numpy(orc.bf16_to_f32(x_bits)).double(), rank, world)
        part = (x_r @ w_r.double()) * s_r.double()[None, :]
        tp.all_reduce_partial(part)
        full = orc.dequant_matmul_f64(x_bits, W, s)
        np.testing.assert_allclose(part.numpy(), full, rtol=1e-12, atol=1e-9)
        # vocab-sharded head: each rank reduces its shard, then gather + combine
        V = 1024
        rs = np.random.RandomState(9)
        logits = orc.f32_to_bf16(rs.standard_normal((3, V)).astype(np.float32) * 3)
        logits[1, 100] = logits[1, 700] = orc.f32_to_bf16(np.float32(40.0))   # tie across the two shards
        n0, n1 = tp.shard_range(V, rank, world)
        mx, am, lse = orc.head_stats(logits[:, n0:n1], n1 - n0, n0)
        g_mx, g_am, g_lse = tp.gather_head_stats(torch.from_numpy(mx), torch.from_numpy(am), torch.from_numpy(lse))
        f_mx, f_am, f_lse = orc.head_stats(logits, V, 0)
        assert np.array_equal(g_mx.numpy(), f_mx)
        assert np.array_equal(g_am.numpy(), f_am)
        np.testing.assert_allclose(g_lse.numpy(), f_lse, rtol=1e-6)
        assert int(g_am[1]) == 100
        # vocab-sharded temperature draw: every shard draws with noise keyed by the global column; the gathered
        # draw equals the unsharded one
        _, _, _, smp, score, slog, _ = orc.head_sample(logits[:, n0:n1], n1 - n0, 1 / 0.8, 77, 5, n0)
        g_smp, g_slog = tp.gather_head_samples(torch.from_numpy(smp), torch.from_numpy(score.astype(np.float32)),
                                               torch.from_numpy(slog))
        f = orc.head_sample(logits, V, 1 / 0.8, 77, 5, 0)
        assert np.array_equal(g_smp.numpy(), f[3])
        np.testing.assert_allclose(g_slog.numpy(), f[5], rtol=1e-6)
        open(os.path.join(result_dir, f"ok{rank}"), "w").write("ok")
    finally:
        dist.destroy_process_group()


def test_tp_host_logic_two_gloo_ranks(tmp_path):
    world = 2
    mp.start_processes(worker, args=(world, free_port(), str(tmp_path)), nprocs=world, start_method="spawn",
                       join=True)
    for r in range(world):
        assert (tmp_path / f"ok{r}").exists()


def test_combine_rules():
    from qwen_a100_fastpath_b200 import tp
    g = torch.tensor([[[2.0, 5.0, 3.0]], [[2.0, 1.0, 2.5]], [[1.0, 9.0, 1.0]]], dtype=torch.float64)
    mx, am, lse = tp.combine_head_stats(g)
    assert float(mx[0]) == 2.0 and int(am[0]) == 1
    assert abs(float(lse[0]) - float(torch.logsumexp(torch.tensor([3.0, 2.5, 1.0], dtype=torch.float64), 0))) < 1e-6
    with pytest.raises(ValueError):
        tp.shard_range(10, 0, 4)


def test_sample_combine_rules():
    from qwen_a100_fastpath_b200 import tp
    # per shard (score, global column, logit): the largest score wins, lowest column on ties
    g = torch.tensor([[[1.5, 7.0, 0.2]], [[2.5, 130.0, -1.0]], [[2.5, 129.0, 0.7]]], dtype=torch.float64)
    col, logit = tp.combine_head_samples(g)
    assert int(col[0]) == 129 and abs(float(logit[0]) - 0.7) < 1e-7
    parts = [(g[r, :, 0].numpy(), g[r, :, 1].numpy().astype(np.int64), g[r, :, 2].numpy()) for r in range(3)]
    o_col, o_logit = orc.combine_head_samples(parts)
    assert int(o_col[0]) == 129 and abs(float(o_logit[0]) - 0.7) < 1e-12
