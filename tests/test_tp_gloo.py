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


# ------------------------------------------------------------------------------------------------------------------
# the plugin's tensor-parallel routing (patches.row_parallel_forward, the vocab-sharded int8 draft head) on gloo
# ranks, with the CUDA kernels replaced by stand-ins computed from the oracle (the routing, shard bookkeeping and
# collectives are what is tested here; the kernels have their own GPU tests)
# ------------------------------------------------------------------------------------------------------------------
def plugin_worker(rank: int, world: int, port: int, result_dir: str):
    import types

    import torch.distributed as dist

    from qwen_a100_fastpath_b200 import patches, w8a16
    from tests.conftest import from_dev_bf16
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    group = types.SimpleNamespace(cpu_group=None, device_group=None)
    patches._tp_group = lambda: group
    calls = []

    def t16(bits):
        return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)

    try:
        # ---- row-parallel layer: this rank's K-shard, the all-reduce fused into the GEMM (stand-in: the oracle's
        # bf16 partial, summed over the ranks in rank order in fp32)
        M, N, K = 5, 256, 512
        x_bits, W, s = orc.make_inputs(31, 16, N, K)
        k0, k1 = rank * K // world, (rank + 1) * K // world

        def fused_stand_in(x, w_q, w_s, comm, out=None, pdl=None):
            calls.append(("fused", tuple(x.shape), comm))
            part = torch.from_numpy(orc.bf16_to_f32(orc.w8a16_mm(from_dev_bf16(x), w_q.t().contiguous().numpy(),
                                                                 w_s.reshape(-1).numpy(), "bf16")))
            parts = [torch.empty_like(part) for _ in range(world)]
            dist.all_gather(parts, part)
            acc = torch.zeros_like(part)
            for p in parts:
                acc += p
            return acc.to(torch.bfloat16)

        w8a16.w8a16_mm_allreduce = fused_stand_in
        patches.row_comm = lambda g, count: "comm"

        class Kernel:
            def apply_weights(self, layer, x, bias=None):
                raise AssertionError("the fused path replaces apply_weights + all-reduce")
            apply_weights._qwen_fastpath = True

            def _get_layer_params(self, layer):
                return layer.w_q, layer.w_s, None, None, None

        w_shard = torch.from_numpy(np.ascontiguousarray(W[:, k0:k1]))
        layer = types.SimpleNamespace(reduce_results=True, tp_size=world, tp_rank=rank, input_is_parallel=True,
                                      bias=None, skip_bias_add=False, return_bias=False,
                                      scheme=types.SimpleNamespace(kernel=Kernel()),
                                      w_q=w_shard.t(), w_s=torch.from_numpy(s).view(N, 1))
        x_shard = t16(np.ascontiguousarray(x_bits[:M, k0:k1]))
        y = patches.row_parallel_forward(layer, x_shard)
        want = np.zeros((M, N), np.float32)
        for r in range(world):
            a, b = r * K // world, (r + 1) * K // world
            want += orc.bf16_to_f32(orc.w8a16_mm(np.ascontiguousarray(x_bits[:M, a:b]),
                                                 np.ascontiguousarray(W[:, a:b]), s, "bf16"))
        assert np.array_equal(from_dev_bf16(y), orc.f32_to_bf16(want))
        # not for this path: 17 rows, fp16, no reduction, one rank, another kernel
        assert patches.row_parallel_forward(layer, t16(np.ascontiguousarray(x_bits[:16, k0:k1])).repeat(2, 1)[:17]) is None
        assert patches.row_parallel_forward(layer, x_shard.half()) is None
        for attr, val in (("reduce_results", False), ("tp_size", 1)):
            other = types.SimpleNamespace(**{**vars(layer), attr: val})
            assert patches.row_parallel_forward(other, x_shard) is None
        plain = types.SimpleNamespace(**{**vars(layer), "scheme": types.SimpleNamespace(kernel=object())})
        assert patches.row_parallel_forward(plain, x_shard) is None
        # input split here when the layer's input is not yet parallel; bias added once, after the sum
        b_bits = orc.make_bias(3, N)
        full = types.SimpleNamespace(**{**vars(layer), "input_is_parallel": False, "bias": t16(b_bits)})
        y2 = patches.row_parallel_forward(full, t16(np.ascontiguousarray(x_bits[:M])))
        assert np.array_equal(from_dev_bf16(y2), orc.add_bias_bf16(orc.f32_to_bf16(want), b_bits))
        assert [c[0] for c in calls] == ["fused", "fused"]

        # ---- vocab-sharded int8 draft head: each rank quantizes its shard; get_top_tokens combines the shards'
        # (max, argmax, lse), compute_logits gathers the shards' logits as vLLM's LogitsProcessor does
        V, H, pad, Mh = 1024, 256, 24, 3
        rs = np.random.RandomState(17)
        wb = orc.f32_to_bf16(rs.standard_normal((V, H)).astype(np.float32) * 0.05)
        wb[V - pad:] = 0                                     # vocab padding rows (last shard)
        wb[300] = wb[800]                                    # equal rows on different shards: lowest index wins
        Vl = V // world
        n_org = Vl - (pad if rank == world - 1 else 0)

        def head_stand_in(h, w_t, scale, n_valid=None, vocab_offset=0, want_logits=True, pdl=None, out=None):
            lg = orc.w8a16_mm(from_dev_bf16(h), w_t.t().contiguous().numpy(), scale.numpy(), "bf16")
            mx, am, lse = orc.head_stats(lg, n_valid, vocab_offset)
            return (t16(lg) if want_logits else None, torch.from_numpy(mx), torch.from_numpy(am),
                    torch.from_numpy(lse))

        w8a16.w8a16_head = head_stand_in

        def gather_logits(lg):
            parts = [torch.empty_like(lg) for _ in range(world)]
            dist.all_gather(parts, lg)
            return torch.cat(parts, dim=-1)

        lm_head = types.SimpleNamespace(weight=t16(wb[rank * Vl:(rank + 1) * Vl]), tp_size=world,
                                        shard_indices=types.SimpleNamespace(
                                            num_org_vocab_padding=Vl - n_org, org_vocab_start_index=rank * Vl,
                                            num_added_elements=0))
        lp = types.SimpleNamespace(logits_as_input=False, soft_cap=None, scale=1.0, org_vocab_size=V - pad,
                                   _gather_logits=gather_logits)
        model = types.SimpleNamespace(lm_head=lm_head, logits_processor=lp)
        assert patches.attach_int8_head(model)
        h_bits = orc.make_inputs(41, Mh, 8, H)[0]
        h_bits[1] = orc.f32_to_bf16(orc.bf16_to_f32(wb[300]) * 40)   # row 1 points at the duplicated rows
        q, sc = orc.quantize_rows(wb)
        ref_logits = orc.w8a16_mm(h_bits, q, sc, "bf16")

        def never(*a, **k):
            raise AssertionError("original method called although the int8 head applies")

        top = patches.draft_get_top_tokens(model, t16(h_bits), never, never)
        assert np.array_equal(top.numpy(), orc.top_tokens(ref_logits, pad, 0))
        assert int(top[1]) == 300
        lg = patches.draft_compute_logits(model, t16(h_bits), 0, never)
        assert lg.shape == (Mh, V - pad) and np.array_equal(from_dev_bf16(lg), ref_logits[:, : V - pad])
        mx_f, am_f, lse_f = orc.head_stats(ref_logits, V - pad, 0)
        np.testing.assert_allclose(model._qf_head_stats[2].numpy(), lse_f, rtol=1e-6)
        open(os.path.join(result_dir, f"ok{rank}"), "w").write("ok")
    finally:
        dist.destroy_process_group()


def test_plugin_tensor_parallel_routing_two_gloo_ranks(tmp_path):
    world = 2
    mp.start_processes(plugin_worker, args=(world, free_port(), str(tmp_path)), nprocs=world, start_method="spawn",
                       join=True)
    for r in range(world):
        assert (tmp_path / f"ok{r}").exists()
