"""vLLM patches of the B200 W8A16 decode path (the drop-in boundary).

Same patch targets, guards and fallbacks as ``qwen_fastpath.patches`` of EurekaZang/qwen-a100-fastpath
(plugin/qwen_fastpath/patches.py:10-189); the kernels behind them are ``libqf_b200.so``:

* ``patch_flash_attention``: ``FlashAttentionImpl.forward`` sends uniform speculative-verification batches
  (every request with the same ``1 < Q <= 8`` query tokens) to the split-KV GQA-packed kernel ``qf_spec_attn``
  (patches.py:10-69, spec_attn.py:139-173); everything else stays on FlashAttention.

* ``patch_int8_linear``: ``CutlassInt8ScaledMMLinearKernel.apply_weights(self, layer, x, bias=None)`` routes
  dynamic symmetric per-token W8A8 linears (patches.py:110) to the opaque custom op
  ``torch.ops.vllm.qf_int8_linear(x, w_q, w_s, bias)`` (patches.py:84-106).  bf16 rows on a K-major weight with
  per-channel scales run on libqf_b200: ``M <= 16`` on the W8A16 kernel (bias fused, rounded like the reference's
  ``y + bias``), more rows (prefill) on the tcgen05 W8A8 kernel with the arithmetic of the reference's vLLM
  fallback (patches.py:99-101); anything else (fp16 activations, weights the tensor maps cannot take) keeps
  vLLM's CUTLASS W8A8 path.
* ``patch_draft_lm_head``: an int8 per-row copy of the MTP draft lm_head made at load time
  (patches.py:133-152), ``compute_logits`` through the int8 head (patches.py:157-174), and ``get_top_tokens``
  taken from the head kernel's fused argmax (patches.py:176-185), which also yields the per-row logsumexp
  probabilistic drafting needs (left on the model as ``_qf_head_stats``).

vLLM is imported lazily inside the patch functions; hooks missing from the installed vLLM are skipped with a
log line instead of failing ``register()``.
"""
from __future__ import annotations

import logging

import torch

logger = logging.getLogger("vllm.qwen_fastpath")

MAX_SPEC_QUERY_LEN = 8


# ----------------------------------------------------------------------------------------------
# QWEN_FAST_ATTN
# ----------------------------------------------------------------------------------------------
def spec_attn_eligible(impl) -> bool:
    """Whether a FlashAttention layer can take the split-KV verification kernel (the reference's layer guard,
    patches.py:23-42, with attributes read defensively across vLLM versions; the FlashAttention version does not
    matter here because the kernel only reads the paged cache).  Cached on the layer."""
    ok = getattr(impl, "_qf_eligible", None)
    if ok is None:
        from vllm.v1.attention.backends import flash_attn as fa
        from .spec_attn import supported
        sw = getattr(impl, "sliding_window", None)
        ok = bool(
            getattr(impl, "attn_type", None) == fa.AttentionType.DECODER
            and getattr(impl, "dcp_world_size", 1) == 1
            and not getattr(impl, "fa4_hd256", False)
            and (sw is None or tuple(sw) == (-1, -1))
            and getattr(impl, "alibi_slopes", None) is None
            and not getattr(impl, "logits_soft_cap", None)
            and getattr(impl, "sinks", None) is None
            and not fa.is_quantized_kv_cache(impl.kv_cache_dtype)
            and impl.num_heads % impl.num_kv_heads == 0
            and impl.head_size in (64, 128, 256)
            and supported(impl.num_heads, impl.num_kv_heads, impl.head_size, 2, 16)
            and getattr(impl, "kv_sharing_target_layer_name", None) is None)
        impl._qf_eligible = ok
    return ok


def spec_attn_caches(kv_cache: torch.Tensor, head_size: int):
    """(key_cache, value_cache) views ``[num_blocks, page, num_kv_heads, head_size]`` of a layer's KV cache: vLLM's
    FlashAttention layout ``[2, num_blocks, page, HKV, D]`` (``unbind(0)``), or the interleaved layout the reference
    reads (``[num_blocks, HKV, page, 2 D]``, ``transpose(1, 2).split(D, -1)``, patches.py:55); None otherwise."""
    if kv_cache.dim() == 5 and kv_cache.shape[0] == 2 and kv_cache.shape[-1] == head_size:
        return kv_cache.unbind(0)
    if kv_cache.dim() == 4 and kv_cache.shape[-1] == 2 * head_size:
        k, v = kv_cache.transpose(1, 2).split(head_size, dim=-1)
        return k, v
    return None


def spec_attn_forward(impl, query, kv_cache, md, output, output_scale=None, output_block_scale=None):
    """The body of the patched ``FlashAttentionImpl.forward`` for one call: runs the split-KV kernel and returns
    ``output`` for a uniform speculative-verification batch (every request has the same ``1 < Q <= 8`` query tokens,
    causal, no cascade), None when the call must stay on FlashAttention (patches.py:44-66 of the reference)."""
    if (md is None or output_scale is not None or output_block_scale is not None
            or not 1 < md.max_query_len <= MAX_SPEC_QUERY_LEN or getattr(md, "use_cascade", False)
            or getattr(md, "causal", True) is not True
            or getattr(md, "mm_prefix_query_range_tensor", None) is not None
            or getattr(md, "rswa_prefix_lens", None) is not None
            or query.dtype != torch.bfloat16 or not spec_attn_eligible(impl)):
        return None
    num_reqs = md.query_start_loc.shape[0] - 1
    q_len = md.max_query_len
    if md.num_actual_tokens != num_reqs * q_len:  # uniform: every request has exactly q_len tokens
        return None
    caches = spec_attn_caches(kv_cache, impl.head_size)
    if caches is None or caches[0].dtype != torch.bfloat16:
        return None
    from .spec_attn import gqa_packed_spec_attention, supported
    key_cache, value_cache = caches
    if not supported(impl.num_heads, impl.num_kv_heads, impl.head_size, q_len, key_cache.shape[1]):
        return None
    q3 = query.view(query.shape[0], impl.num_heads, impl.head_size)
    o3 = output.view(output.shape[0], impl.num_heads, impl.head_size)
    gqa_packed_spec_attention(q3, key_cache, value_cache, o3, md.seq_lens, md.block_table, num_reqs, q_len,
                              impl.num_kv_heads, impl.scale)
    return output


def patch_flash_attention() -> bool:
    """Route uniform speculative-decode batches (every request has Q = 1 + k query tokens, 1 < Q <= 8) through the
    split-KV GQA-packed kernel; prefill, mixed batches and Q == 1 stay on FlashAttention (patches.py:10-69)."""
    try:
        from vllm.v1.attention.backends import flash_attn as fa
    except Exception as e:  # noqa: BLE001 -- any import failure of the backend disables only this patch
        logger.info("qwen_fastpath: attention patch skipped (%s)", e)
        return False
    orig_forward = fa.FlashAttentionImpl.forward
    if getattr(orig_forward, "_qwen_fastpath", False):
        return False

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale=None,
                output_block_scale=None):
        out = spec_attn_forward(self, query, kv_cache, attn_metadata, output, output_scale, output_block_scale)
        if out is not None:
            return out
        return orig_forward(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale,
                            output_block_scale)

    forward._qwen_fastpath = True
    forward._qf_orig = orig_forward
    fa.FlashAttentionImpl.forward = forward
    logger.info("qwen_fastpath: split-KV GQA-packed attention enabled for speculative-decode verification")
    return True


# ----------------------------------------------------------------------------------------------
# QWEN_FAST_LINEAR
# ----------------------------------------------------------------------------------------------
def w8a8_fallback(x2: torch.Tensor, w_q: torch.Tensor, w_s: torch.Tensor, bias: torch.Tensor | None,
                  out_dtype: torch.dtype) -> torch.Tensor:
    """vLLM's stock W8A8 path for what the small-M kernel does not take (patches.py:99-100 of the reference):
    dynamic per-token int8 activations and the CUTLASS int8 GEMM."""
    from vllm import _custom_ops as ops
    x_q, x_s, _ = ops.scaled_int8_quant(x2.contiguous(), None, None, symmetric=True)
    return ops.cutlass_scaled_mm(x_q, w_q, scale_a=x_s, scale_b=w_s, out_dtype=out_dtype, bias=bias)


def make_int8_linear_op():
    """The ``qf_int8_linear`` implementation and its fake (shape-only) counterpart.

    bf16 activations on a K-major int8 weight with per-channel scales run on libqf_b200: ``M <= 16`` rows on the
    small-M W8A16 kernel (the reference's path), more rows on the tcgen05 W8A8 kernel with the reference's own
    fallback arithmetic (per-token int8 activations, scaled int32 GEMM).  Anything else keeps vLLM's path."""
    from ._lib import QF_MAX_N, load_torch_ops
    kernel = load_torch_ops()  # torch.ops.qf_b200.int8_linear (csrc/qf_torch_ops.cpp)
    bf16 = torch.bfloat16

    def qf_int8_linear(x: torch.Tensor, w_q: torch.Tensor, w_s: torch.Tensor,
                       bias: torch.Tensor | None) -> torch.Tensor:
        # the reference's gate (patches.py:91) without its M limit, plus the tensor-map rules for the weight view
        # (16-byte base, 16-byte row stride); the operator checks the rest and picks the kernel by M
        N = w_q.shape[1]
        if (x.dtype is bf16 and w_q.stride(0) == 1 and w_s.numel() == N and 0 < N <= QF_MAX_N and x.shape[-1] > 0
                and w_q.data_ptr() % 16 == 0 and (N == 1 or w_q.stride(1) % 16 == 0)):
            return kernel(x, w_q, w_s, bias)
        x2 = x.reshape(-1, x.shape[-1])
        return w8a8_fallback(x2, w_q, w_s, bias, x.dtype).view(*x.shape[:-1], N)

    def qf_int8_linear_fake(x: torch.Tensor, w_q: torch.Tensor, w_s: torch.Tensor,
                            bias: torch.Tensor | None) -> torch.Tensor:
        return x.new_empty((*x.shape[:-1], w_q.shape[1]))

    return qf_int8_linear, qf_int8_linear_fake


def patch_int8_linear() -> bool:
    """Small-M (decode) W8A8 linears -> B200 W8A16 kernel on the same int8 weights; large M keeps CUTLASS."""
    from vllm.model_executor.kernels.linear.scaled_mm.cutlass import CutlassInt8ScaledMMLinearKernel
    from vllm.utils.torch_utils import direct_register_custom_op

    from .w8a16 import SMALL_M

    orig_apply = CutlassInt8ScaledMMLinearKernel.apply_weights
    if getattr(orig_apply, "_qwen_fastpath", False):
        return False

    op, fake = make_int8_linear_op()
    if not hasattr(torch.ops.vllm, "qf_int8_linear"):
        direct_register_custom_op("qf_int8_linear", op, mutates_args=[], fake_impl=fake)

    def apply_weights(self, layer, x, bias=None):
        w_q, w_s, i_s, i_zp, azp_adj = self._get_layer_params(layer)
        if i_s is None and i_zp is None and azp_adj is None:  # dynamic symmetric per-token activations
            return torch.ops.vllm.qf_int8_linear(x, w_q, w_s, bias)
        return orig_apply(self, layer, x, bias)

    apply_weights._qwen_fastpath = True
    apply_weights._qf_orig = orig_apply
    CutlassInt8ScaledMMLinearKernel.apply_weights = apply_weights
    logger.info("qwen_fastpath: B200 W8A16 decode path for W8A8-int8 linears (M <= %d), CUTLASS above", SMALL_M)
    return True


# ----------------------------------------------------------------------------------------------
# QWEN_FAST_DRAFT_HEAD
# ----------------------------------------------------------------------------------------------
def quantize_head_rows(weight: torch.Tensor, block_rows: int = 16384):
    """Per-row symmetric int8 copy of an lm_head weight ``[V, H]`` (patches.py:143-147): ``s = max|w| / 127``
    (at least 1e-8 / 127), ``q = clamp(round_half_even(w / s), -127, 127)``.  Returns (int8 ``[V, H]``, fp32
    ``[V]``) on the weight's device.  A bf16 CUDA weight is quantized by the library's device kernel
    (``qf_quantize_rows_int8``, one pass, bit-identical); a weight still on the host (loading) goes through the
    reference's torch arithmetic in 16384-row blocks so the fp32 temporaries stay small."""
    V, H = weight.shape
    w8 = torch.empty((V, H), dtype=torch.int8, device=weight.device)
    scale = torch.empty((V,), dtype=torch.float32, device=weight.device)
    if weight.is_cuda and weight.dtype == torch.bfloat16 and weight.stride(1) == 1 and H <= 8192:
        from ._lib import LIB, check
        check("qf_quantize_rows_int8", LIB.qf_quantize_rows_int8(
            weight.data_ptr(), weight.stride(0), V, H, w8.data_ptr(), H, scale.data_ptr(),
            torch.cuda.current_stream(weight.device).cuda_stream))
        return w8, scale
    with torch.no_grad():
        for r0 in range(0, V, block_rows):
            rows = weight[r0:r0 + block_rows].float()
            s = rows.abs().amax(dim=1).clamp_(min=1e-8) / 127.0
            w8[r0:r0 + block_rows] = torch.round(rows / s[:, None]).clamp_(-127, 127).to(torch.int8)
            scale[r0:r0 + block_rows] = s
    return w8, scale


def attach_int8_head(draft_model) -> bool:
    """Give a draft model (``Qwen3_5MTP``-like: ``lm_head.weight`` 2-D) its int8 head copy (patches.py:133-152).
    The reference requires ``lm_head.tp_size == 1`` (patches.py:138); here a vocab-sharded head (tensor parallel) is
    taken too: each rank quantizes its own shard (the quantizer is per row), its statistics are combined over the
    ranks in ``get_top_tokens`` and its logits gathered as vLLM's LogitsProcessor does in ``compute_logits``.  Heads
    with added (LoRA) vocabulary keep the original path.  Returns True if attached."""
    lm_head = getattr(draft_model, "lm_head", None)
    weight = getattr(lm_head, "weight", None)
    si = getattr(lm_head, "shard_indices", None)
    if weight is None or weight.dim() != 2 or si is None or getattr(si, "num_added_elements", 0):
        return False
    from .w8a16 import pick_config
    V, H = weight.shape
    w8, scale = quantize_head_rows(weight)
    num_pad = si.num_org_vocab_padding
    draft_model._qf_head_i8 = (w8.t(), scale, num_pad, pick_config(V, H))
    draft_model._qf_head_tp = int(getattr(lm_head, "tp_size", 1))
    logger.info("qwen_fastpath: int8 draft lm_head (%d x %d, %.2f GB, tp %d) for MTP proposals", V, H,
                w8.numel() / 1e9, draft_model._qf_head_tp)
    return True


def int8_head(model, hidden_states: torch.Tensor, want_logits: bool = True):
    """Run the int8 head if the model and inputs qualify (patches.py:157-166); else None.

    Returns (logits bf16 [M, V] or None, row_max, row_argmax (+ vocab start), row_lse)."""
    from .w8a16 import SMALL_M, w8a16_head
    q = model.__dict__.get("_qf_head_i8")
    lp = getattr(model, "logits_processor", None)
    if (q is None or lp is None or hidden_states.dim() != 2 or hidden_states.shape[0] > SMALL_M
            or hidden_states.shape[0] < 1 or hidden_states.dtype != torch.bfloat16 or lp.logits_as_input
            or lp.soft_cap is not None or lp.scale != 1.0
            or getattr(model, "draft_id_to_target_id", None) is not None):
        return None
    w_t, scale, num_pad, cfg = q
    if cfg is None:
        return None
    si = model.lm_head.shard_indices
    V = w_t.shape[1]
    out = w8a16_head(hidden_states, w_t, scale, n_valid=V - num_pad, vocab_offset=si.org_vocab_start_index,
                     want_logits=want_logits, pdl=True)
    if model.__dict__.get("_qf_head_tp", 1) > 1:
        # vocab shards: combine the per-shard (max, argmax, lse) over the tensor-parallel ranks (collective: every
        # rank takes this path with the same shapes)
        from .tp import gather_head_stats
        out = (out[0], *gather_head_stats(out[1], out[2], out[3], group=_tp_group().device_group))
    model._qf_head_stats = out[1:]
    return out


def draft_compute_logits(model, hidden_states: torch.Tensor, spec_step_idx, orig_logits):
    """Body of the patched ``Qwen3_5MTP.compute_logits`` (patches.py:168-174 of the reference): the int8 head's
    logits cut to ``org_vocab_size``, or the original method where the int8 head does not apply."""
    out = int8_head(model, hidden_states)
    if out is None:
        return orig_logits(model, hidden_states, spec_step_idx)
    logits = out[0]
    if model.__dict__.get("_qf_head_tp", 1) > 1:  # vocab shards: gather them as vLLM's LogitsProcessor does
        logits = model.logits_processor._gather_logits(logits)
        if logits is None:  # ranks other than 0 under a gather (not all-gather)
            return None
    return logits[..., : model.logits_processor.org_vocab_size]


def draft_get_top_tokens(model, hidden_states: torch.Tensor, orig_logits, orig_top=None):
    """Body of the patched ``Qwen3_5MTP.get_top_tokens`` (patches.py:176-185 of the reference): the int8 head's
    fused argmax (vocab padding excluded, + ``org_vocab_start_index``), else the original method, else the argmax of
    the original logits with the padding masked."""
    out = int8_head(model, hidden_states, want_logits=False)
    if out is not None:
        return out[2]
    if orig_top is not None:
        return orig_top(model, hidden_states)
    logits = orig_logits(model, hidden_states)
    si = model.lm_head.shard_indices
    if si.num_org_vocab_padding > 0:
        logits[..., -si.num_org_vocab_padding:] = -float("inf")
    return logits.argmax(dim=-1) + si.org_vocab_start_index


# ----------------------------------------------------------------------------------------------
# tensor parallelism: row-parallel linears with the all-reduce fused into the GEMM
# ----------------------------------------------------------------------------------------------
def _tp_group():
    """vLLM's tensor-parallel GroupCoordinator (``cpu_group`` for the buffer exchange, ``device_group`` for the
    small gathers)."""
    from vllm.distributed import get_tp_group
    return get_tp_group()


_ROW_COMMS: dict = {}


def _make_row_comm(group, max_count: int):
    from .tp import NVLinkAllReduce
    return NVLinkAllReduce(max_count, group=group.cpu_group)


def row_comm(group, count: int):
    """The NVLink buffers of this process's tensor-parallel group, made on first use (collective: the ranks run the
    same layers in the same order).  None while a CUDA graph is being captured and no buffers exist yet (the IPC
    exchange cannot be captured); the layer then keeps vLLM's path for that call on every rank."""
    key = (torch.cuda.current_device(), id(group))
    comm = _ROW_COMMS.get(key)
    if comm is None or comm.max_count < count:
        if torch.cuda.is_current_stream_capturing():
            return None
        comm = _make_row_comm(group, max(count, 16 * 8192))
        _ROW_COMMS[key] = comm
    return comm


def row_parallel_forward(layer, input_: torch.Tensor):
    """Body of the patched ``RowParallelLinear.forward`` for a W8A8-int8 layer under tensor parallelism whose
    output is reduced (o_proj, down): this rank's K-shard GEMM with the all-reduce in its epilogue over NVLink
    (``qf_w8a16_gemm_allreduce``; vLLM would run the shard GEMM and then ``tensor_model_parallel_all_reduce``).
    Returns None where it does not apply (the caller then runs vLLM's forward): no reduction, one rank, another
    quant kernel or static activation scales, more than 16 rows, non-bf16 activations, a weight view the tensor maps
    cannot take.  The bias is added once after the sum (vLLM adds it on rank 0 before the sum: the same value up
    to the bf16 rounding of the partial)."""
    from .w8a16 import SMALL_M, w8a16_mm_allreduce
    if not getattr(layer, "reduce_results", False) or getattr(layer, "tp_size", 1) <= 1:
        return None
    kernel = getattr(getattr(layer, "scheme", None), "kernel", None)
    if kernel is None or not getattr(getattr(type(kernel), "apply_weights", None), "_qwen_fastpath", False):
        return None
    w_q, w_s, i_s, i_zp, azp_adj = kernel._get_layer_params(layer)
    if i_s is not None or i_zp is not None or azp_adj is not None:
        return None
    if layer.input_is_parallel:
        x = input_
    else:
        x = input_.chunk(layer.tp_size, dim=-1)[layer.tp_rank].contiguous()
    K = x.shape[-1]
    N = w_q.shape[1]
    M = x.numel() // K if K else 0
    if (x.dtype is not torch.bfloat16 or not 1 <= M <= SMALL_M or w_q.stride(0) != 1 or w_s.numel() != N
            or w_q.data_ptr() % 16 or (N > 1 and w_q.stride(1) % 16)):
        return None
    comm = row_comm(_tp_group(), M * ((N + 127) // 128 * 128))
    if comm is None:
        return None
    y = w8a16_mm_allreduce(x.reshape(M, K), w_q, w_s, comm, pdl=True).view(*x.shape[:-1], N)
    bias = getattr(layer, "bias", None)
    if bias is not None and not layer.skip_bias_add:
        y = y + bias
    if not getattr(layer, "return_bias", False):
        return y
    return y, (bias if layer.skip_bias_add else None)


def patch_row_parallel() -> bool:
    """Route reduced row-parallel int8 layers through the fused GEMM + NVLink all-reduce under tensor parallelism."""
    from vllm.model_executor.layers.linear import RowParallelLinear
    orig = RowParallelLinear.forward
    if getattr(orig, "_qwen_fastpath", False):
        return False

    def forward(self, input_):
        out = row_parallel_forward(self, input_)
        return orig(self, input_) if out is None else out

    forward._qwen_fastpath = True
    forward._qf_orig = orig
    RowParallelLinear.forward = forward
    logger.info("qwen_fastpath: row-parallel int8 linears (M <= 16) with the all-reduce fused over NVLink")
    return True


def patch_draft_lm_head() -> bool:
    """MTP drafting through an int8 per-row copy of the lm_head: half the bytes of the bf16 head per draft
    token, and argmax / logsumexp fused into the GEMM."""
    try:
        from vllm.model_executor.models import qwen3_5_mtp
    except Exception as e:  # noqa: BLE001 -- any import failure of the host model disables only this patch
        logger.info("qwen_fastpath: draft head patch skipped (%s)", e)
        return False
    cls = qwen3_5_mtp.Qwen3_5MTP
    if getattr(cls.compute_logits, "_qwen_fastpath", False):
        return False

    try:
        from vllm.v1.worker.gpu.spec_decode.mtp.speculator import MTPSpeculator
    except Exception:  # noqa: BLE001
        MTPSpeculator = None
    if MTPSpeculator is not None:
        orig_load = MTPSpeculator.load_draft_model
        if not getattr(orig_load, "_qwen_fastpath", False):
            def load_draft_model(self, target_model, target_attn_layer_names):
                draft_model = orig_load(self, target_model, target_attn_layer_names)
                if isinstance(draft_model, cls):
                    attach_int8_head(draft_model)
                return draft_model

            load_draft_model._qwen_fastpath = True
            MTPSpeculator.load_draft_model = load_draft_model
    else:
        logger.info("qwen_fastpath: this vLLM has no MTPSpeculator.load_draft_model hook; call "
                    "patches.attach_int8_head(draft_model) after loading the drafter")

    orig_logits = cls.compute_logits
    orig_top = getattr(cls, "get_top_tokens", None)

    def compute_logits(self, hidden_states, spec_step_idx=0):
        return draft_compute_logits(self, hidden_states, spec_step_idx, orig_logits)

    def get_top_tokens(self, hidden_states):
        return draft_get_top_tokens(self, hidden_states, orig_logits, orig_top)

    compute_logits._qwen_fastpath = True
    get_top_tokens._qwen_fastpath = True
    cls.compute_logits = compute_logits
    cls.get_top_tokens = get_top_tokens
    logger.info("qwen_fastpath: int8 draft lm_head enabled")
    return True
