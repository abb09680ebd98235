"""vLLM general plugin: B200 (sm_100a) decode fast path for W8A8-int8 Qwen checkpoints.

Drop-in for EurekaZang/qwen-a100-fastpath's ``qwen_fastpath`` plugin (plugin/qwen_fastpath/__init__.py:17-28)
on its W8A16 decode-GEMM path and its speculative-verification attention.  vLLM loads it in every process through the ``vllm.general_plugins`` entry
point; ``register()`` is idempotent and each patch can be switched off with an environment variable:

  QWEN_FAST_ATTN=0        keep FlashAttention for speculative-verification batches
  QWEN_FAST_LINEAR=0      keep CUTLASS W8A8 for small-batch (decode) linear layers
  QWEN_FAST_DRAFT_HEAD=0  keep the bf16 lm_head for MTP draft proposals
"""
import logging
import os

logger = logging.getLogger("vllm.qwen_fastpath")
_registered = False


def register():
    global _registered
    if _registered:
        return
    _registered = True
    from . import patches
    if os.environ.get("QWEN_FAST_ATTN", "1") == "1":
        patches.patch_flash_attention()
    if os.environ.get("QWEN_FAST_LINEAR", "1") == "1":
        patches.patch_int8_linear()
        patches.patch_row_parallel()
    if os.environ.get("QWEN_FAST_DRAFT_HEAD", "1") == "1":
        patches.patch_draft_lm_head()
