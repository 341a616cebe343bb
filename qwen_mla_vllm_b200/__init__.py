"""qwen_mla_vllm_b200 — B200-native paged latent-KV MLA / GLA decode attention.

A drop-in for the decode hot path of the qwen-mla-vllm plugin: the Triton
entry point ``decode_attention_fwd`` (``mla_decode_attention``), the
FlashInfer adapter ``forward_mqa`` / ``plan_for_step`` (``fi_decode``), the
FP8 cache writer (``kv_cache``), the prefill context gather (``mla_gather``),
the decode-context-parallel merge (``dcp``) and ``torch.library`` ops for
compiled graphs (``ops``: ``torch.ops.qmla.mla_decode`` / ``gather_cache``),
all over hand-written sm_100a kernels in ``libqmla.so`` (C ABI:
``include/qmla.h``).
"""
from . import _lib  # noqa: F401

__all__ = ["_lib"]
