"""qwen_mla_vllm_b200 — B200-native paged latent-KV MLA / GLA decode attention.

A drop-in for the decode hot path of the qwen-mla-vllm plugin: the Triton
entry point ``decode_attention_fwd`` (``mla_decode_attention``), the
FlashInfer adapter ``forward_mqa`` / ``plan_for_step`` (``fi_decode``), the
FP8 cache writer and layout helpers (``mla_impl``) and the decode-context-
parallel merge (``dcp``), all over hand-written sm_100a kernels in
``libqmla.so`` (C ABI: ``include/qmla.h``).
"""
from . import _lib  # noqa: F401

__all__ = ["_lib"]
