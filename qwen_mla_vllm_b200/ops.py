"""``torch.library`` custom ops over libqmla: ``torch.ops.qmla.mla_decode`` and
``torch.ops.qmla.gather_cache``.

vLLM compiles its model with torch.compile and captures CUDA graphs around it. A ctypes call
inside a compiled region would break the graph. These ops are opaque to the compiler: each
declares which arguments it writes (``o`` / ``lse``, ``dst``) and has a fake kernel that does
nothing, so tracing never touches the library. The real kernels run the same entry points as
``mla_decode_attention.decode_attention_fwd`` and ``mla_gather.gather_cache_torch``.

    qmla::mla_decode(Tensor q, Tensor kv_cache, Tensor(a!) o, Tensor(b!) lse, Tensor block_table,
                     Tensor seq_lens, Tensor workspace, int rank, int qk_dim, int rms_offset,
                     int rms_mode, int page_size, float sm_scale, float logit_cap,
                     Tensor? k_scale, int qrows) -> ()
    qmla::gather_cache(Tensor src_cache, Tensor(a!) dst, Tensor block_table, Tensor cu_seq_lens,
                       Tensor token_to_seq, int num_tokens, str kv_cache_dtype, Tensor scale,
                       Tensor? seq_starts, int rms_offset, int rms_heads, str rms_mode) -> ()

``rms_mode`` of mla_decode is a ``QMLA_RMS_*`` code (0 none, 1 native, 2 bf16 bytes, 3 log8).
Set ``rms_offset`` < 0 in gather_cache for a 2-byte cache (no rms layout).
"""
from __future__ import annotations

from typing import Optional

import torch

from .mla_decode_attention import build_params, run_params
from .mla_gather import gather_cache_torch


@torch.library.custom_op("qmla::mla_decode", mutates_args=("o", "lse"), device_types="cuda")
def mla_decode(q: torch.Tensor, kv_cache: torch.Tensor, o: torch.Tensor, lse: torch.Tensor,
               block_table: torch.Tensor, seq_lens: torch.Tensor, workspace: torch.Tensor, rank: int,
               qk_dim: int, rms_offset: int, rms_mode: int, page_size: int, sm_scale: float,
               logit_cap: float, k_scale: Optional[torch.Tensor], qrows: int) -> None:
    """Paged latent decode into ``o`` / ``lse`` (``qmla_mla_decode``).  ``workspace`` backs the
    kernel's split scratch when it is large enough (vLLM's ``attn_logits`` qualifies)."""
    p = build_params(q, kv_cache, o, lse, block_table, seq_lens, rank=rank, qk_dim=qk_dim,
                     rms_offset=rms_offset, rms_mode=rms_mode, page_size=page_size, sm_scale=sm_scale,
                     logit_cap=logit_cap, k_scale=k_scale, qrows=qrows)
    run_params(p, q.device, scratch=workspace)


@mla_decode.register_fake
def _mla_decode_fake(q, kv_cache, o, lse, block_table, seq_lens, workspace, rank, qk_dim, rms_offset,
                     rms_mode, page_size, sm_scale, logit_cap, k_scale, qrows) -> None:
    return None


@torch.library.custom_op("qmla::gather_cache", mutates_args=("dst",), device_types="cuda")
def gather_cache(src_cache: torch.Tensor, dst: torch.Tensor, block_table: torch.Tensor,
                 cu_seq_lens: torch.Tensor, token_to_seq: torch.Tensor, num_tokens: int,
                 kv_cache_dtype: str, scale: torch.Tensor, seq_starts: Optional[torch.Tensor],
                 rms_offset: int, rms_heads: int, rms_mode: str) -> None:
    """Chunked-prefill context gather into ``dst`` (``qmla_gather_cache``)."""
    gather_cache_torch(src_cache=src_cache, dst=dst, block_table=block_table, cu_seq_lens=cu_seq_lens,
                       token_to_seq=token_to_seq, num_tokens=num_tokens, kv_cache_dtype=kv_cache_dtype,
                       scale=scale, seq_starts=seq_starts,
                       mla_rms=(rms_offset, rms_heads, rms_mode) if rms_offset >= 0 else None)


@gather_cache.register_fake
def _gather_cache_fake(src_cache, dst, block_table, cu_seq_lens, token_to_seq, num_tokens, kv_cache_dtype,
                       scale, seq_starts, rms_offset, rms_heads, rms_mode) -> None:
    return None
