"""Decode context parallelism (DCP): split-KV decode over the GPUs of one node.

Each rank holds a contiguous slice of every sequence's KV cache, decodes the same
queries against its slice (``qmla_mla_decode``), and the per-rank ``(o, lse)``
partials are combined with the log-sum-exp merge of the reference's DCP output
correction (``qwen_mla/dcp_fix.py:31-130``, patched into vLLM's
``cp_lse_ag_out_rs`` at ``:133-142``):

    lse_g = logsumexp_n lse_n          (NaN / +inf count as -inf)
    o     = sum_n exp(lse_n - lse_g) * o_n

Collective choreography (one process per GPU, ``torch.distributed`` over NCCL):
all-gather of the small ``lse`` tensor, a local correction kernel that scales the
rank's own partial (``qmla_dcp_correct``), then one all-reduce (or reduce-scatter
over heads) of the scaled partials.  The choreography takes the correction as a
callable so the host logic can be exercised with the ``gloo`` backend on CPU.
"""
from __future__ import annotations

import ctypes
from typing import Callable

import torch
import torch.distributed as dist

from . import _lib
from .mla_decode_attention import _dt


def correct_attn_out(out: torch.Tensor, lses: torch.Tensor, cp_rank: int, ctx=None,
                     is_lse_base_on_e: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """In-place DCP correction of this rank's output; returns ``(out, lse_global)``.

    Same signature, shapes and semantics as ``_mla_correct_attn_out``
    (``qwen_mla/dcp_fix.py:102-130``): ``out`` [B,H,D] or [B,1,H,D], ``lses`` [N,B,H]
    (or with singleton dims), any head dim D.
    """
    del ctx
    if out.ndim == 4 and out.shape[1] == 1:
        out = out.squeeze(1)
    if out.ndim != 3:
        raise ValueError(f"expected out [B,H,D] or [B,1,H,D], got {tuple(out.shape)}")
    if lses.ndim == 4 and lses.shape[-1] == 1:
        lses = lses.squeeze(-1)
    if lses.ndim == 4 and lses.shape[1] == 1:
        lses = lses.squeeze(1)
    if lses.ndim != 3 or lses.dtype != torch.float32:
        raise ValueError(f"expected fp32 lses [N,B,H], got {tuple(lses.shape)} {lses.dtype}")
    if out.stride(-1) != 1 or lses.stride(-1) != 1:
        raise ValueError("out and lses need a unit stride on the last dim")
    B, H, D = out.shape
    N = lses.shape[0]
    lse = torch.empty(B, H, dtype=torch.float32, device=out.device)
    lib = _lib.load()
    stream = torch.cuda.current_stream(out.device).cuda_stream
    _lib.check("qmla_dcp_correct", lib.qmla_dcp_correct(
        ctypes.c_void_p(out.data_ptr()), _dt(out), out.stride(0), out.stride(1),
        ctypes.c_void_p(lses.data_ptr()), lses.stride(0), lses.stride(1), ctypes.c_void_p(lse.data_ptr()),
        N, cp_rank, B, H, D, 1 if is_lse_base_on_e else 0, ctypes.c_void_p(stream)))
    return out, lse


def merge_partials(parts: torch.Tensor, part_lses: torch.Tensor, o: torch.Tensor | None = None,
                   lse: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused merge of N partials held on one GPU: parts [N,B,H,D], part_lses [N,B,H] fp32."""
    N, B, H, D = parts.shape
    parts = parts.contiguous()
    part_lses = part_lses.contiguous().float()
    if o is None:
        o = torch.empty(B, H, D, dtype=parts.dtype, device=parts.device)
    if lse is None:
        lse = torch.empty(B, H, dtype=torch.float32, device=parts.device)
    lib = _lib.load()
    stream = torch.cuda.current_stream(parts.device).cuda_stream
    _lib.check("qmla_dcp_merge", lib.qmla_dcp_merge(
        ctypes.c_void_p(parts.data_ptr()), _dt(parts), ctypes.c_void_p(part_lses.data_ptr()),
        ctypes.c_void_p(o.data_ptr()), _dt(o), ctypes.c_void_p(lse.data_ptr()), N, B, H, D,
        ctypes.c_void_p(stream)))
    return o, lse


def shard_bounds(seq_len: int, world: int, rank: int) -> tuple[int, int]:
    """Token range [lo, hi) of one sequence held by ``rank`` (contiguous, even split)."""
    return seq_len * rank // world, seq_len * (rank + 1) // world


def shard_lengths(seq_lens: list[int], world: int, rank: int) -> list[int]:
    """Per-sequence token counts of this rank's KV shard."""
    return [hi - lo for lo, hi in (shard_bounds(int(L), world, rank) for L in seq_lens)]


def lse_all_gather(lse: torch.Tensor, group=None) -> torch.Tensor:
    """[B,H] fp32 per rank -> [N,B,H] on every rank."""
    world = dist.get_world_size(group)
    out = torch.empty((world,) + tuple(lse.shape), dtype=lse.dtype, device=lse.device)
    dist.all_gather(list(out.unbind(0)), lse.contiguous(), group=group)
    return out


def merge_across_ranks(o_part: torch.Tensor, lse_part: torch.Tensor, group=None,
                       correct: Callable | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Combine this rank's (o_part [B,H,D] fp32, lse_part [B,H] fp32) with the other ranks'.

    all-gather lse -> correct(o_part, lses, rank) scales the local partial in place ->
    all-reduce(sum) of the scaled partials.  Every rank ends with the merged (o, lse).
    ``correct`` defaults to :func:`correct_attn_out` (the CUDA kernel).
    """
    rank = dist.get_rank(group)
    lses = lse_all_gather(lse_part, group)
    fn = correct or correct_attn_out
    o_scaled, lse_g = fn(o_part, lses, rank)
    dist.all_reduce(o_scaled, op=dist.ReduceOp.SUM, group=group)
    return o_scaled, lse_g
