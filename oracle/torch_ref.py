"""torch (CPU) restatement of the reference's own decode references (oracle; test infrastructure).

TEST INFRASTRUCTURE ONLY: imported by ``bench.py``'s CPU legs (``cpu_baseline`` and
``--impl reference``), which time it on the host cores as the reference's CPU path, and by
``tests/``.  The product path never imports it.

The reference checks its decode kernels against small torch functions in its tests:
``ref_out`` (``tests/test_fi_partial_rope.py:49-58``, bf16 caches) and ``ref``
(``tests/test_fp8_kv.py:61-72``, FP8 caches).  Both gather one sequence's cache rows through
its block-table row, compute ``s = q . K^T / rms^T * sm_scale`` in float32, take ``softmax(s)``
and multiply by the latent part.  ``decode_paged`` below does the same per row of a paged
batch, with the per-row LSE (natural log, as the Triton stage 2 writes it,
``qwen_mla/ops/mla_decode_attention.py:1133``) and the FP8 rules of the Triton kernel:
K = e4m3 * k_scale rounded to bf16 (``:451-452``), rms from the log8 code (``:467-476``).
"""
from __future__ import annotations

import torch

_LOG8_STEP = 6.0 / 255.0


def _rms(rows: torch.Tensor, heads: int, rms_offset: int, mode: str, fp8: bool, k_scale: float):
    """[L, H] float32 divisor from the row tail (same rules as ``oracle.decode._rms_values``)."""
    if mode == "log8":
        return torch.exp2(-3.0 + rows[:, rms_offset:rms_offset + heads].float() * _LOG8_STEP)
    if mode == "bf16":
        b = rows[:, rms_offset:rms_offset + 2 * heads].contiguous()
        return b.view(torch.bfloat16).float()
    if fp8:
        return rows[:, rms_offset:rms_offset + heads].view(torch.float8_e4m3fn).float() * k_scale
    return rows[:, rms_offset:rms_offset + heads].float()


def decode_paged(q: torch.Tensor, cache: torch.Tensor, block_table: torch.Tensor, seq_lens, *, rank: int,
                 qk_dim: int, page_size: int, sm_scale: float, rms_offset: int, rms_mode: str = "native",
                 k_scale: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    """(o [rows, H, rank] f32, lse [rows, H] f32) for CPU tensors.

    cache: [pages, page_size, W] bf16, or uint8 bytes of an FP8 e4m3 cache.
    q: [rows, H, >= qk_dim] (bf16 or float32); seq_lens: ints (<= 0: o = 0, lse = -inf).
    """
    rows_n, H = q.shape[0], q.shape[1]
    fp8 = cache.dtype == torch.uint8
    o = torch.zeros(rows_n, H, rank, dtype=torch.float32)
    lse = torch.full((rows_n, H), float("-inf"), dtype=torch.float32)
    for r in range(rows_n):
        L = int(seq_lens[r])
        if L <= 0:
            continue
        npg = (L + page_size - 1) // page_size
        flat = cache[block_table[r, :npg].long()].reshape(npg * page_size, -1)[:L]
        if fp8:
            K = (flat[:, :qk_dim].view(torch.float8_e4m3fn).float() * k_scale).to(torch.bfloat16).float()
        else:
            K = flat[:, :qk_dim].float()
        qf = q[r, :, :qk_dim].float()
        s = qf @ K.T
        if rms_offset >= 0 and rms_mode != "none":
            m = _rms(flat, H, rms_offset, rms_mode, fp8, k_scale)
            s = s / torch.where(m > 0, m, torch.ones_like(m)).T
        s = s * sm_scale
        lse[r] = torch.logsumexp(s, -1)
        o[r] = torch.softmax(s, -1) @ K[:, :rank]
    return o, lse
