"""FP8 latent-cache writer: the producer of the FP8 row format the decode kernel reads.

``fp8_kv_cache_update`` keeps the arguments and semantics of
``QwenMLATritonImpl.do_kv_cache_update`` (``qwen_mla/mla_impl.py:309-342``) for an FP8
cache: row = [latent e4m3 | packed rope e4m3 | rms tail | pad] with ``x * (1/k_scale)``
clamped to +-448 and rounded to nearest-even e4m3; the rms tail is the log8 code
(one byte per head) or raw bf16 (two bytes per head); padding tokens (slot -1) are
redirected to slot 0.  One CUDA kernel, no allocation (graph-capturable).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib


def fp8_kv_cache_update(kv_c_normed: torch.Tensor, k_pe: torch.Tensor, kv_cache: torch.Tensor,
                        slot_mapping: torch.Tensor, k_scale: torch.Tensor, packed_rope: int,
                        local_heads: int, rms_mode: str = "log8") -> None:
    """Write FP8 rows for ``slot_mapping.numel()`` tokens into ``kv_cache`` in place.

    kv_c_normed [>=n, rank] bf16, k_pe [>=n, ...] bf16 holding [rope (packed_rope) | rms (heads)],
    kv_cache [blocks, block, 1, width] float8_e4m3fn or uint8, slot_mapping [n] int64,
    k_scale 0-d fp32 device tensor.
    """
    if rms_mode not in ("log8", "bf16"):
        raise ValueError(f"rms_mode {rms_mode!r}: expected log8 or bf16")
    if kv_cache.numel() == 0:
        return
    slots = slot_mapping.flatten()
    n = slots.shape[0]
    if slots.dtype != torch.int64:
        slots = slots.to(torch.int64)
    if kv_c_normed.dtype != torch.bfloat16 or k_pe.dtype != torch.bfloat16:
        raise TypeError("kv_c_normed and k_pe must be bf16")
    k_pe2 = k_pe.reshape(k_pe.shape[0], -1)
    if kv_c_normed.stride(-1) != 1 or k_pe2.stride(-1) != 1:
        raise ValueError("kv_c_normed and k_pe need a unit stride on the last dim")
    width = kv_cache.shape[-1]
    if kv_cache.element_size() != 1:
        raise TypeError("kv_cache must be an FP8 (1-byte) cache")
    row_stride = kv_cache.stride(-3) if kv_cache.ndim >= 3 else width
    if kv_cache.ndim == 4 and kv_cache.stride(0) != kv_cache.shape[1] * row_stride:
        raise ValueError("kv_cache blocks must be contiguous (slot = block * block_size + offset)")
    rank = kv_c_normed.shape[-1]
    if k_scale.dtype != torch.float32:
        k_scale = k_scale.float()
    lib = _lib.load()
    mode = _lib.RMS_LOG8 if rms_mode == "log8" else _lib.RMS_BF16
    stream = torch.cuda.current_stream(kv_cache.device).cuda_stream
    _lib.check("qmla_fp8_cache_write", lib.qmla_fp8_cache_write(
        ctypes.c_void_p(kv_c_normed.data_ptr()), kv_c_normed.stride(0), ctypes.c_void_p(k_pe2.data_ptr()),
        k_pe2.stride(0), ctypes.c_void_p(slots.data_ptr()), n, rank, packed_rope, local_heads, mode,
        ctypes.c_void_p(k_scale.data_ptr()), ctypes.c_void_p(kv_cache.data_ptr()), row_stride,
        ctypes.c_void_p(stream)))
