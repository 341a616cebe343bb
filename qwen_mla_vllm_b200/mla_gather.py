"""Chunked-prefill context gather: paged latent cache rows -> a dense destination.

``gather_cache_torch`` keeps the name, keyword arguments, in-place output and errors of
``qwen_mla/ops/mla_gather.py:28-76``.  For destination row j, s = token_to_seq[j] and
tok = j - cu_seq_lens[s] (+ seq_starts[s]), the row is token tok of sequence s, found
through ``block_table``.  A 2-byte cache row is copied whole.  An FP8 row is dequantised:
[latent | rope] e4m3 * scale, then the rms tail (log8 code, raw bf16 bytes, or e4m3 *
scale) as one element per head at the rms offset.  Later columns are left as they were.
The work is one CUDA kernel (``qmla_gather_cache``), with no slicing and no fp32
intermediates in memory.  The reference runs 8192-row slices only to bound the memory
those intermediates take.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

_DT = {torch.bfloat16: _lib.DT_BF16, torch.float16: _lib.DT_F16, torch.float32: _lib.DT_F32}
_RMS = {"log8": _lib.RMS_LOG8, "bf16": _lib.RMS_BF16, "e4m3": _lib.RMS_NATIVE}
_status: dict[int, torch.Tensor] = {}


def _i32(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.int32 and t.is_contiguous() else t.to(torch.int32).contiguous()


def _status_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _status:
        _status[idx] = torch.zeros(1, dtype=torch.int32, device=device)
    return _status[idx]


def gather_status(device: torch.device | int | None = None, clear: bool = True) -> int:
    """Status bits of this device's gathers since the last clear (2 = a row had an index
    outside the tables and was skipped).  Synchronises the current stream."""
    dev = torch.device("cuda", device) if isinstance(device, int) else (device or torch.device("cuda"))
    w = _status_word(dev)
    v = int(w.item())
    if clear:
        w.zero_()
    return v


def gather_cache_torch(*, src_cache: torch.Tensor, dst: torch.Tensor, block_table: torch.Tensor,
                       cu_seq_lens: torch.Tensor, token_to_seq: torch.Tensor, num_tokens: int,
                       kv_cache_dtype: str, scale: torch.Tensor, seq_starts: torch.Tensor | None = None,
                       mla_rms=None, check: bool = False) -> None:
    """Write rows [0, num_tokens) of ``dst`` in place (``qwen_mla/ops/mla_gather.py:28-76``).

    src_cache [pages, page_size, ...]: bf16 / f16 ("auto", "bfloat16", "float16") or an FP8
    byte cache ("fp8*"); mla_rms = (rms_offset, heads[, "bf16" | "log8" | "e4m3"]) is
    required for FP8.  dst [>= num_tokens, width] bf16 / f16 / f32 with unit column stride.
    Index tensors may be any integer dtype (converted to int32 when they are not).
    ``check=True`` synchronises and raises IndexError when a row's sequence, token or page
    index fell outside the tables (such rows are skipped); the reference raises there too.
    """
    fp8 = str(kv_cache_dtype).startswith("fp8")
    if not fp8 and kv_cache_dtype not in ("auto", "bfloat16", "float16"):
        raise NotImplementedError(f"MLA gather has no dequant path for kv_cache_dtype={kv_cache_dtype}")
    if fp8 and mla_rms is None:
        raise NotImplementedError("FP8 MLA gather needs the row layout (rms offset, heads)")
    if num_tokens <= 0:
        return
    if not src_cache.is_cuda or not dst.is_cuda:
        raise ValueError("gather_cache_torch: src_cache and dst must be CUDA tensors")
    if dst.dim() != 2 or dst.stride(1) != 1 or dst.shape[0] < num_tokens:
        raise ValueError(f"dst must be [>= {num_tokens}, width] with unit column stride, got "
                         f"{tuple(dst.shape)} strides {dst.stride()}")
    if dst.dtype not in _DT:
        raise TypeError(f"dst dtype {dst.dtype}: expected bf16, f16 or f32")
    if src_cache.dim() < 3:
        raise ValueError("src_cache must be [pages, page_size, ...]")
    # one row = the trailing dims, densely packed (a [pages, page, 1, width] cache is the usual form)
    row_elems, dense = 1, 1
    for d in range(src_cache.dim() - 1, 1, -1):
        if src_cache.shape[d] != 1 and src_cache.stride(d) != dense:
            raise ValueError("src_cache rows (dims 2..) must be contiguous")
        dense *= src_cache.shape[d]
        row_elems *= src_cache.shape[d]
    p = _lib.GatherParams()
    if fp8:
        if src_cache.element_size() != 1:
            raise TypeError("an fp8 kv_cache_dtype needs a 1-byte cache")
        off, nh = int(mla_rms[0]), int(mla_rms[1])
        mode = mla_rms[2] if len(mla_rms) > 2 else "bf16"
        if mode not in _RMS:
            raise ValueError(f"mla_rms mode {mode!r}: expected bf16, log8 or e4m3")
        need = off + (2 if mode == "bf16" else 1) * nh
        if row_elems < need or dst.shape[1] < off + nh:
            raise ValueError(f"row of {row_elems} bytes / dst width {dst.shape[1]} too small for "
                             f"rms_offset {off} + {nh} heads ({mode})")
        p.src_dtype = _lib.DT_FP8E4M3
        p.rms_offset, p.rms_heads, p.rms_mode = off, nh, _RMS[mode]
        sc = scale if isinstance(scale, torch.Tensor) else torch.tensor(float(scale))
        sc = sc.to(device=dst.device, dtype=torch.float32).reshape(-1)[:1].contiguous()
        p.scale = sc.data_ptr()
    else:
        if src_cache.dtype not in (torch.bfloat16, torch.float16):
            raise TypeError(f"src_cache dtype {src_cache.dtype}: expected bf16 or f16")
        if dst.shape[1] != row_elems:
            raise ValueError(f"dst width {dst.shape[1]} != cache row width {row_elems}")
        p.src_dtype = _DT[src_cache.dtype]
        p.row_elems = row_elems
    bt = block_table if block_table.dtype == torch.int32 and block_table.stride(-1) == 1 \
        else block_table.to(torch.int32).contiguous()
    cu, t2s = _i32(cu_seq_lens), _i32(token_to_seq)
    st = _i32(seq_starts) if seq_starts is not None else None
    num_seqs = min(bt.shape[0], cu.shape[0] - 1, st.shape[0] if st is not None else bt.shape[0])
    if t2s.shape[0] < num_tokens:
        raise ValueError(f"token_to_seq has {t2s.shape[0]} entries, need {num_tokens}")
    status = _status_word(dst.device)
    p.src_cache = src_cache.data_ptr()
    p.src_stride_page, p.src_stride_token = src_cache.stride(0), src_cache.stride(1)
    p.page_size, p.num_pages = src_cache.shape[1], src_cache.shape[0]
    p.block_table, p.block_table_stride, p.block_table_cols = bt.data_ptr(), bt.stride(0), bt.shape[1]
    p.cu_seq_lens, p.token_to_seq = cu.data_ptr(), t2s.data_ptr()
    p.seq_starts = st.data_ptr() if st is not None else None
    p.num_seqs, p.num_tokens = max(num_seqs, 0), int(num_tokens)
    p.dst, p.dst_stride_row, p.dst_dtype = dst.data_ptr(), dst.stride(0), _DT[dst.dtype]
    p.status = status.data_ptr()
    p.device = dst.device.index if dst.device.index is not None else torch.cuda.current_device()
    stream = torch.cuda.current_stream(dst.device).cuda_stream
    _lib.check("qmla_gather_cache", _lib.load().qmla_gather_cache(ctypes.byref(p), ctypes.c_void_p(stream)))
    if check and gather_status(dst.device) & _lib.DEV_ERR_INDEX:
        raise IndexError("gather_cache_torch: a row's sequence, token or page index is outside the tables")
