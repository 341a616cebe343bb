"""Drop-in for the reference's Triton decode entry point, backed by libqmla.

``decode_attention_fwd`` keeps the signature, argument meaning, in-place
outputs and error behaviour of
``qwen_mla/ops/mla_decode_attention.py:1264-1359`` (the function
``QwenMLATritonImpl._mla_kernel`` calls, ``qwen_mla/mla_impl.py:302-307``).
The work runs in one persistent sm_100a kernel (plus a plan and a merge
kernel); there is no Triton, FlashInfer or CPU path.

``attn_logits`` stays caller-owned scratch as in the reference: when it is
large enough it backs the kernel's split workspace, otherwise a per-device
buffer cached by this module is used (allocated on first use, so make the
first call outside CUDA-graph capture, as vLLM's warm-up does).
"""
from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib

_TORCH_DT = {torch.bfloat16: _lib.DT_BF16, torch.float16: _lib.DT_F16, torch.float32: _lib.DT_F32}
_FP8_TYPES = tuple(t for t in (getattr(torch, "float8_e4m3fn", None),) if t is not None)

_ws_lock = threading.Lock()
_ws_cache: dict[int, torch.Tensor] = {}


def _page_stride(buf: torch.Tensor, page_size: int) -> int:
    """Stride between pages in elements; 3-D buffers pack pages along tokens.

    Same contract as ``_page_stride`` in the reference
    (``qwen_mla/ops/mla_decode_attention.py:78-84``): the real stride is read,
    so cross-layer views with gaps work.
    """
    if buf.ndim == 3:
        buf = buf.unflatten(-3, (-1, page_size))
    return buf.stride(-4)


def _workspace(device: torch.device, nbytes: int, scratch: torch.Tensor | None) -> torch.Tensor:
    if scratch is not None and scratch.is_contiguous() and scratch.numel() * scratch.element_size() >= nbytes \
            and scratch.data_ptr() % 256 == 0 and scratch.device == device:
        return scratch
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _ws_lock:
        ws = _ws_cache.get(idx)
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _ws_cache[idx] = ws
        return ws


def _dt(t: torch.Tensor) -> int:
    if t.dtype in _TORCH_DT:
        return _TORCH_DT[t.dtype]
    raise TypeError(f"unsupported dtype {t.dtype}")


def build_params(q: torch.Tensor, kv: torch.Tensor, o: torch.Tensor, lse: torch.Tensor | None,
                 block_table: torch.Tensor, seq_lens: torch.Tensor, *, rank: int, qk_dim: int,
                 rms_offset: int, rms_mode: int, page_size: int, sm_scale: float,
                 logit_cap: float = 0.0, k_scale: torch.Tensor | None = None,
                 q_pe: torch.Tensor | None = None, qrows: int = 1, num_ctas: int = 0,
                 plan_tile_prefix: torch.Tensor | None = None) -> _lib.DecodeParams:
    """Fill a ``qmla_decode_params`` from tensors (no launch, no allocation).

    kv: [pages, page_size, 1, W] or [pages*page_size, 1, W] cache (bf16 or FP8 bytes).
    q:  [rows, heads, >= rank] (the latent part, plus the rope part when q_pe is None).
    """
    if kv.ndim not in (3, 4):
        raise ValueError(f"cache must be 3-D or 4-D, got {tuple(kv.shape)}")
    fp8 = kv.dtype in _FP8_TYPES or kv.dtype == torch.uint8
    es = 1 if fp8 else 2
    if not fp8 and kv.dtype != torch.bfloat16:
        raise TypeError(f"cache dtype {kv.dtype} not supported (bf16 or float8_e4m3fn)")
    num_pages = kv.shape[0] if kv.ndim == 4 else kv.shape[0] // page_size
    if kv.ndim == 4 and kv.shape[1] != page_size:
        raise ValueError(f"page_size {page_size} != cache page dim {kv.shape[1]}")
    for name, t in (("q", q), ("o", o), ("block_table", block_table), ("seq_lens", seq_lens)):
        if not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor")
    if q.stride(-1) != 1 or o.stride(-1) != 1 or kv.stride(-1) != 1:
        raise ValueError("q, o and the cache need a unit stride on the last dim")
    if block_table.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise TypeError("block_table and seq_lens must be int32")
    if seq_lens.stride(0) != 1 or block_table.stride(-1) != 1:
        raise ValueError("seq_lens and block_table rows must be contiguous")
    p = _lib.DecodeParams()
    p.q = q.data_ptr()
    p.q_stride_row, p.q_stride_head = q.stride(0), q.stride(1)
    if q_pe is not None:
        if q_pe.stride(-1) != 1:
            raise ValueError("q_pe needs a unit stride on the last dim")
        p.q_pe = q_pe.data_ptr()
        p.qpe_stride_row, p.qpe_stride_head = q_pe.stride(0), q_pe.stride(1)
    else:
        p.q_pe = q.data_ptr() + rank * q.element_size()
        p.qpe_stride_row, p.qpe_stride_head = q.stride(0), q.stride(1)
    p.q_dtype = _dt(q)
    p.kv_cache = kv.data_ptr()
    p.kv_stride_page = _page_stride(kv, page_size)
    p.kv_stride_token = kv.stride(-3)
    p.kv_num_pages = num_pages
    p.kv_row_width = kv.shape[-1]
    p.kv_dtype = _lib.DT_FP8E4M3 if fp8 else _lib.DT_BF16
    p.page_size = page_size
    p.block_table = block_table.data_ptr()
    p.block_table_stride = block_table.stride(0)
    p.seq_lens = seq_lens.data_ptr()
    p.num_rows = q.shape[0]
    p.num_heads = q.shape[1]
    p.rank = rank
    p.qk_dim = qk_dim
    p.rms_offset = rms_offset
    p.rms_mode = rms_mode
    p.sm_scale = float(sm_scale)
    p.logit_cap = float(logit_cap or 0.0)
    p.k_scale = k_scale.data_ptr() if k_scale is not None else None
    p.qrows = qrows
    p.o = o.data_ptr()
    p.o_stride_row, p.o_stride_head = o.stride(0), o.stride(1)
    p.o_dtype = _dt(o)
    if lse is not None:
        p.lse = lse.data_ptr()
        p.lse_stride_row = lse.stride(0)
        p.lse_dtype = _dt(lse)
        if lse.stride(-1) != 1:
            raise ValueError("lse needs a unit stride on the head dim")
    p.num_ctas = num_ctas
    p.device = q.device.index if q.device.index is not None else torch.cuda.current_device()
    if plan_tile_prefix is not None:
        p.plan_tile_prefix = plan_tile_prefix.data_ptr()
    del es
    return p


def run_params(p: _lib.DecodeParams, device: torch.device, scratch: torch.Tensor | None = None,
               workspace: torch.Tensor | None = None) -> None:
    """Size the workspace, attach it and launch on the current stream."""
    lib = _lib.load()
    need = ctypes.c_int64(0)
    _lib.check("qmla_decode_workspace_bytes", lib.qmla_decode_workspace_bytes(ctypes.byref(p), ctypes.byref(need)))
    ws = workspace if workspace is not None else _workspace(device, int(need.value), scratch)
    if ws.numel() * ws.element_size() < need.value:
        raise ValueError(f"workspace of {ws.numel() * ws.element_size()} bytes < {need.value} needed")
    p.workspace = ws.data_ptr()
    p.workspace_bytes = ws.numel() * ws.element_size()
    stream = torch.cuda.current_stream(device).cuda_stream
    _lib.check("qmla_mla_decode", lib.qmla_mla_decode(ctypes.byref(p), ctypes.c_void_p(stream)))


def rms_mode_for(kv_dtype: torch.dtype, rms_offset: int, rms_bf16: bool, rms_log8: bool) -> int:
    """Map the reference's (rms_offset, rms_bf16, rms_log8) flags to QMLA_RMS_*."""
    if rms_offset < 0:
        return _lib.RMS_NONE
    fp8 = kv_dtype in _FP8_TYPES or kv_dtype == torch.uint8
    if fp8 and rms_log8:
        return _lib.RMS_LOG8
    if fp8 and rms_bf16:
        return _lib.RMS_BF16
    return _lib.RMS_NATIVE


def decode_attention_fwd(q, k_buffer, v_buffer, o, lse, req_to_token, b_seq_len, attn_logits,
                         num_kv_splits, sm_scale, page_size=1, logit_cap=0.0, k_scale=None,
                         v_scale=None, is_mla=False, rms_offset=-1, rms_bf16=False, rms_log8=False,
                         qrows=1):
    """Paged MLA decode with the reference's signature; writes ``o`` and ``lse`` in place.

    q [B, H, Lk+], k_buffer [pages, page_size, 1, W] (bf16, or FP8 e4m3 bytes with
    ``k_scale``), v_buffer = k_buffer[..., :rank], o [B, H, rank], lse [B, H],
    req_to_token [B, max_pages] int32, b_seq_len [B] int32.  ``qrows`` > 1 marks
    MTP verify rows that are already flattened with lengths L-(q-1-j); each row
    is decoded with its own length (the reference folds them for speed only).
    """
    assert num_kv_splits == attn_logits.shape[2]
    if q.shape[1] == v_buffer.shape[-2]:
        raise NotImplementedError("MHA decode (kv_group_num == 1) is outside this build's MLA path")
    if not is_mla and v_buffer.data_ptr() != k_buffer.data_ptr():
        raise NotImplementedError("only the MLA layout (v_buffer = k_buffer[..., :rank]) is supported")
    rank = v_buffer.shape[-1]
    qk_dim = rms_offset if rms_offset >= 0 else k_buffer.shape[-1]
    mode = rms_mode_for(k_buffer.dtype, rms_offset, rms_bf16, rms_log8)
    if k_scale is not None and not torch.is_tensor(k_scale):
        k_scale = torch.tensor(float(k_scale), dtype=torch.float32, device=q.device)
    if k_scale is not None and k_scale.dtype != torch.float32:
        k_scale = k_scale.float()
    p = build_params(q, k_buffer, o, lse, req_to_token, b_seq_len, rank=rank, qk_dim=qk_dim,
                     rms_offset=rms_offset, rms_mode=mode, page_size=page_size, sm_scale=sm_scale,
                     logit_cap=logit_cap, k_scale=k_scale, qrows=qrows)
    run_params(p, q.device, scratch=attn_logits)
