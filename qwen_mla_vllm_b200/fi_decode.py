"""Drop-in for the plugin's FlashInfer adapter (``qwen_mla/fi_decode.py``), backed by this build's
sm_100a decode instead of the forked FlashInfer kernel.

Same contract as the reference:

* ``plan_for_step(builder, md, common=None)`` runs in the metadata builder, outside any CUDA
  graph (``fi_decode.py:291-326``).  It plans from host sequence lengths when vLLM has them
  (no device sync), with MTP rows flattened as the builder does, into buffers whose device
  addresses never change, and attaches the plan to the metadata as ``_mla_fi_plan``.
* ``forward_mqa(impl, q, kv_c_and_k_pe_cache, attn_metadata, layer)`` returns ``(o, lse)`` (or
  ``(o, None)``), or ``None`` to decline so the caller falls back to the Triton-signature path
  (``fi_decode.py:338-384``).  It declines on the same mismatches: no plan, batch or head count,
  softmax scale, rope window or latent rank differing from the plan.
* The LSE is returned in base 2, as the FlashInfer kernel returns it unless
  ``return_lse_base_on_e`` is set (``kernels/qwen_mla.cuh:1085``).

The cache is read in place: latent ``[..., :rank]``, rope window ``[..., rank:rank+win]``, rms
at ``impl.rms_offset``.  q may be the ``(q_nope, q_pe)`` tuple vLLM passes or one tensor.
"""
from __future__ import annotations

import ctypes
import math
import os

import numpy as np
import torch

from . import _lib
from .mla_decode_attention import _FP8_TYPES, build_params, rms_mode_for, run_params

_LOG2E = 1.0 / math.log(2.0)


def fp8_rms_mode() -> str:
    """The FP8 rms tail format selected by QWEN_MLA_FP8_RMS, as the plugin reads it
    (``mla_impl.py:134-139``): log8 (default), bf16 or e4m3."""
    m = os.environ.get("QWEN_MLA_FP8_RMS", "log8")
    if m not in ("log8", "bf16", "e4m3"):
        raise ValueError(f"QWEN_MLA_FP8_RMS={m!r}: expected log8, bf16 or e4m3")
    return m


def rope_window(head_offset: int, n_local: int, rope_group: int, rope_dim: int) -> tuple[int, int]:
    """(offset, width) of the rope slice this rank's heads span (``fi_decode.py:103-114``):
    the cache stores only that window, so the offset is 0 and the width covers the rope groups
    from the rank's first to its last global head."""
    first = head_offset // rope_group
    last = (head_offset + n_local - 1) // rope_group
    return 0, (last - first + 1) * rope_dim


class RankPlan:
    """Per-KV-group decode plan with device buffers that keep their addresses across steps."""

    def __init__(self, device, rank, win, n_local, page_size, max_batch, max_pages=None, kpe=None,
                 spec=False):
        del max_pages, spec
        self.device = torch.device(device)
        self.rank, self.win, self.n_local = rank, win, n_local
        self.kpe = kpe or win
        self.page_size = page_size
        self.max_batch = max_batch
        i32 = dict(dtype=torch.int32, device=self.device)
        self.tile_prefix = torch.zeros(max_batch + 1, **i32)
        self.kv_indptr = torch.zeros(max_batch + 1, **i32)
        self.kv_len = torch.zeros(max_batch, **i32)
        pin = self.device.type == "cuda"
        self._ring = []
        for _ in range(4):  # async H2D copies still in flight are never overwritten
            bufs = [torch.zeros(max_batch + 1, dtype=torch.int32), torch.zeros(max_batch + 1, dtype=torch.int32),
                    torch.zeros(max(max_batch, 1), dtype=torch.int32)]
            self._ring.append([b.pin_memory() for b in bufs] if pin else bufs)
        self._ring_i = 0
        self.block_table = None
        self.seq_lens = None
        self.host_planned = False
        self.planned_batch = -1
        self.planned_scale = None
        self.fits = True
        self.workspace = None

    def plan_cpu(self, block_table, seq_lens, lens_cpu, scale, q_dtype=None, kv_dtype=None):
        """Plan from host lengths (no device->host sync): tile prefix, kv_indptr and kv_len are
        computed on the host by ``qmla_plan`` and copied asynchronously into the fixed buffers."""
        del q_dtype, kv_dtype
        B = int(lens_cpu.shape[0])
        if B > self.max_batch:
            raise ValueError(f"decode batch {B} exceeds the preallocated {self.max_batch}")
        tp, ip, kl = self._ring[self._ring_i]
        self._ring_i = (self._ring_i + 1) % len(self._ring)
        lens = np.ascontiguousarray(lens_cpu.to(torch.int32).numpy())
        tt, tpg = ctypes.c_int64(), ctypes.c_int64()
        _lib.check("qmla_plan", _lib.load().qmla_plan(
            lens.ctypes.data, B, self.page_size, tp.data_ptr(), ip.data_ptr(), kl.data_ptr(),
            ctypes.byref(tt), ctypes.byref(tpg)))
        nb = self.device.type == "cuda"
        self.tile_prefix[:B + 1].copy_(tp[:B + 1], non_blocking=nb)
        self.kv_indptr[:B + 1].copy_(ip[:B + 1], non_blocking=nb)
        self.kv_len[:B].copy_(kl[:B], non_blocking=nb)
        self.block_table, self.seq_lens = block_table, seq_lens
        self.host_planned = True
        self.planned_batch = B
        self.planned_scale = scale

    def plan(self, block_table, seq_lens, scale, q_dtype=None, kv_dtype=None):
        """Plan without host lengths: the decode builds its tile prefix on the device."""
        del q_dtype, kv_dtype
        B = int(seq_lens.shape[0])
        if B > self.max_batch:
            raise ValueError(f"decode batch {B} exceeds the preallocated {self.max_batch}")
        self.block_table, self.seq_lens = block_table, seq_lens
        self.host_planned = False
        self.planned_batch = B
        self.planned_scale = scale


def _decode_lens_cpu(common, nd, exact=False):
    """Host copy of the decode rows' lengths if vLLM already holds one (never syncs)."""
    if common is None:
        return None
    c = getattr(common, "_seq_lens_cpu", None)
    if c is None and not exact:
        c = getattr(common, "seq_lens_cpu_upper_bound", None)
    if c is None:
        return None
    c = torch.as_tensor(c)
    return c[:nd].to(torch.int32) if c.device.type == "cpu" else None


def plan_for_step(builder, md, common=None) -> None:
    """Build or refresh the step's plan and attach it to ``md`` (outside graph capture)."""
    if getattr(md, "decode", None) is None or not getattr(builder, "_mla_fi_ok", True):
        return
    try:
        plan = getattr(builder, "_mla_fi_plan", None)
        if plan is None:
            plan = RankPlan(**builder._mla_fi_cfg)
            builder._mla_fi_plan = plan
        q = getattr(md.decode, "_mla_q", 1)
        rows = md.decode.seq_lens.shape[0]
        lens_cpu = _decode_lens_cpu(common, rows // q, exact=q > 1)
        if lens_cpu is not None and q > 1:  # the builder's MTP flattening (mla_impl.py:628-662)
            lens_cpu = (lens_cpu[:, None] + torch.arange(1 - q, 1, dtype=lens_cpu.dtype)[None, :]).reshape(-1).clamp_(min=0)
        if lens_cpu is not None and os.environ.get("QWEN_MLA_FI_SYNC_PLAN") != "1":
            plan.plan_cpu(md.decode.block_table, md.decode.seq_lens, lens_cpu, builder._mla_fi_scale)
        else:
            plan.plan(md.decode.block_table, md.decode.seq_lens, builder._mla_fi_scale)
    except Exception:  # noqa: BLE001 - a failed plan declines the fast path for this step only
        return
    object.__setattr__(md, "_mla_fi_plan", plan)


def forward_mqa(impl, q, kv_c_and_k_pe_cache, attn_metadata, layer, return_lse_base_on_e=False):
    """Returns ``(out, lse|None)``, or ``None`` when this step has no usable plan."""
    plan = getattr(attn_metadata, "_mla_fi_plan", None)
    if plan is None:
        return None
    if isinstance(q, tuple):
        q_nope_in, q_pe_in = q
        n_rows, n_heads = q_nope_in.shape[0], q_nope_in.shape[1]
    else:
        q_nope_in, q_pe_in = q, None
        n_rows, n_heads = q.shape[0], q.shape[1]
    if n_rows != plan.planned_batch or n_heads != plan.n_local:
        return None
    if impl.scale != plan.planned_scale:
        return None
    rank = plan.rank
    off, win = rope_window(impl.mla_head_offset, n_heads, impl.mla_rope_group, impl.mla_rope_dim)
    if win != plan.win or rank != impl.kv_lora_rank:
        return None

    cache = kv_c_and_k_pe_cache
    if q_pe_in is None:
        q_nope, q_pe = q_nope_in[..., :rank], q_nope_in[..., rank + off:rank + off + win]
    else:
        q_nope, q_pe = q_nope_in[..., :rank], q_pe_in[..., off:off + win]
    fp8 = cache.dtype in _FP8_TYPES or cache.dtype == torch.uint8
    rms_offset = impl.rms_offset
    fmt = fp8_rms_mode() if fp8 else "bf16"
    mode = rms_mode_for(cache.dtype, rms_offset, fp8 and fmt == "bf16", fp8 and fmt == "log8")
    k_scale = getattr(layer, "_k_scale", None) if fp8 else None
    if k_scale is not None and k_scale.dtype != torch.float32:
        k_scale = k_scale.float()
    want_lse = bool(getattr(impl, "need_to_return_lse_for_decode", False))
    o = torch.empty(n_rows, n_heads, rank, dtype=q_nope.dtype, device=q_nope.device)
    lse = torch.empty(n_rows, n_heads, dtype=torch.float32, device=q_nope.device) if want_lse else None
    p = build_params(q_nope, cache, o, lse, plan.block_table, plan.seq_lens, rank=rank, qk_dim=rank + win,
                     rms_offset=rms_offset, rms_mode=mode, page_size=plan.page_size, sm_scale=impl.scale,
                     k_scale=k_scale, q_pe=q_pe,
                     plan_tile_prefix=plan.tile_prefix if plan.host_planned else None)
    run_params(p, q_nope.device, workspace=plan.workspace)
    if lse is not None and not return_lse_base_on_e:
        lse.mul_(_LOG2E)  # the kernel's natural-log LSE in FlashInfer's base 2
    return o, lse
