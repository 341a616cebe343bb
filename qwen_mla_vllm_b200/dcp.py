"""Decode context parallelism (DCP): split-KV decode over the GPUs of one node.

Each rank holds a contiguous slice of every sequence's KV cache, decodes the same
queries against its slice (``qmla_mla_decode``), and the per-rank ``(o, lse)``
partials are combined with the log-sum-exp merge of the reference's DCP output
correction (``qwen_mla/dcp_fix.py:31-130``, patched into vLLM's
``cp_lse_ag_out_rs`` at ``:133-142``):

    lse_g = logsumexp_n lse_n          (NaN / +inf count as -inf)
    o     = sum_n exp(lse_n - lse_g) * o_n

Two ways to combine (one process per GPU):

* :class:`P2PExchange` (the default on GPUs): each rank decodes straight into its
  exchange buffer, and ONE kernel (``qmla_dcp_p2p_merge``) publishes an epoch flag
  to every peer, waits (bounded) for theirs and merges the N partials read over
  NVLink from the peers' buffers (CUDA IPC mappings).  Mode ``"rs"`` leaves rank r
  the heads ``[r*H/N, (r+1)*H/N)`` (vLLM's ``cp_lse_ag_out_rs`` layout), ``"ar"``
  all heads.
* :func:`merge_across_ranks` (the NCCL baseline, and what the ``gloo`` CPU tests
  exercise): all-gather of the small ``lse`` tensor, a local correction kernel that
  scales the rank's own partial (``qmla_dcp_correct``), then an all-reduce or a
  reduce-scatter over heads of the scaled partials.  It takes the correction as a
  callable so the host logic runs on CPU.
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


def head_group_of(rank: int, world: int, groups: int) -> tuple[int, int, int]:
    """GLA head-group sharding: (head group, rank inside the group's split-KV sub-group, sub-group
    size) of ``rank``.  The ``groups`` latent head groups (each with its own cache, rank-local
    latent ``r / groups``: ``qwen_mla/mla_impl.py:182-200``) are spread over the ranks in order:
    group g on ranks [g * world/groups, (g+1) * world/groups).  With world == groups each GPU
    holds one group and nothing is exchanged; with more ranks each group is additionally split by
    KV over its sub-group and merged there (the same LSE merge as DCP)."""
    if world % groups:
        raise ValueError(f"{world} ranks do not split into {groups} head groups")
    per = world // groups
    return rank // per, rank % per, per


def head_group_subgroups(world: int, groups: int) -> list:
    """One process group per head group (ranks of head_group_of).  Every rank must call this, in
    the same order, before using any of them (torch.distributed.new_group's rule)."""
    per = world // groups
    return [dist.new_group(list(range(g * per, (g + 1) * per))) for g in range(groups)]


def lse_all_gather(lse: torch.Tensor, group=None) -> torch.Tensor:
    """[B,H] fp32 per rank -> [N,B,H] on every rank."""
    world = dist.get_world_size(group)
    out = torch.empty((world,) + tuple(lse.shape), dtype=lse.dtype, device=lse.device)
    dist.all_gather(list(out.unbind(0)), lse.contiguous(), group=group)
    return out


def merge_across_ranks(o_part: torch.Tensor, lse_part: torch.Tensor, group=None,
                       correct: Callable | None = None, mode: str = "ar"
                       ) -> tuple[torch.Tensor, torch.Tensor]:
    """Combine this rank's (o_part [B,H,D] fp32, lse_part [B,H] fp32) with the other ranks'.

    all-gather lse -> correct(o_part, lses, rank) scales the local partial in place ->
    all-reduce (mode "ar": every rank gets o [B,H,D]) or reduce-scatter over heads
    (mode "rs": rank r gets o [B, H/N, D] of heads [r*H/N, (r+1)*H/N) and their lse).
    ``correct`` defaults to :func:`correct_attn_out` (the CUDA kernel).
    """
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    lses = lse_all_gather(lse_part, group)
    fn = correct or correct_attn_out
    o_scaled, lse_g = fn(o_part, lses, rank)
    if mode == "ar":
        dist.all_reduce(o_scaled, op=dist.ReduceOp.SUM, group=group)
        return o_scaled, lse_g
    if mode != "rs":
        raise ValueError(f"mode {mode!r}: expected 'ar' or 'rs'")
    B, H, D = o_scaled.shape
    if H % world:
        raise ValueError(f"{H} heads do not split over {world} ranks")
    hs = H // world
    # [N*B, hs, D]: rank n's block is the first dim's n-th B rows (NCCL and gloo agree on that)
    send = o_scaled.view(B, world, hs, D).transpose(0, 1).reshape(world * B, hs, D)
    out = torch.empty(B, hs, D, dtype=o_scaled.dtype, device=o_scaled.device)
    dist.reduce_scatter_tensor(out, send, op=dist.ReduceOp.SUM, group=group)
    return out, lse_g[:, rank * hs:(rank + 1) * hs].contiguous()


class _DeviceArray:
    """A raw device allocation seen through ``__cuda_array_interface__`` (zero copy)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 2, "strides": None}


def _device_view(ptr: int, shape: tuple, device, dtype=torch.float32) -> torch.Tensor:
    typestr = {torch.float32: "<f4", torch.int32: "<i4", torch.int64: "<i8"}[dtype]
    return torch.as_tensor(_DeviceArray(ptr, shape, typestr), device=device)


class ExchangeBuffer:
    """One rank's DCP exchange buffer (``qmla_dcp_buffer_alloc``) and its typed views."""

    def __init__(self, num_rows: int, num_heads: int, head_dim: int, device):
        self.device = torch.device(device)
        self.B, self.H, self.D = num_rows, num_heads, head_dim
        lib = _lib.load()
        vals = [ctypes.c_int64() for _ in range(5)]
        _lib.check("qmla_dcp_buffer_layout", lib.qmla_dcp_buffer_layout(
            num_rows, num_heads, head_dim, *[ctypes.byref(v) for v in vals]))
        self.total, self.o_off, self.o_slot, self.lse_off, self.lse_slot = (v.value for v in vals)
        ptr = ctypes.c_void_p()
        self.handle = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
        _lib.check("qmla_dcp_buffer_alloc", lib.qmla_dcp_buffer_alloc(
            self.device.index, self.total, ctypes.byref(ptr), self.handle))
        self.ptr = ptr.value

    def flags(self) -> torch.Tensor:
        """The header: flags[8] (epoch published by each rank), the status word, the last merged
        epoch (device-epoch mode) and the merge's block counter."""
        return _device_view(self.ptr, (_lib.DCP_MAX_WORLD + 3,), self.device, torch.int32)

    def partial(self, epoch: int) -> tuple[torch.Tensor, torch.Tensor]:
        """(o [B,H,D] f32, lse [B,H] f32) views of slot epoch & 1."""
        slot = epoch & 1
        o = _device_view(self.ptr + self.o_off + slot * self.o_slot, (self.B, self.H, self.D), self.device)
        lse = _device_view(self.ptr + self.lse_off + slot * self.lse_slot, (self.B, self.H), self.device)
        return o, lse

    def merge_stats(self) -> torch.Tensor:
        """The header's merge statistics (int64 view): merges, ns waiting for the peers' flags, ns
        from entry to exit, ns to publish, summed over the merges of this rank since the last
        ``zero_()``."""
        return _device_view(self.ptr + 64, (4,), self.device, torch.int64)

    def status(self) -> int:
        st = ctypes.c_int32()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check("qmla_dcp_read_status", _lib.load().qmla_dcp_read_status(
            ctypes.c_void_p(self.ptr), ctypes.c_void_p(stream), ctypes.byref(st)))
        return st.value

    def free(self) -> None:
        if self.ptr:
            _lib.load().qmla_dcp_buffer_free(ctypes.c_void_p(self.ptr))
            self.ptr = 0


def p2p_merge(bufs: list[int], rank: int, B: int, H: int, D: int, epoch: int, out: torch.Tensor,
              mode: str = "rs", lse_out: torch.Tensor | None = None, timeout_s: float = 2.0) -> None:
    """Launch ``qmla_dcp_p2p_merge`` for this rank over the exchange buffers ``bufs``
    (device addresses on this device, one per rank, this rank's own included).  ``epoch`` 0
    takes the step's epoch from the device (the rank's last merged epoch + 1)."""
    world = len(bufs)
    if not 1 <= world <= _lib.DCP_MAX_WORLD:
        raise ValueError(f"world {world} outside 1..{_lib.DCP_MAX_WORLD}")
    p = _lib.DcpP2PParams()
    for n, b in enumerate(bufs):
        p.bufs[n] = b
    p.world, p.rank = world, rank
    p.num_rows, p.num_heads, p.head_dim = B, H, D
    p.mode = {"ar": _lib.DCP_ALL_HEADS, "rs": _lib.DCP_HEAD_SCATTER}[mode]
    p.epoch = epoch
    p.out = out.data_ptr()
    p.out_stride_row, p.out_stride_head = out.stride(0), out.stride(1)
    if out.stride(2) != 1:
        raise ValueError("out needs a unit stride on the last dim")
    p.out_dtype = _dt(out)
    if lse_out is not None:
        if lse_out.dtype != torch.float32 or not lse_out.is_contiguous():
            raise ValueError("lse_out must be contiguous fp32")
        p.lse_out = lse_out.data_ptr()
    p.timeout_ns = int(timeout_s * 1e9)
    p.device = out.device.index
    stream = torch.cuda.current_stream(out.device).cuda_stream
    _lib.check("qmla_dcp_p2p_merge", _lib.load().qmla_dcp_p2p_merge(ctypes.byref(p), ctypes.c_void_p(stream)))


class P2PExchange:
    """DCP over NVLink peer memory for one rank of ``group`` (one process per GPU).

    ``partial()`` gives the (o, lse) views the rank's decode writes for the next step;
    ``merge()`` runs the one-kernel exchange.  Set-up exchanges the CUDA IPC handles of
    the ranks' buffers with ``all_gather_object`` (once); steps use no collective.
    """

    def __init__(self, num_rows: int, num_heads: int, head_dim: int, group=None, device=None,
                 timeout_s: float = 2.0, device_epoch: bool = True):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > _lib.DCP_MAX_WORLD:
            raise ValueError(f"at most {_lib.DCP_MAX_WORLD} ranks")
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None
                                   else torch.device(device).index)
        self.B, self.H, self.D = num_rows, num_heads, head_dim
        self.timeout_s = timeout_s
        # device_epoch: the merge kernel keeps the step's epoch in device memory (epoch 0 at the
        # C ABI), so steps captured in a CUDA graph can be replayed; self.epoch mirrors it on the
        # host for slot selection (a captured sequence must hold an even number of merges).
        self.device_epoch = device_epoch
        self.buf = ExchangeBuffer(num_rows, num_heads, head_dim, self.device)
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(self.buf.handle.raw), group=group)
        lib = _lib.load()
        self.ptrs, self._opened = [], []
        for n, h in enumerate(handles):
            if n == self.rank:
                self.ptrs.append(self.buf.ptr)
                continue
            ptr = ctypes.c_void_p()
            hb = ctypes.create_string_buffer(h, _lib.IPC_HANDLE_BYTES)
            _lib.check("qmla_dcp_buffer_open", lib.qmla_dcp_buffer_open(self.device.index, hb, ctypes.byref(ptr)))
            self.ptrs.append(ptr.value)
            self._opened.append(ptr.value)
        self.epoch = 0

    def partial(self) -> tuple[torch.Tensor, torch.Tensor]:
        """(o [B,H,D] f32, lse [B,H] f32) for the next step's decode of this rank's shard."""
        return self.buf.partial(self.epoch + 1)

    def merge(self, out: torch.Tensor | None = None, lse_out: torch.Tensor | None = None,
              mode: str = "rs", out_dtype=torch.bfloat16) -> tuple[torch.Tensor, torch.Tensor | None]:
        """Merge this step's partials of all ranks; returns (out, lse_out)."""
        self.epoch += 1
        hs = self.H // self.world if mode == "rs" else self.H
        if out is None:
            out = torch.empty(self.B, hs, self.D, dtype=out_dtype, device=self.device)
        p2p_merge(self.ptrs, self.rank, self.B, self.H, self.D, 0 if self.device_epoch else self.epoch, out,
                  mode, lse_out, self.timeout_s)
        return out, lse_out

    def status(self) -> int:
        """0, or 1 when a merge wait for a peer's flag ran out (synchronises the stream)."""
        return self.buf.status()

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after a barrier, so no peer still reads it)."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        lib = _lib.load()
        for ptr in self._opened:
            lib.qmla_dcp_buffer_close(ctypes.c_void_p(ptr))
        self._opened = []
        self.buf.free()
