"""The DCP merge choreography (all-gather of lse, local correction, then an all-reduce of o or
a reduce-scatter over heads) on two CPU ranks over gloo, with the oracle's correction in place
of the CUDA kernel: the merged result of the two KV shards equals the single-rank decode."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _case():
    rng = np.random.default_rng(7)
    B, H, rank, rope, page = 3, 8, 128, 64, 16
    lens = [200, 9, 1]
    W = rank + rope + H
    pps = (max(lens) + page - 1) // page
    cache = oracle.f32_to_bf16_bits(rng.standard_normal((B * pps, page, W)).astype(np.float32))
    cache[..., rank + rope:] = oracle.f32_to_bf16_bits(rng.uniform(0.5, 2, (B * pps, page, H)).astype(np.float32))
    bt = rng.permutation(B * pps).reshape(B, pps).astype(np.int32)
    q = oracle.bf16_round((rng.standard_normal((B, H, rank + rope)) / 32).astype(np.float32))
    kw = dict(rank=rank, qk_dim=rank + rope, page_size=page, sm_scale=1 / 16, rms_offset=rank + rope)
    return cache, bt, q, lens, kw


def _shard_decode(cache, bt, q, lens, kw, world, r):
    """Decode this rank's contiguous token slice of every sequence (the KV shard it holds)."""
    from qwen_mla_vllm_b200.dcp import shard_bounds
    page = kw["page_size"]
    o = np.zeros((len(lens), q.shape[1], kw["rank"]))
    lse = np.full((len(lens), q.shape[1]), -np.inf)
    for b, L in enumerate(lens):
        lo, hi = shard_bounds(L, world, r)
        if hi <= lo:
            continue
        t = np.arange(lo, hi)
        rows = cache[bt[b, t // page], t % page].reshape(1, hi - lo, -1)
        ob, lb = oracle.decode(q[b:b + 1], rows, np.array([[0]]), np.array([hi - lo]), **{**kw, "page_size": hi - lo})
        o[b], lse[b] = ob[0], lb[0]
    return o, lse


def _oracle_correct(out, lses, cp_rank):
    res, g = oracle.dcp_correct(out.numpy(), lses.numpy(), cp_rank)
    out.copy_(torch.from_numpy(res))
    return out, torch.from_numpy(g)


def _worker(r, world, port, q_out, mode="ar"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=r, world_size=world)
    try:
        from qwen_mla_vllm_b200.dcp import merge_across_ranks
        cache, bt, q, lens, kw = _case()
        o, lse = _shard_decode(cache, bt, q, lens, kw, world, r)
        om, lm = merge_across_ranks(torch.from_numpy(o), torch.from_numpy(lse), correct=_oracle_correct,
                                    mode=mode)
        q_out.put((r, om.numpy(), lm.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["ar", "rs"])
def test_two_rank_merge_equals_full_decode(mode):
    world = 2
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q_out, mode)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q_out.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    cache, bt, q, lens, kw = _case()
    full_o, full_lse = oracle.decode(q, cache, bt, np.array(lens), **kw)
    hs = q.shape[1] // world
    for r, om, lm in res:
        h0, h1 = (r * hs, (r + 1) * hs) if mode == "rs" else (0, q.shape[1])
        assert om.shape[1] == h1 - h0
        assert np.abs(om - full_o[:, h0:h1]).max() < 1e-10, r
        assert np.abs(lm - full_lse[:, h0:h1]).max() < 1e-10, r


def test_shard_bounds_cover_sequence():
    from qwen_mla_vllm_b200.dcp import shard_bounds, shard_lengths
    for L in (0, 1, 7, 64, 262144, 100003):
        for w in (1, 2, 3, 4, 8):
            b = [shard_bounds(L, w, r) for r in range(w)]
            assert b[0][0] == 0 and b[-1][1] == L
            assert all(b[i][1] == b[i + 1][0] for i in range(w - 1))
            assert sum(shard_lengths([L], w, r)[0] for r in range(w)) == L


def _gla_worker(r, world, groups, port, q_out):
    """GLA-g2 over gloo: rank r holds head group g's KV shard (its own cache per group) and merges
    only with the ranks of its group's sub-group."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=r, world_size=world)
    try:
        from qwen_mla_vllm_b200.dcp import head_group_of, head_group_subgroups, merge_across_ranks
        g, sub_rank, per = head_group_of(r, world, groups)
        pgs = head_group_subgroups(world, groups)
        cache, bt, q, lens, kw = _gla_case(g)
        o, lse = _shard_decode(cache, bt, q, lens, kw, per, sub_rank)
        if per > 1:
            om, lm = merge_across_ranks(torch.from_numpy(o), torch.from_numpy(lse), group=pgs[g],
                                        correct=_oracle_correct, mode="rs")
            om, lm = om.numpy(), lm.numpy()
        else:
            om, lm = o, lse
        q_out.put((r, g, sub_rank, per, om, lm))
    finally:
        dist.destroy_process_group()


def _gla_case(g):
    """Head group g's own cache (12 heads, latent 384 | rope 116 | rms 12) and queries."""
    rng = np.random.default_rng(100 + g)
    B, H, rank, rope, page = 3, 12, 128, 116, 16
    lens = [300, 17, 64]
    W = rank + rope + H
    pps = (max(lens) + page - 1) // page
    cache = oracle.f32_to_bf16_bits(rng.standard_normal((B * pps, page, W)).astype(np.float32))
    cache[..., rank + rope:] = oracle.f32_to_bf16_bits(rng.uniform(0.5, 2, (B * pps, page, H)).astype(np.float32))
    bt = rng.permutation(B * pps).reshape(B, pps).astype(np.int32)
    q = oracle.bf16_round((rng.standard_normal((B, H, rank + rope)) / 32).astype(np.float32))
    kw = dict(rank=rank, qk_dim=rank + rope, page_size=page, sm_scale=1 / 16, rms_offset=rank + rope)
    return cache, bt, q, lens, kw


@pytest.mark.parametrize("world", [2, 4])
def test_gla_head_groups_over_ranks(world):
    """2 head groups on 2 ranks (one group each, no exchange) and on 4 ranks (each group split by
    KV over 2 ranks and merged inside its sub-group): every rank's heads equal its group's full
    decode."""
    groups = 2
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gla_worker, args=(r, world, groups, port, q_out)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q_out.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r, g, sub_rank, per, om, lm in res:
        assert g == r // (world // groups)
        cache, bt, q, lens, kw = _gla_case(g)
        full_o, full_lse = oracle.decode(q, cache, bt, np.array(lens), **kw)
        hs = q.shape[1] // per
        h0 = sub_rank * hs if per > 1 else 0
        assert np.abs(om - full_o[:, h0:h0 + om.shape[1]]).max() < 1e-10, r
        assert np.abs(lm - full_lse[:, h0:h0 + lm.shape[1]]).max() < 1e-10, r
