"""Decode context parallelism on 2 GPUs: each rank decodes its contiguous KV shard with the
sm_100a kernel, the partials are merged, and the result must equal the single-GPU decode of
the whole sequences.  Two merges: NCCL (all-gather lse, correction kernel, all-reduce) and
the one-kernel merge over NVLink peer memory (qmla_dcp_p2p_merge, each rank keeping its half
of the heads).  Skipped when fewer than two GPUs are visible."""
from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _case(device):
    from gpu_util import make_bf16_case
    # rank 1's shard starts at L // 2: every length here puts that start on a page boundary,
    # so a shard is addressed by the row's page table from page lo / 16 on
    lens = [5025, 1, 129, 64, 2049]
    return lens, make_bf16_case(len(lens), 24, 768, 232, 16, lens, seed=17, device=device)


def _worker(rank, port, out_q, merge="nccl"):
    import datetime
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import torch.distributed as dist
    # NVLink SHARP (multicast objects) off: these ranks exchange only through plain peer memory
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from qwen_mla_vllm_b200.dcp import merge_across_ranks, shard_bounds
        from qwen_mla_vllm_b200.mla_decode_attention import build_params, run_params
        lens, (cache, q, bt, sl) = _case(dev)
        # this rank's shard: token range [lo, hi) of each row, addressed through a shifted page table
        page = 16
        bts, sls = [], []
        for b, L in enumerate(lens):
            lo, hi = shard_bounds(L, WORLD, rank)
            assert hi <= lo or lo % page == 0
            row = torch.zeros(bt.shape[1], dtype=torch.int32, device=dev)
            row[:bt.shape[1] - lo // page] = bt[b, lo // page:]
            bts.append(row)
            sls.append(max(hi - lo, 0))
        bt_s = torch.stack(bts)
        sl_s = torch.tensor(sls, dtype=torch.int32, device=dev)
        ex = None
        if merge == "p2p":
            from qwen_mla_vllm_b200.dcp import P2PExchange
            ex = P2PExchange(len(lens), 24, 768)
            o, lse = ex.partial()
        else:
            o = torch.zeros(len(lens), 24, 768, dtype=torch.float32, device=dev)
            lse = torch.zeros(len(lens), 24, dtype=torch.float32, device=dev)
        p = build_params(q, cache, o, lse, bt_s, sl_s, rank=768, qk_dim=1000, rms_offset=1000, rms_mode=1,
                         page_size=page, sm_scale=1 / 16)
        run_params(p, dev)
        if ex is not None:
            lm = torch.empty(len(lens), 24 // WORLD, dtype=torch.float32, device=dev)
            om, _ = ex.merge(lse_out=lm, mode="rs", out_dtype=torch.float32)
            h0, h1 = rank * (24 // WORLD), (rank + 1) * (24 // WORLD)
        else:
            om, lm = merge_across_ranks(o, lse)
            h0, h1 = 0, 24
        torch.cuda.synchronize()
        if ex is not None:
            assert ex.status() == 0
        of = torch.zeros(len(lens), 24, 768, dtype=torch.float32, device=dev)
        lf = torch.zeros(len(lens), 24, dtype=torch.float32, device=dev)
        pf = build_params(q, cache, of, lf, bt, sl, rank=768, qk_dim=1000, rms_offset=1000, rms_mode=1,
                          page_size=page, sm_scale=1 / 16)
        run_params(pf, dev)
        torch.cuda.synchronize()
        out_q.put((rank, (om - of[:, h0:h1]).abs().max().item(), (lm - lf[:, h0:h1]).abs().max().item()))
        if ex is not None:
            ex.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD,
                    reason="needs 2 GPUs")
@pytest.mark.parametrize("merge", ["nccl", "p2p"])
def test_dcp_two_gpus_equals_single_gpu(merge):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q, merge)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, d_o, d_l in res:
        assert d_o < 2e-3 and d_l < 1e-3, (merge, rank, d_o, d_l)
