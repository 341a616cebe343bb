"""The FlashInfer-adapter mirror (qwen_mla_vllm_b200/fi_decode.py) without a GPU: rope windows,
host planning into fixed buffers, MTP flattening in plan_for_step, and declining."""
from __future__ import annotations

import types

import numpy as np
import pytest
import torch

import oracle
from qwen_mla_vllm_b200 import fi_decode


@pytest.mark.parametrize("head_offset,n_local,want", [(0, 24, (0, 232)), (0, 12, (0, 116)), (12, 12, (0, 116)),
                                                      (6, 12, (0, 116)), (3, 12, (0, 174)), (23, 1, (0, 58))])
def test_rope_window(head_offset, n_local, want):
    assert fi_decode.rope_window(head_offset, n_local, 6, 58) == want


def test_plan_cpu_matches_oracle_and_keeps_buffers():
    p = fi_decode.RankPlan("cpu", rank=768, win=232, n_local=24, page_size=16, max_batch=8)
    addr = (p.tile_prefix.data_ptr(), p.kv_indptr.data_ptr(), p.kv_len.data_ptr())
    lens = torch.tensor([0, 1, 65, 1000, 4097], dtype=torch.int32)
    bt = torch.zeros(5, 300, dtype=torch.int32)
    for _ in range(5):  # ring reuse
        p.plan_cpu(bt, lens, lens, 1 / 16)
    tp, ip, kl = oracle.plan_arrays(lens.numpy(), 16)
    assert np.array_equal(p.tile_prefix[:6].numpy(), tp)
    assert np.array_equal(p.kv_indptr[:6].numpy(), ip)
    assert np.array_equal(p.kv_len[:5].numpy(), kl)
    assert addr == (p.tile_prefix.data_ptr(), p.kv_indptr.data_ptr(), p.kv_len.data_ptr())
    assert p.host_planned and p.planned_batch == 5 and p.planned_scale == 1 / 16
    with pytest.raises(ValueError):
        p.plan_cpu(bt, torch.zeros(9, dtype=torch.int32), torch.zeros(9, dtype=torch.int32), 1.0)


def test_plan_for_step_flattens_mtp_lengths():
    cfg = dict(device="cpu", rank=768, win=232, n_local=24, page_size=16, max_batch=64)
    builder = types.SimpleNamespace(_mla_fi_cfg=cfg, _mla_fi_plan=None, _mla_fi_scale=1 / 16, _mla_fi_ok=True)
    q = 4
    req_lens = torch.tensor([100, 2, 33], dtype=torch.int32)
    bt_req = torch.arange(3 * 10, dtype=torch.int32).reshape(3, 10)
    bt_rows, lens_rows = oracle.mtp_flatten(bt_req.numpy(), req_lens.numpy(), q)
    decode = types.SimpleNamespace(seq_lens=torch.from_numpy(lens_rows), block_table=torch.from_numpy(bt_rows), _mla_q=q)
    md = types.SimpleNamespace(decode=decode)
    common = types.SimpleNamespace(_seq_lens_cpu=req_lens)
    fi_decode.plan_for_step(builder, md, common)
    plan = md._mla_fi_plan
    assert plan.host_planned and plan.planned_batch == 12
    assert np.array_equal(plan.kv_len[:12].numpy(), lens_rows)
    # no host lengths: the plan is left to the device
    md2 = types.SimpleNamespace(decode=decode)
    fi_decode.plan_for_step(builder, md2, None)
    assert md2._mla_fi_plan is plan and not plan.host_planned


def test_forward_mqa_declines_without_a_matching_plan():
    impl = types.SimpleNamespace(scale=1 / 16, mla_head_offset=0, mla_rope_group=6, mla_rope_dim=58,
                                 kv_lora_rank=768, rms_offset=1000)
    q = torch.zeros(2, 24, 1000)
    assert fi_decode.forward_mqa(impl, q, None, types.SimpleNamespace(), None) is None
    p = fi_decode.RankPlan("cpu", rank=768, win=232, n_local=24, page_size=16, max_batch=8)
    p.plan_cpu(None, torch.tensor([5, 5], dtype=torch.int32), torch.tensor([5, 5], dtype=torch.int32), 1 / 16)
    md = types.SimpleNamespace(_mla_fi_plan=p)
    assert fi_decode.forward_mqa(impl, torch.zeros(3, 24, 1000), None, md, None) is None       # batch
    assert fi_decode.forward_mqa(impl, torch.zeros(2, 12, 1000), None, md, None) is None       # heads
    impl2 = types.SimpleNamespace(**{**impl.__dict__, "scale": 0.1})
    assert fi_decode.forward_mqa(impl2, q, None, md, None) is None                             # scale
    impl3 = types.SimpleNamespace(**{**impl.__dict__, "kv_lora_rank": 512})
    assert fi_decode.forward_mqa(impl3, q, None, md, None) is None                             # rank
