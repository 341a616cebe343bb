"""forward_mqa of the FlashInfer-adapter mirror against decode_attention_fwd on the same inputs:
identical outputs, LSE in base 2 (natural log with return_lse_base_on_e), host and device plans."""
from __future__ import annotations

import math
import types

import pytest
import torch

from gpu_util import make_bf16_case, make_fp8_case

pytestmark = pytest.mark.gpu


def _impl(fp8=False):
    return types.SimpleNamespace(scale=1 / 16, mla_head_offset=0, mla_rope_group=6, mla_rope_dim=58,
                                 kv_lora_rank=768, rms_offset=1000, need_to_return_lse_for_decode=True)


@pytest.mark.parametrize("host_plan", [True, False])
@pytest.mark.parametrize("fp8", [False, True])
def test_forward_mqa_matches_decode_attention_fwd(cuda_device, host_plan, fp8):
    from qwen_mla_vllm_b200 import fi_decode
    from qwen_mla_vllm_b200.mla_decode_attention import decode_attention_fwd
    lens = [3000, 1, 64, 777]
    if fp8:
        cache, q, bt, sl, ks = make_fp8_case(len(lens), 24, 768, 232, 16, lens, seed=5, device=cuda_device)
        kst = torch.tensor(ks, dtype=torch.float32, device=cuda_device)
    else:
        cache, q, bt, sl = make_bf16_case(len(lens), 24, 768, 232, 16, lens, seed=5, device=cuda_device)
        kst = None
    o_ref = torch.empty(len(lens), 24, 768, dtype=torch.bfloat16, device=cuda_device)
    lse_ref = torch.empty(len(lens), 24, dtype=torch.float32, device=cuda_device)
    logits = torch.empty(len(lens), 24, 8, 769, dtype=torch.float32, device=cuda_device)
    decode_attention_fwd(q, cache, cache[..., :768], o_ref, lse_ref, bt, sl, logits, 8, 1 / 16, 16,
                         k_scale=kst, v_scale=kst, is_mla=True, rms_offset=1000, rms_log8=fp8)
    plan = fi_decode.RankPlan(cuda_device, rank=768, win=232, n_local=24, page_size=16, max_batch=16)
    if host_plan:
        plan.plan_cpu(bt, sl, sl.cpu(), 1 / 16)
    else:
        plan.plan(bt, sl, 1 / 16)
    md = types.SimpleNamespace(_mla_fi_plan=plan)
    layer = types.SimpleNamespace(_k_scale=kst)
    q_tuple = (q[..., :768].contiguous(), q[..., 768:].contiguous())
    o, lse2 = fi_decode.forward_mqa(_impl(fp8), q_tuple, cache, md, layer)
    o_e, lse_e = fi_decode.forward_mqa(_impl(fp8), q, cache, md, layer, return_lse_base_on_e=True)
    torch.cuda.synchronize()
    assert torch.equal(o, o_ref) and torch.equal(o_e, o_ref)
    assert torch.equal(lse_e, lse_ref)
    fin = torch.isfinite(lse_ref)
    assert torch.allclose(lse2[fin], lse_ref[fin] / math.log(2.0), rtol=1e-6, atol=1e-6)
