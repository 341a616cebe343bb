"""The torch.library ops on the GPU: ``torch.ops.qmla.mla_decode`` / ``gather_cache`` give the
same bits as the Python entry points, also when called from a ``torch.compile(fullgraph=True)``
function (the ops stay opaque to the tracer and write their outputs in place)."""
from __future__ import annotations

import pytest
import torch

from gpu_util import make_bf16_case, make_fp8_case

pytestmark = pytest.mark.gpu


def _decode_args(cache, q, bt, sl, ws, k_scale=None, rms_mode=1):
    o = torch.zeros(q.shape[0], q.shape[1], 768, dtype=torch.bfloat16, device=q.device)
    lse = torch.zeros(q.shape[0], q.shape[1], dtype=torch.float32, device=q.device)
    return o, lse, (q, cache, o, lse, bt, sl, ws, 768, 1000, 1000, rms_mode, 16, 1 / 16, 0.0, k_scale, 1)


@pytest.mark.parametrize("fp8", [False, True])
def test_mla_decode_op_matches_entry_point(cuda_device, fp8):
    import qwen_mla_vllm_b200.ops  # noqa: F401
    from qwen_mla_vllm_b200.mla_decode_attention import decode_attention_fwd
    lens = [900, 1, 4100]
    if fp8:
        cache, q, bt, sl, scale = make_fp8_case(3, 24, 768, 232, 16, lens, seed=5, device=cuda_device)
        ks = torch.tensor(scale, dtype=torch.float32, device=cuda_device)
    else:
        cache, q, bt, sl = make_bf16_case(3, 24, 768, 232, 16, lens, seed=5, device=cuda_device)
        ks = None
    logits = torch.empty(3, 24, 8, 769, dtype=torch.float32, device=cuda_device)
    o_ref = torch.zeros(3, 24, 768, dtype=torch.bfloat16, device=cuda_device)
    lse_ref = torch.zeros(3, 24, dtype=torch.float32, device=cuda_device)
    decode_attention_fwd(q, cache, cache[..., :768], o_ref, lse_ref, bt, sl, logits, 8, 1 / 16, 16,
                         k_scale=ks, v_scale=ks, is_mla=True, rms_offset=1000, rms_log8=fp8)
    o, lse, args = _decode_args(cache, q, bt, sl, logits, ks, rms_mode=3 if fp8 else 1)
    torch.ops.qmla.mla_decode(*args)
    torch.cuda.synchronize()
    assert torch.equal(o, o_ref) and torch.equal(lse, lse_ref)

    @torch.compile(fullgraph=True, backend="aot_eager")
    def step(q, cache, o, lse, bt, sl, ws):
        torch.ops.qmla.mla_decode(q, cache, o, lse, bt, sl, ws, 768, 1000, 1000, 3 if fp8 else 1, 16,
                                  1 / 16, 0.0, ks, 1)
        return o.float().sum()

    o.zero_()
    lse.zero_()
    step(q, cache, o, lse, bt, sl, logits)
    torch.cuda.synchronize()
    assert torch.equal(o, o_ref) and torch.equal(lse, lse_ref)


def test_gather_op_matches_entry_point(cuda_device):
    import qwen_mla_vllm_b200.ops  # noqa: F401
    from qwen_mla_vllm_b200.mla_gather import gather_cache_torch
    cache, _, bt, _, scale = make_fp8_case(3, 24, 768, 232, 16, [300, 0, 200], seed=9, device=cuda_device)
    cu = torch.tensor([0, 120, 120, 300], dtype=torch.int32, device=cuda_device)
    t2s = torch.repeat_interleave(torch.arange(3, dtype=torch.int32, device=cuda_device),
                                  torch.tensor([120, 0, 180], device=cuda_device))
    starts = torch.tensor([7, 0, 3], dtype=torch.int32, device=cuda_device)
    sc = torch.tensor(scale, dtype=torch.float32, device=cuda_device)
    want = torch.zeros(300, 1024, dtype=torch.bfloat16, device=cuda_device)
    gather_cache_torch(src_cache=cache, dst=want, block_table=bt, cu_seq_lens=cu, token_to_seq=t2s,
                       num_tokens=300, kv_cache_dtype="fp8", scale=sc, seq_starts=starts,
                       mla_rms=(1000, 24, "log8"), check=True)
    got = torch.zeros_like(want)
    torch.ops.qmla.gather_cache(cache, got, bt, cu, t2s, 300, "fp8", sc, starts, 1000, 24, "log8")
    torch.cuda.synchronize()
    assert torch.equal(got, want)
