"""DCP shard layouts on one GPU: every rank's shard of one global cache is decoded in turn
(ranks emulated, no peers), the partials are merged with the fused merge kernel
(qmla_dcp_merge), and the result must equal the single-GPU decode of the whole cache.  Covers the
contiguous split and vLLM's token-interleaved layout (cp_kv_cache_interleave_size 16 and 1), where
a rank's local length differs per row, with MTP verify rows (4 causal drafts, each with its own
local length on every rank) on an FP8 log8 cache and on a bf16 cache."""
from __future__ import annotations

import pytest
import torch

import bench

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("world,interleave", [(2, 0), (4, 16), (8, 1), (3, 0)])
def test_sharded_decode_merges_to_the_full_decode(cuda_device, fp8, world, interleave):
    from qwen_mla_vllm_b200.dcp import merge_partials
    from qwen_mla_vllm_b200.mla_decode_attention import run_params
    w = bench.Workload("t", "dcp layout test", fp8=fp8, heads=24, rank=768, rope=232,
                       lens=[3000, 5, 700, 17, 4100, 129], qrows=4, seed=11 + world)
    full = bench.build_case(w, cuda_device)
    rows = full.q.shape[0]
    o_ref = torch.empty(rows, w.heads, w.rank, dtype=torch.float32, device=cuda_device)
    l_ref = torch.empty(rows, w.heads, dtype=torch.float32, device=cuda_device)
    run_params(bench.params_for(w, full, o_ref, l_ref), cuda_device)
    parts = torch.empty(world, rows, w.heads, w.rank, dtype=torch.float32, device=cuda_device)
    lses = torch.empty(world, rows, w.heads, dtype=torch.float32, device=cuda_device)
    for r in range(world):
        sh = bench.shard_case(w, full, world, r, cuda_device, interleave)
        run_params(bench.params_for(w, sh, parts[r], lses[r]), cuda_device)
    o, lse = merge_partials(parts, lses)
    torch.cuda.synchronize()
    # two decodes of the same data split differently: bf16 P is rounded per weight (2^-9), and rows of
    # a few tokens have |o| ~ 1, so bf16 differs by a few 1e-3; FP8's hi + lo P is finer
    tol = 5e-3 if fp8 else 1e-2
    assert float((o - o_ref).abs().max()) < tol
    fin = l_ref.isfinite()
    assert torch.equal(lse.isfinite(), fin)
    assert float((lse[fin] - l_ref[fin]).abs().max()) < 1e-3
