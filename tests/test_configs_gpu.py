"""GPU parity at every BASELINE config's own shape, on the bench's own workloads (bench.py builds
them, seeded): the whole batch is decoded through the C ABI and the oracle checks the rows below
in full.

* config 1: bf16, 64 rows, L ~ U[1024, 32768]; the 8 longest rows (up to 32,768 tokens).
* config 2: FP8 e4m3 + log8 rms, k_scale = absmax/448, 128 requests x 4 causal drafts, L = 8192;
  16 requests (64 rows).
* config 3: GLA-g2, both head groups (12 heads, 384 | 116 | 12), L ~ U[4096, 65536]; the longest,
  the shortest and two more rows of each group.
* config 4: FP8 e4m3 + log8 rms, 8 rows of 262,144 tokens; one full row (2,048 tiles, spread over
  many CTA segments and merged), the oracle streaming it in float64 chunks.

Tolerances: max abs error < 2e-2 (bf16) and < 5e-2 (FP8), max|d|/max|ref| < 2e-2, lse < 2e-2.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import bench
from gpu_util import compare, oracle_rows

pytestmark = pytest.mark.gpu

BF16_TOL, FP8_TOL = 2e-2, 5e-2


def _decode(w, case, device):
    from qwen_mla_vllm_b200.mla_decode_attention import run_params
    rows = case.q.shape[0]
    o = torch.full((rows, w.heads, w.rank), float("nan"), dtype=torch.bfloat16, device=device)
    lse = torch.full((rows, w.heads), float("nan"), dtype=torch.float32, device=device)
    run_params(bench.params_for(w, case, o, lse), device)
    torch.cuda.synchronize(device)
    assert torch.isfinite(o).all()
    return o, lse


def _check(w, case, o, lse, rows):
    ref_o, ref_lse = oracle_rows(w, case, rows)
    err, rel = compare(o[rows], lse[rows], ref_o, ref_lse, tol=FP8_TOL if w.fp8 else BF16_TOL, rel_tol=2e-2)
    return err, rel


def test_config1_full_batch(cuda_device):
    w = bench.workloads()["cfg1"]
    case = bench.build_case(w, cuda_device)
    o, lse = _decode(w, case, cuda_device)
    longest = sorted(range(len(w.lens)), key=lambda r: -w.lens[r])[:8]
    _check(w, case, o, lse, longest)


def test_config2_fp8_mtp_verify(cuda_device):
    w = bench.workloads()["cfg2"]
    case = bench.build_case(w, cuda_device)
    o, lse = _decode(w, case, cuda_device)
    reqs = list(range(0, 128, 8))  # 16 requests spread over the batch, all 4 drafts each
    rows = [r * w.qrows + j for r in reqs for j in range(w.qrows)]
    _check(w, case, o, lse, rows)


@pytest.mark.parametrize("group", [0, 1])
def test_config3_gla_head_groups(cuda_device, group):
    w = bench.workloads()["cfg3"]
    case = bench.build_case(w, cuda_device, group=group)
    o, lse = _decode(w, case, cuda_device)
    order = sorted(range(len(w.lens)), key=lambda r: w.lens[r])
    _check(w, case, o, lse, [order[-1], order[0], order[len(order) // 2], 17])


def test_config4_fp8_262k_row(cuda_device):
    w = bench.workloads()["cfg4"]
    case = bench.build_case(w, cuda_device)
    o, lse = _decode(w, case, cuda_device)
    _check(w, case, o, lse, [5])
    # the other rows: same length and distribution, so their outputs must be alike in scale
    assert float(o.float().abs().max()) < 1.0
