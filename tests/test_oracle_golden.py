"""The oracle against golden vectors produced by the reference's own torch functions.

Fixtures: tests/golden/*.npz, written by tests/golden/make_golden.py from
tests/test_fi_partial_rope.py, tests/test_fp8_kv.py, tests/test_decode_numerics.py,
qwen_mla/mla_impl.py:do_kv_cache_update, qwen_mla/fi_decode.py:_RankPlan.plan_cpu and
qwen_mla/ops/mla_gather.py:gather_cache_torch.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import DECODE_FIXTURES, GATHER_FIXTURES, gather_expected, load_golden, oracle_args


@pytest.mark.parametrize("name", DECODE_FIXTURES)
def test_decode_matches_reference(name):
    g = load_golden(name)
    q = oracle.bf16_bits_to_f32(g["q"])
    args = oracle_args(g)
    fp8 = args["kv_fp8"]
    # The reference's FP8 test reference keeps dequantised keys in float32: compare like for like.
    o, lse = oracle.decode(q, g["cache"], g["block_table"], g["seq_lens"], dequant_to_bf16=not fp8, **args)
    ref = g["out"].astype(np.float64)
    rel = np.abs(o - ref).max() / np.abs(ref).max()
    assert rel < 2e-6, f"{name}: oracle vs reference max rel {rel:.3e}"
    assert np.isfinite(lse).all()
    if fp8:  # the kernel-order oracle (bf16 dequant) stays within the reference test's own bar
        o2, _ = oracle.decode(q, g["cache"], g["block_table"], g["seq_lens"], **args)
        assert np.abs(o2 - ref).max() / np.abs(ref).max() < 2e-2


@pytest.mark.parametrize("mode", ["log8", "bf16"])
def test_fp8_cache_rows_bit_exact(mode):
    g = load_golden(f"cache_write_{mode}")
    slots = g["slots"].astype(np.int64)
    n = len(slots)
    lat = oracle.bf16_bits_to_f32(g["latent"])[:n]
    kpe = oracle.bf16_bits_to_f32(g["k_pe"])[:n]
    rows = oracle.fp8_cache_rows(lat, kpe, float(g["k_scale"]), int(g["packed_rope"]), int(g["heads"]), mode)
    cache = np.zeros_like(g["cache"]).reshape(-1, g["cache"].shape[-1])
    cache[np.maximum(slots, 0), :rows.shape[1]] = rows
    want = g["cache"].reshape(-1, g["cache"].shape[-1])
    assert np.array_equal(cache, want), f"{int((cache != want).sum())} bytes differ"


def test_rank_plan_arrays_exact():
    g = load_golden("rank_plan")
    qo, indptr, idx, kv_len = oracle.rank_plan_arrays(g["block_table"], g["seq_lens"], int(g["page"]))
    assert np.array_equal(qo, g["qo_indptr"])
    assert np.array_equal(indptr, g["kv_indptr"])
    assert np.array_equal(idx, g["kv_indices"])
    assert np.array_equal(kv_len, g["kv_len"])
    tp, indptr2, kv_len2 = oracle.plan_arrays(g["seq_lens"], int(g["page"]))
    assert np.array_equal(indptr2, g["kv_indptr"]) and np.array_equal(kv_len2, g["kv_len"])
    assert tp[-1] == sum((int(L) + oracle.TILE - 1) // oracle.TILE for L in g["seq_lens"])


@pytest.mark.parametrize("name", GATHER_FIXTURES)
def test_gather_bit_exact(name):
    """Every destination element the reference's gather writes, bit for bit, and the
    sentinel left in the rows and columns it does not write."""
    g = load_golden(name)
    want = g["dst"]
    got = gather_expected(g)
    assert np.array_equal(got, want), f"{name}: {int((got != want).sum())} elements differ"


def test_gather_empty_and_fp8_without_layout():
    g = load_golden("gather_log8")
    assert oracle.gather_cache(g["cache"], g["block_table"], g["cu_seq_lens"], g["token_to_seq"], 0,
                               fp8=True, mla_rms=(488, 24, "log8")).size == 0
    with pytest.raises(NotImplementedError):
        oracle.gather_cache(g["cache"], g["block_table"], g["cu_seq_lens"], g["token_to_seq"], 4, fp8=True)


def test_mtp_flattening_matches_the_reference_builder():
    """oracle.mtp_flatten and the product's plan_for_step flattening against the rows the
    reference's own MLATritonMetadataBuilder._build_decode produced (qwen_mla/mla_impl.py:628-662),
    bit for bit: block table per draft row, lengths L - (q-1-j) clamped at 0."""
    import types

    import torch

    from qwen_mla_vllm_b200 import fi_decode
    g = load_golden("mtp_build_decode")
    q = int(g["qrows"])
    bt, sl = oracle.mtp_flatten(g["block_table"], g["seq_lens"], q)
    assert np.array_equal(bt, g["flat_block_table"])
    assert np.array_equal(sl, g["flat_seq_lens"])
    cfg = dict(device="cpu", rank=768, win=232, n_local=24, page_size=16, max_batch=64)
    builder = types.SimpleNamespace(_mla_fi_cfg=cfg, _mla_fi_plan=None, _mla_fi_scale=1 / 16, _mla_fi_ok=True)
    decode = types.SimpleNamespace(seq_lens=torch.from_numpy(g["flat_seq_lens"]),
                                   block_table=torch.from_numpy(g["flat_block_table"]), _mla_q=q)
    md = types.SimpleNamespace(decode=decode)
    fi_decode.plan_for_step(builder, md, types.SimpleNamespace(_seq_lens_cpu=torch.from_numpy(g["seq_lens"])))
    n = len(g["flat_seq_lens"])
    assert np.array_equal(md._mla_fi_plan.kv_len[:n].numpy(), g["flat_seq_lens"])


@pytest.mark.parametrize("base_e", [True, False])
def test_dcp_correction_matches_the_reference_kernel(base_e):
    """oracle.dcp_correct against the reference's own Triton DCP correction
    (qwen_mla/dcp_fix.py:101-130, run on a GPU by tests/golden/make_golden_gpu.py): NaN / +inf
    partial LSEs, rows empty on every rank or on some, every cp_rank, base e and base 2."""
    g = load_golden("dcp_correct")
    for r in range(int(g["N"])):
        key = f"{'e' if base_e else '2'}{r}"
        got, lse = oracle.dcp_correct(g["out"][r], g["lses"], r, is_base_e=base_e)
        np.testing.assert_allclose(got, g[f"out_{key}"], rtol=2e-6, atol=1e-6)
        want = g[f"lse_{key}"]
        fin = np.isfinite(want)
        assert np.array_equal(np.isfinite(lse), fin)
        np.testing.assert_allclose(lse[fin], want[fin], rtol=1e-6, atol=1e-6)
