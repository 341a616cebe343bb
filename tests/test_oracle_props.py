"""Properties of the oracle that need no reference fixture: number formats against torch's
own conversions, MTP flattening, DCP split-and-merge consistency, and the FP8 writer / context
gather round trip."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle


def test_bf16_round_matches_torch():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 10.0 ** rng.integers(-30, 30, 20000),
                        np.array([0.0, -0.0, 1.0, 65504.0, 3.4e38, -3.4e38, 1e-40, 1.00390625, 1.01171875],
                                 dtype=np.float32)]).astype(np.float32)
    want = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(oracle.f32_to_bf16_bits(x), want)


def test_e4m3_encode_matches_torch_all_ranges():
    rng = np.random.default_rng(1)
    x = np.concatenate([
        rng.uniform(-460, 460, 50000), rng.standard_normal(50000) * 1e-2,
        rng.standard_normal(20000) * 2.0 ** -8,
        # every midpoint between neighbouring codes (ties go to the even code)
        (oracle.e4m3_decode(np.arange(126)) + oracle.e4m3_decode(np.arange(1, 127))) / 2,
        -(oracle.e4m3_decode(np.arange(126)) + oracle.e4m3_decode(np.arange(1, 127))) / 2,
        [0.0, -0.0, 448.0, -448.0, 2.0 ** -10, 2.0 ** -9, 3 * 2.0 ** -10]]).astype(np.float32)
    x = np.clip(x, -448, 448).astype(np.float32)
    want = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    got = oracle.e4m3_encode(x)
    assert np.array_equal(got, want), f"{int((got != want).sum())} codes differ"


def test_e4m3_decode_matches_torch():
    b = np.arange(256, dtype=np.uint8)
    want = torch.from_numpy(b).view(torch.float8_e4m3fn).float().numpy()
    got = oracle.e4m3_decode(b)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan], want[~nan])


def test_log8_round_trip_error_bound():
    x = np.exp2(np.linspace(-3, 3, 10001)).astype(np.float32)
    back = oracle.log8_decode(oracle.log8_encode(x))
    # one code step is 6/255 in log2: half a step bounds the relative error by 2^(3/255) - 1
    assert np.max(np.abs(back / x - 1)) <= 2 ** (3 / 255) - 1 + 1e-6
    assert oracle.log8_encode(np.array([1e-9, 0.0, 100.0], np.float32)).tolist() == [0, 0, 255]


def test_mtp_flatten_lengths():
    bt = np.arange(12, dtype=np.int32).reshape(3, 4)
    lens = np.array([10, 2, 0], np.int32)
    fbt, fl = oracle.mtp_flatten(bt, lens, 4)
    assert fl.tolist() == [7, 8, 9, 10, 0, 0, 1, 2, 0, 0, 0, 0]
    assert np.array_equal(fbt[5], bt[1]) and fbt.shape == (12, 4)


def _rand_case(rng, B, H, rank, rope, page, lens):
    W = rank + rope + H
    W += (-W) % 8
    pps = max(1, (max(lens) + page - 1) // page)
    P = B * pps + 2
    cache = oracle.f32_to_bf16_bits(rng.standard_normal((P, page, W)).astype(np.float32))
    cache[..., rank + rope:] = oracle.f32_to_bf16_bits(rng.uniform(0.5, 2.0, (P, page, W - rank - rope)).astype(np.float32))
    bt = rng.permutation(B * pps).reshape(B, pps).astype(np.int32)
    q = oracle.bf16_round((rng.standard_normal((B, H, rank + rope)) / 32).astype(np.float32))
    return cache, bt, q


@pytest.mark.parametrize("n_shards", [2, 3, 8])
def test_dcp_split_merge_equals_full(n_shards):
    """Decoding contiguous KV shards and merging with the dcp_fix math reproduces the full decode."""
    rng = np.random.default_rng(n_shards)
    B, H, rank, rope, page = 3, 8, 128, 64, 16
    lens = [300, 17, 1]
    cache, bt, q = _rand_case(rng, B, H, rank, rope, page, lens)
    kw = dict(rank=rank, qk_dim=rank + rope, page_size=page, sm_scale=1 / 16, rms_offset=rank + rope)
    full_o, full_lse = oracle.decode(q, cache, bt, np.array(lens), **kw)
    parts, lses = [], []
    for s in range(n_shards):
        # shard s owns tokens [lo, hi) of each row; present them as rows of their own
        o_s, l_s = np.zeros_like(full_o), np.full_like(full_lse, -np.inf)
        for b, L in enumerate(lens):
            lo, hi = L * s // n_shards, L * (s + 1) // n_shards
            if hi <= lo:
                continue
            t = np.arange(lo, hi)
            rows = cache[bt[b, t // page], t % page]
            sub = rows.reshape(1, hi - lo, -1)
            ob, lb = oracle.decode(q[b:b + 1], sub, np.array([[0]]), np.array([hi - lo]),
                                   **{**kw, "page_size": hi - lo})
            o_s[b], l_s[b] = ob[0], lb[0]
        parts.append(o_s)
        lses.append(l_s)
    o, lse = oracle.dcp_merge(np.stack(parts), np.stack(lses))
    assert np.abs(o - full_o).max() < 1e-12
    assert np.abs(lse - full_lse).max() < 1e-12


def test_dcp_correct_special_values():
    out = np.ones((1, 2, 4))
    lses = np.array([[[np.nan, -np.inf]], [[0.0, -np.inf]]])
    res, g = oracle.dcp_correct(out, lses, 0)
    assert np.all(res[0, 0] == 0.0) and np.all(res[0, 1] == 0.0)
    assert g[0, 0] == 0.0 and g[0, 1] == -np.inf
    res1, _ = oracle.dcp_correct(out, lses, 1)
    assert np.allclose(res1[0, 0], 1.0)


def test_plan_arrays_edge_cases():
    tp, indptr, kv_len = oracle.plan_arrays(np.array([0, -5, 1, 64, 65, 128]), 16)
    assert oracle.TILE == 128
    assert tp.tolist() == [0, 0, 0, 1, 2, 3, 4]
    assert indptr.tolist() == [0, 0, 0, 1, 5, 10, 18]
    assert kv_len.tolist() == [0, 0, 1, 64, 65, 128]


def test_log8_decode_bf16_f16_rounding_margin():
    """The gather's bit-exact claim for bf16 / f16 destinations: for every log8 code, the exact
    2^(fl(-3 + fl(code * fl(6/255)))) lies more than 40 float32 ulps from the nearest bf16 /
    f16 rounding midpoint, so any exp2 within a few ulps rounds to the same destination value."""
    import math
    c = np.arange(256, dtype=np.float32)
    x = (np.float32(-3.0) + (c * np.float32(6.0 / 255.0)).astype(np.float32)).astype(np.float32)
    for mant_bits, need in ((7, 150), (10, 40)):
        worst = math.inf
        for v in x:
            e = 2.0 ** float(v)
            _, ex = math.frexp(e)
            step = 2.0 ** (ex - 1 - mant_bits)
            mid = (math.floor(e / step) + 0.5) * step
            worst = min(worst, abs(e - mid) / 2.0 ** (ex - 24))
        assert worst > need, (mant_bits, worst)


@pytest.mark.parametrize("mode", ["log8", "bf16"])
def test_cache_write_then_gather_round_trip(mode):
    """Rows written by the FP8 writer (mla_impl.py:309-342) and gathered back
    (ops/mla_gather.py:28-76) give e4m3(x / k_scale) * k_scale and the rms decode, for a chunk
    whose sequences start mid-page."""
    rng = np.random.default_rng(8)
    rank, rope, heads, page = 256, 232, 24, 16
    n_tok = 40 * page
    lat = oracle.bf16_round(rng.standard_normal((n_tok, rank)).astype(np.float32) * 2)
    kpe = np.concatenate([oracle.bf16_round(rng.standard_normal((n_tok, rope)).astype(np.float32)),
                          oracle.bf16_round(np.exp(rng.standard_normal((n_tok, heads)) * 0.6).astype(np.float32))], 1)
    ks = float(np.abs(lat).max()) / 448
    rows = oracle.fp8_cache_rows(lat, kpe, ks, rope, heads, mode)
    W = rows.shape[1] + (-rows.shape[1]) % 16
    cache = np.zeros((n_tok, W), np.uint8)
    perm = rng.permutation(40)                  # token t lives in page perm[t // page]
    slots = perm[np.arange(n_tok) // page] * page + np.arange(n_tok) % page
    cache[slots, :rows.shape[1]] = rows
    cache = cache.reshape(40, page, W)
    bt = np.stack([perm[:20], perm[20:]]).astype(np.int32)       # two sequences of 320 tokens
    starts = np.array([17, 100], np.int32)
    lens = np.array([300, 220])
    cu = np.array([0, 300, 520], np.int32)
    t2s = np.repeat(np.arange(2, dtype=np.int32), lens)
    got = oracle.gather_cache(cache, bt, cu, t2s, 520, fp8=True, scale=ks, seq_starts=starts,
                              mla_rms=(rank + rope, heads, mode))
    tok = np.concatenate([np.arange(17, 317), 320 + np.arange(100, 320)])
    x = np.concatenate([lat, kpe[:, :rope]], 1)[tok]
    inv = np.float32(1.0) / np.float32(ks)     # the writer multiplies by 1 / k_scale (mla_impl.py:329-332)
    want_lat = oracle.e4m3_decode(oracle.e4m3_encode(np.clip(x * inv, -448, 448))) * np.float32(ks)
    assert np.array_equal(got[:, :rank + rope], want_lat.astype(np.float32))
    r = kpe[tok, rope:]
    want_rms = oracle.log8_decode(oracle.log8_encode(r)) if mode == "log8" else r
    assert np.array_equal(got[:, rank + rope:], want_rms)


def _small_paged(fp8: bool, seed: int = 3):
    rng = np.random.default_rng(seed)
    H, rank, rope, page = 24, 256, 232, 16
    lens = np.array([0, 1, 300, 777], dtype=np.int32)
    pps = 49
    P = len(lens) * pps
    bt = rng.permutation(P).reshape(len(lens), pps).astype(np.int32)
    q = oracle.bf16_round((rng.standard_normal((len(lens), H, rank + rope)) / 32).astype(np.float32))
    if fp8:
        lat = oracle.bf16_round(rng.standard_normal((P * page, rank)).astype(np.float32))
        kpe = oracle.bf16_round(np.concatenate([rng.standard_normal((P * page, rope)),
                                                rng.uniform(0.5, 2.0, (P * page, H))], 1).astype(np.float32))
        rows = oracle.fp8_cache_rows(lat, kpe, 0.0125, rope, H, "log8")
        cache = rows.reshape(P, page, -1)
    else:
        c = rng.standard_normal((P, page, rank + rope + H)).astype(np.float32)
        c[..., rank + rope:] = rng.uniform(0.5, 2.0, (P, page, H))
        cache = oracle.f32_to_bf16_bits(c)
    return q, cache, bt, lens, dict(rank=rank, qk_dim=rank + rope, page_size=page, sm_scale=1 / 16,
                                    rms_offset=rank + rope)


@pytest.mark.parametrize("fp8", [False, True])
def test_chunked_oracle_equals_whole_row(fp8):
    """Streaming a row in chunks (the oracle's long-row mode) gives the whole-row result."""
    q, cache, bt, lens, kw = _small_paged(fp8)
    extra = dict(rms_mode="log8", kv_fp8=True, k_scale=0.0125) if fp8 else {}
    o1, l1 = oracle.decode(q, cache, bt, lens, **kw, **extra)
    o2, l2 = oracle.decode(q, cache, bt, lens, **kw, **extra, chunk=64)
    np.testing.assert_allclose(o2, o1, rtol=1e-12, atol=1e-14)
    np.testing.assert_allclose(l2[np.isfinite(l1)], l1[np.isfinite(l1)], rtol=1e-12)
    assert np.array_equal(np.isfinite(l1), np.isfinite(l2))


@pytest.mark.parametrize("fp8", [False, True])
def test_torch_cpu_reference_matches_oracle(fp8):
    """The torch CPU path timed as the reference arm computes what the oracle computes."""
    from oracle.torch_ref import decode_paged
    q, cache, bt, lens, kw = _small_paged(fp8)
    extra = dict(rms_mode="log8", kv_fp8=True, k_scale=0.0125) if fp8 else {}
    o1, l1 = oracle.decode(q, cache, bt, lens, **kw, **extra)
    tc = torch.from_numpy(cache) if fp8 else torch.from_numpy(cache.view(np.int16)).view(torch.bfloat16)
    o2, l2 = decode_paged(torch.from_numpy(q), tc, torch.from_numpy(bt), lens.tolist(), rank=kw["rank"],
                          qk_dim=kw["qk_dim"], page_size=kw["page_size"], sm_scale=kw["sm_scale"],
                          rms_offset=kw["rms_offset"], rms_mode="log8" if fp8 else "native",
                          k_scale=0.0125 if fp8 else 1.0)
    np.testing.assert_allclose(o2.numpy(), o1, atol=2e-5)
    fin = np.isfinite(l1)
    np.testing.assert_allclose(l2.numpy()[fin], l1[fin], atol=2e-5)
    assert np.array_equal(np.isfinite(l2.numpy()), fin)
