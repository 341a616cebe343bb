"""GPU parity of the sm_100a decode kernel (through the reference-compatible entry point and
the C ABI) against the reference's golden vectors and the oracle.

Tolerances (from the build's contract): max abs error < 2e-2 for bf16 caches, < 5e-2 for
FP8 caches; the reference tests' own relative bars are checked too (max|d|/max|ref| below
2e-2, tests/test_fp8_kv.py:99 and tests/test_fi_partial_rope.py:116).
"""
from __future__ import annotations

import math
import os

import numpy as np
import pytest
import torch

import oracle
from conftest import DECODE_FIXTURES, load_golden, oracle_args
from gpu_util import bf16_tensor, compare, fp8_tensor, make_bf16_case, make_fp8_case, oracle_ref

pytestmark = pytest.mark.gpu

BF16_TOL, FP8_TOL = 2e-2, 5e-2


def _run(q, cache, bt, sl, *, rank, rms_offset, page, sm_scale=1 / 16, k_scale=None, mode="native",
         lse_dtype=torch.float32, o_dtype=torch.bfloat16, splits=8, logit_cap=0.0, qrows=1):
    from qwen_mla_vllm_b200.mla_decode_attention import decode_attention_fwd
    B, H = q.shape[0], q.shape[1]
    o = torch.full((B, H, rank), float("nan"), dtype=o_dtype, device=q.device)
    lse = torch.full((B, H), float("nan"), dtype=lse_dtype, device=q.device)
    logits = torch.empty(B, H, splits, rank + 1, dtype=torch.float32, device=q.device)
    ks = None if k_scale is None else torch.tensor(k_scale, dtype=torch.float32, device=q.device)
    decode_attention_fwd(q, cache, cache[..., :rank], o, lse, bt, sl, logits, splits, sm_scale, page,
                         logit_cap=logit_cap, k_scale=ks, v_scale=ks, is_mla=True, rms_offset=rms_offset,
                         rms_bf16=mode == "bf16", rms_log8=mode == "log8", qrows=qrows)
    torch.cuda.synchronize()
    return o, lse


def _status():
    import ctypes
    from qwen_mla_vllm_b200 import _lib
    from qwen_mla_vllm_b200 import mla_decode_attention as m
    st = ctypes.c_int32(-1)
    for ws in m._ws_cache.values():
        _lib.load().qmla_read_status(ctypes.c_void_p(ws.data_ptr()),
                                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(st))
    return st.value


@pytest.mark.parametrize("name", DECODE_FIXTURES)
def test_golden_fixture(cuda_device, name):
    """Kernel output vs the reference's own torch reference on the same inputs."""
    g = load_golden(name)
    fp8 = str(g["kind"]) == "fp8"
    args = oracle_args(g)
    cache = (fp8_tensor(g["cache"], cuda_device) if fp8 else bf16_tensor(g["cache"], cuda_device)).unsqueeze(2)
    q = bf16_tensor(g["q"], cuda_device)
    bt = torch.from_numpy(g["block_table"]).to(cuda_device)
    sl = torch.from_numpy(g["seq_lens"]).to(cuda_device)
    mode = str(g["rms_mode"]) if fp8 else "native"
    o, lse = _run(q, cache, bt, sl, rank=int(g["rank"]), rms_offset=int(g["rms_offset"]), page=int(g["page"]),
                  sm_scale=float(g["sm_scale"]), k_scale=float(g["k_scale"]) if fp8 else None,
                  mode="native" if mode == "e4m3" else mode)
    ref = g["out"].astype(np.float64)
    _, ref_lse = oracle.decode(oracle.bf16_bits_to_f32(g["q"]), g["cache"], g["block_table"], g["seq_lens"], **args)
    compare(o, lse, ref, ref_lse, tol=FP8_TOL if fp8 else BF16_TOL, rel_tol=2e-2)
    assert _status() == 0


def test_baseline_config0(cuda_device):
    """B=4, H=24, L=2048, page 16 shuffled, row 768|232|24 bf16, seed 0."""
    cache, q, bt, sl = make_bf16_case(4, 24, 768, 232, 16, [2048] * 4, seed=0, device=cuda_device)
    o, lse = _run(q, cache, bt, sl, rank=768, rms_offset=1000, page=16)
    ref_o, ref_lse = oracle_ref(q, cache, bt, sl, rank=768, qk_dim=1000, page=16, sm_scale=1 / 16, rms_offset=1000)
    err, rel = compare(o, lse, ref_o, ref_lse, tol=BF16_TOL, rel_tol=1e-2)
    assert o.shape == (4, 24, 768) and lse.shape == (4, 24)


@pytest.mark.parametrize("page", [1, 8, 16, 64, 400, 784])
@pytest.mark.parametrize("path", ["tma", "tma_one_column", "tma_one_column_v_copied", "cp_async"])
def test_pages_paths_ragged(cuda_device, page, path, monkeypatch):
    """Every page size on every load path (TMA K in the paired two-column slots this shape gets
    by default, with V copied 16 bytes at a time; one-column K slots, whose bf16 V comes by TMA
    boxes; the same with V copied; cp.async), ragged lengths including 0, 1 and tile edges."""
    if path == "cp_async":
        monkeypatch.setenv("QMLA_NO_TMA", "1")
    if path.startswith("tma_one_column"):
        monkeypatch.setenv("QMLA_NO_PAIR", "1")
    if path == "tma_one_column_v_copied":
        monkeypatch.setenv("QMLA_V_TMA", "0")
    lens = [0, 1, 63, 64, 65, 1000, 2049, 130]
    cache, q, bt, sl = make_bf16_case(len(lens), 24, 768, 232, page, lens, seed=page, device=cuda_device)
    o, lse = _run(q, cache, bt, sl, rank=768, rms_offset=1000, page=page)
    ref_o, ref_lse = oracle_ref(q, cache, bt, sl, rank=768, qk_dim=1000, page=page, sm_scale=1 / 16,
                                rms_offset=1000)
    compare(o, lse, ref_o, ref_lse, tol=BF16_TOL, rel_tol=1e-2)
    # empty rows are defined as o = 0, lse = -inf
    assert torch.all(o[0] == 0) and torch.all(lse[0] == -math.inf)
    assert _status() == 0


@pytest.mark.parametrize("mode", ["log8", "bf16", "e4m3"])
@pytest.mark.parametrize("page", [16, 784])
def test_fp8_modes(cuda_device, mode, page):
    lens = [777, 1, 64, 2000]
    cache, q, bt, sl, ks = make_fp8_case(len(lens), 24, 768, 232, page, lens, mode=mode, seed=3, device=cuda_device)
    o, lse = _run(q, cache, bt, sl, rank=768, rms_offset=1000, page=page, k_scale=ks,
                  mode="native" if mode == "e4m3" else mode)
    ref_o, ref_lse = oracle_ref(q, cache, bt, sl, rank=768, qk_dim=1000, page=page, sm_scale=1 / 16,
                                rms_offset=1000, rms_mode="native" if mode == "e4m3" else mode, kv_fp8=True,
                                k_scale=ks)
    compare(o, lse, ref_o, ref_lse, tol=FP8_TOL, rel_tol=2e-2)


@pytest.mark.parametrize("heads,rank,rope", [(12, 384, 116), (16, 512, 128), (32, 256, 232), (8, 768, 232),
                                             (32, 768, 232), (24, 768, 256), (24, 768, 64)])
def test_head_and_rank_shapes(cuda_device, heads, rank, rope):
    """GLA-g2 groups (12 heads, 384 | 116) and the other head counts / ranks the kernel is built for.
    Rank 768 with rope 256 (no partial last column) and rope 64 (an odd number of full columns:
    the last paired slot holds one column) cover the paired layout's edges."""
    lens = [300, 4097, 5]
    cache, q, bt, sl = make_bf16_case(len(lens), heads, rank, rope, 16, lens, seed=heads, device=cuda_device)
    qk = rank + rope
    o, lse = _run(q, cache, bt, sl, rank=rank, rms_offset=qk, page=16)
    ref_o, ref_lse = oracle_ref(q, cache, bt, sl, rank=rank, qk_dim=qk, page=16, sm_scale=1 / 16, rms_offset=qk)
    compare(o, lse, ref_o, ref_lse, tol=BF16_TOL, rel_tol=1e-2)


@pytest.mark.parametrize("path", ["paired_k", "v_boxes", "v_copied"])
def test_nan_past_row_end_is_never_read(cuda_device, path, monkeypatch):
    """Cache rows past a row's length (inside its last page) hold NaN: outputs stay exact on
    every V path (a V box straddling the row end must not carry them into P = 0 times NaN)."""
    if path != "paired_k":
        monkeypatch.setenv("QMLA_NO_PAIR", "1")  # one-column K slots: V by TMA boxes
    if path == "v_copied":
        monkeypatch.setenv("QMLA_V_TMA", "0")
    lens = [37, 100, 64]
    cache, q, bt, sl = make_bf16_case(len(lens), 24, 768, 232, 16, lens, seed=5, device=cuda_device)
    for b, L in enumerate(lens):
        pg = (L + 15) // 16
        last = int(bt[b, pg - 1])
        if L % 16:
            cache[last, L % 16:] = float("nan")
        for j in range(pg, bt.shape[1]):
            cache[int(bt[b, j])] = float("nan")
    o, lse = _run(q, cache, bt, sl, rank=768, rms_offset=1000, page=16)
    ref_o, ref_lse = oracle_ref(q, cache, bt, sl, rank=768, qk_dim=1000, page=16, sm_scale=1 / 16, rms_offset=1000)
    compare(o, lse, ref_o, ref_lse, tol=BF16_TOL, rel_tol=1e-2)



def test_fp8_nan_past_row_end_is_never_read(cuda_device):
    """e4m3 NaN bytes (0x7f) in the rows past each row's length: outputs stay exact."""
    lens = [37, 100, 64, 300]
    cache, q, bt, sl, ks = make_fp8_case(len(lens), 24, 768, 232, 16, lens, seed=9, device=cuda_device)
    ref_o, ref_lse = oracle_ref(q, cache, bt, sl, rank=768, qk_dim=1000, page=16, sm_scale=1 / 16,
                                rms_offset=1000, rms_mode="log8", kv_fp8=True, k_scale=ks)
    raw = cache.view(torch.uint8)
    for b, L in enumerate(lens):
        pg = (L + 15) // 16
        if L % 16:
            raw[int(bt[b, pg - 1]), L % 16:] = 0x7F
        for j in range(pg, bt.shape[1]):
            raw[int(bt[b, j])] = 0x7F
    o, lse = _run(q, cache, bt, sl, rank=768, rms_offset=1000, page=16, k_scale=ks, mode="log8")
    compare(o, lse, ref_o, ref_lse, tol=FP8_TOL, rel_tol=2e-2)

def test_mtp_verify_rows(cuda_device):
    """Speculative verify: 4 draft tokens per request, flattened as the plugin's metadata builder
    does (qwen_mla/mla_impl.py:628-662); FP8 log8 cache (BASELINE config 2 format)."""
    nreq, qd = 5, 4
    lens_req = [1500, 3, 64, 900, 2]
    cache, _, bt_req, sl_req, ks = make_fp8_case(nreq, 24, 768, 232, 16, lens_req, seed=9, device=cuda_device)
    bt_np, sl_np = oracle.mtp_flatten(bt_req.cpu().numpy(), sl_req.cpu().numpy(), qd)
    bt = torch.from_numpy(bt_np).to(cuda_device)
    sl = torch.from_numpy(sl_np).to(cuda_device)
    g = torch.Generator().manual_seed(2)
    q = (torch.randn(nreq * qd, 24, 1000, generator=g) / 32).to(torch.bfloat16).to(cuda_device)
    o, lse = _run(q, cache, bt, sl, rank=768, rms_offset=1000, page=16, k_scale=ks, mode="log8", qrows=qd)
    ref_o, ref_lse = oracle_ref(q, cache, bt, sl, rank=768, qk_dim=1000, page=16, sm_scale=1 / 16,
                                rms_offset=1000, rms_mode="log8", kv_fp8=True, k_scale=ks)
    compare(o, lse, ref_o, ref_lse, tol=FP8_TOL, rel_tol=2e-2)


@pytest.mark.parametrize("num_ctas", [1, 3, 7, 148])
def test_rows_split_across_ctas_merge(cuda_device, num_ctas):
    """Rows cut at persistent-CTA boundaries are merged exactly (the reference's stage 2)."""
    from qwen_mla_vllm_b200.mla_decode_attention import build_params, run_params
    lens = [5000, 70, 1, 3333, 0, 640]
    cache, q, bt, sl = make_bf16_case(len(lens), 24, 768, 232, 16, lens, seed=num_ctas, device=cuda_device)
    o = torch.zeros(len(lens), 24, 768, dtype=torch.float32, device=cuda_device)
    lse = torch.zeros(len(lens), 24, dtype=torch.float32, device=cuda_device)
    p = build_params(q, cache, o, lse, bt, sl, rank=768, qk_dim=1000, rms_offset=1000, rms_mode=1,
                     page_size=16, sm_scale=1 / 16, num_ctas=num_ctas)
    run_params(p, cuda_device)
    torch.cuda.synchronize()
    ref_o, ref_lse = oracle_ref(q, cache, bt, sl, rank=768, qk_dim=1000, page=16, sm_scale=1 / 16, rms_offset=1000)
    compare(o, lse, ref_o, ref_lse, tol=BF16_TOL, rel_tol=1e-2)


def test_split_q_pe_and_strided_cache_view(cuda_device):
    """q given as (q_nope, q_pe) tensors and a cross-layer cache view with gaps between pages."""
    from qwen_mla_vllm_b200.mla_decode_attention import build_params, run_params
    lens = [900, 33]
    cache, q, bt, sl = make_bf16_case(len(lens), 24, 768, 232, 16, lens, seed=21, device=cuda_device)
    big = torch.zeros((cache.shape[0], 3) + tuple(cache.shape[1:]), dtype=cache.dtype, device=cuda_device)
    big[:, 1] = cache
    view = big[:, 1]
    q_nope = q[..., :768].contiguous()
    q_pe = torch.zeros(2, 24, 256, dtype=torch.bfloat16, device=cuda_device)
    q_pe[..., :232] = q[..., 768:]
    o = torch.zeros(2, 24, 768, dtype=torch.bfloat16, device=cuda_device)
    lse = torch.zeros(2, 24, dtype=torch.float32, device=cuda_device)
    p = build_params(q_nope, view, o, lse, bt, sl, rank=768, qk_dim=1000, rms_offset=1000, rms_mode=1,
                     page_size=16, sm_scale=1 / 16, q_pe=q_pe)
    run_params(p, cuda_device)
    torch.cuda.synchronize()
    ref_o, ref_lse = oracle_ref(q, cache, bt, sl, rank=768, qk_dim=1000, page=16, sm_scale=1 / 16, rms_offset=1000)
    compare(o, lse, ref_o, ref_lse, tol=BF16_TOL, rel_tol=1e-2)


@pytest.mark.parametrize("o_dtype,lse_dtype", [(torch.float32, torch.float32), (torch.float16, torch.bfloat16),
                                               (torch.bfloat16, torch.float16)])
def test_output_dtypes(cuda_device, o_dtype, lse_dtype):
    lens = [500, 64]
    cache, q, bt, sl = make_bf16_case(len(lens), 24, 768, 232, 16, lens, seed=4, device=cuda_device)
    o, lse = _run(q, cache, bt, sl, rank=768, rms_offset=1000, page=16, o_dtype=o_dtype, lse_dtype=lse_dtype)
    ref_o, ref_lse = oracle_ref(q, cache, bt, sl, rank=768, qk_dim=1000, page=16, sm_scale=1 / 16, rms_offset=1000)
    compare(o, lse, ref_o, ref_lse, tol=BF16_TOL, lse_tol=5e-2)


def test_logit_cap_and_large_logits(cuda_device):
    """Large scores exercise the lazy-rescale path; logit_cap follows the reference's tanh cap."""
    lens = [3000, 128]
    cache, q, bt, sl = make_bf16_case(len(lens), 24, 768, 232, 16, lens, seed=8, device=cuda_device,
                                      rms_lo=0.05, rms_hi=0.2)
    q = (q.float() * 20).to(torch.bfloat16)
    for cap in (0.0, 30.0):
        o, lse = _run(q, cache, bt, sl, rank=768, rms_offset=1000, page=16, logit_cap=cap)
        ref_o, ref_lse = oracle_ref(q, cache, bt, sl, rank=768, qk_dim=1000, page=16, sm_scale=1 / 16,
                                    rms_offset=1000, logit_cap=cap)
        compare(o, lse, ref_o, ref_lse, tol=BF16_TOL, lse_tol=5e-2)


def test_no_rms_divisor(cuda_device):
    lens = [700]
    cache, q, bt, sl = make_bf16_case(1, 24, 768, 232, 16, lens, seed=12, device=cuda_device)
    from qwen_mla_vllm_b200.mla_decode_attention import decode_attention_fwd
    o = torch.zeros(1, 24, 768, dtype=torch.bfloat16, device=cuda_device)
    lse = torch.zeros(1, 24, dtype=torch.float32, device=cuda_device)
    logits = torch.empty(1, 24, 4, 1024 + 1, dtype=torch.float32, device=cuda_device)
    qq = torch.zeros(1, 24, 1024, dtype=torch.bfloat16, device=cuda_device)
    qq[..., :1000] = q
    decode_attention_fwd(qq, cache, cache[..., :768], o, lse, bt, sl, logits, 4, 1 / 16, 16, is_mla=True)
    torch.cuda.synchronize()
    ref_o, ref_lse = oracle_ref(qq, cache, bt, sl, rank=768, qk_dim=1024, page=16, sm_scale=1 / 16, rms_offset=-1,
                                rms_mode="none")
    compare(o, lse, ref_o, ref_lse, tol=BF16_TOL)


def test_errors_are_raised(cuda_device):
    from qwen_mla_vllm_b200 import _lib
    from qwen_mla_vllm_b200.mla_decode_attention import build_params, run_params
    lens = [100]
    cache, q, bt, sl = make_bf16_case(1, 24, 768, 232, 16, lens, seed=1, device=cuda_device)
    o = torch.zeros(1, 24, 768, dtype=torch.bfloat16, device=cuda_device)
    p = build_params(q, cache, o, None, bt, sl, rank=768, qk_dim=1000, rms_offset=1000, rms_mode=1,
                     page_size=16, sm_scale=1 / 16)
    with pytest.raises(ValueError, match="workspace"):
        run_params(p, cuda_device, workspace=torch.empty(64, dtype=torch.uint8, device=cuda_device))
    # the C entry point itself rejects a short workspace
    import ctypes
    ws = torch.empty(256, dtype=torch.uint8, device=cuda_device)
    p.workspace, p.workspace_bytes = ws.data_ptr(), 256
    rc = _lib.load().qmla_mla_decode(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == -4
    # rank 640 (5 output blocks) has no kernel in this build
    big = torch.zeros(4, 16, 1, 1024, dtype=torch.bfloat16, device=cuda_device)
    q2 = torch.zeros(1, 24, 1024, dtype=torch.bfloat16, device=cuda_device)
    o2 = torch.zeros(1, 24, 640, dtype=torch.bfloat16, device=cuda_device)
    p2 = build_params(q2, big, o2, None, bt, sl, rank=640, qk_dim=872, rms_offset=872, rms_mode=1,
                      page_size=16, sm_scale=1 / 16)
    with pytest.raises(_lib.QmlaError) as e2:
        run_params(p2, cuda_device)
    assert e2.value.code == -2


def test_cuda_graph_replay(cuda_device):
    """The entry point is capture-safe: a captured call replays to the same result."""
    lens = [1200, 17, 640]
    cache, q, bt, sl = make_bf16_case(len(lens), 24, 768, 232, 16, lens, seed=31, device=cuda_device)
    from qwen_mla_vllm_b200.mla_decode_attention import decode_attention_fwd
    o = torch.zeros(3, 24, 768, dtype=torch.bfloat16, device=cuda_device)
    lse = torch.zeros(3, 24, dtype=torch.float32, device=cuda_device)
    logits = torch.empty(3, 24, 8, 769, dtype=torch.float32, device=cuda_device)
    call = lambda: decode_attention_fwd(q, cache, cache[..., :768], o, lse, bt, sl, logits, 8, 1 / 16, 16,
                                        is_mla=True, rms_offset=1000)
    call()  # first call outside capture (workspace sizing)
    torch.cuda.synchronize()
    want_o, want_lse = o.clone(), lse.clone()
    o.zero_()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            call()
    torch.cuda.current_stream().wait_stream(s)
    o.zero_()
    lse.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(o, want_o) and torch.equal(lse, want_lse)
    del graph


def test_entry_points_restore_current_device(cuda_device):
    """qmla_mla_decode and qmla_mla_decode_static make p->device current for the call only: a
    thread whose current device is another GPU keeps it (needs a second GPU)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import ctypes
    from qwen_mla_vllm_b200 import _lib
    from qwen_mla_vllm_b200.mla_decode_attention import build_params, run_params
    lens = [300, 65]
    cache, q, bt, sl = make_bf16_case(len(lens), 24, 768, 232, 16, lens, seed=3, device=cuda_device)
    o = torch.zeros(2, 24, 768, dtype=torch.bfloat16, device=cuda_device)
    p = build_params(q, cache, o, None, bt, sl, rank=768, qk_dim=1000, rms_offset=1000, rms_mode=1,
                     page_size=16, sm_scale=1 / 16)
    run_params(p, cuda_device)  # sizes and attaches a workspace on device 0
    torch.cuda.synchronize(cuda_device)
    lib = _lib.load()
    stream0 = torch.cuda.current_stream(cuda_device).cuda_stream
    prev = torch.cuda.current_device()
    try:
        torch.cuda.set_device(1)
        for fn in (lib.qmla_mla_decode, lib.qmla_mla_decode_static):
            _lib.check(fn.__name__, fn(ctypes.byref(p), ctypes.c_void_p(stream0)))
            assert torch.cuda.current_device() == 1
        torch.cuda.synchronize(cuda_device)
    finally:
        torch.cuda.set_device(prev)
    ref_o, _ = oracle_ref(q, cache, bt, sl, rank=768, qk_dim=1000, page=16, sm_scale=1 / 16, rms_offset=1000)
    compare(o, None, ref_o, None, tol=BF16_TOL)


@pytest.mark.parametrize("fp8,heads,qd,rank,rope", [(True, 24, 4, 768, 232), (False, 24, 2, 768, 232),
                                                     (True, 12, 4, 384, 116), (False, 12, 3, 384, 116),
                                                     (True, 24, 3, 768, 232), (False, 16, 3, 512, 128)])
def test_mtp_rows_decoded_together(cuda_device, fp8, heads, qd, rank, rope, monkeypatch):
    """MTP verify with a request's drafts decoded together (up to 48 query rows: 2 drafts x 24 heads,
    4 x 12, 3 x 12, 3 x 16; 3 x 24 does not fold) against the oracle and, bit for bit where the
    tiles are the same, against the row-by-row decode (QMLA_NO_FOLD).  Ragged requests include
    drafts of length 0 (a request of length 2 with 4 drafts) and tile edges."""
    lens_req = [1500, 2, 64, 900, 129, 1, 4097]
    n = len(lens_req)
    if fp8:
        cache, _, bt_req, sl_req, ks = make_fp8_case(n, heads, rank, rope, 16, lens_req, seed=qd * 7 + heads,
                                                     device=cuda_device)
    else:
        cache, _, bt_req, sl_req = make_bf16_case(n, heads, rank, rope, 16, lens_req, seed=qd * 7 + heads,
                                                  device=cuda_device)
        ks = None
    bt_np, sl_np = oracle.mtp_flatten(bt_req.cpu().numpy(), sl_req.cpu().numpy(), qd)
    bt = torch.from_numpy(bt_np).to(cuda_device)
    sl = torch.from_numpy(sl_np).to(cuda_device)
    g = torch.Generator().manual_seed(qd)
    q = (torch.randn(n * qd, heads, rank + rope, generator=g) / 32).to(torch.bfloat16).to(cuda_device)
    mode = "log8" if fp8 else "native"
    o, lse = _run(q, cache, bt, sl, rank=rank, rms_offset=rank + rope, page=16, k_scale=ks, mode=mode, qrows=qd,
                  o_dtype=torch.float32)
    ref_o, ref_lse = oracle_ref(q, cache, bt, sl, rank=rank, qk_dim=rank + rope, page=16, sm_scale=1 / 16,
                                rms_offset=rank + rope, rms_mode=mode, kv_fp8=fp8, k_scale=ks or 1.0)
    compare(o, lse, ref_o, ref_lse, tol=FP8_TOL if fp8 else BF16_TOL, rel_tol=2e-2)
    # drafts of length 0 are empty rows: o = 0, lse = -inf
    zero = (sl == 0).nonzero().flatten().tolist()
    assert zero and all(torch.all(o[r] == 0) and torch.all(lse[r] == -math.inf) for r in zero)
    monkeypatch.setenv("QMLA_NO_FOLD", "1")
    o1, lse1 = _run(q, cache, bt, sl, rank=rank, rms_offset=rank + rope, page=16, k_scale=ks, mode=mode, qrows=qd,
                    o_dtype=torch.float32)
    assert float((o1 - o).abs().max()) < (5e-3 if fp8 else 1e-2)
    fin = torch.isfinite(lse1)
    assert torch.equal(fin, torch.isfinite(lse)) and float((lse1[fin] - lse[fin]).abs().max()) < 1e-3
    assert _status() == 0


@pytest.mark.parametrize("heads,fp8", [(40, False), (48, True), (33, True)])
def test_more_than_32_heads(cuda_device, heads, fp8):
    """Up to 48 query heads per row (one decode row, no drafts)."""
    lens = [700, 3, 2100]
    if fp8:
        cache, q, bt, sl, ks = make_fp8_case(len(lens), heads, 512, 128, 16, lens, seed=heads, device=cuda_device)
    else:
        cache, q, bt, sl = make_bf16_case(len(lens), heads, 512, 128, 16, lens, seed=heads, device=cuda_device)
        ks = None
    mode = "log8" if fp8 else "native"
    o, lse = _run(q, cache, bt, sl, rank=512, rms_offset=640, page=16, k_scale=ks, mode=mode)
    ref_o, ref_lse = oracle_ref(q, cache, bt, sl, rank=512, qk_dim=640, page=16, sm_scale=1 / 16, rms_offset=640,
                                rms_mode=mode, kv_fp8=fp8, k_scale=ks or 1.0)
    compare(o, lse, ref_o, ref_lse, tol=FP8_TOL if fp8 else BF16_TOL, rel_tol=2e-2)


@pytest.mark.parametrize("heads,rope,page", [(24, 232, 784), (12, 116, 16), (24, 256, 16), (32, 232, 64)])
def test_rank_1792(cuda_device, heads, rope, page):
    """The reference's widest latent (rank 1792: 14 output blocks, QK width up to 2048), with the
    shapes of its tests/test_two_pass_1792.py: 784-token pages, shuffled tables, ragged lengths, rms
    spread; 12 and 24 heads with partial rope, 24 heads with full rope; 32 heads."""
    lens = [4096, 1, 785, 2000, 0, 3333]
    cache, q, bt, sl = make_bf16_case(len(lens), heads, 1792, rope, page, lens, seed=heads + rope, device=cuda_device,
                                      rms_lo=0.2, rms_hi=4.0)
    qk = 1792 + rope
    o, lse = _run(q, cache, bt, sl, rank=1792, rms_offset=qk, page=page)
    ref_o, ref_lse = oracle_ref(q, cache, bt, sl, rank=1792, qk_dim=qk, page=page, sm_scale=1 / 16, rms_offset=qk)
    compare(o, lse, ref_o, ref_lse, tol=BF16_TOL, rel_tol=1e-2)
    assert _status() == 0


@pytest.mark.parametrize("page", [16, 784])
def test_rank_1792_fp8(cuda_device, page):
    """Rank 1792 on an FP8 cache with log8 rms codes (tests/test_fp8_kv.py:137 runs 1792 too)."""
    lens = [3000, 17, 800]
    cache, q, bt, sl, ks = make_fp8_case(len(lens), 24, 1792, 232, page, lens, seed=page, device=cuda_device)
    o, lse = _run(q, cache, bt, sl, rank=1792, rms_offset=2024, page=page, k_scale=ks, mode="log8")
    ref_o, ref_lse = oracle_ref(q, cache, bt, sl, rank=1792, qk_dim=2024, page=page, sm_scale=1 / 16,
                                rms_offset=2024, rms_mode="log8", kv_fp8=True, k_scale=ks)
    compare(o, lse, ref_o, ref_lse, tol=FP8_TOL, rel_tol=2e-2)


@pytest.mark.parametrize("merge_kernel", [False, True])
def test_split_rows_merged_in_kernel_or_by_merge_kernel(cuda_device, merge_kernel, monkeypatch):
    """Rows cut at CTA boundaries: merged by the merge kernel (the default), or inside the decode
    kernel by the CTA that writes a row's last piece (test hook QMLA_ROW_MERGE); both against the
    oracle, with empty rows among them, and each stable across calls."""
    if not merge_kernel:
        monkeypatch.setenv("QMLA_ROW_MERGE", "1")
    g = torch.Generator().manual_seed(5)
    lens = torch.randint(1, 3000, (48,), generator=g).tolist()
    lens[3] = lens[17] = 0
    cache, q, bt, sl = make_bf16_case(len(lens), 24, 768, 232, 16, lens, seed=41, device=cuda_device)
    o, lse = _run(q, cache, bt, sl, rank=768, rms_offset=1000, page=16, o_dtype=torch.float32)
    ref_o, ref_lse = oracle_ref(q, cache, bt, sl, rank=768, qk_dim=1000, page=16, sm_scale=1 / 16, rms_offset=1000)
    compare(o, lse, ref_o, ref_lse, tol=BF16_TOL, rel_tol=1e-2)
    assert torch.all(o[3] == 0) and torch.all(lse[17] == -math.inf)
    o2, lse2 = _run(q, cache, bt, sl, rank=768, rms_offset=1000, page=16, o_dtype=torch.float32)
    assert torch.equal(o, o2) and torch.equal(lse, lse2)  # same partition, same merge order
    assert _status() == 0
