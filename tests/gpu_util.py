"""Helpers shared by the GPU parity tests: fixture tensors on the device, seeded inputs,
and the comparison against the oracle."""
from __future__ import annotations

import math

import numpy as np
import torch

import oracle


def bf16_tensor(bits: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def fp8_tensor(b: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(b)).to(device).view(torch.float8_e4m3fn)


def cache_numpy(cache: torch.Tensor) -> np.ndarray:
    """[P, page, 1, W] device cache -> raw element array [P, page, W] for the oracle."""
    c = cache[:, :, 0, :].contiguous().cpu()
    if c.dtype == torch.bfloat16:
        return c.view(torch.int16).numpy().view(np.uint16)
    return c.view(torch.uint8).numpy()


def make_bf16_case(B, H, rank, rope, page, lens, *, seed=0, device, extra_pages=3, rms_lo=0.5, rms_hi=2.0):
    """bf16 cache [P, page, 1, rank+rope+H (+pad to 8)], shuffled page table, N(0,1) latent/rope,
    U(rms_lo, rms_hi) rms tail, q ~ N(0,1)/sqrt(1024) (the BASELINE config-0 recipe)."""
    g = torch.Generator().manual_seed(seed)
    W = rank + rope + H
    W += (-W) % 8
    pps = max(1, max((int(L) + page - 1) // page for L in lens))
    P = B * pps + extra_pages
    cache = torch.randn(P, page, 1, W, generator=g).to(torch.bfloat16)
    cache[..., rank + rope:] = (torch.rand(P, page, 1, W - rank - rope, generator=g) * (rms_hi - rms_lo) + rms_lo).to(torch.bfloat16)
    bt = torch.randperm(B * pps, generator=g).reshape(B, pps).to(torch.int32)
    q = (torch.randn(B, H, rank + rope, generator=g) / math.sqrt(1024)).to(torch.bfloat16)
    sl = torch.tensor(lens, dtype=torch.int32)
    return cache.to(device), q.to(device), bt.to(device), sl.to(device)


def make_fp8_case(B, H, rank, rope, page, lens, *, mode="log8", seed=0, device, extra_pages=3):
    """FP8 rows written by the oracle's restatement of the reference writer
    (qwen_mla/mla_impl.py:309-342), k_scale = absmax / 448."""
    g = torch.Generator().manual_seed(seed)
    pps = max(1, max((int(L) + page - 1) // page for L in lens))
    P = B * pps + extra_pages
    lat = torch.randn(P * page, rank, generator=g) * 2.0
    rp = torch.randn(P * page, rope, generator=g) * 1.5
    rms = torch.exp(torch.randn(P * page, H, generator=g) * 0.6)
    scale = float(max(lat.abs().max(), rp.abs().max())) / 448
    lat_b = oracle.bf16_round(lat.numpy())
    kpe = np.concatenate([oracle.bf16_round(rp.numpy()), oracle.bf16_round(rms.numpy())], axis=1)
    if mode in ("log8", "bf16"):
        rows = oracle.fp8_cache_rows(lat_b, kpe, scale, rope, H, mode)
    else:  # e4m3 rms: scaled with the row like latent and rope (tests/test_fp8_kv.py:37-43)
        rows = np.concatenate([oracle.fp8_cache_rows(lat_b, kpe, scale, rope, H, "log8")[:, :rank + rope],
                               oracle.e4m3_encode(np.clip(kpe[:, rope:] / np.float32(scale), -448, 448))], axis=1)
    W = rows.shape[1] + (-rows.shape[1]) % 16
    buf = np.zeros((P * page, W), np.uint8)
    buf[:, :rows.shape[1]] = rows
    cache = torch.from_numpy(buf.reshape(P, page, 1, W)).to(device).view(torch.float8_e4m3fn)
    bt = torch.randperm(B * pps, generator=g).reshape(B, pps).to(torch.int32)
    q = (torch.randn(B, H, rank + rope, generator=g) / math.sqrt(1024)).to(torch.bfloat16)
    return cache, q.to(device), bt.to(device), torch.tensor(lens, dtype=torch.int32).to(device), scale


def oracle_ref(q, cache, bt, sl, *, rank, qk_dim, page, sm_scale, rms_offset, rms_mode="native",
               kv_fp8=False, k_scale=1.0, logit_cap=0.0):
    qn = q.float().cpu().numpy()
    return oracle.decode(qn, cache_numpy(cache), bt.cpu().numpy(), sl.cpu().numpy(), rank=rank,
                         qk_dim=qk_dim, page_size=page, sm_scale=sm_scale, rms_offset=rms_offset,
                         rms_mode=rms_mode, kv_fp8=kv_fp8, k_scale=k_scale, logit_cap=logit_cap)


def compare(o, lse, ref_o, ref_lse, *, tol, lse_tol=2e-2, rel_tol=None):
    """max-abs check plus max|d|/max|ref| as the reference tests report."""
    o = o.float().cpu().numpy()
    d = np.abs(o - ref_o)
    err = float(d.max()) if d.size else 0.0
    scale = float(np.abs(ref_o).max()) if ref_o.size else 1.0
    rel = err / max(scale, 1e-30)
    assert np.isfinite(o).all(), "non-finite output"
    assert err < tol, f"max abs err {err:.3e} >= {tol}"
    if rel_tol is not None:
        assert rel < rel_tol, f"max rel err {rel:.3e} >= {rel_tol}"
    if lse is not None:
        l = lse.float().cpu().numpy()
        fin = np.isfinite(ref_lse)
        assert np.array_equal(np.isfinite(l), fin) or np.all(~fin == (l == -np.inf))
        if fin.any():
            le = float(np.abs(l[fin] - ref_lse[fin]).max())
            assert le < lse_tol, f"lse err {le:.3e}"
    return err, rel


def oracle_rows(w, case, rows, chunk=65536):
    """oracle.decode on the given decode rows of a bench workload case (only their pages are
    copied to the host).  Returns (o [len(rows), H, rank], lse [len(rows), H]) in float64."""
    page = w.page
    bt_rows = case.bt_rows.cpu()
    sl = case.sl_rows.cpu().numpy()
    need = sorted({int(p) for r in rows for p in bt_rows[r, :(int(sl[r]) + page - 1) // page].tolist()})
    remap = {p: i for i, p in enumerate(need)}
    idx = torch.tensor(need, device=case.cache.device)
    host = cache_numpy(case.cache[idx])
    bt = np.zeros((len(rows), bt_rows.shape[1]), np.int32)
    for i, r in enumerate(rows):
        npg = (int(sl[r]) + page - 1) // page
        bt[i, :npg] = [remap[int(p)] for p in bt_rows[r, :npg].tolist()]
    q = case.q[rows].float().cpu().numpy()
    return oracle.decode(q, host, bt, sl[rows], rank=w.rank, qk_dim=w.qk, page_size=page, sm_scale=1 / 16,
                         rms_offset=w.qk, rms_mode="log8" if w.fp8 else "native", kv_fp8=w.fp8,
                         k_scale=float(case.k_scale) if case.k_scale is not None else 1.0, chunk=chunk)
