"""GPU checks of the auxiliary kernels: the FP8 cache writer (bit-exact against the reference
writer's golden bytes) and the DCP correction / merge kernels (against the oracle's
restatement of qwen_mla/dcp_fix.py)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden
from gpu_util import bf16_tensor

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", ["log8", "bf16"])
def test_fp8_cache_write_bit_exact(cuda_device, mode):
    from qwen_mla_vllm_b200.kv_cache import fp8_kv_cache_update
    g = load_golden(f"cache_write_{mode}")
    want = g["cache"]
    cache = torch.zeros(want.shape[0], want.shape[1], 1, want.shape[2], dtype=torch.uint8,
                        device=cuda_device).view(torch.float8_e4m3fn)
    kv_c = bf16_tensor(g["latent"], cuda_device)
    k_pe = bf16_tensor(g["k_pe"], cuda_device)
    slots = torch.from_numpy(g["slots"]).to(cuda_device)
    ks = torch.tensor(float(g["k_scale"]), dtype=torch.float32, device=cuda_device)
    fp8_kv_cache_update(kv_c, k_pe, cache, slots, ks, int(g["packed_rope"]), int(g["heads"]), mode)
    torch.cuda.synchronize()
    got = cache.view(torch.uint8)[:, :, 0, :].cpu().numpy()
    assert np.array_equal(got, want), f"{int((got != want).sum())} bytes differ"


@pytest.mark.parametrize("n", [2, 4, 8])
@pytest.mark.parametrize("base_e", [True, False])
def test_dcp_correct_matches_oracle(cuda_device, n, base_e):
    from qwen_mla_vllm_b200.dcp import correct_attn_out
    rng = np.random.default_rng(n)
    B, H, D = 5, 24, 768
    lses = rng.standard_normal((n, B, H)).astype(np.float32) * 3
    lses[0, 0, 0] = np.nan
    lses[:, 1, 1] = -np.inf
    lses[n - 1, 2, 2] = np.inf
    for r in range(n):
        out = rng.standard_normal((B, H, D)).astype(np.float32)
        t = torch.from_numpy(out).to(cuda_device)
        res, lse = correct_attn_out(t, torch.from_numpy(lses).to(cuda_device), r, is_lse_base_on_e=base_e)
        torch.cuda.synchronize()
        want, want_lse = oracle.dcp_correct(out, lses, r, base_e)
        assert np.allclose(res.cpu().numpy(), want, rtol=1e-5, atol=1e-6)
        got_lse = lse.cpu().numpy()
        fin = np.isfinite(want_lse)
        assert np.allclose(got_lse[fin], want_lse[fin], rtol=1e-5, atol=1e-5)
        assert np.array_equal(np.isfinite(got_lse), fin)


@pytest.mark.parametrize("n", [1, 2, 8])
def test_dcp_merge_matches_oracle(cuda_device, n):
    from qwen_mla_vllm_b200.dcp import merge_partials
    rng = np.random.default_rng(10 + n)
    B, H, D = 3, 24, 768
    parts = rng.standard_normal((n, B, H, D)).astype(np.float32)
    lses = rng.standard_normal((n, B, H)).astype(np.float32) * 2
    lses[:, 0, 0] = -np.inf  # empty everywhere
    o, lse = merge_partials(torch.from_numpy(parts).to(cuda_device), torch.from_numpy(lses).to(cuda_device))
    torch.cuda.synchronize()
    want, want_lse = oracle.dcp_merge(parts, lses)
    assert np.allclose(o.cpu().numpy(), want, rtol=1e-5, atol=1e-6)
    fin = np.isfinite(want_lse)
    assert np.allclose(lse.cpu().numpy()[fin], want_lse[fin], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("base_e", [True, False])
def test_dcp_kernels_match_the_reference_correction(cuda_device, base_e):
    """qmla_dcp_correct per rank, and the fused merges (qmla_dcp_merge, and the one-kernel P2P merge
    with ranks emulated on one GPU) against the reference's own Triton correction
    (qwen_mla/dcp_fix.py:101-130, fixture from tests/golden/make_golden_gpu.py): the merged
    output is the sum of the ranks' corrected partials."""
    from conftest import load_golden
    from qwen_mla_vllm_b200.dcp import ExchangeBuffer, correct_attn_out, merge_partials, p2p_merge
    g = load_golden("dcp_correct")
    N, B, H, D = (int(g[k]) for k in ("N", "B", "H", "D"))
    lses = torch.from_numpy(g["lses"]).to(cuda_device)
    total = 0
    for r in range(N):
        key = f"{'e' if base_e else '2'}{r}"
        o = torch.from_numpy(g["out"][r]).to(cuda_device).contiguous()
        o, lse = correct_attn_out(o, lses, r, None, is_lse_base_on_e=base_e)
        torch.cuda.synchronize()
        assert torch.allclose(o.cpu(), torch.from_numpy(g[f"out_{key}"]), rtol=2e-6, atol=1e-6)
        want = torch.from_numpy(g[f"lse_{key}"])
        fin = torch.isfinite(want)
        assert torch.equal(torch.isfinite(lse.cpu()), fin)
        assert torch.allclose(lse.cpu()[fin], want[fin], rtol=1e-6, atol=1e-6)
        total = total + g[f"out_{key}"]
    if not base_e:
        return  # the merges take natural-log LSEs
    want = torch.from_numpy(total)
    parts = torch.from_numpy(g["out"]).to(cuda_device).contiguous()
    o, _ = merge_partials(parts, lses)
    torch.cuda.synchronize()
    assert torch.allclose(o.cpu(), want, rtol=1e-5, atol=1e-5)
    bufs = [ExchangeBuffer(B, H, D, cuda_device) for _ in range(N)]
    try:
        for n, b in enumerate(bufs):
            po, pl = b.partial(1)
            po.copy_(parts[n])
            pl.copy_(lses[n])
            b.flags()[:N] = 1
        out = torch.empty(B, H, D, dtype=torch.float32, device=cuda_device)
        p2p_merge([b.ptr for b in bufs], 0, B, H, D, 1, out, "ar", timeout_s=1.0)
        torch.cuda.synchronize()
        assert bufs[0].status() == 0
        assert torch.allclose(out.cpu(), want, rtol=1e-5, atol=1e-5)
    finally:
        for b in bufs:
            b.free()
