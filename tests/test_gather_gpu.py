"""The prefill context gather kernel (qmla_gather_cache) against the reference's golden rows
and the oracle: bit-exact for bf16 / f16 destinations (the e4m3 * scale product, the bf16
bytes and the log8 decode all round the same way; every log8 code's exact value lies
> 40 float32 ulps from an f16 / bf16 rounding midpoint, so a 2-ulp exp2 cannot move it),
the vector and the scalar (unaligned rows) paths, conversions, index errors, and a
full-size chunk checked by a torch restatement of the reference on the device."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from conftest import GATHER_FIXTURES, load_golden, to_dst_bits

pytestmark = pytest.mark.gpu

_TORCH_DT = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.contiguous().cpu()
    if t.dtype == torch.float32:
        return t.numpy().view(np.uint32)
    return t.view(torch.int16).numpy().view(np.uint16)


def _run(g: dict, device, dst: torch.Tensor, **kw) -> None:
    from qwen_mla_vllm_b200.mla_gather import gather_cache_torch
    mode = str(g["mode"])
    cache = torch.from_numpy(np.ascontiguousarray(g["cache"]))
    if mode == "auto":
        cache = cache.view(torch.int16).view(torch.bfloat16)
    else:
        cache = cache.view(torch.float8_e4m3fn)
    cache = cache.to(device).unsqueeze(2)
    gather_cache_torch(
        src_cache=cache, dst=dst, block_table=torch.from_numpy(g["block_table"]).to(device),
        cu_seq_lens=torch.from_numpy(g["cu_seq_lens"]).to(device),
        token_to_seq=torch.from_numpy(g["token_to_seq"]).to(device), num_tokens=int(g["num_tokens"]),
        kv_cache_dtype="auto" if mode == "auto" else "fp8",
        scale=torch.tensor(float(g["scale"]), device=device),
        seq_starts=torch.from_numpy(g["seq_starts"]).to(device),
        mla_rms=None if mode == "auto" else (int(g["rms_offset"]), int(g["heads"]), mode), **kw)


@pytest.mark.parametrize("name", GATHER_FIXTURES)
def test_gather_golden_bit_exact(cuda_device, name):
    g = load_golden(name)
    dst = torch.full(g["dst"].shape, 7.0, dtype=_TORCH_DT[str(g["dst_dtype"])], device=cuda_device)
    _run(g, cuda_device, dst, check=True)
    torch.cuda.synchronize()
    got = _bits(dst)
    assert np.array_equal(got, g["dst"]), f"{int((got != g['dst']).sum())} elements differ"


def _fp8_case(rng, P, page, off, nh, mode, width):
    """Random valid FP8 rows: every e4m3 byte but the two NaN codes, all 256 log8 codes,
    finite bf16 rms bytes."""
    rows = rng.integers(0, 256, size=(P, page, width), dtype=np.uint8)
    nan = (rows & 0x7F) == 0x7F
    rows[nan] = 0x7E
    if mode == "bf16":
        rms = np.exp(rng.standard_normal((P, page, nh)).astype(np.float32) * 0.6)
        rows[:, :, off:off + 2 * nh] = oracle.f32_to_bf16_bits(rms).view(np.uint8).reshape(P, page, 2 * nh)
    elif mode == "log8":
        rows[:, :, off:off + nh] = rng.integers(0, 256, size=(P, page, nh), dtype=np.uint8)
    return rows


def _chunk(rng, n_seqs, P, page, max_len):
    lens = rng.integers(0, max_len, size=n_seqs)
    lens[1] = 0  # an empty sequence in the chunk
    starts = rng.integers(0, 200, size=n_seqs).astype(np.int32)
    cols = (int((lens + starts).max()) + page - 1) // page
    bt = rng.integers(0, P, size=(n_seqs, cols)).astype(np.int32)
    cu = np.zeros(n_seqs + 1, np.int32)
    cu[1:] = np.cumsum(lens)
    t2s = np.repeat(np.arange(n_seqs, dtype=np.int32), lens)
    return bt, cu, t2s, starts, int(lens.sum())


@pytest.mark.parametrize("mode", ["log8", "bf16", "e4m3"])
@pytest.mark.parametrize("dst_dt", ["bfloat16", "float16"])
@pytest.mark.parametrize("path", ["bulk", "regs", "scalar"])
def test_gather_fp8_config_shapes(cuda_device, monkeypatch, mode, dst_dt, path):
    """rank 768 + rope 232, 24 heads (the TP=1 row).  Aligned rows take the staged kernel
    (bulk copies through shared memory) or, with the QMLA_GATHER_REGS hook, the
    register-staged 16-byte path; a 1030-byte row stride and an odd destination offset take
    the scalar path."""
    from qwen_mla_vllm_b200.mla_gather import gather_cache_torch
    if path == "regs":
        monkeypatch.setenv("QMLA_GATHER_REGS", "1")
    aligned = path != "scalar"
    rng = np.random.default_rng(["log8", "bf16", "e4m3"].index(mode) * 8 + (dst_dt == "float16") * 4 +
                                ["bulk", "regs", "scalar"].index(path))
    off, nh, page, P = 1000, 24, 16, 96
    width = (1056 if mode == "bf16" else 1024) if aligned else 1030 + (24 if mode == "bf16" else 0)
    rows = _fp8_case(rng, P, page, off, nh, mode, width)
    bt, cu, t2s, starts, n = _chunk(rng, 7, P, page, 300)
    scale = np.float32(0.0123)
    want = oracle.gather_cache(rows, bt, cu, t2s, n, fp8=True, scale=scale, seq_starts=starts,
                               mla_rms=(off, nh, mode))
    cols = 1024 + (0 if aligned else 8)
    base = torch.full((n + 2, cols + 1), 5.0, dtype=_TORCH_DT[dst_dt], device=cuda_device)
    dst = base[:, :cols] if aligned else base[:, 1:cols + 1]
    cache = torch.from_numpy(rows).to(cuda_device).view(torch.float8_e4m3fn).unsqueeze(2)
    gather_cache_torch(src_cache=cache, dst=dst, block_table=torch.from_numpy(bt).to(cuda_device),
                       cu_seq_lens=torch.from_numpy(cu).to(cuda_device),
                       token_to_seq=torch.from_numpy(t2s).to(cuda_device), num_tokens=n,
                       kv_cache_dtype="fp8_e4m3", scale=torch.tensor(scale, device=cuda_device),
                       seq_starts=torch.from_numpy(starts).to(cuda_device), mla_rms=(off, nh, mode),
                       check=True)
    torch.cuda.synchronize()
    got = _bits(dst)
    exp = np.full(got.shape, to_dst_bits(np.float32(5.0), dst_dt), np.uint16)
    exp[:n, :off + nh] = to_dst_bits(want, dst_dt)
    assert np.array_equal(got, exp), f"{int((got != exp).sum())} elements differ"


@pytest.mark.parametrize("mode", ["log8", "bf16"])
def test_gather_fp8_wide_rows(cuda_device, mode):
    """rank 1792 + rope 232 (rows of 2 KB and more: 16 and 8 rows per stage); a chunk
    whose row count is not a multiple of the stage's."""
    from qwen_mla_vllm_b200.mla_gather import gather_cache_torch
    rng = np.random.default_rng(17 + (mode == "bf16"))
    off, nh, page, P = 2024, 24, 16, 48
    width = 2048 if mode == "log8" else 2080
    rows = _fp8_case(rng, P, page, off, nh, mode, width)
    bt, cu, t2s, starts, n = _chunk(rng, 5, P, page, 333)
    want = oracle.gather_cache(rows, bt, cu, t2s, n, fp8=True, scale=0.25, seq_starts=starts,
                               mla_rms=(off, nh, mode))
    dst = torch.full((n, off + nh), 5.0, dtype=torch.bfloat16, device=cuda_device)
    gather_cache_torch(src_cache=torch.from_numpy(rows).to(cuda_device).view(torch.float8_e4m3fn).unsqueeze(2),
                       dst=dst, block_table=torch.from_numpy(bt).to(cuda_device),
                       cu_seq_lens=torch.from_numpy(cu).to(cuda_device),
                       token_to_seq=torch.from_numpy(t2s).to(cuda_device), num_tokens=n, kv_cache_dtype="fp8",
                       scale=torch.tensor(0.25, device=cuda_device),
                       seq_starts=torch.from_numpy(starts).to(cuda_device), mla_rms=(off, nh, mode), check=True)
    got = _bits(dst)
    assert np.array_equal(got, to_dst_bits(want, "bfloat16"))


def test_gather_fp8_log8_f32_destination(cuda_device):
    """f32 destination: the e4m3 columns are exact; the log8 column is within 4 ulps (the
    2-ulp error of CUDA's exp2f plus numpy's own float32 exp2 error), which bf16 / f16
    destinations round away."""
    from qwen_mla_vllm_b200.mla_gather import gather_cache_torch
    rng = np.random.default_rng(3)
    off, nh, page, P = 1000, 24, 16, 40
    rows = _fp8_case(rng, P, page, off, nh, "log8", 1024)
    bt, cu, t2s, starts, n = _chunk(rng, 5, P, page, 200)
    want = oracle.gather_cache(rows, bt, cu, t2s, n, fp8=True, scale=0.5, seq_starts=starts,
                               mla_rms=(off, nh, "log8"))
    dst = torch.zeros(n, 1024, dtype=torch.float32, device=cuda_device)
    gather_cache_torch(src_cache=torch.from_numpy(rows).to(cuda_device).view(torch.float8_e4m3fn).unsqueeze(2),
                       dst=dst, block_table=torch.from_numpy(bt).to(cuda_device),
                       cu_seq_lens=torch.from_numpy(cu).to(cuda_device),
                       token_to_seq=torch.from_numpy(t2s).to(cuda_device), num_tokens=n, kv_cache_dtype="fp8",
                       scale=torch.tensor(0.5, device=cuda_device),
                       seq_starts=torch.from_numpy(starts).to(cuda_device), mla_rms=(off, nh, "log8"))
    got = dst.cpu().numpy()
    assert np.array_equal(got[:, :off], want[:, :off])
    assert np.allclose(got[:, off:off + nh], want[:, off:], rtol=5e-7, atol=0)


@pytest.mark.parametrize("src_dt,dst_dt", [(torch.bfloat16, torch.bfloat16), (torch.bfloat16, torch.float16),
                                           (torch.float16, torch.bfloat16), (torch.bfloat16, torch.float32)])
@pytest.mark.parametrize("width", [1024, 1001])
def test_gather_two_byte_copy(cuda_device, src_dt, dst_dt, width):
    """2-byte caches: the whole row copied (and converted like torch's copy_), over the
    16-byte path (width 1024) and the scalar path (1001 elements: unaligned rows)."""
    from qwen_mla_vllm_b200.mla_gather import gather_cache_torch
    rng = np.random.default_rng(width)
    page, P = 16, 64
    src = torch.from_numpy(rng.standard_normal((P, page, 1, width)).astype(np.float32) * 3).to(src_dt)
    bt, cu, t2s, starts, n = _chunk(rng, 6, P, page, 250)
    dst = torch.full((n + 1, width), -1.0, dtype=dst_dt, device=cuda_device)
    gather_cache_torch(src_cache=src.to(cuda_device), dst=dst, block_table=torch.from_numpy(bt).to(cuda_device),
                       cu_seq_lens=torch.from_numpy(cu).to(cuda_device),
                       token_to_seq=torch.from_numpy(t2s).to(cuda_device), num_tokens=n, kv_cache_dtype="auto",
                       scale=torch.tensor(1.0, device=cuda_device),
                       seq_starts=torch.from_numpy(starts).to(cuda_device), check=True)
    s = t2s.astype(np.int64)
    tok = np.arange(n) - cu[s] + starts[s]
    blk = bt[s, tok // page]
    want = src[torch.from_numpy(blk), torch.from_numpy(tok % page)].reshape(n, width).to(dst_dt)
    got = dst.cpu()
    assert torch.equal(got[:n], want)
    assert bool((got[n:] == -1.0).all())


def test_gather_bad_indices_are_skipped_and_flagged(cuda_device):
    """A page id past the cache, a token past the block-table row and a sequence id past the
    chunk: those rows stay untouched, the status word says so, and check=True raises."""
    from qwen_mla_vllm_b200.mla_gather import gather_cache_torch, gather_status
    rng = np.random.default_rng(9)
    off, nh, page, P = 1000, 24, 16, 32
    rows = _fp8_case(rng, P, page, off, nh, "log8", 1024)
    bt = rng.integers(0, P, size=(3, 4)).astype(np.int32)
    bt[0, 1] = P + 5                       # token 16..31 of sequence 0: page id out of range
    cu = np.array([0, 40, 60, 64], np.int32)
    t2s = np.repeat(np.arange(3, dtype=np.int32), [40, 20, 4])
    t2s[62] = 7                            # sequence id out of range
    starts = np.array([0, 50, 0], np.int32)  # sequence 1 runs past its 4 block-table columns
    n = 64
    args = dict(block_table=torch.from_numpy(bt).to(cuda_device), cu_seq_lens=torch.from_numpy(cu).to(cuda_device),
                token_to_seq=torch.from_numpy(t2s).to(cuda_device), num_tokens=n, kv_cache_dtype="fp8",
                scale=torch.tensor(1.0, device=cuda_device), seq_starts=torch.from_numpy(starts).to(cuda_device),
                mla_rms=(off, nh, "log8"))
    cache = torch.from_numpy(rows).to(cuda_device).view(torch.float8_e4m3fn).unsqueeze(2)
    gather_status(cuda_device)  # clear
    dst = torch.full((n, 1024), 9.0, dtype=torch.bfloat16, device=cuda_device)
    gather_cache_torch(src_cache=cache, dst=dst, **args)
    assert gather_status(cuda_device) == 2
    got = dst.float().cpu().numpy()
    bad = np.zeros(n, bool)
    bad[16:32] = True                      # seq 0, page column 1
    bad[40 + (64 - 50):60] = True          # seq 1, tokens 64.. -> column 4 of 4
    bad[62] = True
    assert (got[bad] == 9.0).all()
    good = ~bad
    s = t2s[good].astype(np.int64)
    tok = np.arange(n)[good] - cu[s] + starts[s]
    ref = oracle.e4m3_decode(rows[bt[s, tok // page], tok % page, :off])
    assert np.array_equal(got[good][:, :off], oracle.bf16_round(ref))
    with pytest.raises(IndexError):
        gather_cache_torch(src_cache=cache, dst=dst, check=True, **args)
    assert gather_status(cuda_device) == 0


def test_gather_full_chunk_matches_torch_restatement(cuda_device):
    """A 131,072-row chunk (16 sequences x 8192 tokens, rank 768 + rope 232 + 24 log8 codes)
    against the reference's own torch formula evaluated on the device."""
    from qwen_mla_vllm_b200.mla_gather import gather_cache_torch
    g = torch.Generator(device=cuda_device).manual_seed(4)
    off, nh, page, seqs, L = 1000, 24, 16, 16, 8192
    P = seqs * L // page
    raw = torch.randint(0, 256, (P, page, 1, 1024), dtype=torch.uint8, device=cuda_device, generator=g)
    raw[(raw & 0x7F) == 0x7F] = 0x7E
    cache = raw.view(torch.float8_e4m3fn)
    bt = torch.randperm(P, device=cuda_device, generator=g).reshape(seqs, L // page).to(torch.int32)
    cu = torch.arange(0, (seqs + 1) * L, L, dtype=torch.int32, device=cuda_device)
    t2s = torch.arange(seqs, dtype=torch.int32, device=cuda_device).repeat_interleave(L)
    n = seqs * L
    scale = torch.tensor(0.03, device=cuda_device)
    dst = torch.empty(n, 1024, dtype=torch.bfloat16, device=cuda_device)
    gather_cache_torch(src_cache=cache, dst=dst, block_table=bt, cu_seq_lens=cu, token_to_seq=t2s,
                       num_tokens=n, kv_cache_dtype="fp8", scale=scale, mla_rms=(off, nh, "log8"), check=True)
    j = torch.arange(n, device=cuda_device)
    s = t2s.long()
    tok = j - cu.long()[s]
    blk = bt[s, tok // page].long()
    rows = raw[blk, tok % page, 0]
    want_lat = (rows[:, :off].view(torch.float8_e4m3fn).float() * scale).to(torch.bfloat16)
    code = rows[:, off:off + nh].float()
    want_rms = torch.exp2(-3.0 + code * (6.0 / 255.0)).to(torch.bfloat16)
    assert torch.equal(dst[:, :off], want_lat)
    assert torch.equal(dst[:, off:off + nh], want_rms)
