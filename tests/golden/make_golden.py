#!/usr/bin/env python3
"""Generate the golden fixtures of tests/golden/ from the REFERENCE's own torch functions.

Run in a container where the reference plugin (sootaugur/qwen-mla-vllm) is importable:

    QMLA_REFERENCE=/path/to/qwen-mla-vllm python tests/golden/make_golden.py [name-prefix ...]

Everything runs on the CPU.  The reference functions used (each called unmodified):
  * tests/test_fi_partial_rope.py:27-58   build / layout / ref_out   (bf16 partial-rope decode)
  * tests/test_fp8_kv.py:34-76            make / fp8_cache / deq / rms_decoded / ref (FP8 decode)
  * tests/test_decode_numerics.py:25-44   reference (taken from the file's AST: the module runs
                                          its GPU cases at import time)
  * qwen_mla/mla_impl.py:309-342          QwenMLATritonImpl.do_kv_cache_update (FP8 row writer)
  * qwen_mla/fi_decode.py:235-270         _RankPlan.plan_cpu (work-list arrays)
  * qwen_mla/mla_impl.py:628-662          MLATritonMetadataBuilder._build_decode (MTP rows, its
                                          vLLM parent step stubbed)
  * qwen_mla/ops/mla_gather.py:28-76      gather_cache_torch (prefill context gather)
Module-level constants the tests pin (PAGE, dev, SHUFFLE, ...) are set on the imported
modules before the calls; shapes are kept small so the fixtures stay a few hundred KB each.
Arrays are stored raw: bf16 as uint16 bit patterns, FP8 as uint8 bytes.
"""
from __future__ import annotations

import ast
import importlib.util
import os
import pathlib
import sys
import types

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
REF = pathlib.Path(os.environ.get("QMLA_REFERENCE", "/root/reference"))


def _load(path: pathlib.Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    if t.dtype in (torch.float8_e4m3fn, torch.uint8):
        return t.contiguous().view(torch.uint8).numpy()
    return t.contiguous().numpy()


def partial_rope_case(tag, batch, heads, ctx, rank, rope, page=16):
    """bf16 cache, shuffled pages, ragged lengths, rms spread over ~e^+-2."""
    m = _load(REF / "tests" / "test_fi_partial_rope.py", "ref_partial_rope")
    m.PAGE, m.SHUFFLE, m.RAGGED, m.RMS_SPREAD = page, True, True, True
    dev = torch.device("cpu")
    cache, q, pps = m.build(batch, heads, ctx, rank, rope, dev, seed=rank + heads)
    bt, lens = m.layout(batch, ctx, pps, dev)
    out = m.ref_out(cache, q, batch, heads, ctx, rank, rope, pps, bt, lens)
    np.savez_compressed(
        HERE / f"{tag}.npz", kind="bf16", cache=_bits(cache[:, :, 0, :]), q=_bits(q),
        block_table=bt.numpy(), seq_lens=lens.numpy(), out=out.numpy().astype(np.float32),
        rank=rank, rope=rope, heads=heads, page=page, rms_offset=rank + rope,
        sm_scale=np.float32(1.0 / 256 ** 0.5), source="tests/test_fi_partial_rope.py:27-58")
    print(f"{tag}: cache {tuple(cache.shape)} out {tuple(out.shape)}")


def fp8_case(tag, batch, heads, ctx, rank, rope, mode, page=16):
    """FP8 row [lat e4m3 | rope e4m3 | rms (log8 / bf16 bytes / e4m3)] vs the dequantised reference."""
    m = _load(REF / "tests" / "test_fp8_kv.py", "ref_fp8_kv")
    m.PAGE, m.dev = page, torch.device("cpu")
    lat, rp, rms, q, pps = m.make(batch, heads, ctx, rank, rope, seed=rank + heads)
    scale = torch.tensor(float(max(lat.abs().max(), rp.abs().max())) / 448)
    width = rank + rope + (2 if mode == "bf16" else 1) * heads
    width += (-width) % 16
    cache = m.fp8_cache(lat, rp, rms, scale, width, mode)
    g = torch.Generator().manual_seed(1)
    bt = torch.randperm(batch * pps, generator=g).reshape(batch, pps).to(torch.int32)
    lens = torch.tensor([ctx - (37 * b) % page for b in range(batch)], dtype=torch.int32)
    dl, dr = m.deq(lat, rp, scale)
    rq = m.rms_decoded(rms, scale, mode)
    out = m.ref(q, dl, dr, rq, bt, lens, rank, rms_exact=True)
    np.savez_compressed(
        HERE / f"{tag}.npz", kind="fp8", rms_mode=mode, cache=_bits(cache[:, :, 0, :]), q=_bits(q),
        block_table=bt.numpy(), seq_lens=lens.numpy(), out=out.numpy().astype(np.float32),
        k_scale=np.float32(scale.item()), rank=rank, rope=rope, heads=heads, page=page,
        rms_offset=rank + rope, sm_scale=np.float32(1.0 / 16.0), source="tests/test_fp8_kv.py:34-76")
    print(f"{tag}: cache {tuple(cache.shape)} scale {scale.item():.4g}")


def numerics_case(tag, rank, heads, ctx, batch, page=16, packed_rope=256):
    """tests/test_decode_numerics.py `reference` (exact per-head loop, rms clamp 1e-6)."""
    src = (REF / "tests" / "test_decode_numerics.py").read_text()
    tree = ast.parse(src)
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "reference")
    ns = {"torch": torch, "PAGE": page, "PACKED_ROPE": packed_rope}
    exec(compile(ast.Module(body=[fn], type_ignores=[]), "test_decode_numerics.py", "exec"), ns)
    # inputs: the recipe of the file's case() (seeded; contiguous page table, full lengths)
    torch.manual_seed(rank + heads)
    entry = rank + packed_rope + heads
    ppq = (ctx + page - 1) // page
    kv = torch.randn(batch * ppq + 4, page, 1, entry, dtype=torch.bfloat16) * 0.05
    kv[..., rank + packed_rope:] = kv[..., rank + packed_rope:].abs() + 0.3
    bt = torch.arange(batch * ppq, dtype=torch.int32).reshape(batch, ppq)
    sl = torch.full((batch,), ctx, dtype=torch.int32)
    q = torch.randn(batch, heads, rank + packed_rope, dtype=torch.bfloat16) * 0.05
    out = ns["reference"](q, kv, bt, sl, rank, heads, 1.0 / (256 ** 0.5))
    np.savez_compressed(
        HERE / f"{tag}.npz", kind="bf16", cache=_bits(kv[:, :, 0, :]), q=_bits(q), block_table=bt.numpy(),
        seq_lens=sl.numpy(), out=out.numpy().astype(np.float32), rank=rank, rope=packed_rope, heads=heads,
        page=page, rms_offset=rank + packed_rope, sm_scale=np.float32(1.0 / 16.0),
        source="tests/test_decode_numerics.py:25-44")
    print(f"{tag}: cache {tuple(kv.shape)}")


def cache_write_case(tag, mode, n=40, rank=256, packed_rope=232, heads=24, blocks=4, block=16):
    """The FP8 row writer, called on a stand-in `self` carrying the layout attributes."""
    sys.path.insert(0, str(REF))
    os.environ["QWEN_MLA_FP8_RMS"] = mode
    from qwen_mla.mla_impl import QwenMLATritonImpl
    fake = types.SimpleNamespace(rms_offset=rank + packed_rope, mla_packed_rope=packed_rope,
                                 mla_local_heads=heads)
    g = torch.Generator().manual_seed(11 if mode == "log8" else 12)
    kv_c = (torch.randn(n + 3, rank, generator=g) * 2.0).to(torch.bfloat16)   # 3 graph-padding rows
    k_pe = torch.empty(n + 3, packed_rope + heads)
    k_pe[:, :packed_rope] = torch.randn(n + 3, packed_rope, generator=g) * 1.5
    k_pe[:, packed_rope:] = torch.exp(torch.randn(n + 3, heads, generator=g) * 0.9)
    k_pe = k_pe.to(torch.bfloat16)
    width = rank + packed_rope + (2 if mode == "bf16" else 1) * heads
    width += (-width) % 16
    slots = torch.randperm(blocks * block - 1, generator=g)[:n] + 1     # slot 0 is left to the padding row
    slots[7] = -1
    cache = torch.zeros(blocks, block, 1, width, dtype=torch.uint8).view(torch.float8_e4m3fn)
    scale = torch.tensor(float(kv_c.float().abs().max()) / 448)
    QwenMLATritonImpl.do_kv_cache_update(fake, kv_c, k_pe, cache, slots, "fp8", scale)
    np.savez_compressed(
        HERE / f"{tag}.npz", rms_mode=mode, latent=_bits(kv_c), k_pe=_bits(k_pe), slots=slots.numpy(),
        k_scale=np.float32(scale.item()), cache=_bits(cache[:, :, 0, :]), rank=rank,
        packed_rope=packed_rope, heads=heads, source="qwen_mla/mla_impl.py:309-342")
    print(f"{tag}: {n} tokens, width {width}")


def gather_case(tag, mode, dst_dtype=torch.bfloat16, rank=256, rope=232, heads=24, page=16):
    """qwen_mla/ops/mla_gather.py:28-76 on a chunk of three sequences (one empty) with
    seq_starts, pages in random order, and sentinel-filled destination rows / columns."""
    sys.path.insert(0, str(REF))
    from qwen_mla.ops.mla_gather import gather_cache_torch
    batch, ctx = 3, 100
    g = torch.Generator().manual_seed({"auto": 21, "log8": 22, "bf16": 23, "e4m3": 24}[mode])
    if mode == "auto":
        pps = (ctx + page - 1) // page
        width = rank + rope + heads
        cache = (torch.randn(batch * pps, page, 1, width, generator=g) * 1.5).to(torch.bfloat16)
        scale = torch.tensor(1.0)
        mla_rms = None
    else:
        m = _load(REF / "tests" / "test_fp8_kv.py", "ref_fp8_kv")
        m.PAGE, m.dev = page, torch.device("cpu")
        lat, rp, rms, _, pps = m.make(batch, heads, ctx, rank, rope, seed=rank + heads)
        scale = torch.tensor(float(max(lat.abs().max(), rp.abs().max())) / 448)
        width = rank + rope + (2 if mode == "bf16" else 1) * heads
        width += (-width) % 16
        cache = m.fp8_cache(lat, rp, rms, scale, width, mode)
        mla_rms = (rank + rope, heads, mode)
    bt = torch.randperm(batch * pps, generator=g).reshape(batch, pps).to(torch.int32)
    chunk = torch.tensor([40, 0, 57])
    starts = torch.tensor([5, 0, 23], dtype=torch.int32)
    cu = torch.zeros(batch + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(chunk, 0)
    t2s = torch.repeat_interleave(torch.arange(batch, dtype=torch.int32), chunk)
    n = int(chunk.sum())
    dst = torch.full((n + 3, cache.shape[-1] if mode == "auto" else width), 7.0, dtype=dst_dtype)
    gather_cache_torch(src_cache=cache, dst=dst, block_table=bt, cu_seq_lens=cu, token_to_seq=t2s,
                       num_tokens=n, kv_cache_dtype="auto" if mode == "auto" else "fp8", scale=scale,
                       seq_starts=starts, mla_rms=mla_rms)
    np.savez_compressed(
        HERE / f"{tag}.npz", mode=mode, cache=_bits(cache[:, :, 0, :]), block_table=bt.numpy(),
        cu_seq_lens=cu.numpy(), token_to_seq=t2s.numpy(), seq_starts=starts.numpy(), num_tokens=n,
        scale=np.float32(scale.item()), rms_offset=rank + rope, heads=heads,
        dst_dtype=str(dst_dtype).replace("torch.", ""), dst=_bits(dst) if dst_dtype == torch.bfloat16
        else dst.contiguous().view(torch.int16).numpy().view(np.uint16),
        source="qwen_mla/ops/mla_gather.py:28-76")
    print(f"{tag}: {n} rows, width {dst.shape[1]}")


def rank_plan_case(tag, page=16):
    """fi_decode._RankPlan.plan_cpu on a stand-in object whose flashinfer wrapper records its inputs."""
    sys.path.insert(0, str(REF))
    from qwen_mla.fi_decode import _RankPlan
    seen = {}

    class Rec:
        def plan(self, qo, indptr, indices, lens, *rest):
            seen.update(qo=qo.clone(), indptr=indptr.clone(), indices=indices.clone(), lens=lens.clone())

    maxb, maxp = 8, 256
    p = object.__new__(_RankPlan)
    p.rank, p.win, p.n_local, p.kpe, p.page_size = 768, 232, 24, 256, page
    p.kv_len = torch.zeros(maxb, dtype=torch.int32)
    p.max_pages = maxp
    p._ring = [dict(qo=torch.arange(maxb + 1, dtype=torch.int32), indptr=torch.zeros(maxb + 1, dtype=torch.int32),
                    lens=torch.zeros(maxb, dtype=torch.int32), rows=torch.zeros(maxp, dtype=torch.int64),
                    cols=torch.zeros(maxp, dtype=torch.int64)) for _ in range(4)]
    p._ring_i = 0
    p.w = Rec()
    lens = torch.tensor([0, 1, 16, 17, 1000, 64], dtype=torch.int32)
    g = torch.Generator().manual_seed(5)
    bt = torch.randint(0, 4096, (6, 70), generator=g, dtype=torch.int32)
    p.plan_cpu(bt, lens, lens, 1.0 / 16, torch.bfloat16, torch.bfloat16)
    B = len(lens)
    total = int(seen["indptr"][B])
    np.savez_compressed(
        HERE / f"{tag}.npz", block_table=bt.numpy(), seq_lens=lens.numpy(), page=page,
        qo_indptr=seen["qo"][:B + 1].numpy(), kv_indptr=seen["indptr"][:B + 1].numpy(),
        kv_indices=seen["indices"][:total].numpy(), kv_len=seen["lens"][:B].numpy(),
        source="qwen_mla/fi_decode.py:235-270")
    print(f"{tag}: {total} pages")


def build_decode_case(tag, qd=4, width=70):
    """MLATritonMetadataBuilder._build_decode (qwen_mla/mla_impl.py:628-662), run unmodified on a
    stand-in builder: MTP verify rows flattened to one row per draft.  Its vLLM parent step
    (super()._build_decode) is replaced for the call by a stub that returns the metadata object
    holding the request-level block table and lengths, which the method then flattens."""
    sys.path.insert(0, str(REF))
    from qwen_mla.mla_impl import MLATritonMetadataBuilder as B
    parent = next(c for c in B.__mro__[1:] if "_build_decode" in c.__dict__)
    saved = parent.__dict__["_build_decode"]
    parent._build_decode = lambda self, bt, sl, *a: types.SimpleNamespace(block_table=bt, seq_lens=sl)
    try:
        b = object.__new__(B)
        b.vllm_config = types.SimpleNamespace(scheduler_config=types.SimpleNamespace(max_num_seqs=16))
        b.reorder_batch_threshold = qd
        g = torch.Generator().manual_seed(11)
        n = 7
        bt = torch.randint(0, 5000, (n, width), generator=g, dtype=torch.int32)
        # lengths with drafts that clamp at 0 (CUDA-graph padding rows have length 0)
        sl = torch.tensor([0, 1, 2, 3, 4, 129, 8192], dtype=torch.int32)
        md = B._build_decode(b, bt, sl, int(sl.max()), None, None, n * qd, None)
        q = int(getattr(md, "_mla_q"))
        np.savez_compressed(HERE / f"{tag}.npz", block_table=bt.numpy(), seq_lens=sl.numpy(), qrows=q,
                            flat_block_table=md.block_table.numpy(), flat_seq_lens=md.seq_lens.numpy(),
                            source="qwen_mla/mla_impl.py:628-662")
        print(f"{tag}: {n} requests x {q} drafts -> {md.block_table.shape[0]} rows")
    finally:
        parent._build_decode = saved


CASES = {
    "bf16_tp1_r768": lambda t: partial_rope_case(t, batch=2, heads=24, ctx=100, rank=768, rope=232),
    "bf16_tp1_r256": lambda t: partial_rope_case(t, batch=2, heads=24, ctx=200, rank=256, rope=232),
    "bf16_tp2_r384": lambda t: partial_rope_case(t, batch=2, heads=12, ctx=150, rank=384, rope=116),
    "fp8_log8_r256": lambda t: fp8_case(t, batch=2, heads=24, ctx=150, rank=256, rope=232, mode="log8"),
    "fp8_bf16_r256": lambda t: fp8_case(t, batch=2, heads=24, ctx=150, rank=256, rope=232, mode="bf16"),
    "fp8_e4m3_r256": lambda t: fp8_case(t, batch=2, heads=24, ctx=150, rank=256, rope=232, mode="e4m3"),
    "fp8_log8_r768": lambda t: fp8_case(t, batch=2, heads=24, ctx=100, rank=768, rope=232, mode="log8"),
    "fp8_log8_tp2_r384": lambda t: fp8_case(t, batch=2, heads=12, ctx=130, rank=384, rope=116, mode="log8"),
    "numerics_r256_h24": lambda t: numerics_case(t, rank=256, heads=24, ctx=100, batch=2),
    # rank 1792, the reference's widest latent (tests/test_two_pass_1792.py: 24 heads | rope 232 and
    # 12 heads | rope 116; tests/test_fp8_kv.py:137 covers FP8 at rank 1792)
    "bf16_tp1_r1792": lambda t: partial_rope_case(t, batch=2, heads=24, ctx=90, rank=1792, rope=232),
    "bf16_tp2_r1792": lambda t: partial_rope_case(t, batch=2, heads=12, ctx=90, rank=1792, rope=116),
    "fp8_log8_r1792": lambda t: fp8_case(t, batch=2, heads=24, ctx=90, rank=1792, rope=232, mode="log8"),
    "cache_write_log8": lambda t: cache_write_case(t, "log8"),
    "cache_write_bf16": lambda t: cache_write_case(t, "bf16"),
    "rank_plan": lambda t: rank_plan_case(t),
    "mtp_build_decode": lambda t: build_decode_case(t),
    "gather_auto": lambda t: gather_case(t, "auto"),
    "gather_log8": lambda t: gather_case(t, "log8"),
    "gather_log8_f16": lambda t: gather_case(t, "log8", dst_dtype=torch.float16),
    "gather_bf16": lambda t: gather_case(t, "bf16"),
    "gather_e4m3": lambda t: gather_case(t, "e4m3"),
}


def main():
    """Writes every fixture, or only those whose names start with one of the arguments."""
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for tag, make in CASES.items():
        if len(sys.argv) == 1 or any(tag.startswith(a) for a in sys.argv[1:]):
            make(tag)


if __name__ == "__main__":
    main()
