"""numpy restatement of the reference's paged MLA decode path (oracle; test infrastructure only).

Reference: sootaugur/qwen-mla-vllm.  Each function names the reference lines it follows.
Caches are passed as raw element arrays: bf16 caches as uint16 bit patterns, FP8 caches
as uint8 bytes, shape [pages, page_size, width] (a singleton KV-head dim is squeezed by
the caller).  Queries are float32 arrays holding bf16 values.
"""
from __future__ import annotations

import numpy as np

from .numerics import bf16_bits_to_f32, bf16_round, e4m3_decode, e4m3_encode, f32_to_bf16_bits, \
    log8_decode, log8_encode

TILE = 128  # tokens per work unit of the sm_100a kernel's partition (this build's own plan)


def _rms_values(rows: np.ndarray, heads: int, rms_offset: int, mode: str, kv_fp8: bool,
                k_scale: float) -> np.ndarray:
    """Per-(token, head) score divisor [L, H] read from the row tail.

    qwen_mla/ops/mla_decode_attention.py:464-508: log8 code (FP8 rows), raw bf16 bytes
    (FP8 rows, rms_bf16), e4m3 x k_scale (FP8 rows otherwise), or the bf16 element itself.
    """
    if mode == "log8":
        return log8_decode(rows[:, rms_offset:rms_offset + heads])
    if mode == "bf16":
        b = rows[:, rms_offset:rms_offset + 2 * heads].astype(np.uint16)
        return bf16_bits_to_f32(b[:, 0::2] | (b[:, 1::2] << 8))
    if kv_fp8:
        return e4m3_decode(rows[:, rms_offset:rms_offset + heads]) * np.float32(k_scale)
    return bf16_bits_to_f32(rows[:, rms_offset:rms_offset + heads])


def decode(q: np.ndarray, cache: np.ndarray, block_table: np.ndarray, seq_lens: np.ndarray, *,
           rank: int, qk_dim: int, page_size: int, sm_scale: float, rms_offset: int = -1,
           rms_mode: str = "native", kv_fp8: bool = False, k_scale: float = 1.0,
           logit_cap: float = 0.0, dequant_to_bf16: bool = True,
           chunk: int = 65536) -> tuple[np.ndarray, np.ndarray]:
    """Paged latent decode: returns (o [rows, H, rank], lse [rows, H]) in float64.

    Follows the Triton kernel's order (qwen_mla/ops/mla_decode_attention.py:440-586 for one
    split, merged as in :1064-1137):
      K = cache row[:qk_dim]   (FP8: e4m3 * k_scale rounded to bf16, :451-452)
      s = q[:qk_dim] . K / rms(token, head)   (rms <= 0 -> 1, :508)
      s *= sm_scale; s = cap * tanh(s / cap) when logit_cap > 0 (:510-513)
      o = softmax(s) . K[:rank]  (MLA: V is the latent part of the same row, :548-551)
      lse = max + ln(sum exp)    (natural log, :1133)
    dequant_to_bf16=False keeps the FP8 dequantised keys in float32, as the reference's FP8
    test reference does (tests/test_fp8_kv.py:56-58, 61-72).
    rms_mode: "none" | "native" | "bf16" | "log8".  Rows with length <= 0 give o = 0 and
    lse = -inf (the reference divides 0 by 0 there; this build defines them as empty).
    Rows longer than ``chunk`` tokens are processed ``chunk`` tokens at a time with a running
    max, sum and weighted sum in float64 (the split-K merge of :1064-1137 with equal splits), so a
    262,144-token row needs a few hundred MB, not gigabytes.
    """
    rows_n, H = q.shape[0], q.shape[1]
    o = np.zeros((rows_n, H, rank), dtype=np.float64)
    lse = np.full((rows_n, H), -np.inf, dtype=np.float64)
    ks = np.float32(k_scale)
    bt_all = np.asarray(block_table)
    for r in range(rows_n):
        L = int(seq_lens[r])
        if L <= 0:
            continue
        qr = q[r, :, :qk_dim].astype(np.float64)
        m_run = np.full((H, 1), -np.inf)
        den = np.zeros((H, 1))
        acc = np.zeros((H, rank))
        for t0 in range(0, L, max(1, int(chunk))):
            t = np.arange(t0, min(L, t0 + int(chunk)))
            pages = bt_all[r][t // page_size].astype(np.int64)
            rows = cache[pages, t % page_size]  # [n, W]
            if kv_fp8:
                K = e4m3_decode(rows[:, :qk_dim]) * ks
                if dequant_to_bf16:
                    K = bf16_round(K)
            else:
                K = bf16_bits_to_f32(rows[:, :qk_dim])
            K = K.astype(np.float64)
            s = qr @ K.T  # [H, n]
            if rms_offset >= 0 and rms_mode != "none":
                rms = _rms_values(rows, H, rms_offset, rms_mode, kv_fp8, float(ks)).astype(np.float64)
                s = s / np.where(rms > 0, rms, 1.0).T
            s = s * float(np.float32(sm_scale))
            if logit_cap > 0:
                s = logit_cap * np.tanh(s / logit_cap)
            m_new = np.maximum(m_run, s.max(axis=1, keepdims=True))
            alpha = np.exp(m_run - m_new)  # 0 on the first chunk (m_run = -inf)
            p = np.exp(s - m_new)
            den = den * alpha + p.sum(axis=1, keepdims=True)
            acc = acc * alpha + p @ K[:, :rank]
            m_run = m_new
        o[r] = acc / den
        lse[r] = (m_run + np.log(den))[:, 0]
    return o, lse


def mtp_flatten(block_table: np.ndarray, seq_lens: np.ndarray, q: int) -> tuple[np.ndarray, np.ndarray]:
    """Multi-token (speculative verify) decode as single-token rows.

    qwen_mla/mla_impl.py:628-662 (_build_decode): request i with total length L becomes q
    rows; row j attends to the first L - (q-1-j) tokens (clamped at 0) through the
    request's block-table row.
    """
    n, w = block_table.shape
    bt = np.repeat(block_table[:, None, :], q, axis=1).reshape(n * q, w)
    offs = np.arange(1 - q, 1, dtype=np.int64)
    lens = np.maximum(seq_lens.astype(np.int64)[:, None] + offs[None, :], 0).reshape(-1)
    return bt, lens.astype(np.int32)


def tile_prefix(seq_lens: np.ndarray, tile: int = TILE) -> np.ndarray:
    """Exclusive prefix of ceil(max(L, 0) / tile): the decode kernel's work list (int32)."""
    L = np.maximum(np.asarray(seq_lens, dtype=np.int64), 0)
    out = np.zeros(len(L) + 1, dtype=np.int64)
    np.cumsum((L + tile - 1) // tile, out=out[1:])
    return out.astype(np.int32)


def plan_arrays(seq_lens: np.ndarray, page_size: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """(tile_prefix, kv_indptr, kv_len) as qmla_plan returns them.

    kv_indptr / kv_len follow qwen_mla/fi_decode.py:252-257 (pages = ceil(L / page_size),
    indptr = [0, cumsum(pages)], kv_len = L); tile_prefix is tile_prefix() above.
    """
    L = np.maximum(np.asarray(seq_lens, dtype=np.int64), 0)
    indptr = np.zeros(len(L) + 1, dtype=np.int64)
    np.cumsum((L + page_size - 1) // page_size, out=indptr[1:])
    return tile_prefix(L), indptr.astype(np.int32), L.astype(np.int32)


def rank_plan_arrays(block_table: np.ndarray, seq_lens: np.ndarray, page_size: int):
    """(qo_indptr, kv_indptr, kv_indices, kv_len) of qwen_mla/fi_decode.py:235-270 (plan_cpu).

    kv_indices lists, row by row, the first ceil(L / page_size) page ids of each
    block-table row.
    """
    L = np.asarray(seq_lens, dtype=np.int64)
    B = len(L)
    pages = (L + page_size - 1) // page_size
    indptr = np.zeros(B + 1, dtype=np.int64)
    np.cumsum(pages, out=indptr[1:])
    total = int(indptr[-1]) if B else 0
    rows = np.repeat(np.arange(B), pages)
    cols = np.arange(total) - np.repeat(indptr[:-1], pages)
    flat = np.asarray(block_table)[rows, cols].astype(np.int32)
    return (np.arange(B + 1, dtype=np.int32), indptr.astype(np.int32), flat, L.astype(np.int32))


def fp8_cache_rows(latent: np.ndarray, k_pe: np.ndarray, k_scale: float, packed_rope: int,
                   heads: int, rms_mode: str) -> np.ndarray:
    """FP8 cache row bytes [latent e4m3 | rope e4m3 | rms] for each token (uint8).

    qwen_mla/mla_impl.py:309-342 (do_kv_cache_update): x * (1 / k_scale) in float32,
    clamped to +-448 and rounded to e4m3; the rms tail is the log8 code (one byte per
    head) or the raw bf16 bytes (two per head, little-endian).
    """
    inv = np.float32(1.0) / np.float32(k_scale)
    lat = e4m3_encode(np.clip(latent.astype(np.float32) * inv, -448.0, 448.0))
    rope = e4m3_encode(np.clip(k_pe[:, :packed_rope].astype(np.float32) * inv, -448.0, 448.0))
    rms_src = k_pe[:, packed_rope:packed_rope + heads].astype(np.float32)
    if rms_mode == "log8":
        rms = log8_encode(rms_src)
    elif rms_mode == "bf16":
        rms = np.ascontiguousarray(f32_to_bf16_bits(rms_src)).view(np.uint8).reshape(len(rms_src), 2 * heads)
    else:
        raise ValueError(f"rms_mode {rms_mode!r}: expected log8 or bf16")
    return np.concatenate([lat, rope, rms], axis=1)


def gather_cache(cache: np.ndarray, block_table: np.ndarray, cu_seq_lens: np.ndarray,
                 token_to_seq: np.ndarray, num_tokens: int, *, fp8: bool, scale: float = 1.0,
                 seq_starts: np.ndarray | None = None, mla_rms: tuple | None = None) -> np.ndarray:
    """Chunked-prefill context gather: the float32 values of the destination columns it writes.

    qwen_mla/ops/mla_gather.py:28-76 (gather_cache_torch).  Row j of the destination is
    token tok = j - cu_seq_lens[s] (+ seq_starts[s]) of sequence s = token_to_seq[j], read
    from page block_table[s, tok // page] at tok % page.  ``cache`` is [pages, page, width]:
    uint16 bf16 bit patterns (2-byte cache, the whole row is copied) or uint8 bytes (FP8).
    Index arithmetic :41-47; the 2-byte copy :48-50.  FP8 rows: columns [0, off) =
    e4m3 * scale in float32 (:69); the heads columns from off are the log8 code decoded
    (:70-74), the raw bf16 bytes (:75-76) or, in "e4m3" mode, e4m3 * scale like the
    latent (:66-68).  ``mla_rms`` = (off, heads[, mode]) with mode "bf16" by default
    (:58-59).  The reference's slicing into 8192-row passes (:61-65) does not change the
    values.  The caller rounds to the destination dtype.
    """
    n = int(num_tokens)
    if n <= 0:
        return np.zeros((0, 0), np.float32)
    page = cache.shape[1]
    j = np.arange(n, dtype=np.int64)
    s = np.asarray(token_to_seq, dtype=np.int64)[:n]
    tok = j - np.asarray(cu_seq_lens, dtype=np.int64)[s]
    if seq_starts is not None:
        tok = tok + np.asarray(seq_starts, dtype=np.int64)[s]
    blk = np.asarray(block_table, dtype=np.int64)[s, tok // page]
    rows = cache[blk, tok % page].reshape(n, -1)
    if not fp8:
        return bf16_bits_to_f32(rows)
    if mla_rms is None:
        raise NotImplementedError("FP8 MLA gather needs the row layout (rms offset, heads)")
    off, nh = int(mla_rms[0]), int(mla_rms[1])
    mode = mla_rms[2] if len(mla_rms) > 2 else "bf16"
    sc = np.float32(scale)
    if mode == "e4m3":
        return (e4m3_decode(rows[:, :off + nh]) * sc).astype(np.float32)
    out = np.empty((n, off + nh), np.float32)
    out[:, :off] = e4m3_decode(rows[:, :off]) * sc
    if mode == "log8":
        out[:, off:] = log8_decode(rows[:, off:off + nh])
    else:
        b = rows[:, off:off + 2 * nh].astype(np.uint16)
        out[:, off:] = bf16_bits_to_f32(b[:, 0::2] | (b[:, 1::2] << 8))
    return out


def dcp_correct(out: np.ndarray, lses: np.ndarray, cp_rank: int, is_base_e: bool = True):
    """One rank's DCP output correction: returns (out * exp(lse_rank - lse_global), lse_global).

    qwen_mla/dcp_fix.py:62-98: NaN and +inf LSEs count as -inf; an all -inf max is
    replaced by 0; outputs whose factor is exactly 0 are zeroed.
    """
    lse = np.where(np.isnan(lses) | (lses == np.inf), -np.inf, lses).astype(np.float64)
    mx = lse.max(axis=0)
    mx = np.where(mx == -np.inf, 0.0, mx)
    with np.errstate(divide="ignore"):
        if is_base_e:
            g = np.log(np.exp(lse - mx).sum(axis=0)) + mx
        else:
            g = np.log2(np.exp2(lse - mx).sum(axis=0)) + mx
    with np.errstate(invalid="ignore"):
        fin = lses[cp_rank].astype(np.float64) - g
    fin = np.where(np.isnan(fin) | (fin == np.inf), -np.inf, fin)
    factor = np.exp(fin) if is_base_e else np.exp2(fin)
    res = out.astype(np.float64) * factor[..., None]
    res = np.where((factor == 0.0)[..., None], 0.0, res)
    return res, g


def dcp_merge(parts: np.ndarray, part_lses: np.ndarray, is_base_e: bool = True):
    """Merged output of N KV shards: the sum over ranks of dcp_correct (what the reduce-scatter
    after qwen_mla/dcp_fix.py's correction computes), and the global LSE."""
    acc = None
    g = None
    for n in range(parts.shape[0]):
        c, g = dcp_correct(parts[n], part_lses, n, is_base_e)
        acc = c if acc is None else acc + c
    return acc, g
