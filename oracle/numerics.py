"""Bit-level number formats of the latent cache, restated in numpy (oracle; test infrastructure).

* bf16: round-to-nearest-even truncation of float32 (torch ``.to(torch.bfloat16)``).
* e4m3 (float8_e4m3fn): 1 sign, 4 exponent (bias 7), 3 mantissa bits, no infinities,
  0x7f / 0xff are NaN, max finite 448.  Encoding is round-to-nearest-even after the
  reference clamps to +-448 (``qwen_mla/mla_impl.py:328-334``,
  ``tests/test_fp8_kv.py:37-49``).
* log8 rms code: ``round((log2(max(x, 1e-30)) - LO) * 255 / (HI - LO))`` clamped to
  [0, 255] with LO, HI = -3, 3 (``qwen_mla/mla_impl.py:132, 333-336``); decoded as
  ``2^(-3 + code * 6/255)`` (``qwen_mla/ops/mla_decode_attention.py:467-476``).
"""
from __future__ import annotations

import numpy as np

RMS_LOG2_LO, RMS_LOG2_HI = -3.0, 3.0


def f32_to_bf16_bits(x) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round to nearest even; NaN stays NaN."""
    f = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = f.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        r = np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)
    return r


def bf16_bits_to_f32(b) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32 (exact)."""
    b = np.ascontiguousarray(np.asarray(b, dtype=np.uint16))
    return (b.astype(np.uint32) << 16).view(np.float32)


def bf16_round(x) -> np.ndarray:
    """Round float32 values to the nearest bf16 value (returned as float32)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def _e4m3_table() -> np.ndarray:
    v = np.zeros(256, dtype=np.float64)
    for b in range(256):
        s, e, m = b >> 7, (b >> 3) & 15, b & 7
        if e == 15 and m == 7:
            v[b] = np.nan
        elif e == 0:
            v[b] = (m / 8.0) * 2.0 ** -6
        else:
            v[b] = (1.0 + m / 8.0) * 2.0 ** (e - 7)
        if s:
            v[b] = -v[b]
    return v


_E4M3 = _e4m3_table()
_POS = _E4M3[:127]  # codes 0..126: the non-negative finite values, ascending


def e4m3_decode(b) -> np.ndarray:
    """e4m3 bytes (uint8) -> float32 values (exact)."""
    return _E4M3[np.asarray(b, dtype=np.uint8)].astype(np.float32)


def e4m3_encode(x) -> np.ndarray:
    """float32 -> e4m3 bytes: clamp to +-448, then round to nearest, ties to even code."""
    x = np.asarray(x, dtype=np.float32)
    a = np.minimum(np.abs(x.astype(np.float64)), 448.0)
    hi = np.searchsorted(_POS, a, side="left").clip(0, 126)
    lo = (hi - 1).clip(0, 126)
    dlo = np.abs(a - _POS[lo])
    dhi = np.abs(_POS[hi] - a)
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    code = np.where(np.signbit(x), code | 0x80, code).astype(np.uint8)
    return np.where(np.isnan(x), np.uint8(0x7F), code).astype(np.uint8)


def log8_encode(x) -> np.ndarray:
    """rms (float32) -> 1-byte log2 code, as the reference's FP8 cache writer computes it."""
    x = np.asarray(x, dtype=np.float32)
    lg = np.log2(np.maximum(x, np.float32(1e-30))).astype(np.float32)
    code = ((lg - np.float32(RMS_LOG2_LO)) * np.float32(255.0 / (RMS_LOG2_HI - RMS_LOG2_LO))).astype(np.float32)
    return np.clip(np.rint(code), 0, 255).astype(np.uint8)


def log8_decode(code) -> np.ndarray:
    """1-byte log2 code -> rms value 2^(-3 + code * 6/255) (float32)."""
    c = np.asarray(code, dtype=np.float32)
    return np.exp2(np.float32(-3.0) + c * np.float32(6.0 / 255.0)).astype(np.float32)
