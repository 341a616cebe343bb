"""Shared test setup: the `gpu` marker, golden-fixture loading and CUDA gating."""
from __future__ import annotations

import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz", allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


DECODE_FIXTURES = ["bf16_tp1_r768", "bf16_tp1_r256", "bf16_tp2_r384", "numerics_r256_h24",
                   "fp8_log8_r256", "fp8_bf16_r256", "fp8_e4m3_r256", "fp8_log8_r768",
                   "fp8_log8_tp2_r384", "bf16_tp1_r1792", "bf16_tp2_r1792", "fp8_log8_r1792"]


GATHER_FIXTURES = ["gather_auto", "gather_log8", "gather_log8_f16", "gather_bf16", "gather_e4m3"]


import oracle  # noqa: E402  (the checker; ROOT is on sys.path from here on)


def to_dst_bits(x: np.ndarray, dst_dtype: str) -> np.ndarray:
    """float32 values -> bit patterns (uint16) of the destination dtype, round to nearest even."""
    if dst_dtype == "bfloat16":
        return oracle.f32_to_bf16_bits(x)
    return np.asarray(x, np.float32).astype(np.float16).view(np.uint16)


def gather_expected(g: dict) -> np.ndarray:
    """The destination (bit patterns) the oracle's gather writes over a 7.0-filled buffer."""
    mode = str(g["mode"])
    fp8 = mode != "auto"
    vals = oracle.gather_cache(g["cache"], g["block_table"], g["cu_seq_lens"], g["token_to_seq"],
                               int(g["num_tokens"]), fp8=fp8, scale=float(g["scale"]),
                               seq_starts=g["seq_starts"],
                               mla_rms=(int(g["rms_offset"]), int(g["heads"]), mode) if fp8 else None)
    dt = str(g["dst_dtype"])
    out = np.full(g["dst"].shape, to_dst_bits(np.float32(7.0), dt), dtype=np.uint16)
    out[:vals.shape[0], :vals.shape[1]] = to_dst_bits(vals, dt)
    return out


def oracle_args(g: dict) -> dict:
    """Keyword arguments of oracle.decode for a decode fixture."""
    fp8 = str(g["kind"]) == "fp8"
    mode = str(g["rms_mode"]) if fp8 else "native"
    if fp8 and mode == "e4m3":
        mode = "native"
    return dict(rank=int(g["rank"]), qk_dim=int(g["rms_offset"]), page_size=int(g["page"]),
                sm_scale=float(g["sm_scale"]), rms_offset=int(g["rms_offset"]), rms_mode=mode,
                kv_fp8=fp8, k_scale=float(g["k_scale"]) if fp8 else 1.0)


@pytest.fixture(scope="session")
def cuda_device():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.skip(f"needs sm_100 (B200), found sm_{major}{minor}")
    return torch.device("cuda:0")
