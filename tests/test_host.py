"""Host-side logic of the Python entry points (no GPU needed)."""
from __future__ import annotations

import pytest
import torch

from qwen_mla_vllm_b200 import _lib
from qwen_mla_vllm_b200 import mla_decode_attention as mda


def test_rms_mode_mapping_follows_reference_flags():
    f8 = torch.float8_e4m3fn
    assert mda.rms_mode_for(torch.bfloat16, -1, False, False) == _lib.RMS_NONE
    assert mda.rms_mode_for(torch.bfloat16, 1000, False, False) == _lib.RMS_NATIVE
    assert mda.rms_mode_for(f8, 1000, False, True) == _lib.RMS_LOG8
    assert mda.rms_mode_for(f8, 1000, True, False) == _lib.RMS_BF16
    assert mda.rms_mode_for(f8, 1000, False, False) == _lib.RMS_NATIVE
    assert mda.rms_mode_for(torch.uint8, 1000, False, True) == _lib.RMS_LOG8


def test_page_stride_reads_real_strides():
    base = torch.zeros(10, 16, 1, 1024, dtype=torch.bfloat16)
    assert mda._page_stride(base, 16) == 16 * 1024
    # cross-layer view with a gap between pages
    big = torch.zeros(10, 2, 16, 1, 1024, dtype=torch.bfloat16)
    view = big[:, 0]
    assert mda._page_stride(view, 16) == 2 * 16 * 1024
    flat = torch.zeros(160, 1, 512, dtype=torch.bfloat16)
    assert mda._page_stride(flat, 16) == 16 * 512


def test_build_params_requires_cuda_tensors():
    q = torch.zeros(2, 24, 1000, dtype=torch.bfloat16)
    kv = torch.zeros(4, 16, 1, 1024, dtype=torch.bfloat16)
    o = torch.zeros(2, 24, 768, dtype=torch.bfloat16)
    bt = torch.zeros(2, 2, dtype=torch.int32)
    sl = torch.zeros(2, dtype=torch.int32)
    with pytest.raises(ValueError, match="CUDA"):
        mda.build_params(q, kv, o, None, bt, sl, rank=768, qk_dim=1000, rms_offset=1000,
                         rms_mode=_lib.RMS_NATIVE, page_size=16, sm_scale=1 / 16)


def test_decode_attention_fwd_rejects_mha_and_split_mismatch():
    q = torch.zeros(2, 4, 64)
    kv = torch.zeros(4, 16, 4, 64)
    logits = torch.zeros(2, 4, 8, 65)
    with pytest.raises(AssertionError):
        mda.decode_attention_fwd(q, kv, kv, None, None, None, None, logits, 4, 1.0)
    with pytest.raises(NotImplementedError):
        mda.decode_attention_fwd(q, kv, kv, None, None, None, None, logits, 8, 1.0)


def test_error_type_carries_code():
    e = _lib.QmlaError("qmla_mla_decode", -4)
    assert e.code == -4 and "workspace" in str(e)
    with pytest.raises(_lib.QmlaError):
        _lib.check("x", -2)
