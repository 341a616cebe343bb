"""Host-side behaviour of the context-gather entry point that needs no GPU: the reference's
NotImplementedError cases and the empty-chunk no-op (qwen_mla/ops/mla_gather.py:33-39)."""
from __future__ import annotations

import pytest
import torch

from qwen_mla_vllm_b200.mla_gather import gather_cache_torch


def _args(**kw):
    base = dict(src_cache=torch.zeros(2, 16, 1, 64, dtype=torch.uint8), dst=torch.zeros(4, 64),
                block_table=torch.zeros(1, 2, dtype=torch.int32), cu_seq_lens=torch.tensor([0, 4]),
                token_to_seq=torch.zeros(4, dtype=torch.int32), num_tokens=4, kv_cache_dtype="fp8",
                scale=torch.tensor(1.0), mla_rms=(40, 8, "log8"))
    base.update(kw)
    return base


def test_unknown_cache_dtype_raises():
    with pytest.raises(NotImplementedError):
        gather_cache_torch(**_args(kv_cache_dtype="int8"))


def test_fp8_without_row_layout_raises():
    with pytest.raises(NotImplementedError):
        gather_cache_torch(**_args(mla_rms=None))


@pytest.mark.parametrize("dt", ["fp8", "auto"])
def test_empty_chunk_is_a_no_op(dt):
    a = _args(num_tokens=0, kv_cache_dtype=dt)
    a["dst"].fill_(3.0)
    gather_cache_torch(**a)   # returns before touching the device
    assert bool((a["dst"] == 3.0).all())


def test_host_tensors_are_refused():
    with pytest.raises(ValueError):
        gather_cache_torch(**_args())
