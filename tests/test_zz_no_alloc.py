"""qmla_mla_decode_static, the decode entry point for callers that cannot allocate device memory
(hosts that reach the library through a foreign-function layer with no device allocator, and
serving processes whose memory pool is locked at start-up).  It runs on a fixed array inside the
library instead of a caller workspace.  Checked against qmla_mla_decode on the same inputs: two
consecutive calls, bit-identical outputs, a clear status word, and the oversize refusal.  Collected
last (file name), so it also runs after every other GPU test has used the library; it passes alone
in a fresh process too."""
from __future__ import annotations

import ctypes

import pytest
import torch

from gpu_util import make_bf16_case, make_fp8_case

pytestmark = pytest.mark.gpu


def _static_call(p, device):
    from qwen_mla_vllm_b200 import _lib
    stream = torch.cuda.current_stream(device).cuda_stream
    _lib.check("qmla_mla_decode_static", _lib.load().qmla_mla_decode_static(ctypes.byref(p), ctypes.c_void_p(stream)))


def _static_status(device):
    from qwen_mla_vllm_b200 import _lib
    st = ctypes.c_int32(-1)
    stream = torch.cuda.current_stream(device).cuda_stream
    _lib.check("qmla_static_read_status",
               _lib.load().qmla_static_read_status(device.index or 0, ctypes.c_void_p(stream), ctypes.byref(st)))
    return st.value


@pytest.mark.parametrize("fp8", [False, True])
def test_static_scratch_matches_workspace_entry_point(cuda_device, fp8):
    from qwen_mla_vllm_b200.mla_decode_attention import build_params, run_params
    lens = [4100, 1, 0, 777, 2048, 65]
    if fp8:
        cache, q, bt, sl, ks = make_fp8_case(len(lens), 24, 768, 232, 16, lens, seed=77, device=cuda_device)
        kst = torch.tensor(ks, dtype=torch.float32, device=cuda_device)
        mode = 3
    else:
        cache, q, bt, sl = make_bf16_case(len(lens), 24, 768, 232, 16, lens, seed=77, device=cuda_device)
        kst, mode = None, 1

    def outputs():
        return (torch.full((len(lens), 24, 768), float("nan"), dtype=torch.bfloat16, device=cuda_device),
                torch.full((len(lens), 24), float("nan"), dtype=torch.float32, device=cuda_device))

    o_ref, l_ref = outputs()
    p = build_params(q, cache, o_ref, l_ref, bt, sl, rank=768, qk_dim=1000, rms_offset=1000, rms_mode=mode,
                     page_size=16, sm_scale=1 / 16, k_scale=kst)
    run_params(p, cuda_device)
    for _ in range(2):  # two consecutive calls: scratch state left by one call must not leak into the next
        o, l = outputs()
        ps = build_params(q, cache, o, l, bt, sl, rank=768, qk_dim=1000, rms_offset=1000, rms_mode=mode,
                          page_size=16, sm_scale=1 / 16, k_scale=kst)
        _static_call(ps, cuda_device)
        torch.cuda.synchronize()
        assert torch.equal(o, o_ref)
        assert torch.equal(l, l_ref)
        assert _static_status(cuda_device) == 0  # no device wait gave up


def test_static_scratch_rejects_oversize(cuda_device):
    """A shape whose workspace exceeds the 32 MiB array is refused on the host, before any launch."""
    from qwen_mla_vllm_b200 import _lib
    from qwen_mla_vllm_b200.mla_decode_attention import build_params
    n = 1_000_000  # 160 CTAs x 32 heads x rank 768 fp32 partials (31.5 MB) + a 4 MB row prefix
    cache, q, bt, sl = make_bf16_case(1, 32, 768, 232, 16, [64], seed=1, device=cuda_device)
    q = q.expand(n, -1, -1)
    bt = bt.expand(n, -1)
    sl = sl.expand(n).contiguous()
    o = torch.empty(1, 32, 768, dtype=torch.bfloat16, device=cuda_device).expand(n, -1, -1)
    p = build_params(q, cache, o, None, bt, sl, rank=768, qk_dim=1000, rms_offset=1000, rms_mode=1,
                     page_size=16, sm_scale=1 / 16, num_ctas=160)
    need = ctypes.c_int64()
    _lib.check("qmla_decode_workspace_bytes", _lib.load().qmla_decode_workspace_bytes(ctypes.byref(p), ctypes.byref(need)))
    assert need.value > 32 << 20
    with pytest.raises(_lib.QmlaError) as e:
        _static_call(p, cuda_device)
    assert e.value.code == -4
