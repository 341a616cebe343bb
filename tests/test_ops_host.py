"""The torch.library ops without a GPU: they register with the schemas that declare which
arguments they write, and under fake tensors (what torch.compile traces with) they run their
fake kernels and never reach the library."""
from __future__ import annotations

import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import qwen_mla_vllm_b200.ops  # noqa: F401  (registers torch.ops.qmla.*)


def _written(op) -> set[str]:
    return {a.name for a in op.default._schema.arguments if a.alias_info is not None and a.alias_info.is_write}


def test_schemas_declare_the_written_arguments():
    assert _written(torch.ops.qmla.mla_decode) == {"o", "lse"}
    assert _written(torch.ops.qmla.gather_cache) == {"dst"}
    for op in (torch.ops.qmla.mla_decode, torch.ops.qmla.gather_cache):
        assert len(op.default._schema.returns) == 0
    args = {a.name: str(a.type) for a in torch.ops.qmla.mla_decode.default._schema.arguments}
    assert args["k_scale"] == "Optional[Tensor]" and args["sm_scale"] == "float"


def test_fake_kernels_trace_without_the_library():
    with FakeTensorMode():
        dev = "cuda"
        q = torch.empty(4, 24, 1000, dtype=torch.bfloat16, device=dev)
        kv = torch.empty(64, 16, 1, 1024, dtype=torch.bfloat16, device=dev)
        o = torch.empty(4, 24, 768, dtype=torch.bfloat16, device=dev)
        lse = torch.empty(4, 24, dtype=torch.float32, device=dev)
        bt = torch.empty(4, 16, dtype=torch.int32, device=dev)
        sl = torch.empty(4, dtype=torch.int32, device=dev)
        ws = torch.empty(1 << 20, dtype=torch.uint8, device=dev)
        torch.ops.qmla.mla_decode(q, kv, o, lse, bt, sl, ws, 768, 1000, 1000, 1, 16, 1 / 16, 0.0, None, 1)
        src = torch.empty(64, 16, 1, 1024, dtype=torch.uint8, device=dev)
        dst = torch.empty(100, 1024, dtype=torch.bfloat16, device=dev)
        cu = torch.empty(2, dtype=torch.int32, device=dev)
        t2s = torch.empty(100, dtype=torch.int32, device=dev)
        sc = torch.empty((), dtype=torch.float32, device=dev)
        torch.ops.qmla.gather_cache(src, dst, bt, cu, t2s, 100, "fp8", sc, None, 1000, 24, "log8")
        assert o.shape == (4, 24, 768) and dst.shape == (100, 1024)
