#!/usr/bin/env python3
"""Generate the golden fixtures that need the reference's Triton kernels, on a CUDA machine.

    python tests/golden/make_golden_gpu.py            # writes tests/golden/dcp_correct.npz

The reference plugin must be importable: from QMLA_REFERENCE (its source tree) or, by default,
the unmodified install in baseline/_ref.  The reference function used, called unmodified:
  * qwen_mla/dcp_fix.py:101-130   _mla_correct_attn_out (the DCP output correction, a Triton
                                  kernel, with vLLM's CPTritonContext)
Inputs are seeded partial outputs and LSEs of N KV shards, with the cases the correction must
handle: NaN and +inf partial LSEs (counted as -inf), rows empty on every rank (all -inf), and
rows empty on some ranks; both base-e and base-2 LSEs; every cp_rank.  Arrays are stored raw
(float32).
"""
from __future__ import annotations

import os
import pathlib
import sys

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent.parent
REF = pathlib.Path(os.environ.get("QMLA_REFERENCE", ROOT / "baseline" / "_ref"))


def dcp_correct_case(tag: str = "dcp_correct", N: int = 4, B: int = 5, H: int = 24, D: int = 768) -> None:
    sys.path.insert(0, str(REF))
    from qwen_mla.dcp_fix import _mla_correct_attn_out
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(3)
    out = torch.randn(N, B, H, D, generator=g)
    lses = torch.randn(N, B, H, generator=g) * 4.0
    lses[:, 0, 0] = -torch.inf           # (b=0, h=0) empty on every rank
    lses[1, 1, :] = -torch.inf           # row 1 empty on rank 1
    lses[0, 2, 3] = torch.nan            # NaN and +inf partial LSEs count as -inf
    lses[2, 2, 4] = torch.inf
    lses[:, 3, 5] = torch.nan            # (b=3, h=5): NaN on every rank
    res = {}
    for base_e in (True, False):
        for r in range(N):
            o = out[r].clone().to(dev)
            o_new, lse = _mla_correct_attn_out(o, lses.to(dev), r, None, is_lse_base_on_e=base_e)
            torch.cuda.synchronize()
            key = f"{'e' if base_e else '2'}{r}"
            res[f"out_{key}"] = o_new.float().cpu().numpy()
            res[f"lse_{key}"] = lse.float().cpu().numpy()
    # every (row, head) is corrected on its own: keep the first 4 rows x 8 heads, which hold
    # every special case above, so the fixture stays small
    kb, kh = 4, 8
    res = {k: v[:kb, :kh] for k, v in res.items()}
    np.savez_compressed(HERE / f"{tag}.npz", out=out.numpy()[:, :kb, :kh], lses=lses.numpy()[:, :kb, :kh],
                        N=N, B=kb, H=kh, D=D, source="qwen_mla/dcp_fix.py:101-130", **res)
    print(f"{tag}: N={N} B={B} H={H} D={D}, {len(res)} arrays")


if __name__ == "__main__":
    dcp_correct_case()
