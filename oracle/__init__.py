"""CPU oracle for the paged latent-KV MLA decode path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
package, and only as the checker or the timed CPU baseline.  The product path
(``qwen_mla_vllm_b200``) never imports it and has no CPU fallback.

The oracle is a numpy restatement of the reference plugin's own algorithm for
this path (sootaugur/qwen-mla-vllm): every function cites the reference
file:line it follows.  It is pinned against golden vectors produced by the
reference's own torch functions (``tests/golden/make_golden.py``); see
``tests/test_oracle_golden.py``.
"""
from .numerics import (bf16_bits_to_f32, bf16_round, e4m3_decode, e4m3_encode, f32_to_bf16_bits,
                       log8_decode, log8_encode)
from .decode import (TILE, dcp_correct, dcp_merge, decode, fp8_cache_rows, gather_cache,
                     mtp_flatten, plan_arrays, rank_plan_arrays, tile_prefix)

__all__ = [
    "TILE", "bf16_bits_to_f32", "bf16_round", "e4m3_decode", "e4m3_encode", "f32_to_bf16_bits",
    "log8_decode", "log8_encode", "dcp_correct", "dcp_merge", "decode", "fp8_cache_rows", "gather_cache",
    "mtp_flatten", "plan_arrays", "rank_plan_arrays", "tile_prefix",
]
