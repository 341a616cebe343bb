"""Host logic of bench.py that the GPU runs rely on: the BASELINE workloads (lengths, bytes,
flops) and the DCP shards cut from one global cache (contiguous and token-interleaved, MTP rows
included), checked on CPU tensors."""
from __future__ import annotations

import pytest
import torch

import bench


def test_workload_sums_match_the_contract():
    W = bench.workloads()
    assert sum(W["cfg1"].lens) == 1_192_927 and len(W["cfg1"].lens) == 64
    assert min(W["cfg1"].lens) >= 1024 and max(W["cfg1"].lens) <= 32768
    assert sum(W["cfg3"].lens) == 2_280_724 and len(W["cfg3"].lens) == 64
    assert W["cfg1"].width == 1024 and W["cfg1"].row_read == 2048
    assert W["cfg2"].width == 1024 and W["cfg2"].row_read == 1024
    assert W["cfg3"].width == 512 and W["cfg3"].row_read == 1024
    # algorithmic bytes per call (cache rows once per request + page table + q + o + lse)
    assert abs(W["cfg1"].algorithmic_bytes() / 1e9 - 2.4489) < 1e-3
    # config 2: 1.0737 GB of rows (read once per request) + 43.5 MB of q and o for 512 rows
    assert abs(W["cfg2"].algorithmic_bytes() / 1e9 - 1.1175) < 1e-3
    assert abs(W["cfg4"].algorithmic_bytes() / 1e9 - 2.1486) < 1e-3
    # config 2: 4 causal drafts see L-3 .. L tokens; flops use the exact row lengths
    assert W["cfg2"].row_lens([8192]) == [8189, 8190, 8191, 8192]
    assert abs(W["cfg2"].flops() / 1e11 - 3.56) < 0.01


@pytest.mark.parametrize("interleave", [0, 16, 1])
@pytest.mark.parametrize("world", [2, 4])
def test_dcp_shards_partition_the_global_cache(world, interleave):
    """Every token of the global cache lands in exactly one rank's shard, in order, with the
    right per-row local lengths (MTP rows: the rank's tokens below the row's global length)."""
    w = bench.Workload("t", "test", fp8=False, heads=4, rank=128, rope=16, lens=[37, 1, 0, 200, 64], qrows=3,
                       seed=5)
    dev = torch.device("cpu")
    full = bench.build_case(w, dev)
    page = w.page
    seen = {b: [] for b in range(len(w.lens))}
    for r in range(world):
        sh = bench.shard_case(w, full, world, r, dev, interleave)
        for b, L in enumerate(w.lens):
            toks = bench.shard_tokens(L, world, r, interleave)
            assert sh.lens[b] == len(toks)
            for j, t in enumerate(toks.tolist()):
                got = sh.cache[sh.bt[b, j // page], j % page, 0]
                want = full.cache[full.bt[b, t // page], t % page, 0]
                assert torch.equal(got, want)
            seen[b] += toks.tolist()
            for jq in range(w.qrows):
                Lj = max(L - (w.qrows - 1 - jq), 0)
                assert int(sh.sl_rows[b * w.qrows + jq]) == int((toks < Lj).sum())
        assert torch.equal(sh.q, full.q)
    for b, L in enumerate(w.lens):
        assert sorted(seen[b]) == list(range(L))


def test_cpu_reference_path_runs_on_a_case():
    """The CPU path the reference arm times, on a small CPU-built case (all rows, MTP drafts)."""
    w = bench.Workload("t", "test", fp8=False, heads=4, rank=128, rope=16, lens=[37, 300], qrows=2, seed=6)
    c = bench.build_case(w, torch.device("cpu"))
    o, lse, dt, nbytes = bench.cpu_decode(w, c, list(range(4)))
    assert o.shape == (4, 4, 128) and lse.shape == (4, 4)
    assert torch.isfinite(o).all() and nbytes == (36 + 37 + 299 + 300) * w.row_read
