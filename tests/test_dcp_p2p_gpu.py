"""The one-kernel DCP merge over peer memory (qmla_dcp_p2p_merge) on one GPU.

The N ranks' exchange buffers are N allocations on the same device and every rank's
epoch flag is set by the host before the launches, so no launch waits for another
(each launch's wait finds its flags already there).  The merge of each rank is
compared with the oracle's DCP merge; a flag that nothing sets must end the wait
with the timeout status, not a hang.  The multi-GPU path (real peers, IPC mappings)
is in test_dcp_gpu.py."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _bufs(world, B, H, D, dev):
    from qwen_mla_vllm_b200.dcp import ExchangeBuffer
    return [ExchangeBuffer(B, H, D, dev) for _ in range(world)]


@pytest.mark.parametrize("world,mode,odt", [(1, "ar", torch.float32), (2, "rs", torch.bfloat16),
                                            (4, "ar", torch.float32), (4, "rs", torch.float16),
                                            (8, "rs", torch.bfloat16)])
def test_p2p_merge_matches_oracle(cuda_device, world, mode, odt):
    from qwen_mla_vllm_b200.dcp import p2p_merge
    B, H, D = 5, 24, 768
    rng = np.random.default_rng(world * 7 + len(mode))
    parts = rng.standard_normal((world, B, H, D)).astype(np.float32)
    lses = (rng.standard_normal((world, B, H)) * 3).astype(np.float32)
    lses[:, 0, 0] = -np.inf           # a row/head that is empty on every rank
    lses[0, 1, 2] = np.nan            # NaN / +inf partial LSEs count as -inf (dcp_fix.py:62-98)
    if world > 1:
        lses[1, 2, 3] = np.inf
    want, want_lse = oracle.dcp_merge(parts, lses)
    bufs = _bufs(world, B, H, D, cuda_device)
    epoch = 3
    try:
        for n, b in enumerate(bufs):
            o, lse = b.partial(epoch)
            o.copy_(torch.from_numpy(parts[n]))
            lse.copy_(torch.from_numpy(lses[n]))
            b.flags()[:world] = epoch  # every rank has published this epoch
        hs = H // world if mode == "rs" else H
        for r in range(world):
            out = torch.full((B, hs, D), 7.0, dtype=odt, device=cuda_device)
            lse_out = torch.empty(B, hs, dtype=torch.float32, device=cuda_device)
            p2p_merge([b.ptr for b in bufs], r, B, H, D, epoch, out, mode, lse_out, timeout_s=1.0)
            torch.cuda.synchronize()
            assert bufs[r].status() == 0
            h0 = r * hs if mode == "rs" else 0
            ref = want[:, h0:h0 + hs]
            tol = 1e-5 if odt == torch.float32 else 1e-2
            assert np.allclose(out.float().cpu().numpy(), ref, rtol=tol, atol=tol)
            ref_lse = want_lse[:, h0:h0 + hs]
            got = lse_out.cpu().numpy()
            fin = np.isfinite(ref_lse)
            assert np.array_equal(np.isfinite(got), fin)
            assert np.allclose(got[fin], ref_lse[fin], rtol=1e-5, atol=1e-5)
    finally:
        for b in bufs:
            b.free()


def test_p2p_merge_wait_times_out(cuda_device):
    """Rank 0 of 2 waits for a flag rank 1 never publishes: the kernel gives up after
    its bound, records the timeout in the status word and leaves the output alone."""
    from qwen_mla_vllm_b200.dcp import p2p_merge
    B, H, D = 2, 8, 256
    bufs = _bufs(2, B, H, D, cuda_device)
    try:
        out = torch.full((B, H // 2, D), 3.0, dtype=torch.float32, device=cuda_device)
        p2p_merge([b.ptr for b in bufs], 0, B, H, D, 7, out, "rs", timeout_s=0.05)
        torch.cuda.synchronize()
        assert bufs[0].status() == 1
        assert bool((out == 3.0).all())
        # rank 0 did publish its own epoch into rank 1's flags
        assert int(bufs[1].flags()[0].item()) == 7
    finally:
        for b in bufs:
            b.free()


def test_p2p_merge_device_epoch_and_graph_replay(cuda_device):
    """Device-epoch mode (epoch 0 at the C ABI): each merge takes the rank's last merged epoch
    + 1 from its header, reads slot epoch & 1 and advances the header, so a CUDA graph of two
    merges replays correctly.  The peers' flags are set far ahead, so no wait blocks."""
    from qwen_mla_vllm_b200.dcp import p2p_merge
    B, H, D, world = 3, 8, 256, 2
    rng = np.random.default_rng(11)
    parts = rng.standard_normal((2, world, B, H, D)).astype(np.float32)  # [slot, rank, ...]
    lses = rng.standard_normal((2, world, B, H)).astype(np.float32)
    bufs = _bufs(world, B, H, D, cuda_device)
    try:
        for n, b in enumerate(bufs):
            for slot in (0, 1):
                o, lse = b.partial(slot)
                o.copy_(torch.from_numpy(parts[slot, n]))
                lse.copy_(torch.from_numpy(lses[slot, n]))
            b.flags()[:world] = 1000
        want = [oracle.dcp_merge(parts[slot], lses[slot])[0] for slot in (0, 1)]
        out = torch.empty(B, H, D, dtype=torch.float32, device=cuda_device)
        for step in range(1, 4):  # epochs 1, 2, 3 -> slots 1, 0, 1
            p2p_merge([b.ptr for b in bufs], 0, B, H, D, 0, out, "ar", timeout_s=1.0)
            torch.cuda.synchronize()
            assert int(bufs[0].flags()[9].item()) == step      # last merged epoch
            assert int(bufs[0].flags()[10].item()) == 0        # block counter reset
            assert np.allclose(out.cpu().numpy(), want[step & 1], rtol=1e-5, atol=1e-5)
        outs = [torch.empty_like(out) for _ in range(2)]
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for k in range(2):
                    p2p_merge([b.ptr for b in bufs], 0, B, H, D, 0, outs[k], "ar", timeout_s=1.0)
        torch.cuda.current_stream().wait_stream(s)
        for rep in range(3):  # each replay merges epochs 4+2rep (slot 0) and 5+2rep (slot 1)
            outs[0].zero_()
            outs[1].zero_()
            g.replay()
            torch.cuda.synchronize()
            assert int(bufs[0].flags()[9].item()) == 5 + 2 * rep
            assert np.allclose(outs[0].cpu().numpy(), want[0], rtol=1e-5, atol=1e-5)
            assert np.allclose(outs[1].cpu().numpy(), want[1], rtol=1e-5, atol=1e-5)
        assert bufs[0].status() == 0
        del g
    finally:
        for b in bufs:
            b.free()
