#!/usr/bin/env python3
"""Benchmark of the sm_100a paged MLA decode: achieved HBM TB/s (and seqs/s) on BASELINE config 1.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the plugin's real row split): bf16 latent cache, batch 64,
1 query token, 24 heads, context lengths U[1024, 32768] (torch generator seed 1), 16-token
pages in random order, row = latent 768 | rope 232 | rms 24 (1024 bf16), q ~ N(0,1)/sqrt(1024),
cache ~ N(0,1), rms ~ U(0.5, 2).  Synthetic, seeded; the 2.44 GB cache is larger than L2, so
no L2 flush is needed between steps.

One step = one decode call over the whole batch.  N = 1: qmla_mla_decode on one GPU.  N > 1
(launched with torchrun, one process per GPU): decode context parallelism -- every rank holds a
contiguous 1/N slice of every sequence's KV, decodes it, and the (o, lse) partials are merged
over NCCL (all-gather of lse, the correction kernel, all-reduce of o) -- the total work is fixed
("scaling": "strong").

``--impl reference`` times the reference's algorithm on the host cores instead: the numpy
restatement in oracle/ (the reference's own CPU path is torch code that cannot travel to the GPU
box), on a bounded sample of the same workload; under torchrun only rank 0 runs.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import pathlib
import statistics
import sys
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MLA decode attn achieved HBM TB/s (% peak) and seqs/s at 1/2/4/8 B200"
B, H, RANK, ROPE, PAGE = 64, 24, 768, 232, 16
QK = RANK + ROPE  # attention width = rms offset
ROW = 1024        # elements per cache row (768 | 232 | 24)
ROW_READ = QK * 2 + H * 2  # bytes of a row the decode reads: latent + rope + rms tail
WORKLOAD = ("config1: bf16 latent paged MLA decode, B=64, 1 query token, 24 heads, "
            "row 768|232|24 bf16, L~U[1024,32768] (seed 1), 16-token pages in random order")


# --workload cfg4 (BASELINE config 4 on the decode side: FP8 e4m3 cache with log8 rms codes,
# batch 8 x 262,144 tokens, one query token) instead of the default config 1.  Not the headline
# line: it measures the DCP scaling that BASELINE states at 262k context.
FP8 = False
WORKLOAD4 = ("config4: FP8-e4m3 latent paged MLA decode, B=8 x 262144 tokens, 1 query token, 24 heads, "
             "row 768|232 e4m3 + 24 log8 rms codes, k_scale 0.01, 16-token pages in random order")


def use_cfg4() -> None:
    global FP8, B, ROW_READ, WORKLOAD
    FP8, B = True, 8
    ROW_READ = QK + H  # bytes of a row the decode reads: e4m3 latent + rope + one code per head
    WORKLOAD = WORKLOAD4


def seq_lens_cfg1() -> list[int]:
    import torch
    if FP8:
        return [262144] * B
    return torch.randint(1024, 32769, (B,), generator=torch.Generator().manual_seed(1)).tolist()


def algorithmic_bytes(lens: list[int], rows: int) -> int:
    """Cache rows read once + page table + q + o + lse (the path's unavoidable traffic)."""
    pages = sum((L + PAGE - 1) // PAGE for L in lens)
    return (sum(lens) * ROW_READ + 4 * pages + rows * H * QK * 2 + rows * H * RANK * 2 + rows * H * 4)


def measured_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:  # noqa: BLE001
        return 6650.0, "fallback"


def profile_traffic() -> float | None:
    """DRAM bytes per decode launch from the committed ncu summary of this workload."""
    p = ROOT / "profiles" / "decode_bf16_config1.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("dram_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML (read-only) in a thread."""

    NAMES = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
             0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
             0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, index: int, period_s: float = 0.005):
        self.samples: list[tuple[float, int, int]] = []
        self.period = period_s
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # noqa: BLE001
            self.max_mhz = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((time.perf_counter(), mhz, reasons))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def start(self):
        if self.ok:
            self._t.start()
        return self

    def stop(self):
        self._stop.set()
        if self.ok:
            self._t.join(timeout=2)

    def summary(self, t0: float, t1: float) -> dict:
        win = [s for s in self.samples if t0 <= s[0] <= t1]
        if not win and self.samples:  # timed region shorter than one period: nearest samples
            win = sorted(self.samples, key=lambda s: min(abs(s[0] - t0), abs(s[0] - t1)))[:3]
        if not win:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        bits = 0
        for s in win:
            bits |= s[2]
        reasons = [n for b, n in self.NAMES.items() if bits & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(s[1] for s in win), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(win)}


def make_inputs(lens: list[int], device, seed: int):
    """Cache holding exactly the given sequences (pages shuffled), q, block table, lengths."""
    import torch
    g = torch.Generator(device="cpu").manual_seed(seed)
    pages = [(L + PAGE - 1) // PAGE for L in lens]
    P = max(1, sum(pages))
    gd = torch.Generator(device=device).manual_seed(seed)
    if FP8:  # e4m3 values of N(0,1) / k_scale, then one log8 rms code per head
        cache = torch.randint(0, 256, (P, PAGE, 1, ROW), dtype=torch.uint8, device=device, generator=gd)
        cache[..., :QK] = (torch.randn(P, PAGE, 1, QK, device=device, generator=gd) * 100).clamp(-448, 448) \
            .to(torch.float8_e4m3fn).view(torch.uint8)
        cache = cache.view(torch.float8_e4m3fn)
    else:
        cache = torch.randn(P, PAGE, 1, ROW, device=device, dtype=torch.bfloat16, generator=gd)
        cache[..., QK:] = (torch.rand(P, PAGE, 1, ROW - QK, device=device, generator=gd) * 1.5 + 0.5).to(torch.bfloat16)
    perm = torch.randperm(P, generator=g)
    bt = torch.zeros(len(lens), max(1, max(pages)), dtype=torch.int32)
    off = 0
    for b, n in enumerate(pages):
        bt[b, :n] = perm[off:off + n].to(torch.int32)
        off += n
    q = (torch.randn(len(lens), H, QK, generator=g) / math.sqrt(1024)).to(torch.bfloat16)
    return cache, q, bt, torch.tensor(lens, dtype=torch.int32)


# ------------------------------------------------------------------------------ CPU reference arm
def cpu_reference_sample(lens: list[int], budget_s: float, seed: int = 1):
    """Time the oracle (numpy restatement of the reference algorithm) on whole sequences of the
    workload until ~budget_s of CPU time; returns (bytes, seconds, n_seqs, threads)."""
    import numpy as np

    import oracle
    rng = np.random.default_rng(seed)
    try:
        from threadpoolctl import threadpool_info
        threads = max([i.get("num_threads", 1) for i in threadpool_info()] + [1])
    except Exception:  # noqa: BLE001
        threads = 1
    done_bytes, spent, n = 0, 0.0, 0
    for L in lens:
        pps = (L + PAGE - 1) // PAGE
        cache = oracle.f32_to_bf16_bits(rng.standard_normal((pps, PAGE, ROW), dtype=np.float32))
        cache[..., QK:] = oracle.f32_to_bf16_bits(rng.uniform(0.5, 2.0, (pps, PAGE, ROW - QK)).astype(np.float32))
        bt = rng.permutation(pps).reshape(1, pps).astype(np.int32)
        q = oracle.bf16_round((rng.standard_normal((1, H, QK)) / 32).astype(np.float32))
        t0 = time.perf_counter()
        oracle.decode(q, cache, bt, np.array([L]), rank=RANK, qk_dim=QK, page_size=PAGE, sm_scale=1 / 16,
                      rms_offset=QK)
        spent += time.perf_counter() - t0
        done_bytes += algorithmic_bytes([L], 1)
        n += 1
        if spent >= budget_s:
            break
    return done_bytes, spent, n, threads


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    lens = seq_lens_cfg1()
    # one step = one sequence of the workload (bounded sample), cycling through the batch
    times, nbytes = [], []
    for i in range(args.warmup + args.steps):
        b, s, _, threads = cpu_reference_sample([lens[i % B]], 0.0, seed=i)
        if i >= args.warmup:
            times.append(s)
            nbytes.append(b)
    tot_s, tot_b = sum(times), sum(nbytes)
    value = tot_b / tot_s / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * tot_s / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded), host memory",
        "config": {"workload": WORKLOAD, "sample": "one whole sequence of the batch per step"},
        "cpu_baseline": {"value": value, "unit": "TB/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} sequences of config1 (one per step), numpy oracle"},
        "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------ context gather
# --workload gather: the chunked-prefill context gather (qmla_gather_cache) on one GPU.  Not the
# headline line.  A 131,072-row chunk (16 sequences x 8192 tokens) of an FP8 cache (row 768|232
# e4m3 + 24 log8 codes = 1024 B), pages in random order, into a bf16 [rows, 1024] destination.
GATHER_SEQS, GATHER_LEN = 16, 8192
GATHER_WORKLOAD = ("prefill context gather: FP8-e4m3 cache rows (768|232 e4m3 + 24 log8 codes, 1024 B) "
                   "-> bf16 [131072, 1024], 16 sequences x 8192 tokens, 16-token pages in random order")
GATHER_METRIC = "MLA prefill context gather achieved HBM GB/s (FP8 -> bf16 dequant)"
GATHER_TRAFFIC = 344.8e6  # dram__bytes of the default kernel's ncu launch (profiles/gather_fp8_log8_131k.md)


def gather_row_bytes() -> float:
    """Algorithmic bytes per destination row: the cache row read, the bf16 row written, the
    token's sequence id, and its share of one block-table entry per page."""
    return ROW + 2 * (QK + H) + 4 + 4 / PAGE


def run_gather(args) -> None:
    import torch
    if int(os.environ.get("WORLD_SIZE", "1")) != 1:
        raise SystemExit("--workload gather runs on one GPU")
    from qwen_mla_vllm_b200.mla_gather import gather_cache_torch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    seqs, L = GATHER_SEQS, GATHER_LEN
    n = seqs * L
    P = n // PAGE
    gd = torch.Generator(device=dev).manual_seed(7)
    raw = torch.randint(0, 256, (P, PAGE, 1, ROW), dtype=torch.uint8, device=dev, generator=gd)
    raw[..., :QK] = (torch.randn(P, PAGE, 1, QK, device=dev, generator=gd) * 100).clamp(-448, 448) \
        .to(torch.float8_e4m3fn).view(torch.uint8)
    cache = raw.view(torch.float8_e4m3fn)
    g = torch.Generator().manual_seed(7)
    bt_h = torch.randperm(P, generator=g).reshape(seqs, L // PAGE).to(torch.int32)
    cu_h = torch.arange(0, (seqs + 1) * L, L, dtype=torch.int32)
    t2s_h = torch.arange(seqs, dtype=torch.int32).repeat_interleave(L)
    bt, cu, t2s = bt_h.to(dev), cu_h.to(dev), t2s_h.to(dev)
    scale = torch.tensor(0.01, device=dev)
    dst = torch.empty(n, ROW, dtype=torch.bfloat16, device=dev)
    kw = dict(src_cache=cache, kv_cache_dtype="fp8", scale=scale, mla_rms=(QK, H, "log8"))

    def step(out, b, c, t):
        gather_cache_torch(dst=out, block_table=b, cu_seq_lens=c, token_to_seq=t, num_tokens=n, **kw)

    step(dst, bt, cu, t2s)
    torch.cuda.synchronize()
    t_end = time.perf_counter() + 1.0  # clock ramp
    while time.perf_counter() < t_end:
        for _ in range(20):
            step(dst, bt, cu, t2s)
        torch.cuda.synchronize()
    for _ in range(args.warmup):
        step(dst, bt, cu, t2s)
    stream = torch.cuda.current_stream(dev)
    sampler = ClockSampler(0).start()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(args.steps):
        ev[i][0].record(stream)
        step(dst, bt, cu, t2s)
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    sampler.stop()
    per = [a.elapsed_time(b) for a, b in ev]
    step_ms = statistics.mean(per)
    total = n * gather_row_bytes()
    gbs = total / (step_ms * 1e-3) / 1e9
    peak, peak_kind = measured_peak()

    # end to end: the step's index tables from pinned host memory in, the destination out
    bt_p, cu_p, t2s_p = bt_h.pin_memory(), cu_h.pin_memory(), t2s_h.pin_memory()
    dst_h = torch.empty(n, ROW, dtype=torch.bfloat16).pin_memory()
    bt_d, cu_d, t2s_d = torch.empty_like(bt), torch.empty_like(cu), torch.empty_like(t2s)

    def e2e_step():
        bt_d.copy_(bt_p, non_blocking=True)
        cu_d.copy_(cu_p, non_blocking=True)
        t2s_d.copy_(t2s_p, non_blocking=True)
        step(dst, bt_d, cu_d, t2s_d)
        dst_h.copy_(dst, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    h2d = bt_h.numel() * 4 + cu_h.numel() * 4 + t2s_h.numel() * 4
    d2h = dst_h.numel() * 2

    cpu = None
    if not args.no_cpu_baseline:  # the oracle's gather on a bounded sample of the same chunk
        import oracle
        sample = min(n, 16384)
        rows_np = raw[:, :, 0, :].cpu().numpy()
        bt_np, cu_np, t2s_np = bt_h.numpy(), cu_h.numpy(), t2s_h.numpy()
        reps, spent = 0, 0.0
        while spent < args.cpu_budget:
            c0 = time.perf_counter()
            vals = oracle.gather_cache(rows_np, bt_np, cu_np, t2s_np, sample, fp8=True, scale=0.01,
                                       mla_rms=(QK, H, "log8"))
            oracle.f32_to_bf16_bits(vals)
            spent += time.perf_counter() - c0
            reps += 1
        cpu = {"value": reps * sample * gather_row_bytes() / spent / 1e9, "unit": "GB/s", "cores": 1,
               "kind": "port", "sample": f"{reps} x the first {sample} rows of the chunk, numpy oracle "
                                         f"(gather + bf16 rounding), {spent:.1f} s"}
    clocks = sampler.summary(t0, t1)
    line = {
        "metric": GATHER_METRIC, "value": gbs, "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp8-e4m3->bf16", "data": "synthetic (seeded)",
        "config": {"workload": GATHER_WORKLOAD, "rows": n, "row_bytes_read": ROW, "dst_bytes_per_row": 2 * ROW,
                   "l2": f"inputs larger than L2 ({n * gather_row_bytes() / 1e6:.0f} MB moved per step), no flush"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                     "traffic": GATHER_TRAFFIC,
                     "traffic_note": "dram bytes of one cold ncu launch (profiles/gather_fp8_log8_131k.md); "
                                     "part of the cache was still in L2 and part of the writes still dirty",
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "kernel": "gather_bulk_kernel (one launch per step)"},
        "cpu_baseline": cpu,
        "e2e": {"value": total / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "clocks": {k: clocks[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")},
        "gpu_launches": args.steps,
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------ GPU arm
def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        # NCCL announces its version on stdout while it initialises; the driver reads exactly one
        # JSON line from stdout, so that banner goes to stderr
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
            dist.barrier()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)

    from qwen_mla_vllm_b200.dcp import P2PExchange, merge_across_ranks, shard_lengths
    from qwen_mla_vllm_b200.mla_decode_attention import build_params, run_params

    lens_all = seq_lens_cfg1()[:args.batch]
    lens = shard_lengths(lens_all, world, rank) if world > 1 else lens_all
    cache, q_h, bt_h, sl_h = make_inputs(lens, dev, seed=1000 + rank)
    q, bt, sl = q_h.to(dev), bt_h.to(dev), sl_h.to(dev)
    nb = len(lens_all)
    ks = torch.tensor(0.01, dtype=torch.float32, device=dev) if FP8 else None
    kw = dict(rank=RANK, qk_dim=QK, rms_offset=QK, rms_mode=3 if FP8 else 1, page_size=PAGE, sm_scale=1 / 16,
              k_scale=ks)
    merge_kind = args.dcp_merge if world > 1 else None
    hs = H // world  # heads each rank keeps after the merge (vLLM's cp_lse_ag_out_rs layout)
    ex = None
    if merge_kind == "p2p":
        # each rank decodes straight into slot (epoch & 1) of its exchange buffer; one kernel
        # then merges the ranks' partials over NVLink peer memory
        ex = P2PExchange(nb, H, RANK, device=dev)
        slot_params = []
        for s_epoch in (2, 1):  # slot 0, slot 1
            o_s, l_s = ex.buf.partial(s_epoch)
            slot_params.append(build_params(q, cache, o_s, l_s, bt, sl, **kw))
        o_m = torch.empty(nb, hs, RANK, dtype=torch.bfloat16, device=dev)
        lse_m = torch.empty(nb, hs, dtype=torch.float32, device=dev)
        params = slot_params[0]
    else:
        o = torch.empty(nb, H, RANK, dtype=torch.float32 if world > 1 else torch.bfloat16, device=dev)
        lse = torch.empty(nb, H, dtype=torch.float32, device=dev)
        params = build_params(q, cache, o, lse, bt, sl, **kw)
    run_params(params, dev)  # sizes and attaches the workspace once
    stream = torch.cuda.current_stream(dev)
    # our kernels per step: plan, decode, split merge (+ the P2P merge, or the NCCL path's correction)
    launches_per_step = 3 + (1 if world > 1 else 0)

    def decode():
        if ex is not None:
            run_params(slot_params[(ex.epoch + 1) & 1], dev)
        else:
            run_params(params, dev)

    def merge():
        if ex is not None:
            ex.merge(out=o_m, lse_out=lse_m, mode="rs")
        elif world > 1:
            merge_across_ranks(o, lse, mode="rs")

    def step():
        decode()
        merge()

    # clock ramp: ~1 s of untimed local decode so the SM clock leaves its idle state (no
    # collectives here: the loop is timed per rank, so its iteration count differs between
    # ranks), then W warm-up steps that every rank takes the same number of times
    t_end = time.perf_counter() + 1.0
    while time.perf_counter() < t_end:
        for _ in range(5):
            run_params(params, dev)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    for _ in range(args.warmup):
        step()
    sampler = ClockSampler(local).start()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(args.steps):
        ev[i][0].record(stream)
        decode()
        ev[i][1].record(stream)
        merge()
    stop.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t1 = time.perf_counter()
    sampler.stop()
    ms = start.elapsed_time(stop)
    decode_ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    mine = algorithmic_bytes(lens, nb)
    if world > 1:
        t = torch.tensor([ms, float(mine), decode_ms], dtype=torch.float64, device=dev)
        tmax = t.clone()
        dist.all_reduce(tmax[:1], op=dist.ReduceOp.MAX)
        tsum = t.clone()
        dist.all_reduce(tsum[1:2], op=dist.ReduceOp.SUM)
        ms, total_bytes = float(tmax[0]), float(tsum[1])
    else:
        total_bytes = float(mine)
    step_ms = ms / args.steps
    value = total_bytes / (step_ms * 1e-3) / 1e12
    peak, peak_kind = measured_peak()
    achieved_gbs = mine / (decode_ms * 1e-3) / 1e9
    traffic = profile_traffic() if world == 1 and not FP8 else None
    clocks = sampler.summary(t0, t1)

    # ---- end to end through the public entry point with host buffers (pinned) every step.
    # Every step copies its q / block table / lengths host->device and its (o, lse)
    # device->host.  The copies run on a copy stream, double-buffered, so step i+1's inputs
    # and step i-1's outputs move while step i decodes (as a serving loop would run them);
    # the NCCL merge path keeps them serial.
    from qwen_mla_vllm_b200.mla_decode_attention import decode_attention_fwd
    q_pin, bt_pin, sl_pin = q_h.pin_memory(), bt_h.pin_memory(), sl_h.pin_memory()
    logits = torch.empty(nb, H, 8, RANK + 1, dtype=torch.float32, device=dev)
    heads_kept = hs if world > 1 else H  # a rank keeps its H/N heads after a DCP merge
    out_dtype = o_m.dtype if ex is not None else o.dtype
    pipelined = world == 1 or ex is not None
    nbuf = 2 if pipelined else 1
    ins = [(torch.empty_like(q), torch.empty_like(bt), torch.empty_like(sl)) for _ in range(nbuf)]
    outs_dev = [(torch.empty(nb, heads_kept, RANK, dtype=out_dtype, device=dev),
                 torch.empty(nb, heads_kept, dtype=torch.float32, device=dev)) for _ in range(nbuf)]
    outs_host = [(torch.empty(nb, heads_kept, RANK, dtype=out_dtype).pin_memory(),
                  torch.empty(nb, heads_kept, dtype=torch.float32).pin_memory()) for _ in range(nbuf)]
    cs = torch.cuda.Stream(dev)
    h2d_done = [torch.cuda.Event() for _ in range(nbuf)]
    comp_done = [torch.cuda.Event() for _ in range(nbuf)]

    def copy_in(b):
        with torch.cuda.stream(cs):
            for d, h in zip(ins[b], (q_pin, bt_pin, sl_pin)):
                d.copy_(h, non_blocking=True)
            h2d_done[b].record(cs)

    def compute(b):
        stream.wait_event(h2d_done[b])
        q_d, bt_d, sl_d = ins[b]
        if ex is not None:
            o_w, l_w = ex.partial()
        elif world == 1:
            o_w, l_w = outs_dev[b]
        else:
            o_w, l_w = o, lse
        decode_attention_fwd(q_d, cache, cache[..., :RANK], o_w, l_w, bt_d, sl_d, logits, 8, 1 / 16, PAGE,
                             is_mla=True, rms_offset=QK, k_scale=ks, v_scale=ks, rms_log8=FP8)
        if ex is not None:
            ex.merge(out=outs_dev[b][0], lse_out=outs_dev[b][1], mode="rs")
            res = outs_dev[b]
        elif world > 1:
            res = merge_across_ranks(o, lse, mode="rs")
        else:
            res = outs_dev[b]
        comp_done[b].record(stream)
        return res

    def copy_out(b, res):
        with torch.cuda.stream(cs):
            cs.wait_event(comp_done[b])
            outs_host[b][0].copy_(res[0], non_blocking=True)
            outs_host[b][1].copy_(res[1], non_blocking=True)

    def run_e2e(n):
        if not pipelined:
            for i in range(n):
                copy_in(0)
                res = compute(0)
                copy_out(0, res)
            stream.wait_stream(cs)
            return
        copy_in(0)
        if n > 1:
            copy_in(1)
        for i in range(n):
            b = i % nbuf
            res = compute(b)
            copy_out(b, res)  # after compute(b): the copy stream waits for it
            if i + nbuf < n:
                copy_in(b)  # the next use of buffer b (after this step read its inputs)
        stream.wait_stream(cs)

    run_e2e(max(3, args.warmup))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    cs.wait_event(e0)
    run_e2e(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t[0])
    e2e_value = total_bytes / (e2e_ms / args.steps * 1e-3) / 1e12
    h2d = (q.numel() * q.element_size() + bt.numel() * 4 + sl.numel() * 4) * world
    d2h = (outs_host[0][0].numel() * outs_host[0][0].element_size() + outs_host[0][1].numel() * 4) * world

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not FP8:
        cb, cs, n, threads = cpu_reference_sample(lens_all, args.cpu_budget)
        cpu = {"value": cb / cs / 1e12, "unit": "TB/s", "cores": threads, "kind": "port",
               "sample": f"{n} of the {nb} sequences ({cb / 1e9:.2f} GB of rows), numpy oracle, {cs:.1f} s"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp8-e4m3" if FP8 else "bf16",
            "data": "synthetic (seeded), random-init cache in the plugin's row layout",
            "config": {"workload": WORKLOAD if nb == B else f"{WORKLOAD} -- first {nb} sequences only",
                       "batch": nb, "heads": H, "rank": RANK, "rope": ROPE,
                       "rms": H, "row_bytes_read": ROW_READ, "page_size": PAGE, "sum_context": sum(lens_all),
                       "parallelism": f"dcp{world}" if world > 1 else "single",
                       **({"dcp_merge": "one kernel over NVLink peer memory (qmla_dcp_p2p_merge), heads "
                                        "scattered over ranks" if merge_kind == "p2p" else
                           "NCCL all-gather lse + correction kernel + reduce-scatter over heads"}
                          if world > 1 else {}),
                       "l2": f"inputs larger than L2 ({sum(lens_all) * ROW_READ / 1e9:.2f} GB of rows), no flush"},
            "seqs_per_s": nb / (step_ms * 1e-3),
            "hbm_frac_of_measured_peak": value * 1e3 / peak,
            "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": peak, "unit": "GB/s",
                         "frac": achieved_gbs / peak, "traffic": traffic,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6650 GB/s",
                         "kernel": "qmla_mla_decode call (plan + persistent decode + split merge), rank 0"},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "TB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "clocks": {k: clocks[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")},
            "gpu_launches": launches_per_step * args.steps,
        }
        print(json.dumps(line), flush=True)
    if ex is not None:
        ex.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of CPU baseline sampling")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--dcp-merge", choices=["p2p", "nccl"], default="p2p",
                    help="N>1: merge the ranks' partials with one kernel over NVLink peer memory "
                         "(default) or with NCCL (all-gather + correction + reduce-scatter)")
    ap.add_argument("--workload", choices=["cfg1", "cfg4", "gather"], default="cfg1",
                    help="cfg1 (default, the headline): bf16 config 1; cfg4: FP8 8 x 262,144 tokens; "
                         "gather: the prefill context gather on one GPU")
    ap.add_argument("--batch", type=int, default=None,
                    help="first N sequences of config1 (smaller cases for ncu captures; default: all 64)")
    args = ap.parse_args()
    if args.workload == "cfg4":
        use_cfg4()
    if args.batch is None:
        args.batch = B
    if args.warmup < 3:
        args.warmup = 3
    if args.workload == "gather":
        if args.impl == "reference":
            raise SystemExit("--workload gather has no reference arm; its line carries cpu_baseline")
        run_gather(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
