#!/usr/bin/env python3
"""Benchmark of the sm_100a paged MLA decode: achieved HBM TB/s (and seqs/s) at 1/2/4/8 B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload (the plugin's real row split): bf16 latent cache,
batch 64, 1 query token, 24 heads, context lengths U[1024, 32768] (torch generator seed 1),
16-token pages in random order, row = latent 768 | rope 232 | rms 24 (1024 bf16),
q ~ N(0,1)/sqrt(1024), cache ~ N(0,1), rms ~ U(0.5, 2).  Synthetic and seeded; the 2.44 GB of
cache rows are larger than L2, so no L2 flush is needed between steps.

One step = one decode of the whole batch.  N = 1: one GPU.  N > 1 (torchrun, one process per
GPU): decode context parallelism -- every rank holds a contiguous 1/N of every sequence's KV,
cut from ONE seeded global cache, decodes it into its exchange buffer, and one kernel merges
the ranks' partials over NVLink peer memory (qmla_dcp_p2p_merge); total work is fixed
("scaling": "strong").  Device time is measured over CUDA-graph replays of the step, as vLLM
runs decode; ``e2e`` goes through the public Python entry point with host copies every step.

Sub-objects of the same line: ``cfg2`` (FP8 MTP verify), ``cfg3`` (GLA-g2, both head groups)
and ``cfg4`` (FP8 262k context) at N = 1; ``dcp_cfg4`` (config 4 split over the N ranks) and
``gla_cfg3`` (config 3 sharded by head group, then split-KV inside each group) at N > 1.  Every
multi-GPU sub-object carries ``parity``: the merged output against a single-GPU decode of the
same global cache on each rank (max over ranks).  At N = 1 the CPU baseline leg runs the
reference's CPU path (a torch restatement of the reference's test references, all host cores) on
a sample of each workload and reports its agreement with the GPU output (``cpu_check``).
``gpu_baseline`` times the reference's own Triton ``decode_attention_fwd`` (installed unmodified
in baseline/_ref) on the same GPU and inputs for configs 1 and 2.

``--impl reference`` times the reference's CPU path on the host cores instead, on a bounded
sample of config 1 per step; under torchrun only rank 0 runs.
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
from dataclasses import dataclass, field

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MLA decode attn achieved HBM TB/s (% peak) and seqs/s at 1/2/4/8 B200"


# ------------------------------------------------------------------------------ workloads
def _randint_lens(lo: int, hi: int, n: int, seed: int) -> list[int]:
    import torch
    return torch.randint(lo, hi + 1, (n,), generator=torch.Generator().manual_seed(seed)).tolist()


@dataclass
class Workload:
    """One BASELINE config: shapes, dtypes and the context length of every request."""

    key: str
    desc: str
    fp8: bool
    heads: int
    rank: int
    rope: int
    lens: list = field(default_factory=list)
    qrows: int = 1    # MTP verify tokens per request (causal across the drafts)
    groups: int = 1   # GLA head groups: independent caches with the same lengths
    page: int = 16
    seed: int = 1

    @property
    def qk(self) -> int:
        return self.rank + self.rope

    @property
    def width(self) -> int:
        """Elements per cache row: latent | rope | one rms value (bf16) or code (FP8) per head."""
        w = self.qk + self.heads
        return w + (-w) % (16 if self.fp8 else 8)

    @property
    def row_read(self) -> int:
        """Bytes of a row the decode reads: (latent + rope) elements and the rms tail."""
        return self.qk * (1 if self.fp8 else 2) + self.heads * (1 if self.fp8 else 2)

    def row_lens(self, lens=None) -> list[int]:
        """Decode-row lengths: request L gives rows L - (q-1-j), j < q (qwen_mla/mla_impl.py:628-662)."""
        lens = self.lens if lens is None else lens
        return [max(L - (self.qrows - 1 - j), 0) for L in lens for j in range(self.qrows)]

    def algorithmic_bytes(self, lens=None) -> int:
        """Per call, all groups: cache rows read once per request + page table + q + o + lse."""
        lens = self.lens if lens is None else lens
        rows = len(lens) * self.qrows
        pages = sum((L + self.page - 1) // self.page for L in lens)
        per = (sum(lens) * self.row_read + 4 * pages + rows * self.heads * self.qk * 2
               + rows * self.heads * self.rank * 2 + rows * self.heads * 4)
        return per * self.groups

    def flops(self, lens=None) -> int:
        """Algorithmic flops: 2 x (QK width + rank) per (row, head, token), all groups."""
        return 2 * self.heads * (self.qk + self.rank) * sum(self.row_lens(lens)) * self.groups


def workloads() -> dict[str, Workload]:
    return {
        "cfg1": Workload("cfg1", "config1: bf16 latent paged MLA decode, B=64, 1 query token, 24 heads, row "
                         "768|232|24 bf16, L~U[1024,32768] (seed 1), 16-token pages in random order",
                         fp8=False, heads=24, rank=768, rope=232, lens=_randint_lens(1024, 32768, 64, 1), seed=1),
        "cfg2": Workload("cfg2", "config2: FP8-e4m3 latent cache with log8 rms codes, k_scale = absmax/448, "
                         "MTP verify with 4 causal drafts, 128 requests x 8192 tokens, 24 heads",
                         fp8=True, heads=24, rank=768, rope=232, lens=[8192] * 128, qrows=4, seed=2),
        "cfg3": Workload("cfg3", "config3: GLA-g2, 2 head groups of 12 heads, row 384|116|12 bf16 per group, "
                         "B=64, L~U[4096,65536] (seed 3)",
                         fp8=False, heads=12, rank=384, rope=116, lens=_randint_lens(4096, 65536, 64, 3),
                         groups=2, seed=3),
        "cfg4": Workload("cfg4", "config4: FP8-e4m3 latent cache with log8 rms codes, k_scale = absmax/448, "
                         "B=8 x 262144 tokens, 1 query token, 24 heads",
                         fp8=True, heads=24, rank=768, rope=232, lens=[262144] * 8, seed=4),
    }


@dataclass
class Case:
    """A workload's tensors for one head group on one device."""

    cache: object        # [P, page, 1, width] bf16 or float8_e4m3fn
    bt: object           # [requests, max_pages] int32 (device)
    lens: list           # request lengths
    k_scale: object      # 0-d fp32 device tensor (FP8) or None
    q: object = None     # [rows, heads, qk] bf16 (device)
    bt_rows: object = None  # [rows, max_pages] int32: block table per decode row (MTP rows repeat)
    sl_rows: object = None  # [rows] int32


def build_cache(w: Workload, lens: list[int], device, seed: int):
    """Paged cache holding exactly the given requests, pages in random order.

    bf16: N(0,1) latent and rope, U(0.5, 2) rms.  FP8: the same bf16 values written by this
    build's FP8 cache writer (qmla_fp8_cache_write, bit-exact against the reference's
    do_kv_cache_update) with k_scale = absmax / 448 and one log8 code per head.
    Returns (cache, block_table on the host, k_scale or None)."""
    import torch
    pages = [(L + w.page - 1) // w.page for L in lens]
    P = max(1, sum(pages))
    gd = torch.Generator(device=device).manual_seed(seed)
    k_scale = None
    if not w.fp8:
        cache = torch.randn(P, w.page, 1, w.width, device=device, dtype=torch.bfloat16, generator=gd)
        cache[..., w.qk:] = (torch.rand(P, w.page, 1, w.width - w.qk, device=device, generator=gd) * 1.5
                             + 0.5).to(torch.bfloat16)
    else:
        from qwen_mla_vllm_b200.kv_cache import fp8_kv_cache_update
        n = P * w.page
        raw = torch.zeros(P, w.page, 1, w.width, dtype=torch.uint8, device=device)
        lat = torch.randn(n, w.rank, device=device, dtype=torch.bfloat16, generator=gd)
        kpe = torch.empty(n, w.rope + w.heads, device=device, dtype=torch.bfloat16)
        kpe[:, :w.rope] = torch.randn(n, w.rope, device=device, dtype=torch.bfloat16, generator=gd)
        kpe[:, w.rope:] = (torch.rand(n, w.heads, device=device, generator=gd) * 1.5 + 0.5).to(torch.bfloat16)
        k_scale = (torch.maximum(lat.abs().max(), kpe[:, :w.rope].abs().max()).float() / 448.0).reshape(())
        fp8_kv_cache_update(lat, kpe, raw, torch.arange(n, device=device), k_scale, w.rope, w.heads, "log8")
        del lat, kpe
        cache = raw.view(torch.float8_e4m3fn)
    perm = torch.randperm(P, generator=torch.Generator().manual_seed(seed))
    bt = torch.zeros(len(lens), max(1, max(pages) if pages else 1), dtype=torch.int32)
    off = 0
    for b, n in enumerate(pages):
        bt[b, :n] = perm[off:off + n].to(torch.int32)
        off += n
    return cache, bt, k_scale


def make_query(w: Workload, n_requests: int, device, seed: int):
    import torch
    g = torch.Generator().manual_seed(seed + 12345)
    q = (torch.randn(n_requests * w.qrows, w.heads, w.qk, generator=g) / math.sqrt(1024)).to(torch.bfloat16)
    return q.to(device)


def decode_rows(w: Workload, bt, lens: list[int], device):
    """Per decode row: block table (MTP rows repeat their request's) and length."""
    import torch
    bt_rows = bt.repeat_interleave(w.qrows, dim=0) if w.qrows > 1 else bt
    sl = torch.tensor(w.row_lens(lens), dtype=torch.int32)
    return bt_rows.to(device), sl.to(device)


def build_case(w: Workload, device, group: int = 0, lens=None) -> Case:
    """The whole workload's tensors (one head group) on ``device``; deterministic."""
    lens = w.lens if lens is None else lens
    seed = 1000 * w.seed + group
    cache, bt, ks = build_cache(w, lens, device, seed)
    c = Case(cache=cache, bt=bt.to(device), lens=list(lens), k_scale=ks)
    c.q = make_query(w, len(lens), device, seed)
    c.bt_rows, c.sl_rows = decode_rows(w, bt, lens, device)
    return c


def shard_tokens(L: int, world: int, rank: int, interleave: int = 0):
    """Global token positions of one sequence held by ``rank``: a contiguous 1/world slice, or
    (interleave > 0) the tokens t with (t // interleave) % world == rank, vLLM's
    cp_kv_cache_interleave_size layout.  Kept in increasing order."""
    import torch
    if interleave <= 0:
        return torch.arange(L * rank // world, L * (rank + 1) // world)
    t = torch.arange(L)
    return t[(t // interleave) % world == rank]


def shard_case(w: Workload, full: Case, world: int, rank: int, device, interleave: int = 0) -> Case:
    """This rank's DCP shard of a global case: its tokens of every request, copied into a new
    paged cache (pages in random order), with per-row local lengths (MTP rows included: a row that
    sees the first L_j global tokens sees the rank's tokens below L_j)."""
    import torch
    page = w.page
    toks = [shard_tokens(L, world, rank, interleave) for L in full.lens]
    n_loc = [len(t) for t in toks]
    pages = [(n + page - 1) // page for n in n_loc]
    P = max(1, sum(pages))
    perm = torch.randperm(P, generator=torch.Generator().manual_seed(7919 * (rank + 1) + w.seed))
    bt = torch.zeros(len(toks), max(1, max(pages)), dtype=torch.int32)
    off = 0
    for b, n in enumerate(pages):
        bt[b, :n] = perm[off:off + n].to(torch.int32)
        off += n
    bt_full = full.bt.cpu().long()
    src, dst = [], []
    for b, t in enumerate(toks):
        if len(t) == 0:
            continue
        src.append(bt_full[b, t // page] * page + t % page)
        j = torch.arange(len(t))
        dst.append(bt[b, j // page].long() * page + j % page)
    cache = torch.empty((P, page) + tuple(full.cache.shape[2:]), dtype=full.cache.dtype, device=device)
    if src:
        s = torch.cat(src).to(device)
        d = torch.cat(dst).to(device)
        cv = cache.view(torch.uint8) if w.fp8 else cache
        fv = full.cache.view(torch.uint8) if w.fp8 else full.cache
        cv.view(P * page, -1)[d] = fv.reshape(-1, cv.shape[-1])[s]
    c = Case(cache=cache, bt=bt.to(device), lens=n_loc, k_scale=full.k_scale, q=full.q)
    # local length of each decode row: the rank's tokens below the row's global length
    row_loc = []
    for b, L in enumerate(full.lens):
        for j in range(w.qrows):
            Lj = max(L - (w.qrows - 1 - j), 0)
            row_loc.append(int((toks[b] < Lj).sum()))
    c.bt_rows = (bt.repeat_interleave(w.qrows, dim=0) if w.qrows > 1 else bt).to(device)
    c.sl_rows = torch.tensor(row_loc, dtype=torch.int32, device=device)
    return c


def params_for(w: Workload, c: Case, o, lse):
    from qwen_mla_vllm_b200.mla_decode_attention import build_params
    return build_params(c.q, c.cache, o, lse, c.bt_rows, c.sl_rows, rank=w.rank, qk_dim=w.qk, rms_offset=w.qk,
                        rms_mode=3 if w.fp8 else 1, page_size=w.page, sm_scale=1 / 16, k_scale=c.k_scale,
                        qrows=w.qrows)


# ------------------------------------------------------------------------------ measurement helpers
def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d.get("bf16_tflops", 1590.0)),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", 1400.0)), "kind": "measured"}
    except Exception:  # noqa: BLE001
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "kind": "fallback"}


def profile_traffic() -> float | None:
    """DRAM bytes per decode launch from the committed ncu summary of config 1."""
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


def launches_per_call(work_rows: int, fp8: bool = False) -> int:
    """This build's kernels per qmla_mla_decode call: plan (or bounds), decode, merge, and for
    FP8 caches the Q preparation (e4m3 hi / lo rows) before the decode."""
    del work_rows
    return 4 if fp8 else 3


def capture(fns, device):
    """One CUDA graph per callable (each called once eagerly before, so sizing is done)."""
    import torch
    graphs = []
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        for fn in fns:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                fn()
            graphs.append(g)
    torch.cuda.current_stream(device).wait_stream(s)
    torch.cuda.synchronize(device)
    return graphs


def time_graphs(graphs, steps: int, device) -> float:
    """Device ms per step over ``steps`` replays (the graphs in turn), CUDA events on the
    launching stream with a synchronize on both sides."""
    import torch
    stream = torch.cuda.current_stream(device)
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        graphs[i % len(graphs)].replay()
    e1.record(stream)
    torch.cuda.synchronize(device)
    return e0.elapsed_time(e1) / steps


def ramp(fn, device, seconds: float = 1.0):
    """~1 s of untimed work so the SM clock leaves its idle state (per rank, no collectives)."""
    import torch
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end:
        for _ in range(5):
            fn()
        torch.cuda.synchronize(device)


# ------------------------------------------------------------------------------ CPU path
def cpu_threads() -> int:
    """Use every host core (torchrun sets OMP_NUM_THREADS=1 per rank; override it here)."""
    import torch
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return n


def cpu_decode(w: Workload, c: Case, rows: list[int]):
    """The reference's CPU path (oracle/torch_ref.py) on the given decode rows of a case.
    Returns (o [len(rows), H, rank], lse, seconds, bytes)."""
    import torch
    from oracle.torch_ref import decode_paged
    page = w.page
    bt_rows = c.bt_rows.cpu()
    sl = c.sl_rows.cpu().tolist()
    # copy just the pages these rows use to the host (not timed: the data is host-resident for the CPU)
    need = sorted({int(p) for r in rows for p in bt_rows[r, :(sl[r] + page - 1) // page].tolist()})
    remap = {p: i for i, p in enumerate(need)}
    host = (c.cache.view(torch.uint8) if w.fp8 else c.cache)[torch.tensor(need, device=c.cache.device)][:, :, 0].cpu()
    bt_h = torch.zeros(len(rows), bt_rows.shape[1], dtype=torch.int32)
    for i, r in enumerate(rows):
        npg = (sl[r] + page - 1) // page
        bt_h[i, :npg] = torch.tensor([remap[int(p)] for p in bt_rows[r, :npg].tolist()], dtype=torch.int32)
    q = c.q[rows].cpu()
    ks = float(c.k_scale) if c.k_scale is not None else 1.0
    t0 = time.perf_counter()
    o, lse = decode_paged(q, host, bt_h, [sl[r] for r in rows], rank=w.rank, qk_dim=w.qk, page_size=page,
                          sm_scale=1 / 16, rms_offset=w.qk, rms_mode="log8" if w.fp8 else "native", k_scale=ks)
    dt = time.perf_counter() - t0
    nbytes = sum(sl[r] for r in rows) * w.row_read  # rows read per decode row (the CPU path re-reads per row)
    return o, lse, dt, nbytes


def cpu_check(w: Workload, c: Case, o_gpu, lse_gpu, rows: list[int]) -> dict:
    """CPU baseline leg on a few rows of the workload: timed, and its agreement with the GPU output."""
    o, lse, dt, nbytes = cpu_decode(w, c, rows)
    og = o_gpu[rows].float().cpu()
    lg = lse_gpu[rows].float().cpu()
    fin = lse.isfinite()
    return {"rows": rows, "max_abs": float((og - o).abs().max()),
            "lse_max_abs": float((lg[fin] - lse[fin]).abs().max()) if bool(fin.any()) else 0.0,
            "cpu_s": dt, "cpu_gbs": nbytes / max(dt, 1e-9) / 1e9}


# ------------------------------------------------------------------------------ reference arm
def run_reference(args) -> None:
    """The reference's CPU path (torch restatement of its test references) on all host cores,
    one bounded sample of config 1 per step; rank 0 only under torchrun."""
    import torch
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = cpu_threads()
    w = workloads()["cfg1"]
    per_step = 4  # requests of config 1 per step, cycling through the batch
    sample_lens = w.lens[:16]
    c = build_case(w, torch.device("cpu"), lens=sample_lens)
    times, nbytes = [], []
    for i in range(args.warmup + args.steps):
        rows = [(per_step * i + k) % len(sample_lens) for k in range(per_step)]
        _, _, dt, b = cpu_decode(w, c, rows)
        if i >= args.warmup:
            times.append(dt)
            nbytes.append(b)
    value = sum(nbytes) / sum(times) / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(times) / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded), host memory",
        "config": {"workload": w.desc, "sample": f"{per_step} requests of config1 per step, cycling over the "
                                                  f"first {len(sample_lens)}"},
        "cpu_baseline": {"value": value, "unit": "TB/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} steps x {per_step} config1 requests; torch CPU restatement "
                                   f"of the reference's test references (oracle/torch_ref.py)"},
        "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------ the reference's Triton kernel
def triton_baseline(w: Workload, c: Case, o_ours, lse_ours, steps: int) -> dict:
    """The reference's own Triton decode_attention_fwd (baseline/_ref, unmodified) on the same GPU
    and inputs: device ms per call, TB/s, and its agreement with this build's output."""
    import torch
    ref_dir = ROOT / "baseline" / "_ref"
    if not (ref_dir / "qwen_mla").exists():
        return {"unavailable": "reference not installed in baseline/_ref"}
    try:
        if str(ref_dir) not in sys.path:
            sys.path.insert(0, str(ref_dir))
        import logging
        logging.getLogger("vllm").setLevel(logging.ERROR)
        from qwen_mla.ops.mla_decode_attention import decode_attention_fwd as ref_fwd
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"import failed: {type(e).__name__}: {e}"[:200]}
    dev = c.q.device
    rows, H = c.q.shape[0], c.q.shape[1]
    # num_kv_splits as the plugin sets it: vLLM's split count capped so the fp32 split-K scratch
    # stays within 512 MB (qwen_mla/mla_impl.py:89-103); 64 before the cap
    splits = 64
    while splits > 1 and rows * H * splits * (w.rank + 1) * 4 > (512 << 20):
        splits //= 2
    o = torch.zeros(rows, H, w.rank, dtype=torch.bfloat16, device=dev)
    lse = torch.zeros(rows, H, dtype=torch.float32, device=dev)
    logits = torch.empty(rows, H, splits, w.rank + 1, dtype=torch.float32, device=dev)
    ks = c.k_scale

    def call():
        ref_fwd(c.q, c.cache, c.cache[..., :w.rank], o, lse, c.bt_rows, c.sl_rows, logits, splits, 1 / 16, w.page,
                k_scale=ks, v_scale=ks, is_mla=True, rms_offset=w.qk, rms_bf16=False, rms_log8=w.fp8,
                qrows=w.qrows)

    try:
        t0 = time.perf_counter()
        call()  # JIT compile
        torch.cuda.synchronize(dev)
        compile_s = time.perf_counter() - t0
        for _ in range(2):
            call()
        stream = torch.cuda.current_stream(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(steps):
            call()
        e1.record(stream)
        torch.cuda.synchronize(dev)
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"run failed: {type(e).__name__}: {e}"[:200]}
    ms = e0.elapsed_time(e1) / steps
    nb = w.algorithmic_bytes() // w.groups
    return {"impl": "reference Triton decode_attention_fwd (baseline/_ref, qwen-mla-vllm 0.6.7)", "ms": ms,
            "tb_s": nb / (ms * 1e-3) / 1e12, "num_kv_splits": splits, "compile_s": compile_s,
            "max_abs_vs_ours": float((o.float() - o_ours.float()).abs().max()),
            "lse_max_abs_vs_ours": float((lse - lse_ours.float()).abs()[lse.isfinite()].max()),
            "ours_speedup": None}


# ------------------------------------------------------------------------------ context gather
# --workload gather: the chunked-prefill context gather (qmla_gather_cache) on one GPU.  Not the
# headline line.  A 131,072-row chunk (16 sequences x 8192 tokens) of an FP8 cache (row 768|232
# e4m3 + 24 log8 codes = 1024 B), pages in random order, into a bf16 [rows, 1024] destination.
GATHER_SEQS, GATHER_LEN = 16, 8192
PAGE, ROW, QK, H = 16, 1024, 1000, 24  # FP8 row: 768 | 232 e4m3 + 24 log8 codes
GATHER_WORKLOAD = ("prefill context gather: FP8-e4m3 cache rows (768|232 e4m3 + 24 log8 codes, 1024 B) "
                   "-> bf16 [131072, 1024], 16 sequences x 8192 tokens, 16-token pages in random order")
GATHER_METRIC = "MLA prefill context gather achieved HBM GB/s (FP8 -> bf16 dequant)"
GATHER_TRAFFIC = 344.8e6  # dram__bytes of the default kernel's ncu launch (profiles/gather_fp8_log8_131k.md)


def gather_row_bytes() -> float:
    """Algorithmic bytes per destination row: the cache row read, the bf16 row written, the
    token's sequence id, and its share of one block-table entry per page."""
    return ROW + 2 * (QK + H) + 4 + 4 / PAGE


def run_profile_case(args) -> None:
    """One workload's decode on cuda:0, called --warmup then --steps times with plain launches
    (no graphs, no sub-objects, no baselines): the small cases ncu captures use.  --batch N keeps
    the first N sequences; a GLA workload runs its first head group.  Prints one JSON line."""
    import torch
    from qwen_mla_vllm_b200.mla_decode_attention import run_params
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    w = workloads()[args.profile_case]
    if args.batch and args.batch < len(w.lens):
        w.lens = w.lens[:args.batch]
    c = build_case(w, dev)
    rows = c.q.shape[0]
    o = torch.empty(rows, w.heads, w.rank, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(rows, w.heads, dtype=torch.float32, device=dev)
    p = params_for(w, c, o, lse)
    for _ in range(args.warmup):
        run_params(p, dev)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        run_params(p, dev)
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / args.steps
    nbytes = w.algorithmic_bytes() / w.groups
    print(json.dumps({"profile_case": w.key, "sequences": len(w.lens), "tokens": int(sum(w.lens)),
                      "ms_per_call": round(ms, 4), "algorithmic_bytes": int(nbytes),
                      "tbs": round(nbytes / ms / 1e9, 3)}))


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
    pk = measured_peaks()
    peak, peak_kind = pk["hbm_gbs"], pk["kind"]

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


def triton_child(key: str, steps: int) -> dict:
    """triton_baseline in a child process on the same GPU (its own CUDA context, so nothing the
    reference's kernel does can touch this process's).  The child rebuilds the seeded workload."""
    import subprocess
    cmd = [sys.executable, str(ROOT / "bench.py"), "--triton-baseline", key, "--steps", str(steps)]
    env = dict(os.environ)
    env.pop("RANK", None)
    env.pop("WORLD_SIZE", None)
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env)
    except subprocess.TimeoutExpired:
        return {"unavailable": "reference Triton run exceeded 900 s"}
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    if r.returncode != 0 or not lines:
        tail = (r.stderr or r.stdout).strip().splitlines()[-1:] or ["no output"]
        return {"unavailable": f"child exited {r.returncode}: {tail[0][:200]}"}
    return json.loads(lines[-1])


def run_triton_child(args) -> None:
    import torch
    from qwen_mla_vllm_b200.mla_decode_attention import run_params
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    w = workloads()[args.triton_baseline]
    c = build_case(w, dev)
    rows = c.q.shape[0]
    o = torch.empty(rows, w.heads, w.rank, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(rows, w.heads, dtype=torch.float32, device=dev)
    run_params(params_for(w, c, o, lse), dev)
    torch.cuda.synchronize(dev)
    print(json.dumps(triton_baseline(w, c, o, lse, args.steps)), flush=True)


# ------------------------------------------------------------------------------ GPU arm
class Dist:
    """Rank / world and max/min/sum reductions over ranks (no-ops at N = 1)."""

    def __init__(self, world: int, rank: int, device):
        self.world, self.rank, self.device = world, rank, device

    def reduce(self, values: list[float], op: str) -> list[float]:
        if self.world == 1:
            return list(values)
        import torch
        import torch.distributed as dist
        t = torch.tensor(values, dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op={"max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN, "sum": dist.ReduceOp.SUM}[op])
        return t.tolist()

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()


def single_gpu_line(w: Workload, device, steps: int, warmup: int, peaks: dict, group: int | None = None):
    """Decode of every head group of ``w`` on this GPU: graph-replay timing, roofline, outputs."""
    import torch
    from qwen_mla_vllm_b200.mla_decode_attention import run_params
    groups = range(w.groups) if group is None else [group]
    cases, outs, params = [], [], []
    for g in groups:
        c = build_case(w, device, group=g)
        rows = c.q.shape[0]
        o = torch.empty(rows, w.heads, w.rank, dtype=torch.bfloat16, device=device)
        lse = torch.empty(rows, w.heads, dtype=torch.float32, device=device)
        p = params_for(w, c, o, lse)
        cases.append(c)
        outs.append((o, lse))
        params.append(p)

    def step():
        for p in params:
            run_params(p, device)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(device)
    graphs = capture([step], device)
    ramp(lambda: graphs[0].replay(), device, 0.5)
    ms = time_graphs(graphs, steps, device)
    nb = w.algorithmic_bytes() * len(list(groups)) // w.groups
    fl = w.flops() * len(list(groups)) // w.groups
    tbs = nb / (ms * 1e-3) / 1e12
    res = {"workload": w.desc, "ms_per_step": ms, "value": tbs, "unit": "TB/s",
           "algorithmic_bytes": nb, "seqs_per_s": len(w.lens) * len(list(groups)) / (ms * 1e-3),
           "roofline": {"bound": "hbm", "achieved": tbs * 1e3, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                        "frac": tbs * 1e3 / peaks["hbm_gbs"], "peak_source": peaks["kind"]},
           "gpu_launches_per_step": launches_per_call(len(w.lens) * w.qrows, w.fp8) * len(params)}
    if w.qrows > 1:
        tf = fl / (ms * 1e-3) / 1e12
        res["tensor"] = {"algorithmic_flops": fl, "achieved_tflops": tf, "peak": peaks["bf16_tflops_sustained"],
                         "frac": tf / peaks["bf16_tflops_sustained"],
                         "note": "bf16-equivalent flops (FP8 q and P are split into e4m3 hi + lo terms); "
                                 "peak = measured bf16 sustained"}
    del graphs
    return res, cases, outs


def dcp_line(w: Workload, d: Dist, steps: int, warmup: int, peaks: dict, group_world: int, group_rank: int,
             pg, group: int = 0, interleave: int = 0):
    """Split-KV of ``w`` (head group ``group``) over ``group_world`` ranks (this one is
    ``group_rank`` in process group ``pg``): shards cut from one seeded global cache, each rank
    decodes into its exchange buffer, one kernel merges over NVLink peer memory.  Returns the
    per-rank numbers (the caller reduces over ranks) and the parity of the merged output against
    this rank's single-GPU decode of the global cache."""
    import torch
    from qwen_mla_vllm_b200.dcp import P2PExchange
    from qwen_mla_vllm_b200.mla_decode_attention import run_params
    dev = d.device
    full = build_case(w, dev, group=group)
    rows = full.q.shape[0]
    # single-GPU decode of the whole global cache on this rank: the parity reference
    o_ref = torch.empty(rows, w.heads, w.rank, dtype=torch.float32, device=dev)
    l_ref = torch.empty(rows, w.heads, dtype=torch.float32, device=dev)
    run_params(params_for(w, full, o_ref, l_ref), dev)
    shard = shard_case(w, full, group_world, group_rank, dev, interleave)
    torch.cuda.synchronize(dev)
    del full
    torch.cuda.empty_cache()
    hs = w.heads // group_world
    ex = P2PExchange(rows, w.heads, w.rank, group=pg, device=dev)
    slot_params = {}
    for par in (1, 0):  # the first merge is epoch 1 -> slot 1
        o_s, l_s = ex.buf.partial(par)
        slot_params[par] = params_for(w, shard, o_s, l_s)
    o_m = torch.empty(rows, hs, w.rank, dtype=torch.bfloat16, device=dev)
    lse_m = torch.empty(rows, hs, dtype=torch.float32, device=dev)

    def step_for(par):
        def step():
            run_params(slot_params[par], dev)
            ex.merge(out=o_m, lse_out=lse_m, mode="rs")
        return step

    def decode_only():
        run_params(slot_params[1], dev)

    # eager warm-up steps, the same count on every rank, starting at epoch 1 (slot 1)
    nw = max(2, warmup + warmup % 2)
    for i in range(nw):
        step_for((i + 1) & 1)()
    torch.cuda.synchronize(dev)
    # parity: the merged heads of this rank against its single-GPU decode of the global cache
    h0 = group_rank * hs
    err = float((o_m.float() - o_ref[:, h0:h0 + hs]).abs().max())
    lr = l_ref[:, h0:h0 + hs]
    fin = lr.isfinite()
    lerr = float((lse_m[fin] - lr[fin]).abs().max()) if bool(fin.any()) else 0.0
    status = ex.status()
    # graphs: [odd epoch -> slot 1, even epoch -> slot 0] replayed in turn; decode alone
    g_steps = capture([step_for(1), step_for(0)], dev)
    g_dec = capture([decode_only], dev)
    ramp(lambda: g_dec[0].replay(), dev, 0.5)
    dec_ms = time_graphs(g_dec, steps, dev)
    stats = ex.buf.merge_stats()
    d.barrier()
    stats.zero_()
    torch.cuda.synchronize(dev)
    d.barrier()
    ms = time_graphs(g_steps, steps + steps % 2, dev)
    st = stats.cpu().tolist()
    mine = w.algorithmic_bytes(shard.lens) // w.groups
    out = {"ms": ms, "decode_ms": dec_ms, "bytes": mine, "err": err, "lerr": lerr, "status": status,
           "wait_us": st[1] / max(st[0], 1) / 1e3, "merge_us": (st[2] - st[1]) / max(st[0], 1) / 1e3,
           "publish_us": st[3] / max(st[0], 1) / 1e3,
           "ex": ex, "graphs": g_steps + g_dec, "shard": shard, "o_m": o_m, "lse_m": lse_m,
           "slot_params": slot_params, "o_ref": o_ref}
    return out


def summarize_dcp(name: str, w: Workload, d: Dist, r: dict, steps: int, peaks: dict, n_ranks: int,
                  groups_note: str) -> dict:
    """Reduce one DCP measurement over all ranks into a sub-object of the line."""
    mx = d.reduce([r["ms"], r["decode_ms"], r["err"], r["lerr"], float(r["status"]), r["wait_us"], r["merge_us"],
                   r["publish_us"]], "max")
    mn = d.reduce([r["decode_ms"], r["wait_us"]], "min")
    tot = d.reduce([float(r["bytes"])], "sum")[0]
    ms = mx[0]
    tbs = tot / (ms * 1e-3) / 1e12
    return {"workload": w.desc, "parallelism": groups_note, "ms_per_step": ms, "value": tbs, "unit": "TB/s",
            "algorithmic_bytes": int(tot), "seqs_per_s": len(w.lens) * w.groups / (ms * 1e-3),
            "hbm_frac_of_n_x_measured_peak": tbs * 1e3 / (peaks["hbm_gbs"] * n_ranks),
            "per_rank": {"decode_ms_min": mn[0], "decode_ms_max": mx[1],
                         "merge_flag_wait_us_min": mn[1], "merge_flag_wait_us_max": mx[5],
                         "merge_kernel_us_max": mx[6], "merge_publish_us_max": mx[7],
                         "note": "decode alone timed per rank over graph replays; the merge's flag wait "
                                 "and its merge time come from the kernel's %globaltimer stamps (block 0)"},
            "parity": {"max_abs": mx[2], "lse_max_abs": mx[3], "status": int(mx[4]),
                       "against": "single-GPU decode of the same global cache, every rank's heads",
                       "tol": 5e-2 if w.fp8 else 2e-2}}


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
        # the DCP merge runs over plain peer memory; NCCL carries only barriers and timing
        # reductions here, so its NVLink SHARP (multicast) path stays off
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        # NCCL announces its version on stdout while it initialises; the driver reads exactly one
        # JSON line from stdout, so that banner goes to stderr
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
            dist.barrier()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    d = Dist(world, rank, dev)
    peaks = measured_peaks()
    W = workloads()
    w1 = W["cfg1"]
    if args.batch and args.batch < len(w1.lens):
        w1.lens = w1.lens[:args.batch]
        w1.desc += f" -- first {args.batch} sequences only"
    sampler = ClockSampler(local).start()
    from qwen_mla_vllm_b200.mla_decode_attention import decode_attention_fwd, run_params

    # ---------------------------------------------------------------- headline: config 1
    sub = {}
    if world == 1:
        line1, cases1, outs1 = single_gpu_line(w1, dev, args.steps, args.warmup, peaks)
        # the timed region proper (graph replays), with clocks sampled
        c1 = cases1[0]
        o1, lse1 = outs1[0]
        p1 = params_for(w1, c1, o1, lse1)
        g1 = capture([lambda: run_params(p1, dev)], dev)
        ramp(lambda: g1[0].replay(), dev, 1.0)
        t0 = time.perf_counter()
        step_ms = time_graphs(g1, args.steps, dev)
        t1 = time.perf_counter()
        total_bytes = float(w1.algorithmic_bytes())
        decode_ms = step_ms
        launches = launches_per_call(len(w1.lens))
    else:
        pg = None
        r1 = dcp_line(w1, d, args.steps, args.warmup, peaks, world, rank, pg)
        torch.cuda.synchronize(dev)
        d.barrier()
        t0 = time.perf_counter()
        ms_r = time_graphs(r1["graphs"][:2], args.steps + args.steps % 2, dev)
        t1 = time.perf_counter()
        r1["ms"] = ms_r
        s1 = summarize_dcp("cfg1", w1, d, r1, args.steps, peaks, world, f"dcp{world}")
        step_ms = s1["ms_per_step"]
        total_bytes = float(s1["algorithmic_bytes"])
        decode_ms = r1["decode_ms"]
        launches = launches_per_call(len(w1.lens)) + 1  # + the P2P merge
        sub["dcp_cfg1"] = s1
    clocks = sampler.summary(t0, t1)
    value = total_bytes / (step_ms * 1e-3) / 1e12

    # ---------------------------------------------------------------- e2e through the public entry point
    # Every step copies its q / block table / lengths host->device from pinned memory and (o, lse)
    # device->host; the copies run on a copy stream with double buffers, so step i+1's inputs and
    # step i-1's outputs move while step i decodes (as a serving loop runs them).
    if world == 1:
        c = cases1[0]
        ks = None
    else:
        c = r1["shard"]
        ks = None
    rows = c.q.shape[0]
    heads_kept = w1.heads // world
    q_pin, bt_pin, sl_pin = c.q.cpu().pin_memory(), c.bt_rows.cpu().pin_memory(), c.sl_rows.cpu().pin_memory()
    logits = torch.empty(rows, w1.heads, 8, w1.rank + 1, dtype=torch.float32, device=dev)
    ins = [(torch.empty_like(c.q), torch.empty_like(c.bt_rows), torch.empty_like(c.sl_rows)) for _ in range(2)]
    outs_dev = [(torch.empty(rows, heads_kept, w1.rank, dtype=torch.bfloat16, device=dev),
                 torch.empty(rows, heads_kept, dtype=torch.float32, device=dev)) for _ in range(2)]
    outs_host = [(torch.empty(rows, heads_kept, w1.rank, dtype=torch.bfloat16).pin_memory(),
                  torch.empty(rows, heads_kept, dtype=torch.float32).pin_memory()) for _ in range(2)]
    stream = torch.cuda.current_stream(dev)
    cs = torch.cuda.Stream(dev)
    h2d_done = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]
    ex = r1["ex"] if world > 1 else None

    def copy_in(b):
        with torch.cuda.stream(cs):
            for dst, h in zip(ins[b], (q_pin, bt_pin, sl_pin)):
                dst.copy_(h, non_blocking=True)
            h2d_done[b].record(cs)

    def compute(b):
        stream.wait_event(h2d_done[b])
        q_d, bt_d, sl_d = ins[b]
        o_w, l_w = ex.partial() if ex is not None else outs_dev[b]
        decode_attention_fwd(q_d, c.cache, c.cache[..., :w1.rank], o_w, l_w, bt_d, sl_d, logits, 8, 1 / 16, w1.page,
                             is_mla=True, rms_offset=w1.qk, k_scale=ks, v_scale=ks)
        if ex is not None:
            ex.merge(out=outs_dev[b][0], lse_out=outs_dev[b][1], mode="rs")
        comp_done[b].record(stream)

    def copy_out(b):
        with torch.cuda.stream(cs):
            cs.wait_event(comp_done[b])
            outs_host[b][0].copy_(outs_dev[b][0], non_blocking=True)
            outs_host[b][1].copy_(outs_dev[b][1], non_blocking=True)

    def run_e2e(n):
        copy_in(0)
        if n > 1:
            copy_in(1)
        for i in range(n):
            b = i % 2
            compute(b)
            copy_out(b)
            if i + 2 < n:
                copy_in(b)
        stream.wait_stream(cs)

    n_warm = max(4, args.warmup + args.warmup % 2)  # even: the DCP exchange keeps its slot parity
    run_e2e(n_warm)
    d.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = args.steps + args.steps % 2
    e0.record(stream)
    cs.wait_event(e0)
    run_e2e(e2e_steps)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = d.reduce([e0.elapsed_time(e1)], "max")[0]
    e2e_value = total_bytes / (e2e_ms / e2e_steps * 1e-3) / 1e12
    h2d = (c.q.numel() * 2 + c.bt_rows.numel() * 4 + c.sl_rows.numel() * 4) * world
    d2h = (outs_host[0][0].numel() * 2 + outs_host[0][1].numel() * 4) * world
    e2e_parity = None
    if world == 1:  # the last e2e step's output (host copy) equals the graph-timed decode's
        b = (e2e_steps - 1) % 2
        e2e_parity = float((outs_host[b][0].float() - o1.float().cpu()).abs().max())

    # ---------------------------------------------------------------- CPU baseline and the Triton baseline (N = 1)
    cpu = None
    gpu_base = None
    parity_cpu = None
    if world == 1:
        if not args.no_cpu_baseline:
            threads = cpu_threads()
            # rows of config 1 in batch order until ~cpu_budget seconds; the CPU output is compared
            # with the GPU output of the same rows
            done_rows, spent, nbytes = [], 0.0, 0
            errs, lerrs = [], []
            for r in range(len(w1.lens)):
                chk = cpu_check(w1, c1, o1, lse1, [r])
                done_rows.append(r)
                spent += chk["cpu_s"]
                nbytes += w1.lens[r] * w1.row_read
                errs.append(chk["max_abs"])
                lerrs.append(chk["lse_max_abs"])
                if spent >= args.cpu_budget:
                    break
            cpu = {"value": nbytes / spent / 1e12, "unit": "TB/s", "cores": threads, "kind": "port",
                   "sample": f"{len(done_rows)} of the {len(w1.lens)} config1 sequences ({nbytes / 1e9:.2f} GB of rows), "
                             f"torch CPU restatement of the reference's test references (oracle/torch_ref.py), "
                             f"{spent:.1f} s"}
            parity_cpu = {"rows": len(done_rows), "max_abs": max(errs), "lse_max_abs": max(lerrs), "tol": 2e-2,
                          "against": "the CPU baseline's output on the same rows"}
        if not args.no_gpu_baseline:
            gpu_base = {"cfg1": triton_child("cfg1", max(5, args.steps // 4))}
            if "ms" in gpu_base["cfg1"]:
                gpu_base["cfg1"]["ours_speedup"] = gpu_base["cfg1"]["ms"] / step_ms
        del g1
    sub_keys = [] if args.no_subs else (["cfg2", "cfg3", "cfg4"] if world == 1 else ["cfg4", "cfg3"])
    if world == 1:
        del cases1, outs1, c1, c
        torch.cuda.empty_cache()

    # ---------------------------------------------------------------- the other configs
    for key in sub_keys:
        w = W[key]
        if world == 1:
            res, cases, outs = single_gpu_line(w, dev, args.steps, args.warmup, peaks)
            if not args.no_cpu_baseline:
                cpu_threads()
                rows_chk = [0] if w.qrows == 1 else list(range(w.qrows))  # first request (all its drafts)
                res["cpu_check"] = [dict(cpu_check(w, cases[g], outs[g][0], outs[g][1], rows_chk), group=g)
                                    for g in range(len(cases))]
                res["cpu_check_tol"] = 5e-2 if w.fp8 else 2e-2
            if key == "cfg2" and not args.no_gpu_baseline:
                gb = triton_child("cfg2", max(5, args.steps // 4))
                if "ms" in gb:
                    gb["ours_speedup"] = gb["ms"] / res["ms_per_step"]
                gpu_base = dict(gpu_base or {}, cfg2=gb)
            sub[key] = res
            del cases, outs
            torch.cuda.empty_cache()
        elif key == "cfg4":
            r = dcp_line(w, d, args.steps, args.warmup, peaks, world, rank, None)
            sub["dcp_cfg4"] = summarize_dcp(key, w, d, r, args.steps, peaks, world, f"dcp{world}")
            r["ex"].close()
            del r
            torch.cuda.empty_cache()
        elif key == "cfg3":
            # head group g on ranks [g * N/2, (g+1) * N/2): N = 2 shards by group only (no exchange);
            # N = 4 / 8 add split-KV inside each group, merged among the group's ranks
            from qwen_mla_vllm_b200.dcp import head_group_of, head_group_subgroups
            g, sub_rank, per = head_group_of(rank, world, w.groups)
            pgs = head_group_subgroups(world, w.groups)
            if per == 1:
                res, _, _ = single_gpu_line(w, dev, args.steps, args.warmup, peaks, group=g)
                mx = d.reduce([res["ms_per_step"]], "max")[0]
                tot = w.algorithmic_bytes()
                sub["gla_cfg3"] = {"workload": w.desc, "parallelism": f"head group per GPU ({world} GPUs)",
                                   "ms_per_step": mx, "value": tot / (mx * 1e-3) / 1e12, "unit": "TB/s",
                                   "algorithmic_bytes": tot, "seqs_per_s": len(w.lens) * w.groups / (mx * 1e-3),
                                   "parity": {"note": "no exchange: each GPU runs the single-GPU decode of its "
                                                      "group (parity-tested at this shape)"}}
            else:
                r = dcp_line(w, d, args.steps, args.warmup, peaks, per, sub_rank, pgs[g], group=g)
                sub["gla_cfg3"] = summarize_dcp(key, w, d, r, args.steps, peaks, world,
                                                f"{w.groups} head groups x dcp{per}")
                r["ex"].close()
                del r
            for p_ in pgs:
                dist.destroy_process_group(p_)
            torch.cuda.empty_cache()
    sampler.stop()

    if rank == 0:
        traffic = profile_traffic() if world == 1 and len(w1.lens) == 64 else None
        achieved = float(w1.algorithmic_bytes() if world == 1 else total_bytes / world) / (decode_ms * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded), random-init cache in the plugin's row layout",
            "config": {"workload": w1.desc, "batch": len(w1.lens), "heads": w1.heads, "rank": w1.rank,
                       "rope": w1.rope, "rms": w1.heads, "row_bytes_read": w1.row_read, "page_size": w1.page,
                       "sum_context": sum(w1.lens), "parallelism": f"dcp{world}" if world > 1 else "single",
                       **({"dcp_merge": "one kernel over NVLink peer memory (qmla_dcp_p2p_merge), heads scattered "
                                        "over ranks; shards cut from one seeded global cache"} if world > 1 else {}),
                       "timing": "device time over CUDA-graph replays of the step (CUDA events)",
                       "l2": f"inputs larger than L2 ({sum(w1.lens) * w1.row_read / 1e9:.2f} GB of rows), no flush"},
            "seqs_per_s": len(w1.lens) / (step_ms * 1e-3),
            "hbm_frac_of_measured_peak": value * 1e3 / (peaks["hbm_gbs"] * world),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"], "traffic": traffic,
                         "peak_source": f"{peaks['kind']} (MEASURED_PEAKS.json hbm_gbs)",
                         "kernel": "qmla_mla_decode call (plan + persistent decode + split merge)"
                                   + (", rank 0's shard" if world > 1 else "")},
            "parity": (parity_cpu if world == 1 else sub["dcp_cfg1"]["parity"]),
            "cpu_baseline": cpu,
            "gpu_baseline": gpu_base,
            "e2e": {"value": e2e_value, "unit": "TB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    **({"max_abs_vs_graph_timed": e2e_parity} if e2e_parity is not None else {})},
            "clocks": {k: clocks[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")},
            "gpu_launches": launches * args.steps,
            **sub,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        r1["ex"].close()
        d.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of CPU baseline sampling")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gpu-baseline", action="store_true", help="skip timing the reference's Triton kernel")
    ap.add_argument("--no-subs", action="store_true", help="config 1 only (no cfg2/cfg3/cfg4 sub-objects)")
    ap.add_argument("--workload", choices=["cfg1", "gather"], default="cfg1",
                    help="cfg1 (default, the headline line with its sub-objects) or the prefill context gather")
    ap.add_argument("--triton-baseline", choices=["cfg1", "cfg2"], default=None,
                    help=argparse.SUPPRESS)  # child process of triton_child()
    ap.add_argument("--batch", type=int, default=None,
                    help="first N sequences of config1 (smaller cases for ncu captures; default: all 64)")
    ap.add_argument("--profile-case", choices=["cfg1", "cfg2", "cfg3", "cfg4"], default=None,
                    help="only this workload's decode, plain launches (ncu captures); --batch applies")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.triton_baseline:
        run_triton_child(args)
    elif args.profile_case:
        run_profile_case(args)
    elif args.workload == "gather":
        if args.impl == "reference":
            raise SystemExit("--workload gather has no reference arm; its line carries cpu_baseline")
        run_gather(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
