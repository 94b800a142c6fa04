"""Benchmark of the MaxSim hot path on B200 (one process per GPU).

Default workload ("multi-query rerank"): per GPU a shard of 100,000 ragged
documents, N_d ~ U[64, 300] (about 18.2M tokens, one concatenated fp16 token matrix + int64
offsets), d = 128, L2-normalised Gaussian vectors; 64 queries x 32 tokens; each step scores every
query against the shard (tcgen05 kernel), takes the per-query top-1000 and, at N > 1 GPUs, merges
the per-shard top-1000 lists with one NCCL all-gather. Per-GPU work is fixed (weak scaling).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2|c1|c3_256|c3_768|c5]
    python bench.py --impl reference ...   # the reference algorithm on the host CPU cores

Prints ONE JSON line on rank 0. ``value`` = doc-tokens scored per second over all GPUs
(query x document-token pairs, B_q * T / t, the unit of the reference's throughput tables), timed
on the device with CUDA events, max over ranks, inputs resident in HBM. ``e2e`` is the same metric
through the public API with the queries copied from pinned host memory and the top-k results
copied back every step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    # name: (n_queries, nq, d, n_docs per GPU, nd_lo, nd_hi, k)
    "c2": (64, 32, 128, 100_000, 64, 300, 1000),
    "c1": (1, 32, 128, 1_000, 180, 180, 10),
    "c3_256": (16, 32, 256, 50_000, 256, 256, 1000),
    "c3_768": (16, 32, 768, 50_000, 256, 256, 1000),
    "c5": (256, 32, 128, 1_250_000, 96, 160, 100),  # one eighth of the 10M-doc sharded corpus
    # single query, the reference's best-case V2-MQ shape (Nd = 256, B = 100k): HBM-bound
    "q1_nd256": (1, 32, 128, 100_000, 256, 256, 10),
    "q1_ragged": (1, 32, 128, 400_000, 64, 300, 10),
    # reduced corpora for ncu --set full captures (still larger than L2, a few hundred MB)
    "c2_small": (64, 32, 128, 10_000, 64, 300, 1000),
    "q1_small": (1, 32, 128, 20_000, 256, 256, 10),
}


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


# ------------------------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML every 20 ms while running."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device: torch.device):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._h = None
        try:
            import pynvml
            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(device)
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            self._h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._nv = pynvml
        except Exception:  # NVML missing: report no clock record
            self._h = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self._nv.nvmlDeviceGetClockInfo(self._h, self._nv.NVML_CLOCK_SM))
                r = self._nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.reasons.update(v for k, v in self.REASONS.items() if r & k)
            except Exception:
                pass
            self._stop.wait(0.02)

    def __enter__(self):
        if self._h is not None:
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._h is not None:
            self._t.join()

    last_sm_mhz = None

    def summary(self) -> dict | None:
        if self._h is None or not self.samples:
            return None
        ClockSampler.last_sm_mhz = statistics.median(self.samples)
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "samples": len(self.samples), "reasons": sorted(self.reasons)}


# ------------------------------------------------------------------------------------ workload
def make_corpus(n_docs: int, lo: int, hi: int, d: int, seed: int, device: torch.device):
    lengths = np.random.default_rng(seed).integers(lo, hi + 1, n_docs).astype(np.int64)
    off = np.zeros(n_docs + 1, dtype=np.int64)
    np.cumsum(lengths, out=off[1:])
    T = int(off[-1])
    D = torch.empty(T, d, dtype=torch.float16, device=device)
    g = torch.Generator(device=device).manual_seed(seed)
    step = 1 << 22
    for t0 in range(0, T, step):  # N(0,1) in fp32, L2-normalised per token, fp16
        x = torch.randn(min(step, T - t0), d, device=device, generator=g)
        D[t0:t0 + x.shape[0]] = torch.nn.functional.normalize(x, dim=-1).half()
    return D, torch.from_numpy(off).to(device), T


def make_queries(nqry: int, nq: int, d: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(nqry, nq, d, generator=g)
    return torch.nn.functional.normalize(q, dim=-1).half()


# ------------------------------------------------------------------------------------ arms
def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _cpu_sample(cfg, n_s: int):
    """A bounded sample of the workload for the host CPU: 1 query x the first n_s ragged documents
    (same length distribution), padded in chunks as the reference's CPU scorers take them."""
    from oracle import maxsim_oracle as O
    nqry, nq, d, n_docs, lo, hi, k = cfg
    n_s = min(n_docs, n_s)
    lengths = np.random.default_rng(42).integers(lo, hi + 1, n_s).astype(np.int64)
    off = np.zeros(n_s + 1, np.int64)
    np.cumsum(lengths, out=off[1:])
    g = torch.Generator().manual_seed(1)
    D = torch.nn.functional.normalize(torch.randn(int(off[-1]), d, generator=g), dim=-1).half()
    Q = make_queries(1, nq, d, 42)
    return Q, O.pad_chunks_torch(D, off), n_s, int(off[-1])


def _cpu_threads() -> int:
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    torch.set_num_threads(n)
    return torch.get_num_threads()


def cpu_baseline(cfg, seconds: float = 12.0) -> dict:
    """The reference's CPU scoring (torch fp32 einsum -> masked max -> sum, all host cores) on a
    bounded sample: 1 query against the first documents of the shard."""
    from oracle import maxsim_oracle as O
    threads = _cpu_threads()
    Q, chunks, n_s, T = _cpu_sample(cfg, 5000)
    O.maxsim_padded_chunks_torch(Q, chunks, n_s)  # warm-up
    t0 = time.perf_counter()
    reps = 0
    while True:
        O.maxsim_padded_chunks_torch(Q, chunks, n_s)
        reps += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = (time.perf_counter() - t0) / reps
    return {"value": T / dt, "unit": "doc-tokens/s", "cores": threads, "kind": "port",
            "cpu": cpu_model(), "torch_threads": threads,
            "sample": f"1 query x {n_s} ragged docs ({T} tokens, d={cfg[2]}) x {reps} reps, the reference's "
                      "pytorch_maxsim_score / pytorch_maxsim_naive arithmetic in torch fp32 on padded chunks "
                      "of 4096 docs (oracle/maxsim_oracle.py:maxsim_padded_chunks_torch)"}


def run_reference(args, cfg, rank: int) -> None:
    if rank != 0:
        return
    from oracle import maxsim_oracle as O
    threads = _cpu_threads()
    nqry, nq, d, n_docs, lo, hi, k = cfg
    Q, chunks, n_s, T = _cpu_sample(cfg, 3000)
    kk = min(k, n_s)
    for _ in range(args.warmup):
        torch.topk(O.maxsim_padded_chunks_torch(Q, chunks, n_s), kk)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        torch.topk(O.maxsim_padded_chunks_torch(Q, chunks, n_s), kk)
    dt = (time.perf_counter() - t0) / args.steps
    val = T / dt
    sample = (f"per step 1 query x {n_s} ragged docs ({T} tokens, d={d}) + torch.topk {kk}, the reference's "
              "torch fp32 CPU scoring (pytorch_maxsim_score on padded chunks) on all host cores")
    emit_json({
        "impl": "reference", "metric": "doc-tokens scored/s", "value": val, "unit": "doc-tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{args.config} slice: 1 query x {nq} tokens vs {n_s} ragged docs "
                               f"(N_d ~ U[{lo},{hi}], d={d}), top-{kk}; the full config is {nqry} queries x "
                               f"{n_docs} docs per GPU", "n_queries": 1, "nq": nq, "d": d, "docs": n_s,
                   "nd_range": [lo, hi], "k": kk},
        "cpu_baseline": {"value": val, "unit": "doc-tokens/s", "cores": threads, "kind": "port",
                         "cpu": cpu_model(), "torch_threads": threads, "sample": sample},
        "e2e": {"value": val, "unit": "doc-tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0})


def run_reference_pq(args, cfg, rank: int) -> None:
    """Reference ADC algorithm (oracle port: table build + m-ordered lookups + max + sum) on the host
    cores, on a bounded sample of the PQ workload."""
    if rank != 0:
        return
    from oracle import maxsim_oracle as O
    nqry, nq, M, K, dsub, n_docs, nd, k = cfg
    n_s = min(n_docs, 2000)
    rng = np.random.default_rng(42)
    codes = rng.integers(0, K, (n_s * nd, M), dtype=np.uint8)
    off = np.arange(n_s + 1, dtype=np.int64) * nd
    cb = rng.standard_normal((M, K, dsub), dtype=np.float32)
    Q = make_queries(1, nq, M * dsub, 7)
    for _ in range(args.warmup):
        O.topk(O.pq_maxsim_adc_ragged(Q, cb, codes, off)[0], min(k, n_s))
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.topk(O.pq_maxsim_adc_ragged(Q, cb, codes, off)[0], min(k, n_s))
    dt = (time.perf_counter() - t0) / args.steps
    val = n_s * nd / dt
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    emit_json({
        "impl": "reference", "metric": "doc-tokens scored/s", "value": val, "unit": "doc-tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": args.config},
        "cpu_baseline": {"value": val, "unit": "doc-tokens/s", "cores": cores, "kind": "port",
                         "sample": f"per step 1 query x {n_s} docs x {nd} codes, NumPy ADC restatement"},
        "e2e": {"value": val, "unit": "doc-tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0})


def run_reference_res(args, cfg, rank: int) -> None:
    """Residual-compressed scoring on the host cores: the oracle's decompress + MaxSim + top-k (the
    reference names the storage format but has no implementation of this path), on a bounded
    sample of the workload."""
    if rank != 0:
        return
    from oracle import maxsim_oracle as O
    nqry, nq, d, nbits, n_cent, n_docs, nd, k = cfg
    n_s = min(n_docs, 2000)
    rng = np.random.default_rng(42)
    cent = torch.nn.functional.normalize(torch.from_numpy(rng.standard_normal((n_cent, d), dtype=np.float32)),
                                         dim=-1).half()
    codes = rng.integers(0, n_cent, n_s * nd).astype(np.int32)
    res = rng.integers(0, 256, (n_s * nd, d * nbits // 8), dtype=np.uint8)
    off = np.arange(n_s + 1, dtype=np.int64) * nd
    bw = np.linspace(-0.06, 0.06, 1 << nbits, dtype=np.float32)
    Q = make_queries(nqry, nq, d, 7)

    def one():
        D = torch.from_numpy(O.residual_decompress(cent, codes, res, bw, nbits))
        return O.topk(O.maxsim_ragged(Q, D, off), min(k, n_s))

    for _ in range(args.warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one()
    dt = (time.perf_counter() - t0) / args.steps
    val = nqry * n_s * nd / dt
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    emit_json({
        "impl": "reference", "metric": "doc-tokens scored/s", "value": val, "unit": "doc-tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.config},
        "cpu_baseline": {"value": val, "unit": "doc-tokens/s", "cores": cores, "kind": "port",
                         "sample": f"per step {nqry} queries x {n_s} docs x {nd} residual-compressed tokens, "
                                   "NumPy decompress + MaxSim restatement"},
        "e2e": {"value": val, "unit": "doc-tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0})


def config_dict(args, cfg) -> dict:
    nqry, nq, d, n_docs, lo, hi, k = cfg
    return {"workload": f"{args.config}: {nqry} queries x {nq} tokens vs {n_docs} ragged docs per GPU "
                        f"(N_d ~ U[{lo},{hi}], d={d}, fp16), top-{k}",
            "n_queries": nqry, "nq": nq, "d": d, "docs_per_gpu": n_docs, "nd_range": [lo, hi], "k": k,
            "parallelism": f"corpus-sharded x{args.gpus}, NCCL all-gather of per-shard top-k",
            "l2": "inputs larger than L2 (corpus >> 126 MB)" if n_docs * (lo + hi) / 2 * d * 2 > 126e6
                  else "corpus fits in L2"}


# The JSON result line goes to the process's real standard output; everything libraries print on
# file descriptor 1 while the benchmark runs (NCCL's version banner, for one) is sent to standard
# error, so standard output carries exactly one line per run.
_RESULT_FD: int | None = None


def route_library_output_to_stderr() -> None:
    global _RESULT_FD
    if _RESULT_FD is None:
        sys.stdout.flush()
        _RESULT_FD = os.dup(1)
        os.dup2(2, 1)


def emit_json(obj: dict) -> None:
    line = (json.dumps(obj) + "\n").encode()
    sys.stdout.flush()
    os.write(_RESULT_FD if _RESULT_FD is not None else 1, line)


def percentiles(xs: list[float]) -> list[float]:
    """[p50, p95] of per-launch kernel times (this rank's, CUDA events)."""
    ys = sorted(xs)
    pick = lambda q: ys[min(len(ys) - 1, int(round(q * (len(ys) - 1))))]  # noqa: E731
    return [pick(0.5), pick(0.95)]


def topk_launches(rows: int, n: int, k: int) -> int:
    """Kernels one tms_topk call launches (csrc/topk.cu: one sort for n <= 16384, else a slice
    select, plus a merge sort when the row is split into several slices)."""
    if n <= 16384:
        return 1
    c = min(-(-n // 16384), 16384 // k, 1 if rows >= 296 else 296 // rows)
    return 2 if c >= 2 else 1


def search_launches(rows: int, n: int, k: int, world: int, score_launches: int) -> int:
    """Our kernels per search step: scoring, local top-k, and (N > 1) the merge top-k."""
    return score_launches + topk_launches(rows, n, k) + (topk_launches(rows, world * k, k) if world > 1 else 0)


PQ_CONFIGS = {
    # name: (n_queries, nq, M, K, dsub, n_docs per GPU, nd, k) -- BASELINE config 4, scored with
    # the reference's fp32 table arithmetic (TileMaxSimPQ's default, exact=True)
    "c4": (16, 32, 16, 256, 8, 1_000_000, 128, 100),
    "c4_small": (16, 32, 16, 256, 8, 50_000, 128, 100),
    # single-query PQ over the same corpus (the north star's single-query PQ path)
    "q1_pq": (1, 32, 16, 256, 8, 1_000_000, 128, 100),
    "q1_pq_small": (1, 32, 16, 256, 8, 100_000, 128, 100),  # ncu captures (205 MB of codes)
}
# the same workloads on the tensor-core mode (exact=False: codebook rounded to fp16, ~1e-3 relative)
PQ_CONFIGS.update({f"{k}_fast": v for k, v in list(PQ_CONFIGS.items())})


def pq_route(nqry: int, nq: int, M: int, K: int, dsub: int, exact: bool) -> str:
    """The kernel tms_pq_maxsim picks for fp16 queries (csrc/pq_adc.cu routing): "tokrows" (the
    token-rows tensor kernel) for 1-4 chunks of 32 query rows in fast mode, and at the default
    precision (codebook split into hi + lo) in passes of up to four chunks for queries of up to 128
    rows -- except batches of <= 8-token queries that need several passes; else "lut" (table
    lookups) at the default precision or "decoder" (the dense kernel's decoder warps) in fast
    mode."""
    nchunk = -(-nq // 32)
    chunks = nqry * nchunk
    d = M * dsub
    cb = M * K * dsub * 2 * (2 if exact else 1)
    shape_ok = d % 64 == 0 and d <= 256 and dsub % 8 == 0 and K <= 256 and cb <= (128 if exact else 96) * 1024
    if shape_ok and (chunks <= 4 or (exact and nchunk <= 4 and nq >= 9)):
        return "tokrows"  # at the default precision: in passes of up to four chunks
    return "lut" if exact else "decoder"


def pq_score_launches(nqry: int, nq: int, M: int, K: int, dsub: int, exact: bool) -> int:
    """Kernels one PQ scoring call launches: the scoring kernel (+ query packing for the decoder
    kernel) and the partial-sum kernel when a query spans several slices (8 query tokens per table
    slice, 32 per tensor chunk)."""
    route = pq_route(nqry, nq, M, K, dsub, exact)
    if route == "lut":
        return 1 + (1 if nq > 8 else 0)
    if route == "tokrows":
        passes = -(-nqry // (4 // -(-nq // 32))) if exact else 1
        return passes * (1 + (1 if nq > 32 else 0))
    return 2 + (1 if nq > 32 else 0)


def run_pq(args, cfg, rank: int, world: int, device: torch.device, emit: bool = True) -> dict | None:
    """PQ-ADC scoring (TileMaxSimPQ.score_queries) + per-query top-k over uint8 codes."""
    import tilemaxsim_b200 as tms
    from tilemaxsim_b200.sharded import merge_topk
    nqry, nq, M, K, dsub, n_docs, nd, k = cfg
    exact = not args.config.endswith("_fast")
    T = n_docs * nd
    g = torch.Generator(device=device).manual_seed(42 + rank)
    codes = torch.randint(0, K, (T, M), generator=g, device=device, dtype=torch.uint8)
    off = torch.arange(n_docs + 1, device=device, dtype=torch.int64) * nd
    cb = torch.randn(M, K, dsub, generator=torch.Generator().manual_seed(42)).to(device)
    Qh = make_queries(nqry, nq, M * dsub, 7).pin_memory()
    Qd = Qh.to(device)
    pq = tms.TileMaxSimPQ(cb, exact=exact)
    group = dist.group.WORLD if world > 1 else None
    score_ev = []

    def step(Q, timed=False):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        s = pq.score_queries(Q, codes, off)
        e1.record()
        if timed:
            score_ev.append((e0, e1))
        v, i = tms.topk(s, k, id_base=rank * n_docs)
        return merge_topk(v, i, k, group)

    for _ in range(args.warmup):
        step(Qd)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device) as clk:
        start.record()
        for _ in range(args.steps):
            step(Qd, timed=True)
        end.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    kern_list = [a.elapsed_time(b) for a, b in score_ev]
    kern_ms = sum(kern_list) / len(kern_list)
    if world == 1:  # the captured step (see run_ours)
        from tilemaxsim_b200 import GraphedStep
        def plain_step(Q):  # the search step without the timing events
            v, i = tms.topk(pq.score_queries(Q, codes, off), k, id_base=rank * n_docs)
            return merge_topk(v, i, k, group)
        gstep = GraphedStep(plain_step, Qd)
        e2e_call = lambda: gstep(Qh)  # noqa: E731
    else:
        def e2e_call():
            v, i = step(Qh.to(device, non_blocking=True))
            return v.cpu(), i.cpu()
    e2e_call()
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record()
    for _ in range(args.steps):
        e2e_call()
    e_end.record()
    torch.cuda.synchronize()
    e2e_ms = e_start.elapsed_time(e_end) / args.steps
    t_all = torch.tensor([ms, e2e_ms, kern_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t_all, op=dist.ReduceOp.MAX)
    ms, e2e_ms, kern_ms = t_all.tolist()
    if rank != 0:
        return
    T_total = T * world
    pairs = nqry * T_total
    lookups = nqry * nq * T * M  # per GPU per step
    code_bytes = T * M + nqry * n_docs * 4 + M * K * dsub * 4 + nqry * nq * M * dsub * 2
    pk = peaks()
    clocks = clk.summary()
    mhz = ClockSampler.last_sm_mhz or 1965.0
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    hbm = {"achieved_gbs": code_bytes / (kern_ms * 1e-3) / 1e9, "peak_gbs": pk["hbm_gbs"],
           "frac": code_bytes / (kern_ms * 1e-3) / 1e9 / pk["hbm_gbs"]}
    route = pq_route(nqry, nq, M, K, dsub, exact)
    if route == "lut":
        # table lookups: one fp32 entry per (query token, doc token, subspace), read from shared
        # memory; the port moves 128 B per clock per SM = 32 conflict-free 4-byte lookups
        lk_peak = 32.0 * sms * mhz * 1e6
        roof = {"bound": "smem", "achieved": lookups / (kern_ms * 1e-3) / 1e9, "peak": lk_peak / 1e9,
                "unit": "G lookups/s", "frac": lookups / (kern_ms * 1e-3) / lk_peak, "traffic": None,
                "hbm": hbm,
                "note": "fp32 table lookups straight from uint8 codes (reference arithmetic); peak = "
                        "32 lookups/clk/SM (the 128 B/clk shared-memory port) x SMs x median SM clock"}
    else:
        flops = 2.0 * nqry * nq * T * M * dsub * (2 if exact else 1)  # MMA work (hi and lo halves)
        tmem_bytes = 4.0 * nqry * nq * T
        tmem_peak = 56.0 * sms * mhz * 1e6 / 1e9
        # decoding reads one codebook row (dsub fp16) per code from shared memory -- two (hi and lo)
        # at the default precision
        gather_bytes = float(T) * M * dsub * 2 * (2 if exact else 1)
        smem_peak = 128.0 * sms * mhz * 1e6 / 1e9
        # codes decoded in shared memory, MMA on the tensor cores, the epilogue reading every fp32
        # similarity from TMEM (B_q*Nq*T values) -- the same bound as the dense kernel
        roof = {"bound": "tensor", "achieved": flops / (kern_ms * 1e-3) / 1e12,
                "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": flops / (kern_ms * 1e-3) / 1e12 / pk["bf16_tflops"], "traffic": None,
                "hbm": hbm,
                "tmem_read": {"achieved_gbs": tmem_bytes / (kern_ms * 1e-3) / 1e9, "peak_gbs": tmem_peak,
                              "frac": tmem_bytes / (kern_ms * 1e-3) / 1e9 / tmem_peak},
                # decoding reads one codebook row (dsub fp16) per code from shared memory:
                # T*M*dsub*2 bytes per launch at least, against 128 B/clk per SM
                "smem_gather": {"achieved_gbs": gather_bytes / (kern_ms * 1e-3) / 1e9, "peak_gbs": smem_peak,
                                "frac": gather_bytes / (kern_ms * 1e-3) / 1e9 / smem_peak},
                "note": ("codebook split into fp16 hi + lo (reference precision), " if exact else
                         "codebook rounded to fp16 (exact=False), ") + f"{route} kernel; LUT lookups/s "
                        "counts the table-lookup equivalent (B_q*Nq*T*M) of the work"}
    out = {
        "metric": "doc-tokens scored/s", "value": pairs / (ms * 1e-3), "unit": "doc-tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": f"{args.config}: PQ-ADC, {nqry} queries x {nq} tokens vs {n_docs} docs x {nd} "
                               f"uint8 codes per GPU (M={M}, K={K}, dsub={dsub}, fp32 codebook), top-{k}, "
                               + ("reference precision (" + ("hi/lo tensor cores" if route == "tokrows"
                                                            else "fp32 table lookups") + ")" if exact
                                  else "tensor-core mode (fp16 codebook)"),
                   "l2": "codes larger than L2"},
        "queries_per_s": nqry / (ms * 1e-3), "pq_kernel_ms": kern_ms,
        "pq_kernel_ms_p50_p95": percentiles(kern_list),
        "lut_lookups_per_s": lookups / (kern_ms * 1e-3),
        "roofline": roof,
        "e2e": {"value": pairs / (e2e_ms * 1e-3), "unit": "doc-tokens/s", "h2d_bytes_per_step": Qh.numel() * 2,
                "d2h_bytes_per_step": nqry * k * 12, "ms_per_step": e2e_ms},
        "gpu_launches": search_launches(nqry, n_docs, k, world,
                                        pq_score_launches(nqry, nq, M, K, dsub, exact)) * args.steps,
        "clocks": clocks}
    if emit:
        emit_json(out)
    return out


RES_CONFIGS = {
    # name: (n_queries, nq, d, nbits, n_centroids, n_docs per GPU, nd, k): a ColBERTv2-style
    # residual-compressed corpus (centroid id + 2-bit residuals, 36 bytes per token)
    "q1_res": (1, 32, 128, 2, 65536, 1_000_000, 128, 100),
    "q5_res": (5, 32, 128, 2, 65536, 1_000_000, 128, 100),
    # small case for ncu captures (codes + residuals 230 MB, still larger than L2)
    "q1_res_small": (1, 32, 128, 2, 65536, 50_000, 128, 100),
}


def res_score_launches(nqry: int, nq: int) -> int:
    """Kernels one residual scoring call launches (csrc/dense_maxsim.cu tms_residual_maxsim)."""
    nchunk = -(-nq // 32)
    return (1 + (1 if nchunk > 1 else 0)) if nqry * nchunk <= 4 else 2


def run_res(args, cfg, rank: int, world: int, device: torch.device) -> None:
    """Residual-compressed scoring (ResidualMaxSim.score_queries) + per-query top-k."""
    import tilemaxsim_b200 as tms
    from tilemaxsim_b200.sharded import merge_topk
    nqry, nq, d, nbits, n_cent, n_docs, nd, k = cfg
    T = n_docs * nd
    g = torch.Generator(device=device).manual_seed(42 + rank)
    cent = torch.nn.functional.normalize(torch.randn(n_cent, d, generator=g, device=device), dim=-1).half()
    codes = torch.randint(0, n_cent, (T,), generator=g, device=device, dtype=torch.int32)
    res = torch.randint(0, 256, (T, d * nbits // 8), generator=g, device=device, dtype=torch.uint8)
    off = torch.arange(n_docs + 1, device=device, dtype=torch.int64) * nd
    bw = torch.linspace(-0.06, 0.06, 1 << nbits, device=device)
    Qh = make_queries(nqry, nq, d, 7).pin_memory()
    Qd = Qh.to(device)
    scorer = tms.ResidualMaxSim(cent, bw, nbits)
    group = dist.group.WORLD if world > 1 else None
    score_ev = []

    def step(Q, timed=False):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        s = scorer.score_queries(Q, codes, res, off)
        e1.record()
        if timed:
            score_ev.append((e0, e1))
        v, i = tms.topk(s, k, id_base=rank * n_docs)
        return merge_topk(v, i, k, group)

    for _ in range(args.warmup):
        step(Qd)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device) as clk:
        start.record()
        for _ in range(args.steps):
            step(Qd, timed=True)
        end.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    kern_list = [a.elapsed_time(b) for a, b in score_ev]
    kern_ms = sum(kern_list) / len(kern_list)
    if world == 1:  # the captured step (see run_ours)
        from tilemaxsim_b200 import GraphedStep
        def plain_step(Q):
            v, i = tms.topk(scorer.score_queries(Q, codes, res, off), k, id_base=rank * n_docs)
            return merge_topk(v, i, k, group)
        gstep = GraphedStep(plain_step, Qd)
        e2e_call = lambda: gstep(Qh)  # noqa: E731
    else:
        def e2e_call():
            v, i = step(Qh.to(device, non_blocking=True))
            return v.cpu(), i.cpu()
    e2e_call()
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record()
    for _ in range(args.steps):
        e2e_call()
    e_end.record()
    torch.cuda.synchronize()
    e2e_ms = e_start.elapsed_time(e_end) / args.steps
    t_all = torch.tensor([ms, e2e_ms, kern_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t_all, op=dist.ReduceOp.MAX)
    ms, e2e_ms, kern_ms = t_all.tolist()
    if rank != 0:
        return
    pairs = nqry * T * world
    pk = peaks()
    # algorithmic bytes per launch: codes + residual rows + offsets + scores (the centroid table,
    # 16 MB, is read through L2)
    hbm_bytes = T * (4 + d * nbits // 8) + (n_docs + 1) * 8 + nqry * n_docs * 4
    clocks = clk.summary()
    emit_json({
        "metric": "doc-tokens scored/s", "value": pairs / (ms * 1e-3), "unit": "doc-tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": f"{args.config}: residual-compressed corpus, {nqry} queries x {nq} tokens vs "
                               f"{n_docs} docs x {nd} tokens per GPU (d={d}, nbits={nbits}, {n_cent} centroids, "
                               f"normalised), top-{k}",
                   "l2": "codes and residuals larger than L2"},
        "residual_kernel_ms": kern_ms, "residual_kernel_ms_p50_p95": percentiles(kern_list),
        # up to four query chunks: the token-rows kernel (decoded tokens written to TMEM as the MMA's
        # A operand), bound by its TMEM traffic and the decode; the compressed corpus streams at a
        # fraction of HBM bandwidth
        "roofline": {"bound": "hbm", "achieved": hbm_bytes / (kern_ms * 1e-3) / 1e9, "peak": pk["hbm_gbs"],
                     "unit": "GB/s", "frac": hbm_bytes / (kern_ms * 1e-3) / 1e9 / pk["hbm_gbs"], "traffic": None,
                     "note": "decode / TMEM bound, not HBM bound"},
        "e2e": {"value": pairs / (e2e_ms * 1e-3), "unit": "doc-tokens/s", "h2d_bytes_per_step": Qh.numel() * 2,
                "d2h_bytes_per_step": nqry * k * 12, "ms_per_step": e2e_ms},
        # per scoring call: the token-rows kernel (+ the chunk sum for > 32-token queries) for up to
        # four query chunks, else packing + the decoder kernel; then the top-k (and merge) kernels
        "gpu_launches": search_launches(nqry, n_docs, k, world, res_score_launches(nqry, nq)) * args.steps,
        "clocks": clocks})


def run_ours(args, cfg, rank: int, world: int, device: torch.device, emit: bool = True) -> dict | None:
    import tilemaxsim_b200 as tms
    from tilemaxsim_b200 import _lib
    from tilemaxsim_b200.sharded import ShardedIndex
    nqry, nq, d, n_docs, lo, hi, k = cfg
    D, off, T = make_corpus(n_docs, lo, hi, d, seed=42 + rank, device=device)
    Qh = make_queries(nqry, nq, d, 7).pin_memory()
    Qd = Qh.to(device)
    index = ShardedIndex(D, off, doc_id_base=rank * n_docs, group=dist.group.WORLD if world > 1 else None)
    torch.cuda.synchronize()

    def step(Q):
        return index.search(Q, k)

    dense_ev = []

    def step_timed(Q):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        scores = tms.maxsim_batched(Q, D, off)
        e1.record()
        dense_ev.append((e0, e1))
        return index.search_scores(scores, k)

    for _ in range(args.warmup):
        step_timed(Qd)
    torch.cuda.synchronize()
    dense_ev.clear()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device) as clk:
        start.record()
        for _ in range(args.steps):
            step_timed(Qd)
        end.record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end) / args.steps
    dense_list = [a.elapsed_time(b) for a, b in dense_ev]
    dense_ms = sum(dense_list) / len(dense_list)

    # e2e: public API with host queries in pinned memory and results copied back, every step. On
    # one GPU the step is the captured graph (tilemaxsim_b200.GraphedStep); across GPUs the step
    # holds an NCCL all-gather and runs eagerly.
    if world == 1:
        from tilemaxsim_b200 import GraphedStep
        gstep = GraphedStep(lambda Q: index.search(Q, k), Qd)
        e2e_call = lambda: gstep(Qh)  # noqa: E731
    else:
        def e2e_call():
            v, i = step(Qh.to(device, non_blocking=True))
            return v.to("cpu"), i.to("cpu")
    for _ in range(max(1, args.warmup // 2)):
        e2e_call()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record()
    for _ in range(args.steps):
        e2e_call()
    e_end.record()
    torch.cuda.synchronize()
    e2e_ms = e_start.elapsed_time(e_end) / args.steps

    t_all = torch.tensor([ms, e2e_ms, dense_ms, float(T)], dtype=torch.float64, device=device)
    per_rank = [t_all.tolist()]
    if world > 1:
        g_all = torch.empty(world, 4, dtype=torch.float64, device=device)
        dist.all_gather_into_tensor(g_all, t_all)
        per_rank = g_all.tolist()
        mx = t_all.clone()
        dist.all_reduce(mx[:3], op=dist.ReduceOp.MAX)
        tot = t_all[3:].clone()
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        t_all = torch.cat([mx[:3], tot])
    ms, e2e_ms, dense_ms, T_total = t_all.tolist()
    if rank != 0:
        return
    clocks = clk.summary()

    pairs = nqry * T_total
    value = pairs / (ms * 1e-3)
    pk = peaks()
    flops_launch = 2.0 * nqry * nq * (T_total / world) * d
    bytes_launch = (T_total / world) * d * 2 + nqry * nq * d * 2 + nqry * n_docs * 4 + (n_docs + 1) * 8
    tensor_bound = nqry * nq >= 256
    if tensor_bound:
        ach = flops_launch / (dense_ms * 1e-3) / 1e12
        peak, unit = pk["bf16_tflops"], "TFLOP/s"  # burst: an ~11 ms launch in a sub-second loop
    else:
        ach = bytes_launch / (dense_ms * 1e-3) / 1e9
        peak, unit = pk["hbm_gbs"], "GB/s"
    # The epilogue reads every fp32 similarity once from TMEM: B_q*Nq*T values per launch. TMEM ->
    # register bandwidth measured at ~56 B/clk per SM with a tcgen05.ld microbenchmark.
    tmem_bytes = 4.0 * nqry * nq * (T_total / world)
    clk = ClockSampler.last_sm_mhz or 1965.0
    tmem_peak = 56.0 * torch.cuda.get_device_properties(device).multi_processor_count * clk * 1e6 / 1e9
    traffic = None
    tf = ROOT / "profiles" / f"dense_maxsim_{args.config}_traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get("dram_bytes_per_launch")
    # query packing + the dense kernel (+ the chunk sum for Nq > 32), then the top-k kernels
    launches_per_step = search_launches(nqry, n_docs, k, world, 2 + (1 if nq > 32 else 0))
    out = {
        "metric": "doc-tokens scored/s", "value": value, "unit": "doc-tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": config_dict(args, cfg),
        "queries_per_s": nqry / (ms * 1e-3),
        "corpus_tokens_per_s": T_total / (ms * 1e-3),
        "dense_kernel_ms": dense_ms,
        "dense_kernel_ms_p50_p95": percentiles(dense_list),
        # per rank: (step ms, scoring kernel ms); the slowest rank sets the step time
        "per_rank_ms": [{"step": r[0], "kernel": r[2]} for r in per_rank],
        "dense_hbm_gbs": bytes_launch / (dense_ms * 1e-3) / 1e9,
        "dense_tflops": flops_launch / (dense_ms * 1e-3) / 1e12,
        "roofline": {"bound": "tensor" if tensor_bound else "hbm", "achieved": ach, "peak": peak, "unit": unit,
                     "frac": ach / peak, "traffic": traffic,
                     "peak_src": f"{pk['src']} ({'bf16_tflops' if tensor_bound else 'hbm_gbs'})",
                     "algorithmic": {"flops_per_launch": flops_launch, "bytes_per_launch": bytes_launch},
                     "tmem_read": {"achieved_gbs": tmem_bytes / (dense_ms * 1e-3) / 1e9, "peak_gbs": tmem_peak,
                                   "frac": tmem_bytes / (dense_ms * 1e-3) / 1e9 / tmem_peak,
                                   "note": "epilogue reads B_q*Nq*T fp32 values from TMEM; peak = 56 B/clk/SM ("
                                           "tcgen05.ld microbenchmark) x SMs x median SM clock"}},
        "e2e": {"value": pairs / (e2e_ms * 1e-3), "unit": "doc-tokens/s",
                "h2d_bytes_per_step": Qh.numel() * Qh.element_size(),
                "d2h_bytes_per_step": nqry * k * (4 + 8), "ms_per_step": e2e_ms},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
    }
    if world == 1 and args.config == "c5":
        out["bounded_memory_topk"] = chunked_topk_times(Qd, D, off, k, n_docs)
    if emit and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(cfg)
    if emit and world == 1 and args.config == "c2" and not args.no_legs:
        out["legs"] = run_legs(args, device)
    if emit:
        emit_json(out)
    return out


def chunked_topk_times(Q, D, off, k: int, n_docs: int, reps: int = 3) -> dict:
    """The bounded-memory search (tms_dense_maxsim_topk: documents scored a chunk at a time into
    one reused buffer, each chunk's top-k merged into a running list) against the full-matrix
    path timed above (whole (B_q, n) score matrix, then one top-k): device time per search and
    the score buffer each holds."""
    import tilemaxsim_b200 as tms
    res = {}
    for chunk in (n_docs // 10, n_docs // 2):
        tms.maxsim_topk(Q, D, off, k, chunk_docs=chunk)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            tms.maxsim_topk(Q, D, off, k, chunk_docs=chunk)
        e1.record()
        torch.cuda.synchronize()
        res[f"chunk_docs={chunk}"] = {"ms": e0.elapsed_time(e1) / reps,
                                      "score_buffer_mb": Q.shape[0] * chunk * 4 / 2**20}
    res["full_matrix_score_buffer_mb"] = Q.shape[0] * n_docs * 4 / 2**20
    return res


LEGS = ("q1_ragged", "c3_768", "c4")
LEG_KEYS = ("metric", "value", "unit", "ms_per_step", "dtype", "config", "roofline", "e2e", "clocks",
            "dense_kernel_ms", "pq_kernel_ms", "queries_per_s", "gpu_launches")


def run_legs(args, device: torch.device) -> dict:
    """The north star's other single-GPU targets, measured in the same run as the headline line:
    single-query dense over 400k ragged docs (HBM-bound), the d = 768 sweep (config 3) and PQ at
    the reference's precision (config 4). Each leg has its own timing, roofline and clock record."""
    legs = {}
    for name in LEGS:
        sub = argparse.Namespace(**vars(args))
        sub.config = name
        sub.steps = min(args.steps, 10)
        sub.warmup = 3
        torch.cuda.empty_cache()
        if name in PQ_CONFIGS:
            r = run_pq(sub, PQ_CONFIGS[name], 0, 1, device, emit=False)
        else:
            r = run_ours(sub, CONFIGS[name], 0, 1, device, emit=False)
        legs[name] = {k: r[k] for k in LEG_KEYS if k in r}
        legs[name]["steps"] = sub.steps
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    return legs


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS) + sorted(PQ_CONFIGS) + sorted(RES_CONFIGS), default="c2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-legs", action="store_true",
                    help="c2 on one GPU: skip the single-query, d=768 and PQ legs")
    args = ap.parse_args()
    route_library_output_to_stderr()
    args.warmup = max(3, args.warmup)
    cfg = CONFIGS.get(args.config) or PQ_CONFIGS.get(args.config) or RES_CONFIGS[args.config]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        if args.config in PQ_CONFIGS:
            run_reference_pq(args, cfg, rank)
        elif args.config in RES_CONFIGS:
            run_reference_res(args, cfg, rank)
        else:
            run_reference(args, cfg, rank)
        return 0
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        dist.init_process_group("nccl", device_id=device)
    try:
        if args.config in PQ_CONFIGS:
            run_pq(args, cfg, rank, world, device)
        elif args.config in RES_CONFIGS:
            run_res(args, cfg, rank, world, device)
        else:
            run_ours(args, cfg, rank, world, device)
    finally:
        if world > 1:
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
