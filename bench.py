#!/usr/bin/env python
"""Throughput of the GraphKV compression path on B200: quantize+pack and
dequant of a Qwen2.5-7B-shaped 32k-token bf16 cache (28 layers x 4 kv-heads x
head_dim 128, graphkv profile with importance scores: sink/tail/top-1% kept,
symmetric int4, 35% cold tier with Hadamard-rotated int2 values).

One step = selection + quantize+pack of the whole cache, then dequant of the
whole cache back to [B, H, T, D] bf16.  ``value`` is GB/s of input cache
(K+V bytes) per step with inputs resident in HBM; ``phases`` gives each phase
against the HBM roofline (algorithmic bytes = bytes read + bytes written).

N GPUs (torchrun), headline: weak scaling.  The global cache is the same model
with batch N; its 28 x 4 (layer, kv-head) units are sharded contiguously over
the ranks, each unit holding all N batch rows, so every rank compresses exactly
the work of one 32k cache.  ``strong`` (second leg, on by default): the
8 x 131072-token cache (60 GB of K+V) split over the N ranks by the same units
-- strong scaling of one fixed cache.  No collective runs inside a timed step;
after the timed steps one all-gather of per-layer byte and token counts
rebuilds the whole cache's stats() and one more gathers each rank's phase times.

``--impl reference`` times the CPU port of the reference algorithm (the numpy
oracle) on the host cores, on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOAD = "qwen7b-32k"
STRONG_WORKLOAD = "qwen7b-8x131k"
METRIC = "KV quant+pack and dequant GB/s (% HBM peak), Qwen2.5-7B-shape 32k cache"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default=WORKLOAD)
    ap.add_argument("--strong-workload", default=STRONG_WORKLOAD,
                    help="cache split over the ranks for the strong-scaling leg ('' to skip)")
    ap.add_argument("--strong-steps", type=int, default=12)
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--append", type=int, default=1, help="time QuantizedKvCache.append (0: skip)")
    ap.add_argument("--layers", type=int, default=0, help="use only the first N layers (profiling case)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# CPU side: the oracle port on a bounded sample (process pool, spawn)
# ---------------------------------------------------------------------------

def _oracle_slice(args):
    """Quantize + dequantize one (layer, head) slice with the numpy oracle."""
    wkey, layer, head = args
    from graphkv_b200.workloads import WORKLOADS, make_layer, make_scores
    from oracle import graphkv_oracle as orc

    w = WORKLOADS[wkey]
    k, v = make_layer(w, layer, heads=range(head, head + 1), batch=range(1))
    s = make_scores(w)
    K, V = k.float().numpy(), v.float().numpy()
    sn = s.numpy() if s is not None else None
    t0 = time.perf_counter()
    ql = orc.quantize_layer(K, V, "bf16" if w.dtype.itemsize == 2 else "f32", orc.POLICIES[w.profile], sn)
    orc.dequantize_layer(ql)
    return time.perf_counter() - t0, 2 * K.size * w.dtype.itemsize


def cpu_sample(wkey, n_slices, workers):
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    jobs = [(wkey, i % 28, (i // 28) % 4) for i in range(n_slices)]
    with ctx.Pool(workers) as pool:
        pool.map(_oracle_slice, jobs[:workers])  # import / page-in warm-up
        t0 = time.perf_counter()
        res = pool.map(_oracle_slice, jobs)
        wall = time.perf_counter() - t0
    nbytes = sum(r[1] for r in res)
    return nbytes / wall / 1e9, wall, nbytes


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    workers = os.cpu_count() or 1
    per_step = workers  # one (layer, head) slice of the 32k cache per worker per step
    # size each step so the whole run stays within a few minutes (~0.65 s per slice round trip)
    total_budget = 150.0
    est = 0.65 * math.ceil(per_step / workers)
    steps_total = args.steps + args.warmup
    if est * steps_total > total_budget:
        per_step = max(1, int(workers * total_budget / (0.65 * steps_total)))
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    times, nbytes = [], 0
    with ctx.Pool(workers) as pool:
        for step in range(steps_total):
            jobs = [(args.workload, (step * per_step + i) % 28, ((step * per_step + i) // 28) % 4)
                    for i in range(per_step)]
            t0 = time.perf_counter()
            res = pool.map(_oracle_slice, jobs)
            dt = time.perf_counter() - t0
            if step >= args.warmup:
                times.append(dt)
                nbytes += sum(r[1] for r in res)
    total = sum(times)
    value = nbytes / total / 1e9
    sample = (f"{per_step} (layer, kv-head) slices [1, 1, 32768, 128] bf16 per step, one per process, "
              f"quantize+pack then dequant with the numpy port of the reference algorithm")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / max(len(times), 1), 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": args.workload, "device": "host CPU", "sample": sample},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": workers, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ---------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------

class ClockSampler:
    """NVML clocks and clock-event reasons sampled every 20 ms while running."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting",
               0x1: "gpu_idle"}

    def __init__(self, index):
        self.samples, self.reasons, self.ok = [], set(), False
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            import torch

            try:  # CUDA ordinal -> NVML index (honours CUDA_VISIBLE_DEVICES)
                index = torch.cuda._get_nvml_device_index(index)
            except Exception:
                pass
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # NVML unavailable: report nothing rather than guess
            self.max_mhz = None
        self._stop = threading.Event()

    def _run(self):
        get_reasons = getattr(self.nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            self.nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = get_reasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.02)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def committed_traffic(workload):
    """DRAM bytes per launch from the committed ncu summary, if present."""
    path = os.path.join(ROOT, "profiles", f"dram_traffic_{workload}.txt")
    out = {}
    if os.path.exists(path):
        for line in open(path):
            parts = line.split()
            if len(parts) == 2 and not line.startswith("#"):
                try:
                    out[parts[0]] = float(parts[1])
                except ValueError:
                    pass
    return out


class Dist:
    """Rank bookkeeping; every collective below is issued by every rank in the
    same order, outside the timed steps."""

    def __init__(self):
        import torch

        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            from datetime import timedelta

            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=self.dev)

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier()

    def gather(self, values):
        """All ranks' float vectors, [world][len] (one all-gather)."""
        import torch

        t = torch.tensor(values, dtype=torch.float64, device=self.dev)
        if self.world == 1:
            return [values]
        import torch.distributed as dist

        out = torch.empty(self.world * t.numel(), dtype=torch.float64, device=self.dev)
        dist.all_gather_into_tensor(out, t)
        return out.view(self.world, -1).tolist()

    def close(self):
        if self.world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


def time_compression(d: Dist, w, mode: str, steps: int, warmup: int, with_clocks: bool = False):
    """Prepare this rank's shard of workload `w` on the device and time `steps`
    select + quantize + dequant steps.  mode "weak": the cache has batch
    world * B and every rank holds a whole cache's worth of units; "strong": the
    cache is `w` itself, its units split over the ranks."""
    from dataclasses import replace

    import torch

    import graphkv_b200 as g
    from graphkv_b200 import _lib
    from graphkv_b200.engine import CompressionEngine
    from graphkv_b200.sharding import STAT_FIELDS, gather_stat_rows, piece_stat_row, shard_units, stats_from_rows
    from graphkv_b200.workloads import make_layer, make_scores

    wx = replace(w, batch=w.batch * d.world) if mode == "weak" else w
    shard = shard_units(w.layers, w.heads, d.world, d.rank)
    pairs = [make_layer(wx, l, device=str(d.dev), heads=range(h0, h1)) for (l, h0, h1) in shard]
    scores = make_scores(w, device=str(d.dev))
    cfg = g.get_profile(w.profile).config
    in_bytes = sum(k.numel() * k.element_size() * 2 for k, _ in pairs)
    eng = CompressionEngine(pairs, cfg, scores)
    local = eng.cache()
    rows = torch.zeros(w.layers, len(STAT_FIELDS), dtype=torch.int64)
    for lay, (l, h0, _) in zip(local.layers, shard):
        rows[l] += torch.tensor(piece_stat_row(lay, h0), dtype=torch.int64)
    comp_bytes = int(rows[:, 0].sum())
    launches = eng.launches_per_step()
    stream = torch.cuda.current_stream(d.dev)
    work = [(it[1], it[2], it[3]) for it in eng.items if it[0] == "run"]
    nr = len(work)

    def step(ev=None):
        # ev[i] = 4 events per run: before select, after select, after quantize, after dequantize
        for i, (run, s, needs_select) in enumerate(work):
            if ev is not None:
                ev[i][0].record(stream)
            if needs_select:
                run.select(s)
            if ev is not None:
                ev[i][1].record(stream)
            run.quantize()
            if ev is not None:
                ev[i][2].record(stream)
        for i, (run, _, _) in enumerate(work):
            run.dequantize()
            if ev is not None:
                ev[i][3].record(stream)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(d.dev)
    assert _lib.device_error() == 0
    d.barrier()
    torch.cuda.synchronize(d.dev)
    evs = [[[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(nr)] for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(d.local) if with_clocks else None
    if clocks:
        clocks.__enter__()
    start.record(stream)
    for s in range(steps):
        step(evs[s])
    end.record(stream)
    torch.cuda.synchronize(d.dev)
    if clocks:
        clocks.__exit__()
    d.barrier()
    elapsed_ms = start.elapsed_time(end)
    t_sel = t_q = t_dq = 0.0
    for e in evs:
        for i in range(nr):
            t_sel += e[i][0].elapsed_time(e[i][1])
            t_q += e[i][1].elapsed_time(e[i][2])
            t_dq += (e[nr - 1][2] if i == 0 else e[i - 1][3]).elapsed_time(e[i][3])
    assert _lib.device_error() == 0
    # after the timed steps: per-rank phase times and the whole cache's stats (one all-gather each)
    per_rank = d.gather([elapsed_ms / steps, t_sel / steps, t_q / steps, t_dq / steps,
                         float(in_bytes), float(comp_bytes)])
    stats = stats_from_rows(gather_stat_rows(rows, device=d.dev))
    del eng, local, pairs, work
    torch.cuda.empty_cache()
    return {"per_rank": per_rank, "stats": stats, "launches": launches, "nr": nr,
            "clocks": clocks.summary() if clocks else None, "in_bytes": in_bytes, "comp_bytes": comp_bytes}


def bind_host_to_gpu(dev):
    """Run this process on the CPUs local to the GPU's PCIe attachment, so that the
    pinned host buffers allocated next land in that NUMA node's memory; returns
    (previous CPU set, description), or (None, None) when the topology is not
    visible."""
    import torch

    p = torch.cuda.get_device_properties(dev)
    base = f"/sys/bus/pci/devices/{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
    try:
        with open(f"{base}/local_cpulist") as f:
            spec = f.read().strip()
        with open(f"{base}/numa_node") as f:
            node = int(f.read().strip())
    except (OSError, ValueError):
        return None, None
    cpus = set()
    for part in spec.split(","):
        if part:
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
    before = os.sched_getaffinity(0)
    use = cpus & before
    if not use:
        return None, None
    os.sched_setaffinity(0, use)
    return before, {"numa_node": node, "cpus": len(use)}


def copy_ceiling(host_pairs, dev) -> list:
    """GB/s of plain copies of this rank's pinned cache: host to device alone,
    device to host alone, and both at once on two streams (bytes of both
    directions / time) -- the ceiling the end-to-end figure is measured against.
    Every rank copies at the same time, so the figures show what the ranks'
    shared host memory and PCIe links give each of them."""
    import torch

    hosts = [h for pair in host_pairs for h in pair]
    nbytes = sum(h.numel() * h.element_size() for h in hosts)
    dst = [torch.empty_like(h, device=dev) for h in hosts]
    src = [torch.empty_like(h, device=dev) for h in hosts]
    back = [torch.empty_like(h, pin_memory=True) for h in hosts]
    s1, s2 = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def timed(fns):
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        for st, fn in fns:
            with torch.cuda.stream(st):
                fn()
        torch.cuda.synchronize(dev)
        return time.perf_counter() - t0

    def h2d():
        for h, x in zip(hosts, dst):
            x.copy_(h, non_blocking=True)

    def d2h():
        for b, x in zip(back, src):
            b.copy_(x, non_blocking=True)

    timed([(s1, h2d), (s2, d2h)])  # warm-up
    t_h2d = timed([(s1, h2d)])
    t_d2h = timed([(s2, d2h)])
    t_both = timed([(s1, h2d), (s2, d2h)])
    del dst, src, back
    torch.cuda.empty_cache()
    return [nbytes / t_h2d / 1e9, nbytes / t_d2h / 1e9, 2 * nbytes / t_both / 1e9]


def time_selection(dev, T: int, scores, reps: int = 20) -> float:
    """Device ms of one gkv_select_tiers call (graphkv profile) on fp32 [T] scores."""
    import ctypes

    import torch

    import graphkv_b200 as g
    from graphkv_b200 import _lib as L
    from graphkv_b200.config import resolve_tiers

    tiers = resolve_tiers(g.get_profile("graphkv").config, T, True)
    idx = torch.empty(T, dtype=torch.int32, device=dev)
    r, s, c = torch.split(idx, [tiers.n_retained, tiers.n_standard, tiers.n_cold])
    ws = torch.empty(int(L.lib().gkv_select_workspace_bytes(T)), dtype=torch.uint8, device=dev)
    pol = tiers.policy()
    st = L.stream_handle(dev)

    def call():
        L.check(L.lib().gkv_select_tiers(scores.data_ptr(), None, ctypes.byref(pol), r.data_ptr(), s.data_ptr(),
                                         c.data_ptr(), ws.data_ptr(), ws.numel(), st))

    for _ in range(3):
        call()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(torch.cuda.current_stream(dev))
    for _ in range(reps):
        call()
    b.record(torch.cuda.current_stream(dev))
    torch.cuda.synchronize(dev)
    return a.elapsed_time(b) / reps


def selection_report(dev) -> dict:
    """Selection times: log-normal scores, and scores tied across 64-token chunks
    (what graph-memory requests produce), where both boundaries fall inside runs
    of equal scores and the selection takes its exact tie path."""
    import torch

    out = {}
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    for T in (32768, 131072):
        plain = torch.exp(2.0 * torch.randn(T, generator=gen, device=dev))
        chunks = torch.randint(0, 16, (T // 64,), generator=gen, device=dev).float()
        tied = chunks.repeat_interleave(64).contiguous()
        out[f"{T}"] = {"lognormal_ms": round(time_selection(dev, T, plain), 4),
                       "chunk_ties_ms": round(time_selection(dev, T, tied), 4)}
    return out


def append_report(d, w) -> dict:
    """On the whole compressed cache: device ms of one decode step of attention
    read from the packed codes (against dequantize + fp32 attention), and of
    QuantizedKvCache.append of 1 and of 1024 new tokens (the old tokens are
    dequantized into the grown buffers and everything is requantized, as the
    reference's append does)."""
    import torch

    import graphkv_b200 as g
    from graphkv_b200.sharding import shard_units
    from graphkv_b200.workloads import make_layer, make_scores

    cfg = g.get_profile(w.profile).config
    shard = shard_units(w.layers, w.heads, 1, 0)
    pairs = [make_layer(w, l, device=str(d.dev), heads=range(h0, h1)) for (l, h0, h1) in shard]
    scores = make_scores(w, device=str(d.dev))
    cache = g.QuantizedKvCache.from_past_key_values(pairs, cfg, scores)
    del pairs
    out = {}
    gen = torch.Generator(device=d.dev)
    gen.manual_seed(11)
    # one decode step of attention (1 query per kv-head) over every layer: read from
    # the packed codes, against dequantize + fp32 attention
    B, H, T, D = cache.layers[0].original_shape
    queries = [torch.randn(B, H, 1, D, generator=gen, device=d.dev) for _ in cache.layers]

    def fused():
        for q, lay in zip(queries, cache.layers):
            g.attention_from_quantized(q, lay)

    def unfused():
        for q, lay in zip(queries, cache.layers):
            k, v = lay.dequantize()
            g.attention_from_kv(q, k, v)

    for name, fn in (("fused_ms", fused), ("dequantize_then_attend_ms", unfused)):
        for _ in range(2):
            fn()
        torch.cuda.synchronize(d.dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(5):
            fn()
        b.record()
        torch.cuda.synchronize(d.dev)
        out.setdefault("decode_attention", {})[name] = round(a.elapsed_time(b) / 5, 3)
    # the same 28 layer calls replayed from a CUDA graph: the kernels' device time
    # without the Python calls between them
    try:
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(d.dev)
        side.wait_stream(torch.cuda.current_stream(d.dev))
        with torch.cuda.stream(side):
            fused()
            torch.cuda.synchronize(d.dev)
            with torch.cuda.graph(graph, stream=side):
                fused()
        torch.cuda.current_stream(d.dev).wait_stream(side)
        graph.replay()
        torch.cuda.synchronize(d.dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(20):
            graph.replay()
        b.record()
        torch.cuda.synchronize(d.dev)
        out["decode_attention"]["fused_graph_ms"] = round(a.elapsed_time(b) / 20, 4)
        del graph
    except RuntimeError as e:  # capture unsupported here: report why
        out["decode_attention"]["fused_graph_ms"] = None
        out["decode_attention"]["graph_note"] = str(e)[:120]
    out["decode_attention"]["compressed_bytes"] = cache.memory_bytes()
    for n in (1, 1024):
        B, H, T, D = cache.layers[0].original_shape
        new = [(torch.randn(B, H, n, D, generator=gen, device=d.dev).to(w.dtype),
                torch.randn(B, H, n, D, generator=gen, device=d.dev).to(w.dtype)) for _ in cache.layers]
        s_new = torch.cat([scores, torch.exp(2.0 * torch.randn(n, generator=gen, device=d.dev))])
        for _ in range(2):
            cache.append(new, cfg, s_new)
        torch.cuda.synchronize(d.dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        reps = 5
        for _ in range(reps):
            cache.append(new, cfg, s_new)
        b.record()
        torch.cuda.synchronize(d.dev)
        out[f"tokens_{n}_ms"] = round(a.elapsed_time(b) / reps, 3)
    del cache
    torch.cuda.empty_cache()
    return out


def phase_report(res, peak):
    """Max-over-ranks phase times and their roofline fractions (per-rank bytes)."""
    pr = res["per_rank"]
    worst = max(range(len(pr)), key=lambda r: pr[r][0])
    ms = max(r[0] for r in pr)
    sel, q, dq = (max(r[i] for r in pr) for i in (1, 2, 3))
    in_b, comp_b = pr[worst][4], pr[worst][5]
    algo = in_b + comp_b
    return ms, {
        "select": {"ms": round(sel, 4)},
        "quantize": {"ms": round(q, 4), "input_gbs": round(in_b / q / 1e6, 1), "algo_gbs": round(algo / q / 1e6, 1),
                     "frac": round(algo / q / 1e6 / peak, 4)},
        "dequant": {"ms": round(dq, 4), "input_gbs": round(in_b / dq / 1e6, 1),
                    "algo_gbs": round(algo / dq / 1e6, 1), "frac": round(algo / dq / 1e6 / peak, 4)},
    }


def run_ours(args):
    import torch

    import graphkv_b200 as g
    from dataclasses import replace
    from graphkv_b200.workloads import WORKLOADS, make_layer, make_scores

    d = Dist()
    peak, peak_kind = measured_peak()
    w = WORKLOADS[args.workload]
    if args.layers:
        w = replace(w, layers=args.layers)

    # --- headline: weak scaling of the 32k cache ------------------------------------
    head = time_compression(d, w, "weak", args.steps, args.warmup, with_clocks=True)
    ms, phases = phase_report(head, peak)
    in_bytes_rank = head["in_bytes"]

    select_times = selection_report(d.dev) if d.rank == 0 else None
    append_times = append_report(d, w) if d.rank == 0 and args.append else None

    # --- strong scaling of the 8 x 131k (60 GB) cache ---------------------------------
    strong = None
    if args.strong_workload:
        ws = WORKLOADS[args.strong_workload]
        from graphkv_b200.sharding import shard_units

        units = shard_units(ws.layers, ws.heads, d.world, d.rank)
        unit_bytes = ws.batch * ws.seq * ws.head_dim * ws.dtype.itemsize * 2  # K+V of one (layer, head)
        need = sum(h1 - h0 for _, h0, h1 in units) * unit_bytes * 2.3 + (6 << 30)  # in + out + arena
        free, _ = torch.cuda.mem_get_info(d.dev)
        fits = min(r[0] for r in d.gather([1.0 if free > need else 0.0])) > 0
        if fits:
            res = time_compression(d, ws, "strong", args.strong_steps, 3)
            s_ms, s_phases = phase_report(res, peak)
            strong = {"workload": args.strong_workload, "scaling": "strong", "n_gpus": d.world,
                      "value": round(ws.input_bytes / (s_ms * 1e6), 2), "unit": "GB/s",
                      "ms_per_step": round(s_ms, 4), "steps": args.strong_steps,
                      "input_bytes_total": ws.input_bytes, "phases": s_phases,
                      "units_per_rank": [len([0 for _ in shard_units(ws.layers, ws.heads, d.world, r)])
                                         for r in range(d.world)],
                      "cache_stats": res["stats"]}
        else:
            strong = {"workload": args.strong_workload, "skipped": f"needs {need / 2**30:.0f} GiB per GPU"}

    # --- end to end through the public API with host (pinned) buffers -----------------
    e2e = None
    if args.e2e_steps > 0:
        from graphkv_b200.sharding import shard_units

        wN = replace(w, batch=w.batch * d.world)
        shard = shard_units(w.layers, w.heads, d.world, d.rank)
        saved_cpus, binding = bind_host_to_gpu(d.dev)
        host_pairs = []
        for (l, h0, h1) in shard:
            k, v = make_layer(wN, l, device=str(d.dev), heads=range(h0, h1))
            hk = torch.empty(k.shape, dtype=k.dtype, pin_memory=True)
            hv = torch.empty(v.shape, dtype=v.dtype, pin_memory=True)
            hk.copy_(k)
            hv.copy_(v)
            host_pairs.append((hk, hv))
            del k, v
        torch.cuda.empty_cache()
        host_scores = make_scores(w)
        out = g.quantize_hf_cache(tuple(host_pairs), w.profile, importance_scores=host_scores, output="legacy")
        del out
        torch.cuda.synchronize(d.dev)
        d.barrier()
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            out = g.quantize_hf_cache(tuple(host_pairs), w.profile, importance_scores=host_scores, output="legacy")
            torch.cuda.synchronize(d.dev)
            del out
        e2e_s = (time.perf_counter() - t0) / args.e2e_steps
        d.barrier()
        e2e_s = max(r[0] for r in d.gather([e2e_s]))
        ceiling = d.gather(copy_ceiling(host_pairs, d.dev))  # all ranks at once: the shared host limit
        del host_pairs
        if saved_cpus is not None:
            os.sched_setaffinity(0, saved_cpus)
        e2e = {"value": round(d.world * in_bytes_rank / e2e_s / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": in_bytes_rank + 4 * w.seq, "d2h_bytes_per_step": in_bytes_rank,
               "ms_per_step": round(1e3 * e2e_s, 3), "steps": args.e2e_steps,
               "path": "quantize_hf_cache(host pinned legacy cache, output='legacy') -> host tensors",
               "copy_ceiling_gbs_per_rank": {k: [round(r[i], 1) for r in ceiling]
                                             for i, k in enumerate(("h2d", "d2h", "both_ways"))},
               "host_binding": binding or "none (PCIe topology not visible)"}

    if d.rank != 0:
        d.close()
        return
    q_ms, dq_ms = phases["quantize"]["ms"], phases["dequant"]["ms"]
    algo = in_bytes_rank + head["comp_bytes"]
    dominant = "quantize" if q_ms >= dq_ms else "dequant"
    nr = head["nr"]
    dom_ms = (q_ms if dominant == "quantize" else dq_ms) / nr
    dom_bytes = algo / nr
    achieved = dom_bytes / dom_ms / 1e6
    traffic = committed_traffic(args.workload).get(dominant)
    roofline = {"bound": "hbm",
                "kernel": ("quantize call: quantize_tile_kernel launches (keys, values, rotated cold values)"
                           if dominant == "quantize" else
                           "dequantize call: dequantize_tile_kernel launches (keys, values, rotated cold values)"),
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else peak_kind,
                "traffic": traffic, "algorithmic_bytes_per_launch": dom_bytes}
    cpu = None
    if d.world == 1 and not args.no_cpu_baseline:
        workers = os.cpu_count() or 1
        gbs, wall, nb = cpu_sample(args.workload, workers * 2, workers)
        cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": workers, "kind": "port",
               "sample": f"{workers * 2} (layer, kv-head) slices [1, 1, 32768, 128] bf16 "
                         f"({nb / 1e6:.0f} MB of K+V), quantize+pack then dequant, numpy oracle, "
                         f"{workers} processes, {wall:.1f} s"}
    line = {
        "metric": METRIC,
        "value": round(d.world * in_bytes_rank / (ms * 1e6), 2),
        "unit": "GB/s",
        "n_gpus": d.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": args.workload, "layers": w.layers, "kv_heads": w.heads, "head_dim": w.head_dim,
                   "batch_per_gpu": w.batch, "seq_len": w.seq, "profile": w.profile,
                   "input_bytes_per_gpu": in_bytes_rank, "compressed_bytes_per_gpu": head["comp_bytes"],
                   "l2": "inputs (1.88 GB) larger than L2; no flush",
                   "value_definition": "K+V input bytes of all ranks / max over ranks of the device time of one "
                                       "select+quantize+pack+dequant step",
                   "parallelism": f"weak shards of (layer, kv-head) units over {d.world} GPU(s)"},
        "phases": phases,
        "select": select_times,
        "append_and_attention": append_times,
        "rank_ms": [round(r[0], 4) for r in head["per_rank"]],
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "strong": strong,
        "gpu_launches": args.steps * head["launches"],
        "cache_stats": head["stats"],
        "clocks": head["clocks"],
    }
    print(json.dumps(line), flush=True)
    d.close()


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
