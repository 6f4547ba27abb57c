#!/usr/bin/env python
"""Benchmark of the W4A16 decode GEMV (and GQA decode attention) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload sweep|tp70b]

Default workload ("sweep"): the W4A16 linear shape sweep — M in {1,2,4,8} x
K in {4096,8192} x N in {4096,8192,11008}, plus K=11008/N=4096: 28 calls per
step, each on its own seeded weights (benchmark generator: random 32-bit
words, fp16 scales U[0.005,0.02], integer zeros 0..15, group 128).  A step
streams 704 MB of distinct weights, so every call reads its weights from HBM
(126 MB L2).  The step is one CUDA graph of the 28 public-API calls; the timed
region is K replays between a barrier + synchronize on both sides.

One JSON line (rank 0):
  value       aggregate algorithmic GB/s over all ranks: (packed weights +
              fp16 scales + zeros) bytes of every call / max-over-ranks time
  ms_per_step time of one 28-call step; us_per_call = ms_per_step*1000/28
  step_ms     per-step durations (one event per step): min/median/p90/max
  roofline    the GEMV kernel: algorithmic bytes per launch / average launch
              duration (CUDA events on the launching stream), against the
              measured HBM copy bandwidth; traffic = mean algorithmic bytes x
              the DRAM/algorithmic ratio of single-shape ncu captures
              (profiles/w4a16_gemv_traffic.json)
  e2e         same metric through the C ABI (ctypes) with host buffers: per
              call, pinned x -> device, the call, y -> pinned host
  cpu_baseline the oracle's dequant-then-matmul (numpy port of the
              reference's baseline_dequant_matmul) on host threads, bounded sample
  per_shape   each sweep shape alone: L2-cold graph time (median of 7), L2-warm
              graph time, eager time
  decode_bundle / mlp_bundle  the Llama-2-7B 7-projection decode bundle (M=1)
              and the gate/up(SiLU*up) -> down MLP (M=1,4,8), L2-cold and warm
  tp70b       the 70B-shaped tensor-parallel layer over all N ranks (fused
              collective kernels, NCCL between GEMVs, GEMVs alone)
With --gpus N under torchrun each rank runs its own sweep replica (weak scaling);
the tp70b object is the one leg with a collective.
--impl reference times the reference algorithm (numpy port) on the host CPU.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "µs/call and % of ~8 TB/s HBM roofline: W4A16 GEMV M=1–8 and GQA decode attn"
SWEEP = [(M, K, N) for M in (1, 2, 4, 8) for K in (4096, 8192) for N in (4096, 8192, 11008)] + [
    (M, 11008, 4096) for M in (1, 2, 4, 8)]
ATTN_SHAPES = [(B, L) for B in (1, 4, 8) for L in (512, 4096, 32768)]
PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
FALLBACK_HBM_GBS = 6650.0
TRAFFIC_FILE = ROOT / "profiles" / "w4a16_gemv_traffic.json"


def alg_bytes(K: int, N: int) -> int:
    """Packed int4 weights + fp16 scales + fp16 zeros (the weight+scale bytes)."""
    return N * K // 2 + 2 * 2 * N * (K // 128)


def attn_bytes(B: int, L: int, Hkv: int = 8, D: int = 128) -> int:
    return 2 * B * Hkv * L * D * 2


def hbm_peak():
    try:
        d = json.loads(PEAKS_FILE.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def committed_traffic(mean_alg_bytes: float):
    """Per-launch DRAM bytes of the GEMV kernel: the sweep's mean algorithmic
    bytes per launch times the DRAM/algorithmic ratio measured by single-shape
    ncu captures (profiles/w4a16_gemv_traffic.json, written from the captures'
    CSV by `bench.py --traffic-from-ncu`).  None if the file is absent."""
    try:
        d = json.loads(TRAFFIC_FILE.read_text())
        ratios = [r["dram_bytes"] / r["alg_bytes"] for r in d["captures"]]
        return int(round(mean_alg_bytes * statistics.mean(ratios)))
    except Exception:
        return None


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """NVML sampler of SM clock and throttle reasons during the timed region."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            return
        self._period = period_s
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        # the SM clock every period; the throttle reasons (a slower query) every
        # fourth sample and once more at the end, so a short timed region still
        # gets several clock samples
        nv = self._nv
        i = 0
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                if i % 4 == 0:
                    self._reasons()
            except Exception:
                pass
            i += 1
            time.sleep(self._period)
        try:
            self._reasons()
        except Exception:
            pass

    def _reasons(self):
        r = self._nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        for bit, name in self.REASONS.items():
            if r & bit:
                self.reasons.add(name)

    def __enter__(self):
        if self.ok:
            self._t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml_unavailable"], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons - {"gpu_idle"}),
                "samples": len(self.samples)}


# ------------------------------------------------------------- distributed
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def dist_init(world, local):
    import datetime

    import torch
    import torch.distributed as dist

    if world > 1 and not dist.is_initialized():
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return dist if world > 1 else None


def max_over_ranks(value: float, dist, device):
    import torch

    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(dist, device):
    import torch

    torch.cuda.synchronize(device)
    if dist is not None:
        dist.barrier()
        torch.cuda.synchronize(device)


# ------------------------------------------------------------- CPU legs
def cpu_threads():
    n = os.cpu_count() or 1
    try:
        n = len(os.sched_getaffinity(0))
    except Exception:
        pass
    return max(1, n)


def cpu_sweep_sample(budget_s: float, threads: int, shapes=SWEEP, start: int = 0):
    """Run the oracle's threaded dequant-then-matmul over the sweep shapes, one
    call each per pass, repeating passes until `budget_s` seconds of calls have
    been timed (at least one full pass)."""
    from oracle import w4a16 as ow

    cases = {}
    done, total_t, total_b = [], 0.0, 0
    i = 0
    while i < len(shapes) or total_t < budget_s:
        M, K, N = shapes[(start + i) % len(shapes)]
        if (M, K, N) not in cases:
            cases[(M, K, N)] = ow.baseline_case(M, K, N, seed=7 + i % len(shapes))
        x, wq, s, z = cases[(M, K, N)]
        t0 = time.perf_counter()
        ow.linear_threaded(x, wq, s, z, threads)
        total_t += time.perf_counter() - t0
        total_b += alg_bytes(K, N)
        done.append((M, K, N))
        i += 1
    return total_b / total_t / 1e9, total_t, done


def run_reference(args, rank, world):
    """--impl reference: the reference's dequant-then-matmul (numpy port) on the
    host CPU.  Each step is one full pass over the 28 sweep shapes (the same
    step as the GPU arm's)."""
    if rank != 0:
        return
    from oracle import w4a16 as ow

    threads = cpu_threads()
    cases = {}

    for i, (M, K, N) in enumerate(SWEEP):
        cases[(M, K, N)] = ow.baseline_case(M, K, N, seed=1000 + i)

    def step(i):
        t, b = 0.0, 0
        for (M, K, N) in SWEEP:
            x, wq, s, z = cases[(M, K, N)]
            t0 = time.perf_counter()
            ow.linear_threaded(x, wq, s, z, threads)
            t += time.perf_counter() - t0
            b += alg_bytes(K, N)
        return t, b

    for i in range(args.warmup):
        step(i)
    tt, tb = 0.0, 0
    for i in range(args.steps):
        dt, b = step(args.warmup + i)
        tt += dt
        tb += b
    value = tb / tt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(tt / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "w4a16_shape_sweep", "shapes": len(SWEEP),
                   "step": "one pass over the 28 sweep shapes per step",
                   "parallelism": "host CPU"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} passes over the 28 sweep shapes, numpy dequant + "
                                   f"sgemm on {threads} threads"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- GPU legs
def graph_time_us(calls, device, repeats=7, min_calls=64):
    """Median over `repeats` of the per-call time (µs) of `calls` (a list of
    zero-argument callables) captured back to back in one CUDA graph; the graph
    is replayed enough times per repeat that at least `min_calls` calls are
    timed.  Returns (median, [per-repeat values])."""
    import torch

    for c in calls:
        c()
    torch.cuda.synchronize(device)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for c in calls:
                c()
    torch.cuda.current_stream(device).wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize(device)
    reps = max(1, -(-min_calls // len(calls)))
    out = []
    for _ in range(repeats):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize(device)
        out.append(e0.elapsed_time(e1) * 1e3 / (reps * len(calls)))
    del g
    return statistics.median(out), out


def summarize(samples):
    s = sorted(samples)
    return {"min": round(s[0], 3), "median": round(statistics.median(s), 3),
            "p90": round(s[int(0.9 * (len(s) - 1))], 3), "max": round(s[-1], 3), "n": len(s)}


def weight_copies(case, n, device, seed):
    """`case` plus n - 1 copies of its weights at distinct addresses, made on the
    device (packed words XOR-ed with fresh random words; scales and zeros
    cloned), so rotating through them reads every byte from HBM."""
    import torch

    x, wq, s, z = case
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out = [case]
    for _ in range(n - 1):
        r = torch.randint(-2**31, 2**31 - 1, wq.shape, generator=g, device=device, dtype=torch.int32)
        out.append((x, wq ^ r, s.clone(), z.clone()))
    return out


def refstyle_us(fn, device, warmup=30, iters=120, repeats=7):
    """The reference benchmark's own timing (bench/bench_w4a16.py and
    bench/bench_decode_bundle.py, time_cuda + summarize): `warmup` eager calls,
    then per repeat `iters` eager calls back to back between two events, mean
    per call; min / median / p90 / max over `repeats` (µs)."""
    import torch

    out = []
    for _ in range(repeats):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize(device)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize(device)
        out.append(e0.elapsed_time(e1) * 1e3 / iters)
    return summarize(out)


def event_pair_floor_us(device, n=32, reps=3):
    """Median time between two events around one trivial kernel (a 1-element
    in-place multiply), queued behind a GPU sleep: the floor under any
    single-call event measurement on this GPU (µs)."""
    import torch

    z = torch.zeros(1, device=device)
    vals = []
    for _ in range(reps):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        torch.cuda._sleep(20_000_000)
        for a, b in evs:
            a.record()
            z.mul_(1)
            b.record()
        torch.cuda.synchronize(device)
        vals += [a.elapsed_time(b) * 1e3 for a, b in evs]
    return round(statistics.median(vals), 3)


def per_shape_graph(device, peak, repeats=7):
    """Each sweep shape alone: L2-cold (enough weight copies, rotated, to exceed
    the 126 MB L2 several times over) and L2-warm (one weight set called back to
    back), both as CUDA graphs of public-API calls, median of `repeats`."""
    import torch

    import focal_b200 as F

    rows = []
    for i, (M, K, N) in enumerate(SWEEP):
        nb = alg_bytes(K, N)
        copies = max(3, -(-400_000_000 // nb))
        cases = weight_copies(F.baseline_case(M, K, N, seed=3000 + i, device=device), copies, device, 77 + i)
        cold, _ = graph_time_us([(lambda c=c: F.w4a16_linear(*c)) for c in cases], device, repeats)
        warm, _ = graph_time_us([lambda: F.w4a16_linear(*cases[0])] * 16, device, repeats)
        refstyle = refstyle_us(lambda c=cases[0]: F.w4a16_linear(*c), device)
        rows.append({"M": M, "K": K, "N": N, "us": round(cold, 3), "GBps": round(nb / cold / 1e3, 1),
                     "frac": round(nb / cold / 1e3 / peak, 3), "us_warm": round(warm, 3),
                     "us_refstyle": refstyle["median"], "us_refstyle_stats": refstyle})
        del cases
    torch.cuda.empty_cache()
    return rows


# Llama-2-7B decode projections (the reference's bench/bench_decode_bundle.py
# LAYERS): (name, M, K, N)
DECODE_BUNDLE = [("q_proj", 1, 4096, 4096), ("k_proj", 1, 4096, 4096), ("v_proj", 1, 4096, 4096),
                 ("o_proj", 1, 4096, 4096), ("gate_proj", 1, 4096, 11008), ("up_proj", 1, 4096, 11008),
                 ("down_proj", 1, 11008, 4096)]


def bundles(device, peak, repeats=7):
    """The 7-projection Llama-2-7B decode bundle at M=1 and the MLP bundle
    (fused gate/up with SiLU*up, then down; hidden 4096, intermediate 11008) at
    M = 1, 4, 8.  L2-cold: weight copies rotate across graph replays; L2-warm:
    one weight set, the way the reference's own bundle benchmark times it."""
    import torch

    import focal_b200 as F

    out = {}
    nb = sum(alg_bytes(K, N) for (_, _, K, N) in DECODE_BUNDLE)
    copies = max(2, -(-400_000_000 // nb))
    per_layer = [weight_copies(F.baseline_case(M, K, N, seed=9000 + i, device=device), copies, device, 900 + i)
                 for i, (_, M, K, N) in enumerate(DECODE_BUNDLE)]
    sets = [[per_layer[i][c] for i in range(len(DECODE_BUNDLE))] for c in range(copies)]
    calls = [(lambda cs=cs: [F.w4a16_linear(*c) for c in cs]) for cs in sets]
    cold, cold_s = graph_time_us(calls, device, repeats, min_calls=8)
    warm, warm_s = graph_time_us([calls[0]] * 8, device, repeats, min_calls=8)
    # the reference's bundle timing: the seven eager calls on one weight set per
    # iteration, 30 warm-up and 7 x 120 timed iterations
    ref = refstyle_us(calls[0], device)
    out["decode_bundle"] = {
        "layers": [{"name": n, "M": M, "K": K, "N": N} for (n, M, K, N) in DECODE_BUNDLE],
        "bytes": nb, "us_cold": summarize(cold_s), "us_warm": summarize(warm_s), "us_refstyle": ref,
        "GBps_cold": round(nb / cold / 1e3, 1), "frac_cold": round(nb / cold / 1e3 / peak, 3)}
    del sets, calls
    mlp = []
    H, I = 4096, 11008
    nb = 2 * alg_bytes(H, I) + alg_bytes(I, H)
    copies = max(2, -(-400_000_000 // nb))
    for M in (1, 4, 8):
        gate = weight_copies(F.baseline_case(M, H, I, seed=500, device=device), copies, device, 51)
        up = weight_copies(F.baseline_case(M, H, I, seed=501, device=device), copies, device, 52)
        down = weight_copies(F.baseline_case(M, I, H, seed=502, device=device), copies, device, 53)
        x = gate[0][0]
        calls = [(lambda c=c: F.decode_mlp(x, gate[c][1:], up[c][1:], down[c][1:])) for c in range(copies)]
        cold, cold_s = graph_time_us(calls, device, repeats, min_calls=16)
        warm, warm_s = graph_time_us([calls[0]] * 8, device, repeats, min_calls=16)
        mlp.append({"M": M, "us_cold": summarize(cold_s), "us_warm": summarize(warm_s),
                    "GBps_cold": round(nb / cold / 1e3, 1), "frac_cold": round(nb / cold / 1e3 / peak, 3)})
        del gate, up, down, calls
    out["mlp_bundle"] = {"hidden": H, "intermediate": I, "bytes": nb, "shapes": mlp,
                         "kernels": "gate/up fused with SiLU*up (one launch) + down (one launch)"}
    torch.cuda.empty_cache()
    return out


def build_sweep(device, seed0=1000):
    import focal_b200 as F

    return [F.baseline_case(M, K, N, seed=seed0 + i, device=device) for i, (M, K, N) in enumerate(SWEEP)]


def per_launch_profile(cases, reps=3):
    """Per-call kernel durations: eager calls queued behind a GPU sleep (so the
    CPU runs ahead and each event pair brackets only its kernel)."""
    import torch

    import focal_b200 as F

    n = len(cases)
    acc = [0.0] * n
    for _ in range(reps):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        torch.cuda._sleep(50_000_000)  # ~25 ms of GPU time while the calls are queued
        for i, c in enumerate(cases):
            evs[i][0].record()
            F.w4a16_linear(*c)
            evs[i][1].record()
        torch.cuda.synchronize()
        for i in range(n):
            acc[i] += evs[i][0].elapsed_time(evs[i][1]) * 1e3 / reps
    return acc  # microseconds


def e2e_sweep(cases, steps, device):
    """Through the C ABI with host buffers: each step copies the 28 calls' x from
    one pinned host buffer to the device (one H2D copy), makes the 28 calls, and
    reads the 28 outputs back into one pinned host buffer (one D2H copy)."""
    import torch

    from focal_b200 import _lib

    L = _lib.lib()
    stream = torch.cuda.current_stream(device)
    sp = stream.cuda_stream
    x_off, y_off, xo, yo = [], [], 0, 0
    for (M, K, N) in SWEEP:
        x_off.append(xo)
        y_off.append(yo)
        xo += -(-M * K // 8) * 8  # elements, 16-byte aligned slices
        yo += -(-M * N // 8) * 8
    hx = torch.empty(xo, dtype=torch.bfloat16).pin_memory()
    for i, (M, K, N) in enumerate(SWEEP):
        hx[x_off[i]:x_off[i] + M * K].copy_(cases[i][0].reshape(-1).cpu())
    dx = torch.empty(xo, dtype=torch.bfloat16, device=device)
    dy = torch.empty(yo, dtype=torch.bfloat16, device=device)
    hy = torch.empty(yo, dtype=torch.bfloat16).pin_memory()
    ws_n = max(int(L.focal_w4a16_workspace_size(M, K, N)) for (M, K, N) in SWEEP)
    ws = torch.zeros(ws_n, dtype=torch.uint8, device=device)  # zeroed once, as the C ABI requires
    xp, yp = dx.data_ptr(), dy.data_ptr()
    args = [(xp + 2 * x_off[i], c[1].data_ptr(), c[2].data_ptr(), c[3].data_ptr(), yp + 2 * y_off[i], M, K, N)
            for i, (c, (M, K, N)) in enumerate(zip(cases, SWEEP))]
    wsp = ws.data_ptr()
    gemv = L.focal_w4a16_gemv

    def step():
        dx.copy_(hx, non_blocking=True)
        for a in args:
            if gemv(*a, wsp, ws_n, sp):
                raise RuntimeError(_lib.last_error())
        hy.copy_(dy, non_blocking=True)

    for _ in range(3):
        step()
    torch.cuda.synchronize(device)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1) / steps
    h2d = sum(M * K * 2 for (M, K, N) in SWEEP)
    d2h = sum(M * N * 2 for (M, K, N) in SWEEP)
    return ms, h2d, d2h


def attention_secondary(device, reps=20):
    """GQA decode attention contract shapes (B, L), KV read cold from HBM: a
    CUDA graph of calls on rotating KV copies, median of 7 timed replays."""
    import torch

    import focal_b200 as F

    out = []
    budget = 1_200_000_000
    for (B, L) in ATTN_SHAPES:
        nb = attn_bytes(B, L)
        copies = max(1, min(64, -(-400_000_000 // nb)))
        if copies * nb > budget:
            copies = 1
        g = torch.Generator(device="cpu").manual_seed(B * 100 + L)
        q = torch.randn((B, 32, 128), generator=g).to(torch.bfloat16).to(device)
        kv = [(torch.randn((B, 8, L, 128), device=device, dtype=torch.bfloat16),
               torch.randn((B, 8, L, 128), device=device, dtype=torch.bfloat16)) for _ in range(copies)]
        for c in kv:
            F.gqa_decode_attention(q, *c)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device)
        s.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                for c in kv:
                    F.gqa_decode_attention(q, *c)
        torch.cuda.current_stream(device).wait_stream(s)
        graph.replay()
        torch.cuda.synchronize()
        n = max(1, reps // copies) if copies > 1 else reps
        samples = []
        for _ in range(7):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(n):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            samples.append(e0.elapsed_time(e1) * 1e3 / (n * copies))
        us = statistics.median(samples)
        out.append({"B": B, "L": L, "us": round(us, 3), "GBps": round(nb / us / 1e3, 1),
                    "us_stats": summarize(samples)})
        del graph, kv
        torch.cuda.empty_cache()
    return out


def run_ours(args, rank, world, local):
    import torch

    import focal_b200 as F
    from focal_b200 import _lib

    dist = dist_init(world, local)
    device = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(device)
    torch.backends.cuda.matmul.allow_tf32 = False
    peak, peak_kind = hbm_peak()

    cases = build_sweep(device, seed0=1000 + 97 * rank)
    step_bytes = sum(alg_bytes(K, N) for (M, K, N) in SWEEP)

    # one step = one CUDA graph of the 28 public-API calls
    for c in cases:
        F.w4a16_linear(*c)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream(device)
    cap.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(cap):
        with torch.cuda.graph(graph, stream=cap):
            for c in cases:
                F.w4a16_linear(*c)
    torch.cuda.current_stream(device).wait_stream(cap)
    for _ in range(max(3, args.warmup)):
        graph.replay()
    barrier(dist, device)

    # one event before each step and one after the last: per-step durations
    # (median and spread) besides the total
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with ClockSampler(device.index, period_s=0.0002) as clk:
        evs[0].record()
        for i in range(args.steps):
            graph.replay()
            evs[i + 1].record()
        torch.cuda.synchronize(device)
    barrier(dist, device)
    clocks = clk.summary()
    if (clocks.get("samples") or 0) < 10:
        # A short timed region leaves the sampler few samples (NVML queries
        # take a while); the same graph replayed right after it for ~0.25 s
        # gives a clock record of the same load, reported beside the in-region
        # one (not timed).
        n_adj = max(1, int(0.25 / max(1e-4, evs[0].elapsed_time(evs[-1]) * 1e-3 / args.steps)))
        with ClockSampler(device.index, period_s=0.0002) as clk_adj:
            for _ in range(n_adj):
                graph.replay()
            torch.cuda.synchronize(device)
        clocks["adjacent_replays"] = {**clk_adj.summary(), "replays": n_adj}
    barrier(dist, device)
    step_ms = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
    ms_local = evs[0].elapsed_time(evs[-1]) / args.steps
    ms = max_over_ranks(ms_local, dist, device)
    value = world * step_bytes / (ms * 1e-3) / 1e9

    # Roofline of the GEMV launches: the timed region is the 28 calls back to
    # back (one kernel each, chained by programmatic launch), so the average
    # launch time is ms_local / 28.  Per-shape times come from eager calls.
    launch_us = ms_local * 1e3 / len(SWEEP)
    achieved = step_bytes / len(SWEEP) / (launch_us * 1e-6) / 1e9
    us_eager = per_launch_profile(cases)
    floor_us = event_pair_floor_us(device)
    per_shape = None
    extra = {}
    if world == 1 and not args.no_secondary:
        per_shape = per_shape_graph(device, peak)
        for row, u in zip(per_shape, us_eager):
            row["us_eager"] = round(u, 3)
        extra = bundles(device, peak)
    e2e_ms, h2d, d2h = e2e_sweep(cases, max(3, min(args.steps, 50)), device)
    e2e_ms = max_over_ranks(e2e_ms, dist, device)
    attn = attention_secondary(device) if (world == 1 and not args.no_secondary) else None
    tp = None if args.no_tp else tp70b_measure(args, rank, world, dist, device)

    status = __import__("ctypes").c_int(0)
    _lib.lib().focal_device_status(status)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 5), "us_per_call": round(ms * 1e3 / len(SWEEP), 3),
            "step_ms": summarize(step_ms),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int4xbf16->f32", "data": "synthetic",
            "config": {"workload": "w4a16_shape_sweep", "shapes": "M{1,2,4,8} x K{4096,8192} x "
                       "N{4096,8192,11008} + K11008/N4096 (28 calls per step)",
                       "group": 128, "l2": "cold: 28 distinct weight sets per step (704 MB > 126 MB L2)",
                       "step": "one CUDA graph of 28 w4a16_linear calls",
                       "parallelism": f"replica{world}" if world > 1 else "single"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": committed_traffic(step_bytes / len(SWEEP)),
                         "bytes_per_launch_mean": step_bytes // len(SWEEP),
                         "launch_us_mean": round(launch_us, 3),
                         "timing": "CUDA events over the timed graph replays"},
            "e2e": {"value": round(world * step_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": round(e2e_ms, 4), "path": "C ABI via ctypes, eager; one pinned H2D copy of the step's x and one D2H copy of its y"},
            "gpu_launches": len(SWEEP) * args.steps,  # one GEMV kernel per call
            "clocks": clocks,
            "device_status": status.value,
            "per_shape": per_shape,
            "per_shape_note": "us: CUDA graph of L2-cold calls (rotating weight copies), median of 7; "
                              "us_warm: same weights back to back in a graph; us_refstyle: the reference "
                              "benchmark's method (30 warm-up eager calls on one weight set, then 120 back to "
                              "back between two events, mean per call; median of 7 repeats, stats beside it); "
                              "us_eager: one eager call between two events, queued behind a GPU sleep "
                              "(event_pair_floor_us is the same measurement around a trivial kernel)",
            "event_pair_floor_us": floor_us,
            **extra,
        }
        if tp is not None:
            line["tp70b"] = tp
        if attn is not None:
            line["attention"] = {"shapes": attn, "unit": "GB/s of KV bytes",
                                 "frac_of_peak": [round(a["GBps"] / peak, 3) for a in attn]}
        if world == 1 and not args.no_cpu_baseline:
            v, t, done = cpu_sweep_sample(args.cpu_budget, cpu_threads())
            line["cpu_baseline"] = {"value": round(v, 3), "unit": "GB/s", "cores": cpu_threads(),
                                    "kind": "port",
                                    "sample": f"{len(done)} sweep calls ({len(done) / len(SWEEP):.1f} "
                                              f"passes over the 28 shapes, {t:.1f} s of numpy "
                                              f"dequant + sgemm on {cpu_threads()} threads)"}
        print(json.dumps(line), flush=True)
    del graph
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def tp70b_measure(args, rank, world, dist, device):
    """70B-shaped tensor-parallel decode layer at M=8 over `world` GPUs (strong
    scaling): column-parallel K=8192, N=28672 (N sharded, bf16 all-gather of
    y), then row-parallel K=28672, N=8192 (K sharded, fp32 all-reduce).  Times
    the fused kernels (collective inside the GEMV over peer memory), the same
    GEMVs with NCCL collectives between them (N > 1), and the GEMVs alone;
    max over ranks.  Returns the summary dict on rank 0, None elsewhere."""
    import torch

    import focal_b200 as F
    from focal_b200 import tp

    peak, peak_kind = hbm_peak()
    M, K1, N1, K2, N2 = 8, 8192, 28672, 28672, 8192
    n1, k2 = N1 // world, K2 // world
    per_rank = alg_bytes(K1, n1) + alg_bytes(k2, N2)
    copies = max(1, -(-400_000_000 // per_rank))  # rotate weights so every step reads HBM
    col = [F.baseline_case(1, K1, n1, seed=10_000 + 100 * rank + c, device=device)[1:] for c in range(copies)]
    row = [F.baseline_case(1, k2, N2, seed=20_000 + 100 * rank + c, device=device)[1:] for c in range(copies)]
    x = F.baseline_case(M, K1, 64, seed=5, device=device)[0]

    group = tp.TpGroup(max_m=M, max_n=max(n1, N2), device=device)

    def layer(c, mode):
        if mode == "fused":  # one kernel per projection, the collective inside it
            y = group.allgather_linear(x, *col[c])
            return group.allreduce_linear(y[:, rank * k2:(rank + 1) * k2].contiguous(), *row[c])
        collectives = mode == "nccl"
        y_local = F.w4a16_linear(x, *col[c])
        y = tp.gather_columns(y_local) if collectives else y_local
        x2 = y[:, rank * k2:(rank + 1) * k2].contiguous() if collectives else y_local
        part = F.w4a16_linear_f32(x2, *row[c])
        return tp.reduce_partials(part) if collectives else part

    modes = ("fused", "nccl", "local") if world > 1 else ("fused", "local")
    graphs = {}
    for mode in modes:
        for c in range(copies):
            layer(c, mode)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device)
        s.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for c in range(copies):
                    layer(c, mode)
        torch.cuda.current_stream(device).wait_stream(s)
        graphs[mode] = g
    reps = max(1, args.steps // copies)
    res = {}
    clk_summary = None
    for mode in modes:
        for _ in range(max(3, args.warmup // copies + 1)):
            graphs[mode].replay()
        barrier(dist, device)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with ClockSampler(device.index) as clk:
            e0.record()
            for _ in range(reps):
                graphs[mode].replay()
            e1.record()
            torch.cuda.synchronize(device)
        barrier(dist, device)
        if mode == "fused":
            clk_summary = clk.summary()
        res[mode] = max_over_ranks(e0.elapsed_time(e1) / (reps * copies), dist, device)
    status = ctypes.c_int(-1)
    from focal_b200 import _lib as flib

    flib.lib().focal_device_status(status)
    if status.value != 0:
        raise RuntimeError(f"rank {rank}: device status {status.value} after the fused layers")
    del graphs
    group.close()
    if rank != 0:
        return None
    ms, ms_k = res["fused"], res["local"]
    out = {
        "n_gpus": world, "M": M, "column": [K1, N1], "row": [K2, N2], "parallelism": f"tp{world}",
        "fused_us": round(ms * 1e3, 2), "GBps": round(world * per_rank / (ms * 1e-3) / 1e9, 2),
        "kernel_only_us": round(ms_k * 1e3, 2),
        "kernel_only_GBps": round(world * per_rank / (ms_k * 1e-3) / 1e9, 2),
        "kernel_only_frac_of_aggregate_peak": round(per_rank / (ms_k * 1e-3) / 1e9 / peak, 4),
        "collective_us": round((ms - ms_k) * 1e3, 2), "ranks_seen": world,
        "timing": "CUDA events around graph replays of L2-cold layers, max over ranks",
        "collectives": "bf16 all-gather + fp32 all-reduce inside the two GEMV kernels "
                       "(64-bit {value, epoch} stores to peer memory over NVLink)",
        "l2": f"cold: {copies} rotating weight copies per rank", "steps": reps * copies,
        "clocks": clk_summary,
    }
    if "nccl" in res:
        out["nccl_us"] = round(res["nccl"] * 1e3, 2)
        out["nccl_GBps"] = round(world * per_rank / (res["nccl"] * 1e-3) / 1e9, 2)
    return out


def run_tp70b(args, rank, world, local):
    """--workload tp70b: the tensor-parallel layer alone, as its own JSON line."""
    import torch

    dist = dist_init(world, local)
    device = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(device)
    r = tp70b_measure(args, rank, world, dist, device)
    if rank == 0:
        line = {
            "metric": METRIC, "value": r["GBps"], "unit": "GB/s", "n_gpus": world, "steps": r["steps"],
            "warmup": args.warmup, "ms_per_step": r["fused_us"] / 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int4xbf16->f32", "data": "synthetic",
            "config": {"workload": "tp70b_decode_layer", "M": r["M"], "column": r["column"], "row": r["row"],
                       "parallelism": r["parallelism"], "collectives": r["collectives"], "l2": r["l2"]},
            "gpu_launches": 2 * r["steps"], "clocks": r["clocks"], "tp70b": r,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_timeline(args):
    """--timeline M,K,N[;M,K,N...]: per-unit phase timeline of one GEMV call in
    the middle of an eager chain of L2-cold calls, from the diagnostic build
    (python -m focal_b200.build --timeline; stamps described in
    csrc/w4a16_gemv.cu).  Prints one JSON summary per shape: phase times in µs
    as [min, p50, p90, max] over CTAs and sub-pipelines."""
    import numpy as np
    import torch

    import focal_b200 as F
    from focal_b200 import _lib

    path = Path(_lib.__file__).resolve().parent / "libfocal_b200_timeline.so"
    if not path.exists():
        raise SystemExit(f"{path.name} is not built: python -m focal_b200.build --timeline")
    h = ctypes.CDLL(str(path))
    for name, (res, argt) in _lib.SIGNATURES.items():
        fn = getattr(h, name)
        fn.restype, fn.argtypes = res, argt
    h.focal_tl_set.restype, h.focal_tl_set.argtypes = ctypes.c_int, [ctypes.c_void_p]
    CT, PR, UN = 160, 4, 64
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    for spec in args.timeline.split(";"):
        M, K, N = (int(v) for v in spec.split(","))
        copies = max(3, -(-400_000_000 // alg_bytes(K, N)))
        cases = weight_copies(F.baseline_case(M, K, N, seed=50, device=dev), copies, dev, 5)
        y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        nws = int(h.focal_w4a16_workspace_size(M, K, N))
        ws = torch.zeros(nws, dtype=torch.uint8, device=dev)
        buf = torch.zeros(CT * PR * UN * 8 + CT * 8, dtype=torch.int64, device=dev)

        def run(c):
            rc = h.focal_w4a16_gemv(c[0].data_ptr(), c[1].data_ptr(), c[2].data_ptr(), c[3].data_ptr(),
                                    y.data_ptr(), M, K, N, ws.data_ptr(), nws,
                                    torch.cuda.current_stream(dev).cuda_stream)
            if rc:
                raise RuntimeError(h.focal_last_error().decode())

        for _ in range(2):
            for c in cases:
                run(c)
        torch.cuda.synchronize()
        if h.focal_tl_set(buf.data_ptr()):
            raise RuntimeError("focal_tl_set failed")
        torch.cuda._sleep(30_000_000)  # queue the chain so it runs back to back
        for c in cases:
            run(c)  # every call stamps; the last call's stamps remain
        torch.cuda.synchronize()
        h.focal_tl_set(None)
        a = buf.cpu().numpy()
        ev = a[:CT * PR * UN * 8].reshape(CT, PR, UN, 8).astype(np.float64)
        hd = a[CT * PR * UN * 8:].reshape(CT, 8).astype(np.float64)
        live = hd[:, 0] > 0
        ghz = 1.965  # cycles -> ns at the SM clock the runs here hold
        g0 = hd[live, 1]
        off = g0 - g0.min()  # CTA start offsets from %globaltimer
        rel = ev[live] / ghz + off[:, None, None, None]
        rel[ev[live] == 0] = np.nan
        end = (hd[live, 2] - hd[live, 0]) / ghz + off
        gdw = (hd[live, 4] - hd[live, 0]) / ghz + off
        RS, RE = rel[..., 63, 0].copy(), rel[..., 63, 3].copy()
        rel[..., 63, :] = np.nan
        E = [rel[..., i] for i in range(8)]

        def q(v):
            v = np.asarray(v, dtype=np.float64)
            v = v[~np.isnan(v)]
            return [round(float(np.percentile(v, x)) / 1e3, 3) for x in (0, 50, 90, 100)] if v.size else None

        out = {"shape": {"M": M, "K": K, "N": N}, "ctas": int(live.sum()),
               "us_min_p50_p90_max": {
                   "cta_start": q(off), "first_issue": q(E[0][..., 0]), "griddep_done": q(gdw),
                   "first_data_ready": q(E[2][..., 0]), "first_unit_done": q(E[3][..., 0]),
                   "last_unit_done": q(np.nanmax(E[3], axis=2)), "run_end": q(RE - RS), "cta_end": q(end),
                   "per_unit_consumer_busy": q(E[3] - E[2]),
                   "per_unit_between_units": q(E[2][..., 1:] - E[3][..., :-1]),
                   "per_unit_full_wait": q(E[2] - E[4]), "per_unit_smem_loads_and_sums": q(E[5] - E[2]),
                   "per_unit_mma_block": q(E[6] - E[5]), "per_unit_epilogue": q(E[3] - E[6]),
                   "per_unit_issue_interval": q(np.diff(E[0], axis=2)[..., 3:]),
                   "per_unit_data_ready_after_issue": q((E[2] - E[0])[..., 3:]),
                   "per_unit_record_after_issue": q((E[1] - E[0])[..., 3:])}}
        print(json.dumps(out), flush=True)
        del cases


def write_traffic_json(specs):
    """Per-launch DRAM bytes of single-shape GEMV captures (`ncu --csv
    --metrics dram__bytes_read.sum,dram__bytes_write.sum -k regex:w4a16_gemv
    -c 1 python bench.py --profile-shape M,K,N`), one CSV per shape, into
    profiles/w4a16_gemv_traffic.json beside each shape's algorithmic bytes."""
    import csv

    units = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}
    caps = []
    for spec in specs:
        shape, path = spec.split("=", 1)
        M, K, N = (int(v) for v in shape.split(","))
        rows = [r for r in csv.reader(line for line in open(path) if not line.startswith("=="))]
        h = rows[0]
        tot = 0.0
        for r in rows[1:]:
            d = dict(zip(h, r))
            if d.get("Metric Name") in ("dram__bytes_read.sum", "dram__bytes_write.sum"):
                tot += float(d["Metric Value"].replace(",", "")) * units.get(d.get("Metric Unit", "byte"), 1)
        caps.append({"M": M, "K": K, "N": N, "dram_bytes": int(tot), "alg_bytes": alg_bytes(K, N),
                     "ratio": round(tot / alg_bytes(K, N), 4)})
    TRAFFIC_FILE.write_text(json.dumps({
        "kernel": "w4a16_gemv_kernel", "metric": "dram__bytes_read.sum + dram__bytes_write.sum, one launch",
        "command": "ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum --clock-control none "
                   "-k regex:w4a16_gemv -s 2 -c 1 --csv python bench.py --profile-shape M,K,N",
        "captures": caps}, indent=1) + "\n")
    print(TRAFFIC_FILE.read_text())


def run_profile_case(args):
    """A few calls of one shape, for ncu captures of a single kernel:
    --profile-shape M,K,N (W4A16), --profile-attn B,L (attention) or
    --profile-paged B,L,page_size (paged attention, pages shuffled)."""
    import torch

    import focal_b200 as F

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if args.profile_sweep:
        cases = build_sweep(dev)
        fn = lambda: [F.w4a16_linear(*c) for c in cases]  # noqa: E731
    elif args.profile_shape:
        M, K, N = (int(v) for v in args.profile_shape.split(","))
        case = F.baseline_case(M, K, N, seed=1, device=dev)
        fn = lambda: F.w4a16_linear(*case)  # noqa: E731
    elif args.profile_paged:
        B, L, ps = (int(v) for v in args.profile_paged.split(","))
        g = torch.Generator(device="cpu").manual_seed(1)
        per = (L + ps - 1) // ps
        q = torch.randn((B, 32, 128), generator=g).to(torch.bfloat16).to(dev)
        kp = torch.randn((B * per, 8, ps, 128), generator=g).to(torch.bfloat16).to(dev)
        vp = torch.randn((B * per, 8, ps, 128), generator=g).to(torch.bfloat16).to(dev)
        table = torch.randperm(B * per, generator=g).to(torch.int32).view(B, per).to(dev)
        lens = torch.full((B,), L, dtype=torch.int32, device=dev)
        fn = lambda: F.gqa_decode_attention_paged(q, kp, vp, table, lens, L)  # noqa: E731
    else:
        B, L = (int(v) for v in args.profile_attn.split(","))
        g = torch.Generator(device="cpu").manual_seed(1)
        q = torch.randn((B, 32, 128), generator=g).to(torch.bfloat16).to(dev)
        k = torch.randn((B, 8, L, 128), generator=g).to(torch.bfloat16).to(dev)
        v = torch.randn((B, 8, L, 128), generator=g).to(torch.bfloat16).to(dev)
        fn = lambda: F.gqa_decode_attention(q, k, v)  # noqa: E731
    for _ in range(args.profile_calls):
        fn()
    torch.cuda.synchronize()
    print("profile case done")


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["sweep", "tp70b"], default="sweep")
    ap.add_argument("--cpu-budget", type=float, default=15.0, help="seconds for the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the per-shape, bundle and attention legs")
    ap.add_argument("--no-tp", action="store_true", help="skip the tensor-parallel 70B layer leg")
    ap.add_argument("--timeline", default=None, metavar="M,K,N[;M,K,N]",
                    help="per-unit phase timeline of the GEMV (needs python -m focal_b200.build --timeline)")
    ap.add_argument("--traffic-from-ncu", nargs="+", default=None, metavar="M,K,N=CSV",
                    help="write profiles/w4a16_gemv_traffic.json from single-shape ncu CSV captures "
                         "of dram__bytes_read.sum and dram__bytes_write.sum")
    ap.add_argument("--profile-shape", default=None, help="M,K,N: only run a few calls (ncu)")
    ap.add_argument("--profile-attn", default=None, help="B,L: only run a few attention calls (ncu)")
    ap.add_argument("--profile-paged", default=None, help="B,L,page_size: a few paged attention calls (ncu)")
    ap.add_argument("--profile-sweep", action="store_true", help="each sweep shape once per call round (ncu)")
    ap.add_argument("--profile-calls", type=int, default=3)
    args = ap.parse_args(argv)
    if args.traffic_from_ncu:
        write_traffic_json(args.traffic_from_ncu)
        return 0
    if args.timeline:
        run_timeline(args)
        return 0
    if args.profile_shape or args.profile_attn or args.profile_sweep or args.profile_paged:
        run_profile_case(args)
        return 0
    if args.warmup < 3:
        args.warmup = 3
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return 0
    if args.workload == "tp70b":
        run_tp70b(args, rank, world, local)
    else:
        run_ours(args, rank, world, local)
    return 0


if __name__ == "__main__":
    sys.exit(main())
