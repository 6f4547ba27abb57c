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
  roofline    the GEMV kernel: algorithmic bytes per launch / average launch
              duration (CUDA events on the launching stream), against the
              measured HBM copy bandwidth; traffic from the committed ncu summary
  e2e         same metric through the C ABI (ctypes) with host buffers: per
              call, pinned x -> device, the call, y -> pinned host
  cpu_baseline the oracle's dequant-then-matmul (numpy port of the
              reference's baseline_dequant_matmul) on host threads, bounded sample
With --gpus N under torchrun each rank runs its own sweep replica (weak scaling).
--impl reference times the reference algorithm (numpy port) on the host CPU.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import re
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
TRAFFIC_FILE = ROOT / "profiles" / "w4a16_gemv_sweep.md"


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


def committed_traffic():
    """Per-launch DRAM bytes of the GEMV kernel from the committed ncu summary."""
    try:
        m = re.search(r"^traffic_per_launch_bytes:\s*(\d+)", TRAFFIC_FILE.read_text(), re.M)
        return int(m.group(1)) if m else None
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
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self._period)

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
    host CPU.  Each step is one sweep call (cycling through the 28 shapes)."""
    if rank != 0:
        return
    from oracle import w4a16 as ow

    threads = cpu_threads()
    cases = {}

    def step(i):
        M, K, N = SWEEP[i % len(SWEEP)]
        if (M, K, N) not in cases:
            cases[(M, K, N)] = ow.baseline_case(M, K, N, seed=1000 + i % len(SWEEP))
        x, wq, s, z = cases[(M, K, N)]
        t0 = time.perf_counter()
        ow.linear_threaded(x, wq, s, z, threads)
        return time.perf_counter() - t0, alg_bytes(K, N)

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
                   "step": "one sweep call per step, cycling through the 28 shapes",
                   "parallelism": "host CPU"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} sweep calls (one shape each), numpy dequant + "
                                   f"sgemm on {threads} threads"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- GPU legs
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
    """GQA decode attention contract shapes (B, L), KV read cold from HBM."""
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
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (n * copies)
        out.append({"B": B, "L": L, "us": round(us, 3), "GBps": round(nb / us / 1e3, 1)})
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

    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index) as clk:
        e0.record()
        for _ in range(args.steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize(device)
    barrier(dist, device)
    ms_local = e0.elapsed_time(e1) / args.steps
    ms = max_over_ranks(ms_local, dist, device)
    value = world * step_bytes / (ms * 1e-3) / 1e9

    # Roofline of the GEMV launches: the timed region is the 28 calls back to
    # back (one kernel each, chained by programmatic launch), so the average
    # launch time is ms_local / 28.  Per-shape times come from eager calls.
    launch_us = ms_local * 1e3 / len(SWEEP)
    achieved = step_bytes / len(SWEEP) / (launch_us * 1e-6) / 1e9
    us = per_launch_profile(cases)
    per_shape = [{"M": M, "K": K, "N": N, "us": round(u, 3),
                  "GBps": round(alg_bytes(K, N) / u / 1e3, 1),
                  "frac": round(alg_bytes(K, N) / u / 1e3 / peak, 3)}
                 for (M, K, N), u in zip(SWEEP, us)]
    e2e_ms, h2d, d2h = e2e_sweep(cases, max(3, min(args.steps, 50)), device)
    e2e_ms = max_over_ranks(e2e_ms, dist, device)
    attn = attention_secondary(device) if (world == 1 and not args.no_secondary) else None

    status = __import__("ctypes").c_int(0)
    _lib.lib().focal_device_status(status)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 5), "us_per_call": round(ms * 1e3 / len(SWEEP), 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int4xbf16->f32", "data": "synthetic",
            "config": {"workload": "w4a16_shape_sweep", "shapes": "M{1,2,4,8} x K{4096,8192} x "
                       "N{4096,8192,11008} + K11008/N4096 (28 calls per step)",
                       "group": 128, "l2": "cold: 28 distinct weight sets per step (704 MB > 126 MB L2)",
                       "step": "one CUDA graph of 28 w4a16_linear calls",
                       "parallelism": f"replica{world}" if world > 1 else "single"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": committed_traffic(),
                         "bytes_per_launch_mean": step_bytes // len(SWEEP),
                         "launch_us_mean": round(launch_us, 3),
                         "timing": "CUDA events over the timed graph replays"},
            "e2e": {"value": round(world * step_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": round(e2e_ms, 4), "path": "C ABI via ctypes, eager; one pinned H2D copy of the step's x and one D2H copy of its y"},
            "gpu_launches": len(SWEEP) * args.steps,  # one GEMV kernel per call
            "clocks": clk.summary(),
            "device_status": status.value,
            "per_shape": per_shape,
        }
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


def run_tp70b(args, rank, world, local):
    """70B-shaped tensor-parallel decode layer at M=8 over `world` GPUs (strong
    scaling): column-parallel K=8192, N=28672 (N sharded, bf16 all-gather of
    y), then row-parallel K=28672, N=8192 (K sharded, fp32 all-reduce)."""
    import torch

    import focal_b200 as F
    from focal_b200 import tp

    dist = dist_init(world, local)
    device = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(device)
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

    modes = ("fused", "nccl", "local")
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
    if rank == 0:
        ms, ms_k, ms_n = res["fused"], res["local"], res["nccl"]
        line = {
            "metric": METRIC, "value": round(world * per_rank / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "n_gpus": world, "steps": reps * copies, "warmup": args.warmup, "ms_per_step": round(ms, 5),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int4xbf16->f32", "data": "synthetic",
            "config": {"workload": "tp70b_decode_layer", "M": M, "column": [K1, N1], "row": [K2, N2],
                       "parallelism": f"tp{world}",
                       "collectives": "bf16 all-gather + fp32 all-reduce inside the two GEMV kernels "
                                      "(64-bit {value, epoch} stores to peer memory over NVLink)",
                       "l2": f"cold: {copies} rotating weight copies per rank"},
            "kernel_only": {"value": round(world * per_rank / (ms_k * 1e-3) / 1e9, 2), "unit": "GB/s",
                            "ms_per_step": round(ms_k, 5),
                            "frac_of_aggregate_peak": round(per_rank / (ms_k * 1e-3) / 1e9 / peak, 4),
                            "peak_per_gpu": peak, "peak_kind": peak_kind},
            "collective_ms": round(ms - ms_k, 5),
            "nccl_collectives": {"value": round(world * per_rank / (ms_n * 1e-3) / 1e9, 2), "unit": "GB/s",
                                 "ms_per_step": round(ms_n, 5),
                                 "how": "the same GEMVs with torch.distributed all_gather_into_tensor / "
                                        "all_reduce (NCCL) between them"},
            "gpu_launches": 2 * reps * copies,
            "clocks": clk_summary,
        }
        print(json.dumps(line), flush=True)
    del graphs
    group.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


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
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["sweep", "tp70b"], default="sweep")
    ap.add_argument("--cpu-budget", type=float, default=15.0, help="seconds for the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true", help="skip the attention shapes")
    ap.add_argument("--profile-shape", default=None, help="M,K,N: only run a few calls (ncu)")
    ap.add_argument("--profile-attn", default=None, help="B,L: only run a few attention calls (ncu)")
    ap.add_argument("--profile-paged", default=None, help="B,L,page_size: a few paged attention calls (ncu)")
    ap.add_argument("--profile-sweep", action="store_true", help="each sweep shape once per call round (ncu)")
    ap.add_argument("--profile-calls", type=int, default=3)
    args = ap.parse_args(argv)
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
