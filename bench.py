#!/usr/bin/env python3
"""Benchmark of the quantised-linear hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload gemv_q4k|stack]

Prints ONE JSON line (rank 0).  See DESIGN.md ("Measurement") for the
definition of every field.  Inputs are seeded synthetic ggml blocks with the
benchmark configs' distributions (vkflame_b200/synth.py): no model weights
or datasets exist on this machine.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

from vkflame_b200 import synth as S  # noqa: E402

HBM_FALLBACK_GBS = 6650.0


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            pass
    return {}


# ---------------------------------------------------------------- clocks ----
class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=2)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------- distributed -----
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_dist(world: int, local: int):
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1 and not dist.is_initialized():
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return dist if world > 1 else None


def barrier(dist):
    import torch
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(dist, v: float) -> float:
    import torch
    if dist is None:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------ workloads ----
def make_quant_weight_gpu(qtype: int, N: int, K: int, seed: int):
    """Random ggml blocks generated on the device: uniform random bytes (every
    code, 6-bit scale/min and int8 sub-scale is then uniform over its range),
    with the fp16 block scales overwritten by U[1e-3, 1e-2] values."""
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    bb, qk = S.BLOCK_BYTES[qtype], S.BLOCK_VALUES[qtype]
    nb = K // qk
    w = torch.randint(0, 256, (N, nb, bb), dtype=torch.uint8, device="cuda", generator=g)
    fields = {S.Q4_K: [0, 2], S.Q5_K: [0, 2], S.Q6_K: [208], S.Q8_0: [0], S.Q4_0: [0]}[qtype]
    lo, hi = (1e-3, 2e-2) if qtype == S.Q4_0 else (1e-3, 1e-2)
    for off in fields:
        d = (torch.rand((N, nb), device="cuda", generator=g) * (hi - lo) + lo).half()
        w[:, :, off:off + 2] = d.view(torch.uint8).view(N, nb, 2)
    if qtype == S.Q8_0:  # int8 quants uniform in [-127, 127] (never -128)
        q = w[:, :, 2:34].view(torch.int8)
        q[q == -128] = -127
    return w.view(N, nb * bb)


def cpu_baseline_gemv(qtype, N, K, M, budget_s=12.0):
    """The oracle's restatement of the reference pipeline (dequant W to fp32,
    k-serial fp32 dot products; shim/hip_runtime_shim.cpp:1129-1166) on all
    host cores, over a bounded sample of rows; scaled to GB/s of weights."""
    from oracle import pyoracle as po
    cores = os.cpu_count() or 1
    rows = min(N, 2048)
    w = S.quant_matrix(qtype, rows, K, seed=3)
    x = S.normal_f16((M, K), seed=4)
    po.quant_linear(qtype, w, x, M, rows, K, xtype=0, ytype=1, threads=cores)  # warm
    t0 = time.perf_counter()
    reps = 0
    while True:
        po.quant_linear(qtype, w, x, M, rows, K, xtype=0, ytype=1, threads=cores)
        reps += 1
        el = time.perf_counter() - t0
        if el > budget_s or reps >= 200:
            break
    per = el / reps
    gbs = (w.nbytes + M * K * 2 + M * rows * 2) / per / 1e9
    return {"value": gbs, "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{S.NAMES[qtype]} {rows} rows x K={K}, M={M}, {reps} reps ({el:.1f}s)"}


def bench_gemv(args, world, rank, local, dist):
    """Config 3: Q4_K decode GEMV, gate/up shape (K=5120, N=13824), M=1."""
    import torch
    from vkflame_b200 import rt
    rt.lib()
    qtype, K, Ntot, M = S.Q4_K, 5120, 13824, 1
    assert Ntot % world == 0
    N = Ntot // world  # column shard of this rank (rows of W)
    wbytes = N * S.row_bytes(qtype, K)
    # Rotate enough weight copies that every step reads from HBM, not L2.
    l2 = torch.cuda.get_device_properties(local).L2_cache_size
    copies = max(4, int(np.ceil(3 * l2 / wbytes)))
    ws = [make_quant_weight_gpu(qtype, N, K, seed=1000 * rank + i) for i in range(copies)]
    x = torch.randn((M, K), device="cuda").half()
    y = torch.empty((M, N), device="cuda", dtype=torch.float16)
    yfull = torch.empty((world, M, N), device="cuda", dtype=torch.float16)
    stream = torch.cuda.current_stream().cuda_stream

    def step(i):
        w = ws[i % copies]
        rt.quant_linear(w.data_ptr(), qtype, x.data_ptr(), rt.X_F16, y.data_ptr(), rt.Y_F16, M, N, K, K, N, stream)
        if dist is not None:
            dist.all_gather_into_tensor(yfull, y)

    for i in range(args.warmup):
        step(i)
    barrier(dist)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    sampler.start()
    l0 = rt.launch_count()
    ev0.record()
    for i in range(args.steps):
        step(i)
    ev1.record()
    barrier(dist)
    launches = rt.launch_count() - l0
    ms = ev0.elapsed_time(ev1) / args.steps
    ms = max_over_ranks(dist, ms)
    clocks = sampler.stop()
    rt.check_kernel_errors()

    # Kernel-only roofline: GEMV launches alone (no collective), CUDA events
    # on the launching stream.
    kev0, kev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    kev0.record()
    for i in range(args.steps):
        w = ws[i % copies]
        rt.quant_linear(w.data_ptr(), qtype, x.data_ptr(), rt.X_F16, y.data_ptr(), rt.Y_F16, M, N, K, K, N, stream)
    kev1.record()
    torch.cuda.synchronize()
    kms = kev0.elapsed_time(kev1) / args.steps
    alg_bytes = wbytes + M * K * 2 + M * N * 2
    total_bytes = alg_bytes * world  # all ranks' weight shards
    value = total_bytes / (ms * 1e-3) / 1e9

    # End to end through the public C ABI with host buffers: pinned x -> device,
    # GEMV, y -> pinned host, every step.
    xh = torch.randn((M, K)).half().pin_memory()
    yh = torch.empty((M, N), dtype=torch.float16).pin_memory()
    for i in range(args.warmup):
        x.copy_(xh, non_blocking=True)
        w = ws[i % copies]
        rt.quant_linear(w.data_ptr(), qtype, x.data_ptr(), rt.X_F16, y.data_ptr(), rt.Y_F16, M, N, K, K, N, stream)
        yh.copy_(y, non_blocking=True)
    barrier(dist)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        x.copy_(xh, non_blocking=True)
        w = ws[i % copies]
        rt.quant_linear(w.data_ptr(), qtype, x.data_ptr(), rt.X_F16, y.data_ptr(), rt.Y_F16, M, N, K, K, N, stream)
        if dist is not None:
            dist.all_gather_into_tensor(yfull, y)
        yh.copy_(y if dist is None else yfull[rank], non_blocking=True)
    e1.record()
    barrier(dist)
    ems = max_over_ranks(dist, e0.elapsed_time(e1) / args.steps)
    e2e = {"value": total_bytes / (ems * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": M * K * 2,
           "d2h_bytes_per_step": M * N * 2}

    peaks = measured_peaks()
    peak = peaks.get("hbm_gbs")
    achieved = alg_bytes / (kms * 1e-3) / 1e9
    line = {
        "metric": "Q4_K linear HBM GB/s at M=1 (config 3 gate/up, 5120x13824)",
        "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "q4_K x f16 -> f32 acc", "data": "synthetic (seeded random ggml blocks, N(0,1) fp16 x)",
        "config": {"workload": "q4_K GEMV K=5120 N=13824 M=1", "column_shards": world,
                   "l2": f"{copies} weight copies rotated ({copies * wbytes / 1e6:.0f} MB > L2 {l2 / 1e6:.0f} MB)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak or HBM_FALLBACK_GBS, "unit": "GB/s",
                     "frac": achieved / (peak or HBM_FALLBACK_GBS),
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs" if peak else "fallback", "traffic": None,
                     "kernel_ms": kms, "alg_bytes_per_launch": alg_bytes},
        "e2e": e2e, "gpu_launches": launches, "clocks": clocks,
    }
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="gemv_q4k", choices=["gemv_q4k"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_env()

    if args.impl == "reference":
        if rank != 0:
            return
        cb = cpu_baseline_gemv(S.Q4_K, 13824, 5120, 1, budget_s=max(2.0, min(60.0, 0.5 * args.steps)))
        line = {"impl": "reference", "metric": "Q4_K linear HBM GB/s at M=1 (config 3 gate/up, 5120x13824)",
                "value": cb["value"], "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "config": {"workload": "q4_K GEMV K=5120 N=13824 M=1"},
                "cpu_baseline": cb,
                "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    dist = init_dist(world, local)
    line = bench_gemv(args, world, rank, local, dist)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_gemv(S.Q4_K, 13824, 5120, 1)
    if rank == 0:
        print(json.dumps(line))
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
