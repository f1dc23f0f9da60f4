#!/usr/bin/env python3
"""Benchmark of the quantised-linear hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload stack|<config 1-4 case>] [--no-extras] [--no-cpu-baseline]

Default workload: the 48-layer linear stack of a
Qwen2-architecture 14B decoder with Q4_K_M-style random weights (Q6_K for
attn_v, ffn_down and the output head, Q4_K elsewhere), batch-1 decode (M=1),
column-sharded over the ranks with an NCCL all-gather of every linear
group's output slices.  A step is one token: every weight of the stack is
streamed once.  Metric: aggregate weight-streaming GB/s.

Prints ONE JSON line (rank 0): the base fields, plus "roofline" (per-GPU
weight bytes per token / device time per token against the measured HBM
copy bandwidth), "cpu_baseline" (the CPU restatement of the reference
pipeline on this host's cores, bounded sample), "e2e" (the same metric with a
pinned-host input copy and a logits read-back inside the timed region),
"gpu_launches" and "clocks".  `--workload <case>` runs one config 1-4 case
alone and prints its device time (used for ncu captures).  Inputs are seeded synthetic ggml blocks with the
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


# ------------------------------------------------------------ config 5 -----
HIDDEN, FFN, VOCAB, LAYERS = 5120, 13824, 152064, 48
HEADS, KV_HEADS, HEAD_DIM = 40, 8, 128
METRIC = "aggregate weight-streaming GB/s, 48-layer Qwen2-14B Q4_K_M linear stack, M=1 decode"
# DRAM bytes read / algorithmic weight bytes of one gemv_kernel launch, from
# ncu captures of the Q4_K (K=5120, N=13824: 39.890 / 39.855 MB) and Q6_K
# (K=13824, N=5120: 58.172 / 58.099 MB) shapes of the stack.
GEMV_TRAFFIC_RATIO = 1.001


def stack_groups():
    """The linear groups of one layer: (name, qtype, K, N, input) with the
    same-input, same-format matrices fused (q+k, gate+up)."""
    q_n, kv_n = HEADS * HEAD_DIM, KV_HEADS * HEAD_DIM
    return [("qk", S.Q4_K, HIDDEN, q_n + kv_n, "h"), ("v", S.Q6_K, HIDDEN, kv_n, "h"),
            ("o", S.Q4_K, q_n, HIDDEN, "h"), ("gate_up", S.Q4_K, HIDDEN, 2 * FFN, "h"),
            ("down", S.Q6_K, FFN, HIDDEN, "f")]


class Stack:
    """One rank's column shard of the stack, run as a CUDA graph of GEMV
    launches.  N = 1: vkflame_quant_linear_ex.  N > 1: each linear is
    vkflame_quant_linear_gather, the decode GEMV fused with the all-gather
    (every rank stores its output slice into all ranks' gathered buffers over
    NVLink as {fp16 pair, epoch} words), and each linear's X is an earlier
    linear's gathered output (the layer's data flow: qk and the previous down output
    feed the next layer, o reads qk's, gate/up o's, down gate/up's, the head
    the last down's), so every gather is waited for, word by word, inside the
    kernel that reads it.  No NCCL call in the timed region."""

    def __init__(self, world, rank, dist, stream):
        import torch
        from vkflame_b200 import rt, shard
        self.rt, self.world, self.rank, self.dist, self.stream = rt, world, rank, dist, stream
        self.linears = []  # (qtype, K, Nshard, weight, input tensor, output, gather struct or None)
        self.x_h = torch.randn((1, HIDDEN), device="cuda").half()
        self.x_f = torch.randn((1, FFN), device="cuda").half()
        self.weight_bytes = 0
        self.gg = None
        if world > 1:
            from vkflame_b200.gather import GatherGroup
            self.gg = GatherGroup(dist, world, rank)
        seed = 1000 * rank
        groups = [g for _ in range(LAYERS) for g in stack_groups()] + [("head", S.Q6_K, HIDDEN, VOCAB, "h")]
        prev = []  # gathered outputs so far, newest last
        for i, (name, q, K, N, inp) in enumerate(groups):
            r0, r1 = shard.row_range(N, world, rank)  # this rank's output rows (vkflame_b200/shard.py)
            n = r1 - r0
            seed += 1
            w = make_quant_weight_gpu(q, n, K, seed)
            if world > 1:
                y = self.gg.buffer(N)
                src = next((t for t in reversed(prev) if t.N >= K), None)
                g = self.gg.op(y, x=src)
                x = src.tensor if src is not None else (self.x_h if inp == "h" else self.x_f)
                prev.append(y)
            else:
                y = torch.empty((1, n), device="cuda", dtype=torch.float16)
                x, g = (self.x_h if inp == "h" else self.x_f), None
            self.linears.append((q, K, n, w, x, y, g))
            self.weight_bytes += w.numel()
        self.out = self.linears[-1][5] if world == 1 else self.linears[-1][5].tensor
        torch.cuda.synchronize()
        barrier(dist)  # every rank's counters initialised before any kernel signals

    def step(self):
        rt = self.rt
        for q, K, n, w, x, y, g in self.linears:
            if g is None:
                rt.quant_linear_ex(w.data_ptr(), q, x.data_ptr(), rt.X_F16, y.data_ptr(), rt.Y_F16, 1, n, K, K, n,
                                   rt.FLAG_STATIC_WEIGHTS, self.stream)
            else:
                ldx = x.shape[2] * 2 if g.x_gathered else x.shape[1]  # gathered X: words of 2 values
                rt.quant_linear_gather(w.data_ptr(), q, x.data_ptr(), rt.Y_F16, 1, n, K, ldx, y.N,
                                       rt.FLAG_STATIC_WEIGHTS, g, self.stream)


def timed_graph(graph, stream, steps):
    import torch
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        graph.replay()
    e1.record(stream)
    return e0, e1


def bench_stack(args, world, rank, local, dist):
    import torch
    from vkflame_b200 import rt
    rt.lib()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        st = Stack(world, rank, dist, s.cuda_stream)
        torch.cuda.synchronize()
        st.step()  # warms NCCL and the kernels' one-time setup before capture
        torch.cuda.synchronize()
        l0 = rt.launch_count()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            st.step()
        launches_per_step = rt.launch_count() - l0
        for _ in range(args.warmup):
            g.replay()
        barrier(dist)
        sampler = ClockSampler(local)
        sampler.start()
        e0, e1 = timed_graph(g, s, args.steps)
        barrier(dist)
        clocks = sampler.stop()
        ms = max_over_ranks(dist, e0.elapsed_time(e1) / args.steps)
        rt.check_kernel_errors()

        # End to end through the public API with host buffers: pinned token
        # activations -> device, the stack, output-head logits -> pinned host.
        xh = torch.randn((1, HIDDEN)).half().pin_memory()
        # N > 1: the head's gathered buffers ({fp16 pair, epoch} words, both parities)
        outh = torch.empty(st.out.shape, dtype=st.out.dtype).pin_memory()
        def e2e_step():
            st.x_h.copy_(xh, non_blocking=True)
            g.replay()
            outh.copy_(st.out, non_blocking=True)
        for _ in range(args.warmup):
            e2e_step()
        barrier(dist)
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(s)
        for _ in range(args.steps):
            e2e_step()
        f1.record(s)
        barrier(dist)
        ems = max_over_ranks(dist, f0.elapsed_time(f1) / args.steps)

    total_bytes = st.weight_bytes * world  # every rank streams its shard once per token
    value = total_bytes / (ms * 1e-3) / 1e9
    peaks = measured_peaks()
    peak = peaks.get("hbm_gbs") or HBM_FALLBACK_GBS
    per_gpu = st.weight_bytes / (ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "q4_K/q6_K weights x f16 activations, f32 accumulation",
        "data": "synthetic: seeded random ggml blocks (fp16 scales U[1e-3,1e-2]), N(0,1) fp16 activations",
        "config": {"workload": "config 5: Qwen2-14B linear stack, 48 layers + output head, M=1 decode",
                   "layers": LAYERS, "hidden": HIDDEN, "ffn": FFN, "vocab": VOCAB,
                   "weight_gb_per_token": total_bytes / 1e9, "column_shards": world,
                   "launches_per_token": launches_per_step,
                   "dataflow": ("chained: each linear reads an earlier linear's gathered output" if world > 1
                             else "independent: each linear reads its layer input"),
                "collective": ("all-gather fused into each GEMV: output slices stored into every rank's buffer over "
                                  "NVLink (CUDA IPC peer memory) as {fp16 pair, epoch} words, waited for word by word "
                                  "in the kernel that reads them") if world > 1 else "none",
                   "l2": "weights (9.0 GB) exceed L2; no flush needed"},
        "roofline": {"bound": "hbm", "achieved": per_gpu, "peak": peak, "unit": "GB/s", "frac": per_gpu / peak,
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)" if peaks.get("hbm_gbs") else "fallback",
                     "traffic": st.weight_bytes / launches_per_step * GEMV_TRAFFIC_RATIO,
                     "note": "dominant kernel = gemv_kernel, every launch of the timed graph: algorithmic weight "
                             "bytes per launch / average launch time (graph time / launches); traffic = DRAM "
                             "bytes per launch, from the ncu captures of the same kernel on the stack's shapes "
                             "(ratio to algorithmic bytes, profiles/gemv_*.md)"},
        "e2e": {"value": total_bytes / (ems * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": HIDDEN * 2,
                "d2h_bytes_per_step": int(st.out.numel()) * st.out.element_size(), "ms_per_step": ems},
        "gpu_launches": launches_per_step * args.steps, "clocks": clocks,
    }
    return line


# ------------------------------------------------------- sub-benchmarks -----
def graph_time(fn, iters=20):
    import torch
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for _ in range(3):
            fn(s.cuda_stream)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(iters):
                fn(s.cuda_stream)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = timed_graph(g, s, 1)
        torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


GEMV_CASES = {"config3_q4K_gate_up_M1": (S.Q4_K, 5120, 13824, 1),
              "config3_q4K_gate_up_M8": (S.Q4_K, 5120, 13824, 8),
              "config3_q4K_qo_M1": (S.Q4_K, 5120, 5120, 1),
              "config3_q4K_down_M1": (S.Q4_K, 13824, 5120, 1),
              "config1_q4_0_M1": (S.Q4_0, 4096, 4096, 1),
              "config1_q4_0_M32": (S.Q4_0, 4096, 4096, 32),
              "q8_0_gate_up_M1": (S.Q8_0, 5120, 13824, 1),
              "q6K_down_M1": (S.Q6_K, 13824, 5120, 1)}


def bench_gemv_case(name, iters_per_copy=4):
    """One quantised linear (config 1/3 shapes): device time per call under a
    CUDA graph, with the weights rotated over copies that together exceed 3x L2
    so every call streams its weights from HBM."""
    import torch
    from vkflame_b200 import rt
    q, K, N, M = GEMV_CASES[name]
    l2 = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size
    wb = N * S.row_bytes(q, K)
    copies = max(2, int(np.ceil(3 * l2 / wb)))
    ws = [make_quant_weight_gpu(q, N, K, seed=i) for i in range(copies)]
    x = torch.randn((M, K), device="cuda").half()
    y = torch.empty((M, N), device="cuda", dtype=torch.float16)
    it = [0]
    def fn(sp):
        w = ws[it[0] % copies]
        it[0] += 1
        rt.quant_linear_ex(w.data_ptr(), q, x.data_ptr(), rt.X_F16, y.data_ptr(), rt.Y_F16, M, N, K, K, N,
                           rt.FLAG_STATIC_WEIGHTS, sp)
    ms = graph_time(fn, iters=iters_per_copy * copies)
    return {"us": ms * 1e3, "GB/s": (wb + M * K * 2 + M * N * 2) / (ms * 1e-3) / 1e9}


def bench_int8_linear():
    """Config 2: int8 linear with per-row / per-channel scales and bias (the
    hipblasLt BIAS-epilogue call)."""
    import torch
    from vkflame_b200 import rt
    M, N, K = 512, 11008, 4096
    xi = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda")
    wi = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda")
    sx, sw = torch.rand(M, device="cuda") * 1e-2, torch.rand(N, device="cuda") * 1e-2
    bias = (torch.randn(N, device="cuda") * 0.02).half()
    yi = torch.empty((M, N), device="cuda", dtype=torch.float16)
    ms = graph_time(lambda sp: rt.linear_int8(xi.data_ptr(), wi.data_ptr(), sx.data_ptr(), sw.data_ptr(),
                                              bias.data_ptr(), yi.data_ptr(), 0, M, N, K, 0, sp))
    return {"us": ms * 1e3, "TOPS": 2 * M * N * K / (ms * 1e-3) / 1e12}


def bench_q8_prefill():
    """Config 4: fp32 X -> on-device Q8_1 -> Q8_0 x Q8_1 prefill GEMM, fp32 out."""
    import torch
    from vkflame_b200 import rt
    M, N, K = 512, 13824, 5120
    wq = make_quant_weight_gpu(S.Q8_0, N, K, 7)
    xf = torch.randn((M, K), device="cuda")
    xq = torch.empty(M * K // 32 * 36, dtype=torch.uint8, device="cuda")
    yo = torch.empty((M, N), device="cuda")
    def c4(sp):
        rt.quantize_q8_1(xf.data_ptr(), xq.data_ptr(), M, K, K, sp)
        # model weights are written by no kernel: the GEMM may stream them while
        # the activation quantiser and widening run (VKF_FLAG_STATIC_WEIGHTS)
        rt.quant_linear_ex(wq.data_ptr(), S.Q8_0, xq.data_ptr(), rt.X_Q8_1, yo.data_ptr(), rt.Y_F32, M, N, K,
                           K // 32, N, rt.FLAG_STATIC_WEIGHTS, sp)
    ms = graph_time(c4, iters=5)
    return {"us": ms * 1e3, "TOPS": 2 * M * N * K / (ms * 1e-3) / 1e12}


SUB_CASES = dict({n: (lambda n=n: bench_gemv_case(n)) for n in GEMV_CASES},
                 config2_int8_linear_M512=bench_int8_linear, config4_q8_0_x_q8_1_M512=bench_q8_prefill)


def sub_benchmarks(names=None):
    """Configs 1-4 at one shape each (device time, CUDA graphs)."""
    from vkflame_b200 import rt
    out = {n: SUB_CASES[n]() for n in (names or SUB_CASES)}
    rt.check_kernel_errors()
    return out


def cpu_baseline_stack(budget_s=12.0):
    """The oracle's restatement of the reference pipeline (dequantise W to
    fp32, then k-serial fp32 dot products, as shim/hip_runtime_shim.cpp:
    1129-1166 sequences it) on all host cores, over a bounded sample of the
    stack's matrices (the first rows of one Q4_K and one Q6_K group),
    reported as weight-streaming GB/s."""
    from oracle import pyoracle as po
    cores = os.cpu_count() or 1
    samples = [(S.Q4_K, HIDDEN, 2048), (S.Q6_K, FFN, 1024)]
    mats = [(q, K, n, S.quant_matrix(q, n, K, seed=3 + q), S.normal_f16((1, K), seed=4)) for q, K, n in samples]
    for q, K, n, w, x in mats:
        po.quant_linear(q, w, x, 1, n, K, xtype=0, ytype=1, threads=cores)
    t0 = time.perf_counter()
    nbytes = 0
    reps = 0
    while time.perf_counter() - t0 < budget_s and reps < 400:
        for q, K, n, w, x in mats:
            po.quant_linear(q, w, x, 1, n, K, xtype=0, ytype=1, threads=cores)
            nbytes += w.nbytes
        reps += 1
    el = time.perf_counter() - t0
    return {"value": nbytes / el / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{reps} passes over a 2048-row Q4_K (K=5120) and a 1024-row Q6_K (K=13824) slice "
                      f"of the stack ({el:.1f} s)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="stack", choices=["stack"] + list(SUB_CASES),
                    help="stack (config 5, the headline) or one config 1-4 case alone (device time only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the config 1-4 sub-benchmarks")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_env()

    if args.impl == "reference":
        # The reference's own path is Vulkan compute shaders; no graphics stack
        # exists on this machine, so its arithmetic runs as the CPU oracle
        # restatement (reference pipeline: dequant to fp32 + fp32 dot products).
        if rank != 0:
            return
        cb = cpu_baseline_stack(budget_s=max(2.0, min(60.0, 0.25 * args.steps)))
        line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "GB/s", "n_gpus": 1,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None,
                "config": {"workload": "config 5: Qwen2-14B linear stack, 48 layers + output head, M=1 decode"},
                "cpu_baseline": cb,
                "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    if args.workload != "stack":
        init_dist(world, local)
        print(json.dumps({"workload": args.workload, **sub_benchmarks([args.workload])[args.workload]}))
        return

    dist = init_dist(world, local)
    line = bench_stack(args, world, rank, local, dist)
    if rank == 0 and world == 1:
        if not args.no_extras:
            line["configs"] = sub_benchmarks()
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_stack()
    if rank == 0:
        print(json.dumps(line))
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
