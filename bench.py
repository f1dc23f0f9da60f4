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
# Same ratio for the per-token chain kernel, from an ncu capture of a
# 4-layer + head cut of the stack (1.33684 GB read / 1.33639 GB algorithmic).
CHAIN_TRAFFIC_RATIO = 1.0003


def stack_groups():
    """The linear groups of one layer: (name, qtype, K, N, input) with the
    same-input, same-format matrices fused (q+k, gate+up)."""
    q_n, kv_n = HEADS * HEAD_DIM, KV_HEADS * HEAD_DIM
    return [("qk", S.Q4_K, HIDDEN, q_n + kv_n, "h"), ("v", S.Q6_K, HIDDEN, kv_n, "h"),
            ("o", S.Q4_K, q_n, HIDDEN, "h"), ("gate_up", S.Q4_K, HIDDEN, 2 * FFN, "h"),
            ("down", S.Q6_K, FFN, HIDDEN, "f")]


def stack_links(layers=None):
    """The stack's linears in order: (name, qtype, K, N, input), the output
    head last.  layers: fewer than the model's 48 only for profiler captures."""
    n = LAYERS if layers is None else layers
    return [g for _ in range(n) for g in stack_groups()] + [("head", S.Q6_K, HIDDEN, VOCAB, "h")]


def link_seed(rank: int, i: int) -> int:
    """Seed of rank `rank`'s shard of stack link i (make_quant_weight_gpu)."""
    return 1000 * rank + i + 1


class Stack:
    """One rank's column shard of the stack as ONE persistent kernel per token
    (vkflame_chain_*).  Default dataflow "chained", the same at every N: each
    linear reads an earlier linear's gathered output (qk and v the previous
    layer's down, o qk's, gate/up o's, down gate/up's, the head the last
    down's; the first layer's qk and v read the token's input row), and every rank
    stores its output slice into all ranks' gathered buffers as {fp16 pair,
    epoch} words (NVLink peer stores; world size 1: its own buffer), which the
    consumers wait for word by word.  "independent" (world size 1 only): every
    linear reads its layer input and writes a plain fp16 row, the pure
    weight-streaming form.  "launches": the same chained dataflow as one
    vkflame_quant_linear_gather launch per linear (N = 1: independent
    vkflame_quant_linear_ex launches), for comparison."""

    def __init__(self, world, rank, dist, stream, mode="chained", trace=False, layers=None):
        import torch
        from vkflame_b200 import rt, shard
        from vkflame_b200.gather import GatherGroup
        self.rt, self.world, self.rank, self.dist, self.stream, self.mode = rt, world, rank, dist, stream, mode
        # Chained forms: a small input row (N(0,1) x 1e-6) so that the first
        # layer's outputs stay finite in fp16 (with these random weights each
        # link multiplies the magnitudes by ~100) and can be checked; the
        # deeper layers' values overflow, which changes no timing.
        scale = 1.0 if mode == "independent" else 1e-6
        gen = torch.Generator(device="cuda")
        gen.manual_seed(1234)  # the same token row on every rank
        self.x_h = (torch.randn((1, HIDDEN), device="cuda", generator=gen) * scale).half()
        self.x_f = torch.randn((1, FFN), device="cuda", generator=gen).half()
        self.weight_bytes = 0
        self.gg = GatherGroup(dist, world, rank)
        self.links = []   # (name, q, K, n, weight, out buffer or plain tensor, x source index or -1)
        self.ops = []     # "launches" mode: (q, K, n, w, x tensor, out, vkf_gather_t)
        chain = []
        links = stack_links(layers)
        if mode == "independent":
            # same input row and format next to each other: the kernel keeps
            # a quantised row resident across consecutive links
            order = {"qk": 0, "o": 1, "gate_up": 2, "v": 3, "down": 4, "head": 5}
            links = [l for lay in range(len(links) // 5) for l in sorted(links[5 * lay:5 * lay + 5],
                                                                            key=lambda t: order[t[0]])] + links[-1:]
        for i, (name, q, K, N, inp) in enumerate(links):
            r0, r1 = shard.row_range(N, world, rank)  # this rank's output rows (vkflame_b200/shard.py)
            n = r1 - r0
            w = make_quant_weight_gpu(q, n, K, link_seed(rank, i))
            self.weight_bytes += w.numel()
            xin = self.x_h if inp == "h" else self.x_f
            if mode == "independent":
                y = torch.empty((1, n), device="cuda", dtype=torch.float16)
                chain.append(self.gg.chain_linear(w.data_ptr(), q, K, n, None, x_plain=xin.data_ptr(),
                                                  y_plain=y.data_ptr()))
                self.links.append((name, q, K, n, w, y, -1))
                continue
            y = self.gg.buffer(N)
            src = self._source(name)
            if mode == "launches":
                g = self.gg.op(y, x=self.links[src][5] if src >= 0 else None)
                self.ops.append((q, K, n, w, self.links[src][5].tensor if src >= 0 else self.x_h, y, g, name))
            chain.append(self.gg.chain_linear(w.data_ptr(), q, K, n, y, x_src=src,
                                              x_plain=self.x_h.data_ptr() if src < 0 else 0))
            self.links.append((name, q, K, n, w, y, src))
        self.chain = None if mode == "launches" else rt.Chain(chain, world, rank, rt.CHAIN_TRACE if trace else 0)
        last = self.links[-1][5]
        self.out = last if mode == "independent" else last.tensor
        torch.cuda.synchronize()
        barrier(dist)  # every rank's buffers zeroed before any kernel stores into them

    def _source(self, name: str) -> int:
        """Link whose gathered output is this link's X (-1: the token's input
        row): qk and v read the layer input (the previous layer's down), o
        reads qk (standing in for the attention output), gate/up o, down
        gate/up, the head the last down."""
        want = {"qk": "down", "v": "down", "o": "qk", "gate_up": "o", "down": "gate_up", "head": "down"}[name]
        return next((j for j in range(len(self.links) - 1, -1, -1) if self.links[j][0] == want), -1)

    def step(self):
        if self.chain is not None:
            self.chain.run(self.stream)
            return
        rt = self.rt
        for q, K, n, w, x, y, g, name in self.ops:
            ldx = x.shape[2] * 2 if g.x_gathered else x.shape[1]  # gathered X: words of 2 values
            rt.quant_linear_gather(w.data_ptr(), q, x.data_ptr(), rt.Y_F16, 1, n, K, ldx, y.N,
                                   rt.FLAG_STATIC_WEIGHTS, g, self.stream)

    def runs(self) -> int:
        """Completed runs (the chain's epoch; "launches": the first call site's)."""
        if self.chain is not None:
            return self.chain.epoch()
        return int(self.gg.epochs[0].item())

    def close(self):
        if self.chain is not None:
            self.chain.close()
        self.gg.close()

    # ---------------------------------------------------------- parity ----
    def parity(self, sample=(0, 1, 2, 3)):
        """Checks of the last run's outputs, outside the timed region.
        ranks_identical: every rank holds the same gathered words (a
        position-weighted checksum per buffer, all-gathered).  vs_unsharded:
        on rank 0, the full (unsharded) weights of the first layer's links
        (qk and v read the token's row, o reads qk's gathered output, gate_up
        o's; Q4_K and Q6_K) regenerated from every rank's seeds, run through
        the single-GPU decode GEMV (vkflame_quant_linear_ex) on the same
        gathered input, against the gathered output; normwise
        max |y - r| / max |r|.  Deeper layers' values overflow fp16 (random
        weights), so they are covered by ranks_identical only."""
        import torch
        from vkflame_b200 import shard
        if self.mode == "independent":
            return self._parity_independent()
        ep = self.runs()
        words = [lk[5].tensor[ep & 1] for lk in self.links]  # [1][N/2][2] int32
        sums = []
        for wds in words:
            v = wds.reshape(-1).to(torch.int64)
            pos = torch.arange(1, v.numel() + 1, device=v.device, dtype=torch.int64)
            sums.append(((v & 0xFFFFFFFF) * pos).remainder_(2 ** 61 - 1).sum())
        local = torch.stack(sums)
        epochs_ok = all(bool((wds[..., 1] == ep).all()) for wds in words)
        if self.world > 1:
            allv = [torch.empty_like(local) for _ in range(self.world)]
            self.dist.all_gather(allv, local)
            same = all(bool(torch.equal(allv[0], a)) for a in allv)
        else:
            same = True
        out = {"ranks_identical": same, "epochs_current": epochs_ok, "runs": ep}
        if self.rank != 0:
            return out
        errs = {}
        for i in sample:
            name, q, K, n, w, y, src = self.links[i]
            N = n * self.world
            wfull = torch.cat([make_quant_weight_gpu(q, shard.row_range(N, self.world, r)[1] -
                                                     shard.row_range(N, self.world, r)[0], K, link_seed(r, i))
                               for r in range(self.world)]) if self.world > 1 else w
            xin = (self.x_h if src < 0 else self.links[src][5].tensor[ep & 1][..., 0].contiguous().view(
                torch.float16).reshape(1, -1)[:, :K]).contiguous()
            ref = torch.empty((1, N), device="cuda", dtype=torch.float16)
            self.rt.quant_linear_ex(wfull.data_ptr(), q, xin.data_ptr(), self.rt.X_F16, ref.data_ptr(),
                                    self.rt.Y_F16, 1, N, K, K, N, 0, self.stream)
            torch.cuda.synchronize()
            got = words[i][..., 0].contiguous().view(torch.float16).reshape(1, -1).double()
            r = ref.double()
            errs[f"{name}#{i}"] = float((got - r).abs().max() / r.abs().max().clamp_min(1e-30))
            del wfull
        tol = 1e-3
        finite = {k: v for k, v in errs.items() if np.isfinite(v)}
        worst = max(finite.values()) if finite else float("nan")
        out["vs_unsharded"] = {"links": errs, "max_normwise_err": worst, "tol": tol,
                               "nonfinite": sorted(k for k in errs if k not in finite),
                               "reference": "vkflame_quant_linear_ex on the full weights (one GPU)",
                               "pass": bool(finite) and len(finite) == len(errs) and worst < tol}
        return out


    def _parity_independent(self):
        """Independent form (one rank): the first layer's five links, the
        last layer's five and the head, each run again through the decode
        GEMV (vkflame_quant_linear_ex) on the same weights and input row,
        against the chain kernel's plain fp16 output; normwise
        max |y - r| / max |r|.  The last layer's links read an input row
        the kernel has kept resident across the whole stack."""
        import torch
        L = len(self.links)
        sample = sorted(set(range(min(5, L))) | set(range(max(0, L - 6), L)))
        errs = {}
        for i in sample:
            name, q, K, n, w, y, _ = self.links[i]
            xin = self.x_h if K == HIDDEN else self.x_f
            ref = torch.empty((1, n), device="cuda", dtype=torch.float16)
            self.rt.quant_linear_ex(w.data_ptr(), q, xin.data_ptr(), self.rt.X_F16, ref.data_ptr(),
                                    self.rt.Y_F16, 1, n, K, K, n, 0, self.stream)
            torch.cuda.synchronize()
            r, got = ref.double(), y.double()
            errs[f"{name}#{i}"] = float((got - r).abs().max() / r.abs().max().clamp_min(1e-30))
        tol = 1e-3
        finite = {k: v for k, v in errs.items() if np.isfinite(v)}
        worst = max(finite.values()) if finite else float("nan")
        return {"runs": self.runs(), "vs_gemv": {
            "links": errs, "max_normwise_err": worst, "tol": tol,
            "nonfinite": sorted(k for k in errs if k not in finite),
            "reference": "vkflame_quant_linear_ex on the same weights and input (one launch per link)",
            "pass": bool(finite) and len(finite) == len(errs) and worst < tol}}


def timed_graph(graph, stream, steps):
    import torch
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        graph.replay()
    e1.record(stream)
    return e0, e1


def run_stack(args, world, rank, local, dist, mode, steps, e2e=True, trace=False):
    """Builds the stack, captures one token as a CUDA graph, times `steps`
    replays (max over ranks) and, optionally, the end-to-end step."""
    import torch
    from vkflame_b200 import rt
    s = torch.cuda.Stream()
    res = {}
    with torch.cuda.stream(s):
        st = Stack(world, rank, dist, s.cuda_stream, mode=mode, trace=trace, layers=args.layers)
        st.step()  # one-time setup outside the capture
        torch.cuda.synchronize()
        l0 = rt.launch_count()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            st.step()
        res["launches_per_step"] = rt.launch_count() - l0
        for _ in range(args.warmup):
            g.replay()
        barrier(dist)
        sampler = ClockSampler(local)
        sampler.start()
        e0, e1 = timed_graph(g, s, steps)
        barrier(dist)
        res["clocks"] = sampler.stop()
        res["ms"] = max_over_ranks(dist, e0.elapsed_time(e1) / steps)
        rt.check_kernel_errors()
        res["parity"] = st.parity()
        if trace and st.chain is not None:
            res["trace"] = st.chain.trace()
        if e2e:
            # End to end through the public API with host buffers: pinned token
            # activations -> device, the stack, output-head logits -> pinned host
            # (chained: the head's gathered buffers, {fp16 pair, epoch} words).
            xh = torch.randn((1, HIDDEN)).half().pin_memory()
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
            for _ in range(steps):
                e2e_step()
            f1.record(s)
            barrier(dist)
            res["e2e_ms"] = max_over_ranks(dist, f0.elapsed_time(f1) / steps)
            res["d2h"] = int(st.out.numel()) * st.out.element_size()
        res["weight_bytes"] = st.weight_bytes
        torch.cuda.synchronize()
        st.close()
        del st, g
        torch.cuda.empty_cache()
    return res


def e2e_through_hip(steps=20, warmup=3):
    """The N = 1 weight-streaming token through the reference's own API, as
    ggml-hip drives it: the layer input row as Q8_1 blocks copied in with
    hipMemcpyAsync, one hipLaunchKernel("mul_mat_<fmt>_q8_1") per linear
    (libamdhip64 drop-in -> vkflame_quant_linear, fp32 outputs), the head's
    fp32 logits copied out with hipMemcpyAsync; timed with hipEvents, host
    launches included (no CUDA graph)."""
    import ctypes as C
    import torch
    from vkflame_b200 import LIBS, rt
    hip = C.CDLL(str(LIBS["hip"]))

    class Dim3(C.Structure):
        _fields_ = [("x", C.c_uint), ("y", C.c_uint), ("z", C.c_uint)]
    hip.hipLaunchKernel.argtypes = [C.c_void_p, Dim3, Dim3, C.POINTER(C.c_void_p), C.c_size_t, C.c_void_p]
    hip.__hipRegisterFunction.argtypes = [C.c_void_p, C.c_void_p, C.c_char_p, C.c_char_p, C.c_int] + [C.c_void_p] * 5
    hip.hipMemcpyAsync.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int, C.c_void_p]
    hip.hipEventRecord.argtypes = [C.c_void_p, C.c_void_p]
    hip.hipEventElapsedTime.argtypes = [C.POINTER(C.c_float), C.c_void_p, C.c_void_p]
    hip.hipStreamSynchronize.argtypes = [C.c_void_p]
    stubs, names = [], {}
    for fmt, nm in ((S.Q4_K, "mul_mat_q4_K_q8_1"), (S.Q6_K, "mul_mat_q6_K_q8_1")):
        stub = C.create_string_buffer(8)
        stubs.append(stub)
        hip.__hipRegisterFunction(None, C.addressof(stub), nm.encode(), nm.encode(), -1, None, None, None, None, None)
        names[fmt] = C.addressof(stub)
    links = stack_links()
    xs = {K: torch.randn((1, K), device="cuda") for K in (HIDDEN, FFN)}
    xq = {K: torch.empty(K // 32 * 36, dtype=torch.uint8, device="cuda") for K in (HIDDEN, FFN)}
    for K in xq:
        rt.quantize_q8_1(xs[K].data_ptr(), xq[K].data_ptr(), 1, K, K)
    xq_host = {K: xq[K].cpu().pin_memory() for K in xq}
    ws, ys = [], {}
    for i, (name, q, K, N, inp) in enumerate(links):
        ws.append(make_quant_weight_gpu(q, N, K, link_seed(0, i)))
        ys.setdefault(N, torch.empty(N, device="cuda"))
    out_host = torch.empty(VOCAB).pin_memory()
    stream, e0, e1 = C.c_void_p(), C.c_void_p(), C.c_void_p()
    assert hip.hipStreamCreate(C.byref(stream)) == 0
    hip.hipEventCreateWithFlags(C.byref(e0), 0)
    hip.hipEventCreateWithFlags(C.byref(e1), 0)
    holders = []

    def launch_token():
        for K in xq:  # ggml's activation row, Q8_1, host -> device
            assert hip.hipMemcpyAsync(C.c_void_p(xq[K].data_ptr()), C.c_void_p(xq_host[K].data_ptr()),
                                      xq[K].numel(), 1, stream) == 0
        for i, (name, q, K, N, inp) in enumerate(links):
            a = [C.c_void_p(ws[i].data_ptr()), C.c_void_p(xq[K].data_ptr()), C.c_void_p(ys[N].data_ptr()),
                 C.c_int(K), C.c_int(N), C.c_int(K), C.c_int(1), C.c_int(N)]
            holders[:] = a
            argv = (C.c_void_p * len(a))(*[C.addressof(h) for h in a])
            assert hip.hipLaunchKernel(C.c_void_p(names[q]), Dim3(1, 1, 1), Dim3(32, 1, 1), argv, 0, stream) == 0
        assert hip.hipMemcpyAsync(C.c_void_p(out_host.data_ptr()), C.c_void_p(ys[VOCAB].data_ptr()), VOCAB * 4, 2,
                                  stream) == 0
    for _ in range(warmup):
        launch_token()
    hip.hipStreamSynchronize(stream)
    hip.hipEventRecord(e0, stream)
    for _ in range(steps):
        launch_token()
    hip.hipEventRecord(e1, stream)
    hip.hipStreamSynchronize(stream)
    ms = C.c_float()
    hip.hipEventElapsedTime(C.byref(ms), e0, e1)
    per = ms.value / steps
    nbytes = sum(w.numel() for w in ws)
    rt.check_kernel_errors()
    del ws
    torch.cuda.empty_cache()
    return {"value": nbytes / (per * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": per,
            "h2d_bytes_per_step": sum(v.numel() for v in xq.values()), "d2h_bytes_per_step": VOCAB * 4,
            "path": "libamdhip64: hipMemcpyAsync + 241 x hipLaunchKernel(mul_mat_*_q8_1) + hipMemcpyAsync, "
                    "no CUDA graph (host launch rate included)"}


def bench_stack(args, world, rank, local, dist):
    """The headline.  Default (--stack-mode auto): at N = 1 the stack's
    weight-streaming figure, every linear reading its layer input, as one
    persistent kernel per token; at N > 1 the tensor-parallel form, every
    linear waiting for the previous linear's gathered output, one fused
    GEMV + all-gather launch per linear (measured faster than the persistent
    kernel in chained form).  At N = 1 the chained form is also measured,
    both ways, and reported in config (the like-for-like N = 1 figure for
    the N > 1 runs)."""
    mode = args.stack_mode
    if mode == "auto":
        mode = "independent" if world == 1 else "launches"
    args.stack_mode = mode
    res = run_stack(args, world, rank, local, dist, mode, args.steps, trace=args.trace)
    extra = {}
    if world == 1 and not args.no_extras:
        for alt in ("launches", "chained"):
            if alt == mode:
                continue
            r = run_stack(args, world, rank, local, dist, alt, args.steps, e2e=False)
            extra[f"{alt}_ms_per_token"] = r["ms"]
            extra[f"{alt}_gb_s"] = r["weight_bytes"] / (r["ms"] * 1e-3) / 1e9
            extra[f"{alt}_parity"] = r["parity"]
        if args.e2e_hip:
            extra["e2e_through_hip"] = e2e_through_hip()
    ms, ems = res["ms"], res["e2e_ms"]
    weight_bytes = res["weight_bytes"]
    total_bytes = weight_bytes * world  # every rank streams its shard once per token
    value = total_bytes / (ms * 1e-3) / 1e9
    peaks = measured_peaks()
    peak = peaks.get("hbm_gbs") or HBM_FALLBACK_GBS
    per_gpu = weight_bytes / (ms * 1e-3) / 1e9
    chained = args.stack_mode != "independent"
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "q4_K/q6_K weights x f16 activations, f32 accumulation",
        "data": "synthetic: seeded random ggml blocks (fp16 scales U[1e-3,1e-2]), N(0,1) fp16 activations",
        "config": {"workload": "config 5: Qwen2-14B linear stack, 48 layers + output head, M=1 decode"
                               if args.layers == LAYERS else f"profiling cut: {args.layers} layers + output head",
                   "layers": args.layers, "hidden": HIDDEN, "ffn": FFN, "vocab": VOCAB,
                   "weight_gb_per_token": total_bytes / 1e9, "column_shards": world,
                   "kernel": ("one persistent kernel per token (vkflame_chain_run)" if args.stack_mode != "launches"
                              else "one decode GEMV launch per linear"),
                   "launches_per_token": res["launches_per_step"],
                   "dataflow": ("chained at every N: each linear reads an earlier linear's gathered output"
                                if chained else "independent: each linear reads its layer input"),
                   "collective": ("all-gather fused into the decode: output slices stored into every rank's "
                                  "buffer over NVLink (CUDA IPC peer memory) as {fp16 pair, epoch} words, "
                                  "waited for word by word by the linear that reads them") if world > 1 else "none",
                   "l2": "weights (9.0 GB) exceed L2; no flush needed", **extra},
        "roofline": {"bound": "hbm", "achieved": per_gpu, "peak": peak, "unit": "GB/s", "frac": per_gpu / peak,
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)" if peaks.get("hbm_gbs") else "fallback",
                     "traffic": (weight_bytes * CHAIN_TRAFFIC_RATIO if args.stack_mode != "launches"
                                 else weight_bytes / max(1, res["launches_per_step"]) * GEMV_TRAFFIC_RATIO),
                     "note": ("dominant kernel = the per-token chain kernel (the only launch of the timed graph): "
                              "algorithmic weight bytes per launch (this rank's shard of the token) / launch time; "
                              "traffic = DRAM bytes per launch scaled from an ncu capture of the same kernel")
                             if args.stack_mode != "launches" else
                             ("dominant kernel = gemv_kernel (every launch of the timed graph): algorithmic weight "
                              "bytes per launch / average launch time (graph time / launches); traffic = DRAM bytes "
                              "per launch from ncu captures of the kernel on the stack's shapes")},
        "e2e": {"value": total_bytes / (ems * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": HIDDEN * 2,
                "d2h_bytes_per_step": res["d2h"], "ms_per_step": ems},
        "parity": res["parity"],
        "gpu_launches": res["launches_per_step"] * args.steps, "clocks": res["clocks"],
    }
    if "trace" in res:
        out = Path(args.trace)
        out.mkdir(parents=True, exist_ok=True)
        np.save(out / f"chain_trace_w{world}_r{rank}.npy", res["trace"])
    return line


# ------------------------------------------------------- sub-benchmarks -----
def graph_time(fn, iters=20, replays=5):
    """Device time per call: `iters` calls captured in one CUDA graph,
    replayed `replays` times after a warm-up replay (CUDA events on the
    launching stream); the median replay."""
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
        times = []
        for _ in range(replays):
            e0, e1 = timed_graph(g, s, 1)
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1) / iters)
    return float(np.median(times))


def hbm_roofline(bytes_per_call, ms):
    peaks = measured_peaks()
    peak = peaks.get("hbm_gbs") or HBM_FALLBACK_GBS
    a = bytes_per_call / (ms * 1e-3) / 1e9
    return {"bound": "hbm", "achieved": a, "peak": peak, "unit": "GB/s", "frac": a / peak,
            "peak_source": "of measured" if peaks.get("hbm_gbs") else "of fallback"}


def tensor_roofline(ops_per_call, ms, kind):
    """kind "f16": the measured cuBLAS bf16 burst; "i8": twice it (no int8
    figure is measured; the dense int8 rate of B200 is twice its bf16 rate)."""
    peaks = measured_peaks()
    bf16 = peaks.get("bf16_tflops") or 1590.0
    peak = bf16 * (2 if kind == "i8" else 1)
    a = ops_per_call / (ms * 1e-3) / 1e12
    return {"bound": "tensor", "achieved": a, "peak": peak, "unit": "TOPS" if kind == "i8" else "TFLOP/s",
            "frac": a / peak, "peak_source": ("2 x measured bf16 burst (int8 assumption)" if kind == "i8" else
                                             "measured bf16 burst") if peaks.get("bf16_tflops") else "fallback"}


# Config 1 and 3 cases (K, N per BASELINE.json): name -> (format, K, N, M)
GEMV_CASES = {f"config1_q4_0_M{m}": (S.Q4_0, 4096, 4096, m) for m in (1, 32)}
for _shape, (_k, _n) in {"qo": (5120, 5120), "kv": (5120, 1024), "gate_up": (5120, 13824),
                         "down": (13824, 5120)}.items():
    for _m in (1, 2, 4, 8):
        GEMV_CASES[f"config3_q4K_{_shape}_M{_m}"] = (S.Q4_K, _k, _n, _m)
GEMV_CASES.update({"q8_0_gate_up_M1": (S.Q8_0, 5120, 13824, 1), "q6K_down_M1": (S.Q6_K, 13824, 5120, 1)})


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
    nbytes = wb + M * K * 2 + M * N * 2
    return {"us": ms * 1e3, "GB/s": nbytes / (ms * 1e-3) / 1e9, "roofline": hbm_roofline(nbytes, ms),
            "l2": f"weights rotated over {copies} copies ({copies * wb / 1e6:.0f} MB > 3x L2)"}


def _lt(rt):
    import ctypes as C
    from vkflame_b200 import LIBS
    lt = C.CDLL(str(LIBS["hipblaslt"]))
    lt.hipblasLtMatrixLayoutCreate.argtypes = [C.POINTER(C.c_void_p), C.c_int, C.c_uint64, C.c_uint64, C.c_int64]
    return lt


def bench_int8_linear():
    """Config 2 through the hipBLASLt drop-in, as the config states:
    hipblasLtMatmul with int8 X (M x K) x int8 W (N x K, TRANSB = T),
    per-row / per-channel scale pointers and the fp16 BIAS epilogue."""
    import ctypes as C
    import torch
    from vkflame_b200 import rt
    M, N, K = 512, 11008, 4096
    xi = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda")
    wi = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda")
    sx = torch.rand(M, device="cuda") * 9e-3 + 1e-3
    sw = torch.rand(N, device="cuda") * 9e-3 + 1e-3
    bias = (torch.randn(N, device="cuda") * 0.02).half()
    yi = torch.empty((M, N), device="cuda", dtype=torch.float16)
    lt = _lt(rt)
    h, desc, la, lb, ld = (C.c_void_p() for _ in range(5))
    assert lt.hipblasLtCreate(C.byref(h)) == 0 and lt.hipblasLtMatmulDescCreate(C.byref(desc), 0, 0) == 0
    assert lt.hipblasLtMatrixLayoutCreate(C.byref(la), 2, M, K, K) == 0
    assert lt.hipblasLtMatrixLayoutCreate(C.byref(lb), 2, N, K, K) == 0
    assert lt.hipblasLtMatrixLayoutCreate(C.byref(ld), 0, M, N, N) == 0
    def setattr_(attr, value, ctype):
        v = ctype(value)
        assert lt.hipblasLtMatmulDescSetAttribute(desc, attr, C.byref(v), C.sizeof(v)) == 0
    setattr_(1, 112, C.c_int)                  # TRANSB = T
    setattr_(5, 2, C.c_int)                    # EPILOGUE_BIAS
    setattr_(6, bias.data_ptr(), C.c_void_p)   # BIAS_POINTER
    setattr_(7, sx.data_ptr(), C.c_void_p)     # A_SCALE_POINTER (per row)
    setattr_(8, sw.data_ptr(), C.c_void_p)     # B_SCALE_POINTER (per channel)
    one, zero = C.c_float(1.0), C.c_float(0.0)
    def fn(sp):
        rc = lt.hipblasLtMatmul(h, desc, C.byref(one), C.c_void_p(xi.data_ptr()), la, C.c_void_p(wi.data_ptr()), lb,
                                C.byref(zero), None, None, C.c_void_p(yi.data_ptr()), ld, None, None, C.c_size_t(0),
                                C.c_void_p(sp))
        assert rc == 0
    ms = graph_time(fn, iters=20)
    ops = 2 * M * N * K
    return {"us": ms * 1e3, "TOPS": ops / (ms * 1e-3) / 1e12, "path": "hipblasLtMatmul (libhipblaslt.so.0)",
            "roofline": tensor_roofline(ops, ms, "i8"),
            "l2": "inputs 49 MB re-read from L2 between calls (fit in L2; tensor-bound)"}


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
    ms = graph_time(c4, iters=10)
    ops = 2 * M * N * K
    return {"us": ms * 1e3, "TOPS": ops / (ms * 1e-3) / 1e12, "roofline": tensor_roofline(ops, ms, "i8"),
            "includes": "the on-device fp32 -> Q8_1 quantiser of X"}


def bench_prefill_stack(M=512):
    """Config 5 at M = 512: the 48-layer stack's 241 linears as a 512-token
    prefill (vkflame_quant_linear_ex, tensor-core GEMMs), one CUDA graph per
    step; 2 M N K flops summed over the linears."""
    import torch
    from vkflame_b200 import rt
    links = stack_links()
    xs = {K: torch.randn((M, K), device="cuda").half() for K in (HIDDEN, FFN)}
    ys = {}
    ws = []
    flops = 0
    for i, (name, q, K, N, inp) in enumerate(links):
        ws.append(make_quant_weight_gpu(q, N, K, link_seed(0, i)))
        ys.setdefault(N, torch.empty((M, N), device="cuda", dtype=torch.float16))
        flops += 2 * M * N * K
    def step(sp):
        for i, (name, q, K, N, inp) in enumerate(links):
            rt.quant_linear_ex(ws[i].data_ptr(), q, xs[K].data_ptr(), rt.X_F16, ys[N].data_ptr(), rt.Y_F16, M, N, K,
                               K, N, rt.FLAG_STATIC_WEIGHTS, sp)
    ms = graph_time(step, iters=1, replays=3)
    wbytes = sum(w.numel() for w in ws)
    del ws
    torch.cuda.empty_cache()
    return {"ms": ms, "TFLOP/s": flops / (ms * 1e-3) / 1e12, "tflop_per_step": flops / 1e12,
            "weight_gb": wbytes / 1e9, "roofline": tensor_roofline(flops, ms, "f16"),
            "note": "every link on the fused-dequant tcgen05 prefill (Q4_K and Q6_K)"}


# Prefill GEMMs of the stack's shapes at M = 512 (config 5's components).
PREFILL_CASES = {"prefill_q4K_gate_up_M512": (S.Q4_K, 5120, 27648, 512),
                 "prefill_q6K_down_M512": (S.Q6_K, 13824, 5120, 512),
                 "prefill_q6K_head_M512": (S.Q6_K, 5120, 152064, 512)}


def bench_prefill_case(name):
    """One fused-dequant prefill GEMM (vkflame_quant_linear_ex, M = 512)."""
    import torch
    from vkflame_b200 import rt
    q, K, N, M = PREFILL_CASES[name]
    w = make_quant_weight_gpu(q, N, K, 5)
    x = torch.randn((M, K), device="cuda").half()
    y = torch.empty((M, N), device="cuda", dtype=torch.float16)
    def fn(sp):
        rt.quant_linear_ex(w.data_ptr(), q, x.data_ptr(), rt.X_F16, y.data_ptr(), rt.Y_F16, M, N, K, K, N,
                           rt.FLAG_STATIC_WEIGHTS, sp)
    ms = graph_time(fn, iters=3 if N > 100000 else 10)
    flops = 2 * M * N * K
    return {"us": ms * 1e3, "TFLOP/s": flops / (ms * 1e-3) / 1e12, "roofline": tensor_roofline(flops, ms, "f16")}


SUB_CASES = dict({n: (lambda n=n: bench_gemv_case(n)) for n in GEMV_CASES},
                 **{n: (lambda n=n: bench_prefill_case(n)) for n in PREFILL_CASES},
                 config2_int8_linear_M512=bench_int8_linear, config4_q8_0_x_q8_1_M512=bench_q8_prefill,
                 config5_prefill_stack_M512=bench_prefill_stack)


def sub_benchmarks(names=None):
    """Configs 1-4 at their shapes and config 5 at M = 512 (device time, CUDA
    graphs).  Each case is checked for kernel error bits (a bounded wait that
    gave up) on its own; a failing case reports {"error": ...} and the others
    still run."""
    import torch
    from vkflame_b200 import rt
    rt.check_kernel_errors()
    out = {}
    for n in (names or SUB_CASES):
        try:
            r = SUB_CASES[n]()
            torch.cuda.synchronize()
            rt.check_kernel_errors()
            out[n] = r
        except Exception as e:  # noqa: BLE001 - recorded in the JSON line
            out[n] = {"error": f"{type(e).__name__}: {e}"[:300]}
            print(f"sub-benchmark {n} failed: {e}", file=sys.stderr)
    return out


def cpu_baseline_int8(budget_s=3.0):
    """Config 2 on the host: the oracle's int8 linear (int32 accumulators +
    fp16 epilogue, OpenMP over rows) on a 32-row sample of the 512 x 4096 x
    11008 problem, in TOPS."""
    from oracle import pyoracle as po
    cores = os.cpu_count() or 1
    rng = np.random.default_rng(1)
    M, N, K = 32, 11008, 4096
    x = rng.integers(-127, 128, (M, K), dtype=np.int8)
    w = rng.integers(-127, 128, (N, K), dtype=np.int8)
    sx, sw = rng.uniform(1e-3, 1e-2, M).astype(np.float32), rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    po.linear_int8(x[:2], w, sx[:2], sw, want_acc=False, threads=cores)
    t0, reps = time.perf_counter(), 0
    while time.perf_counter() - t0 < budget_s and reps < 50:
        po.linear_int8(x, w, sx, sw, want_acc=False, threads=cores)
        reps += 1
    el = time.perf_counter() - t0
    return {"value": 2 * M * N * K * reps / el / 1e12, "unit": "TOPS", "cores": cores, "kind": "port",
            "sample": f"M=32 of 512 rows, N=11008, K=4096, {reps} reps ({el:.1f} s)"}


def cpu_baseline_q8(budget_s=3.0):
    """Config 4 on the host: the reference's mul_mat sequence (dequant Q8_0 W
    and Q8_1 X to fp32, fp32 dot products) over a 1024-row, 32-token sample."""
    from oracle import pyoracle as po
    cores = os.cpu_count() or 1
    M, N, K = 32, 1024, 5120
    w = S.quant_matrix(S.Q8_0, N, K, seed=3)
    xq = po.quantize_q8_1(S.normal_f32((M, K), seed=4))
    po.quant_linear(S.Q8_0, w, xq, M, N, K, xtype=1, ytype=0, threads=cores)
    t0, reps = time.perf_counter(), 0
    while time.perf_counter() - t0 < budget_s and reps < 50:
        po.quant_linear(S.Q8_0, w, xq, M, N, K, xtype=1, ytype=0, threads=cores)
        reps += 1
    el = time.perf_counter() - t0
    return {"value": 2 * M * N * K * reps / el / 1e12, "unit": "TOPS", "cores": cores, "kind": "port",
            "sample": f"M=32 of 512 rows, N=1024 of 13824, K=5120, {reps} reps ({el:.1f} s)"}


def config_cpu_baselines(configs: dict) -> None:
    """Attaches a bounded host baseline (the oracle's restatement of the
    reference pipeline, all host cores) to each measured config entry."""
    for name, c in configs.items():
        if name in GEMV_CASES:
            q, K, N, M = GEMV_CASES[name]
            if M in (1, 32) or name.endswith("_M8"):
                c["cpu_baseline"] = cpu_baseline_gemv(q, N, K, M, budget_s=1.5)
        elif name.startswith("config2"):
            c["cpu_baseline"] = cpu_baseline_int8()
        elif name.startswith("config4"):
            c["cpu_baseline"] = cpu_baseline_q8()


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


def gemv_timeline(args, world, rank, dist):
    """One token of the per-linear-launch stack with the diagnostic GEMV build:
    for each launch the first CTA start and last CTA end, and per CTA the
    start, dependency release, activations ready, decode loop end and reducer
    end (globaltimer ns).  Prints a per-shape summary (medians over layers)."""
    import ctypes as C
    import torch
    from vkflame_b200 import rt
    lib = rt.lib()
    if not hasattr(lib, "vkf_gemv_timeline"):
        raise SystemExit("--gemv-timeline needs the diagnostic build (VKFLAME_RT_LIB=.../lib/timing/libvkflame_rt.so)")
    lib.vkf_gemv_timeline.argtypes = [C.c_void_p, C.c_int]
    lib.vkf_gemv_cta_times.argtypes = [C.c_void_p, C.c_int]
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        st = Stack(world, rank, dist, s.cuda_stream, mode="launches", layers=args.layers)
        st.step()
        torch.cuda.synchronize()
        lib.vkf_gemv_timeline(None, 1)  # launch ids restart at 0 for the captured graph
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            st.step()
        for _ in range(args.warmup):
            g.replay()
        barrier(dist)
        lib.vkf_gemv_timeline(None, 1)
        barrier(dist)
        e0, e1 = timed_graph(g, s, 1)
        torch.cuda.synchronize()
    n = len(st.ops)
    tl = np.zeros((4096, 3), np.uint64)
    lib.vkf_gemv_timeline(tl.ctypes.data, 0)
    cta = np.zeros((n, 512, 5), np.uint64)
    for i in range(n):
        lib.vkf_gemv_cta_times(cta[i].ctypes.data, i)
    tl, cta = tl[:n].astype(np.int64), cta.astype(np.int64)
    rows = {}
    for i, (name, q, K, nn, *_) in enumerate(st.links):
        c = cta[i][cta[i][:, 0] > 0]
        prev_end = tl[i - 1][1] if i else tl[i][0]
        rows.setdefault(name, []).append([(c[:, 0].max() - c[:, 0].min()) / 1e3, np.median(c[:, 1] - c[:, 0]) / 1e3,
                                          np.median(c[:, 2] - c[:, 1]) / 1e3, np.median(c[:, 3] - c[:, 2]) / 1e3,
                                          np.median(c[:, 4] - c[:, 3]) / 1e3, (tl[i][1] - tl[i][0]) / 1e3,
                                          (tl[i][1] - prev_end) / 1e3, len(c)])
    if rank == 0:
        print(f"token {e0.elapsed_time(e1):.3f} ms (diagnostic build), {n} launches, world {world}")
        print("linear | CTAs | CTA start spread | start->dep release | dep->X ready | decode loop | "
              "reducer tail | launch span | end - previous end  (us, medians over layers)")
        for name, r in rows.items():
            m = np.median(np.array(r), axis=0)
            print(f"{name} | {int(m[7])} | {m[0]:.2f} | {m[1]:.2f} | {m[2]:.2f} | {m[3]:.2f} | {m[4]:.2f} | "
                  f"{m[5]:.2f} | {m[6]:.2f}")
    st.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="stack", choices=["stack"] + list(SUB_CASES),
                    help="stack (config 5, the headline) or one config 1-4 case alone (device time only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the config 1-4 sub-benchmarks")
    ap.add_argument("--stack-mode", default="auto", choices=["auto", "chained", "independent", "launches"],
                    help="auto: independent (persistent kernel) at N = 1, launches (chained) at N > 1")
    ap.add_argument("--layers", type=int, default=LAYERS, help="fewer layers only for profiler captures")
    ap.add_argument("--e2e-hip", action="store_true",
                    help="N = 1: also time the token through libamdhip64 (hipLaunchKernel per linear)")
    ap.add_argument("--watchdog", type=float, default=0,
                    help="dump every thread's Python stack and exit after this many seconds (0: off)")
    ap.add_argument("--trace", default=None, metavar="DIR",
                    help="record per-linear chain timestamps; saved as DIR/chain_trace_w<N>_r<rank>.npy")
    ap.add_argument("--gemv-timeline", action="store_true",
                    help="with --stack-mode launches and the diagnostic build (make -C vkflame_b200/csrc timing; "
                         "VKFLAME_RT_LIB=vkflame_b200/lib/timing/libvkflame_rt.so): per-launch and per-CTA "
                         "timestamps of one token, summarised on stdout")
    args = ap.parse_args()
    if args.watchdog > 0:
        import faulthandler
        faulthandler.dump_traceback_later(args.watchdog, exit=True)
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
    if args.gemv_timeline:
        gemv_timeline(args, world, rank, dist)
        if dist is not None:
            dist.destroy_process_group()
        return
    line = bench_stack(args, world, rank, local, dist)
    if rank == 0 and world == 1:
        if not args.no_extras:
            line["configs"] = sub_benchmarks()
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_stack()
            if "configs" in line:
                config_cpu_baselines(line["configs"])
    if rank == 0:
        print(json.dumps(line))
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
