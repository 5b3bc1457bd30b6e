#!/usr/bin/env python
"""Benchmark: dequantize-fused decode GEMV over Qwen2-7B-shaped quantized linears.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--fmt log4|w4zp8|w8] [--batch B]

Workload: the linears of one Qwen2-7B decode token --
28 layers x (q 3584x3584, k/v 512x3584, o 3584x3584, gate/up 18944x3584,
down 3584x18944) + lm_head 152064x3584 -- in the 4-bit log format, weights
~N(0, 0.02) packed on the device by this repo's packer, activations ~N(0, 1),
batch 1.  One step = every linear once (q|k|v and gate|up share an input and
run as one launch each: 113 GEMV launches per step, issued as one GEMV chain in
which each launch requests the next one's weights into L2).  Synthetic data;
the 3.55 GB of packed weights per step exceed the 126 MB L2, so no flush is
needed.  The same weights are then run at batch 8 and 64 (`batch_lines`).

N > 1: the linears of at least --shard-min-mb MB of packed weights are
column-sharded (output rows split across ranks): each such GEMV's epilogue
stores its rows into every rank's copy of the output over NVLink and publishes
the launch, and whatever reads that output waits for every rank's publication.
Smaller linears run whole on every rank (a column shard of a launch-latency-bound
GEMV costs more in cross-GPU waits than it saves in weight bytes).  Strong
scaling: total work fixed, each linear counted once.  The linears' inputs are
independent synthetic vectors, the same on every rank.

Prints ONE JSON line on rank 0.  `value` is algorithmic GB/s over the whole job
(packed weights + scales + x + y per GEMV); `e2e` is the same metric through the
public host-buffer C-ABI call for a whole step (bramha_cuda_gemv_chain: pinned
host inputs in, every output back in host memory, synchronous).
`--impl reference` times the CPU restatement of the reference's GEMV loop on
this host's cores over the same whole step (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Quant GEMV HBM GB/s vs 8 TB/s peak; decode tokens/s at 1/2/4/8 B200"
H, I, V, LAYERS, NQ, NKV, HD = 3584, 18944, 152064, 28, 28, 4, 128
GROUPS = [  # (name, [(part, N)], K) -- parts in one group share the input
    ("qkv", [("q", NQ * HD), ("k", NKV * HD), ("v", NKV * HD)], H),
    ("o", [("o", H)], H),
    ("gate_up", [("gate", I), ("up", I)], H),
    ("down", [("down", H)], I),
]
BITS = {"log4": 4, "w4zp8": 4, "w8": 8}


def gemv_bytes(n, k, batch, bits):
    """Algorithmic bytes of one GEMV: packed weights + scales + x + y."""
    return n * k * bits // 8 + 4 * n + 4 * batch * k + 4 * batch * n


def token_linears(layers=LAYERS):
    """[(name, N, K)] for every linear of one decode token."""
    out = []
    for _ in range(layers):
        for _, parts, k in GROUPS:
            out += [(p, n, k) for p, n in parts]
    out.append(("lm_head", V, H))
    return out


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.path = os.path.join(tempfile.gettempdir(), f"bramha_bench_clocks_{os.getpid()}_dev{device}.csv")

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) != 6:
                continue
            try:
                sm.append(float(parts[0]))
                smax.append(float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[2:]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------ distributed
def dist_setup(args):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws != args.gpus:
        if ws == 1 and args.gpus > 1:
            raise SystemExit("--gpus N > 1 must be launched with torch.distributed.run (one process per GPU)")
    return ws, rank, local


# ------------------------------------------------------------- reference arm
class CpuStep:
    """The reference's CPU decode GEMV loop over a whole decode step: the C
    restatement of `matvec_mul_into` (src/inference/cpu_engine.rs:1307-1444;
    log4 through its tables) on every linear of `layers` Qwen2-7B layers + the
    lm_head, OpenMP over rows on all host threads, built -march=native as the
    reference builds with target-cpu=native.  The packed codes of the whole
    step (3.55 GB at 4 bits for 28 layers) sit in host memory and are streamed
    once per step, as the GPU arm streams them from HBM; they are drawn as
    uniform random bytes (the CPU loop's time does not depend on code values).
    Each linear has its own N(0, 1) input."""

    def __init__(self, fmt, batch, layers=LAYERS, seed=2024):
        import oracle
        self.oracle = oracle
        self.native = oracle.use_native_build()
        self.threads = oracle.max_threads()
        self.fmt, self.batch = fmt, batch
        bits = BITS[fmt]
        rng = np.random.Generator(np.random.PCG64(seed))
        self.work = []
        for _, n, k in token_linears(layers):
            q = np.frombuffer(rng.bytes(n * k * bits // 8), dtype=np.uint8)
            if fmt == "w8":
                q = q.view(np.int8)
            s = rng.uniform(1e-4, 1e-3, n).astype(np.float32)
            x = rng.standard_normal((batch, k), dtype=np.float32)
            self.work.append((n, k, q, s, x))
        self.nbytes = sum(gemv_bytes(n, k, batch, bits) for n, k, _, _, _ in self.work)
        self.layers = layers

    def step(self):
        o = self.oracle
        for n, k, q, s, x in self.work:
            for b in range(self.batch):
                if self.fmt == "log4":
                    o.matvec_fused_log4(x[b], q, s, n, threads=self.threads)
                else:
                    o.matvec_mul_into(self.fmt, x[b], q, s, n, threads=self.threads)

    def timed(self, steps):
        t0 = time.perf_counter()
        for _ in range(steps):
            self.step()
        return (time.perf_counter() - t0) / steps

    def describe(self, steps, repeats):
        return (f"{'whole step' if self.layers == LAYERS else f'{self.layers} layers'}: {self.layers} layers x 7 "
                f"linears + lm_head ({self.nbytes / 1e9:.2f} GB packed, streamed from host memory), batch "
                f"{self.batch}, {steps} steps x {repeats} timed regions; C restatement of matvec_mul_into "
                f"(cpu_engine.rs:1307-1444), OpenMP over rows, "
                + ("-march=native" if self.native else "-march=x86-64-v3 (native build unavailable)"))


def run_reference(args, ws, rank):
    """The reference's CPU GEMV loop (restated in C) on all host threads, over
    the same workload as the GPU arm: every linear of the decode step."""
    if rank != 0:
        return
    cs = CpuStep(args.fmt, args.batch)
    for _ in range(args.warmup):
        cs.step()
    reps = [cs.timed(args.steps) for _ in range(max(1, args.repeats))]
    dt = reps[0]
    gbs = cs.nbytes / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random packed codes and scales, N(0,1) activations)",
        "config": {"workload": f"qwen2-7b linears ({LAYERS} layers + lm_head), {args.fmt}, batch {args.batch} "
                               "decode GEMV",
                   "batch": args.batch, "fmt": args.fmt, "hidden": H, "intermediate": I, "vocab": V,
                   "layers": LAYERS, "parallelism": "host threads (CPU)",
                   "l2": f"no flush: {cs.nbytes / 1e9:.2f} GB of packed weights per step >> host LLC"},
        "tokens_per_s": round(args.batch / dt, 3),
        "spread": {"repeats": len(reps), "steps_each": args.steps,
                   "ms_per_step_median": round(statistics.median(reps) * 1e3, 3),
                   "ms_per_step_min": round(min(reps) * 1e3, 3), "ms_per_step_max": round(max(reps) * 1e3, 3)},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cs.threads, "kind": "port",
                         "sample": cs.describe(args.steps, len(reps))},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_sample(fmt, batch, steps=3):
    """The reference arm's CPU loop on the same whole-step workload, a few steps
    (rank 0 at N = 1 only)."""
    cs = CpuStep(fmt, batch)
    cs.step()
    dt = cs.timed(steps)
    return {"value": round(cs.nbytes / dt / 1e9, 3), "unit": "GB/s", "cores": cs.threads, "kind": "port",
            "ms_per_step": round(dt * 1e3, 2), "sample": cs.describe(steps, 1)}


# ------------------------------------------------------------------ batch 8 / 64 (config 4)
def batch_lines(plane, dev, layers, fmt, batches=(8, 64), reps=5):
    """BASELINE config 4 at batch 8 and 64 on the step's registered weights:
    the step's 113 launches (q|k|v and gate|up fused) as one GEMV chain in a
    CUDA graph, device time over `reps` replays.  Batch 8 runs on the tensor-core
    GEMV (HBM-bound); batch 64 on the tcgen05 GEMM with the f32 rows split into
    bf16 hi + lo halves of the MMA's N (twice the MMA work of 2*B*N*K, so it is
    bound by the tensor pipe).  The roofline object covers the dominant linear
    (per-group launches timed from their own graphs)."""
    import torch
    bits = BITS[fmt]
    hbm, hbm_kind = load_peaks()
    pk_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    tflops_peak = json.load(open(pk_path))["bf16_tflops"] if os.path.exists(pk_path) else 1590.0
    stream = torch.cuda.Stream(device=dev)
    gen = torch.Generator(device=dev).manual_seed(64)
    out = {}
    for B in batches:
        ops, groups, nbytes, flops = [], {}, 0, 0
        for entry in layers:
            for gname, wts, x, _, _ in entry:
                k = x.shape[1]
                xb = torch.randn((B, k), generator=gen, device=dev)
                yb = [torch.empty((B, w.N), device=dev) for w in wts]
                ops.append((wts, xb, yb))
                groups.setdefault(gname, []).append((wts, xb, yb))
                nbytes += sum(gemv_bytes(w.N, k, B, bits) for w in wts)
                flops += sum(2 * B * w.N * k for w in wts)
        with torch.cuda.stream(stream):
            plane.gemv_chain_dev(ops, B, stream)
        torch.cuda.synchronize()

        def graph_ms(items, n_rep):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                plane.gemv_chain_dev(items, B, stream)
            with torch.cuda.stream(stream):
                g.replay()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                for _ in range(n_rep):
                    g.replay()
                b.record()
            torch.cuda.synchronize()
            del g
            return a.elapsed_time(b) / n_rep

        ms = graph_ms(ops, reps)
        plane.stream_sync(stream)
        per = {}
        for gname, items in groups.items():
            gms = graph_ms(items, 3)
            gb = sum(sum(gemv_bytes(w.N, x.shape[1], B, bits) for w in wts) for wts, x, _ in items)
            gf = sum(sum(2 * B * w.N * x.shape[1] for w in wts) for wts, x, _ in items)
            per[gname] = {"launches": len(items), "us_mean": round(gms * 1e3 / len(items), 2),
                          "gbs": round(gb / (gms * 1e-3) / 1e9, 1), "tflops": round(gf / (gms * 1e-3) / 1e12, 1),
                          "ms": gms}
        tot = sum(v["ms"] for v in per.values())
        for v in per.values():
            v["share"] = round(v.pop("ms") / tot, 3)
        dom = max(per, key=lambda g_: per[g_]["share"])
        if B <= 8:
            ach = per[dom]["gbs"]
            roof = {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": round(ach / hbm, 4),
                    "kernel": f"tc_gemv_kernel<{fmt}, {B}> ({dom})", "peak_source": f"{hbm_kind} hbm_gbs"}
        else:
            ach = per[dom]["tflops"]
            roof = {"bound": "tensor", "achieved": ach, "peak": tflops_peak, "unit": "TFLOP/s",
                    "frac": round(ach / tflops_peak, 4), "kernel": f"gemm_kernel<{fmt}> ({dom}), bf16 hi+lo",
                    "peak_source": "measured bf16_tflops (burst)" if os.path.exists(pk_path) else "fallback",
                    "note": "achieved counts the GEMV's 2*B*N*K; the hi+lo split issues twice that on the tensor pipe"}
        out[str(B)] = {"ms_per_step": round(ms, 4), "value": round(nbytes / (ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                       "tokens_per_s": round(B / (ms * 1e-3), 1), "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
                       "frac_of_hbm_peak_step": round(nbytes / (ms * 1e-3) / 1e9 / hbm, 4),
                       "roofline": roof, "per_linear": per,
                       "timing": f"CUDA graph of the step's chain, {reps} replays, device time"}
        del ops, groups
    return out


# ------------------------------------------------------------------ prefill (config 3)
QWEN05 = [("q", 896, 896), ("k", 128, 896), ("v", 128, 896), ("o", 896, 896), ("gate", 4864, 896),
          ("up", 4864, 896), ("down", 896, 4864), ("lm_head", 151936, 896)]


def prefill_bench(plane, dev, reps=10, m=2048):
    """tcgen05 dequant-GEMM, M = 2048 bf16 tokens on the Qwen2-0.5B
    linears (log4 and int8 weights ~N(0,0.02)); TFLOP/s = 2*M*N*K / CUDA-event time of
    `reps` calls replayed from a CUDA graph (per-call time includes the per-token-sum
    kernel that log4 needs)."""
    import torch
    pk_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    measured = os.path.exists(pk_path)
    peaks = json.load(open(pk_path)) if measured else {"bf16_tflops": 1590.0}
    out = {"workload": f"qwen2-0.5b linears, M={m} bf16 tokens", "peak_tflops": peaks["bf16_tflops"],
           "peak_source": "measured bf16_tflops (burst), MEASURED_PEAKS.json" if measured
           else "fallback 1.59 PFLOP/s (MEASURED_PEAKS.json absent)",
           "timing": f"CUDA graph of {reps} calls per shape, device time", "shapes": {}}
    gen = torch.Generator(device=dev).manual_seed(5)
    stream = torch.cuda.Stream(device=dev)
    for fmt in ("log4", "w8"):
        tot_flop, tot_ms = 0.0, 0.0
        for name, n, k in QWEN05:
            wf = torch.randn((n, k), generator=gen, device=dev) * 0.02
            nb = n * k * (4 if fmt == "log4" else 8) // 8
            qd = torch.empty(nb, dtype=torch.uint8, device=dev)
            sd = torch.empty(n, dtype=torch.float32, device=dev)
            plane.quantize_dev(fmt, wf, qd, sd)
            del wf
            w = plane.register_dev(f"pf:{fmt}:{name}", fmt, n, k, qd, sd)
            x = torch.randn((m, k), generator=gen, device=dev).to(torch.bfloat16)
            y = torch.empty((m, n), dtype=torch.float32, device=dev)
            torch.cuda.synchronize()
            with torch.cuda.stream(stream):
                for _ in range(3):
                    plane.gemm_dev(w, x, y)
            torch.cuda.synchronize()
            # device time: `reps` calls captured in a CUDA graph (the host-side cost of a
            # call -- tensor-map encoding, launch -- is not part of the tensor-pipe figure)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for _ in range(reps):
                    plane.gemm_dev(w, x, y)
            graph.replay()
            torch.cuda.synchronize()
            with torch.cuda.stream(stream):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(3):
                    graph.replay()
                e1.record()
            torch.cuda.synchronize()
            plane.stream_sync(stream)
            del graph
            ms = e0.elapsed_time(e1) / (3 * reps)
            flop = 2.0 * m * n * k
            tot_flop += flop
            tot_ms += ms
            out["shapes"][f"{fmt}:{name}"] = {"n": n, "k": k, "us": round(ms * 1e3, 2),
                                              "tflops": round(flop / (ms * 1e-3) / 1e12, 1)}
            plane.evict(w.key)
            del qd, sd, x, y
        out[f"{fmt}_total_tflops"] = round(tot_flop / (tot_ms * 1e-3) / 1e12, 1)
    lm = out["shapes"]["log4:lm_head"]["tflops"]
    out["frac_lm_head_log4"] = round(lm / out["peak_tflops"], 3)
    return out


# ------------------------------------------------------------------ 2:4 sparse GEMV
SP_VB = {"f32": 8, "w8": 2, "w4zp8": 1}  # device bytes of one group's kept pair


def sp24_bytes(fmt, n, k):
    """Algorithmic bytes of one 2:4 GEMV launch: kept code pairs + 4-bit column
    pairs of the K/4 groups, the row scales, x and y."""
    g = k // 4
    return n * g * SP_VB[fmt] + n * g // 2 + 4 * n + 4 * k + 4 * n


def sparse24_bench(plane, dev, layers=4, reps=5):
    """2:4 structured-sparse GEMV (sparse_matvec_mul_2_4_tensor_into /
    sparse_matvec_2_4_compressed) on the Qwen2-7B MLP shapes: gate and up
    (18944 x 3584) and down (3584 x 18944) of `layers` layers, weights ~N(0,0.02)
    quantized on the device (f32, w8, w4zp8) and registered as 2:4.  One pass =
    the 3*layers launches (more bytes than the 126 MB L2 in every format),
    captured in a CUDA graph and replayed `reps` times between CUDA events;
    the dense GEMV of the same codes is timed the same way for comparison.
    The CPU figure is the oracle's restatement (OpenMP over rows, all host
    threads) on one gate matrix."""
    import torch
    import oracle
    hbm, kind = load_peaks()
    shapes = [("gate", I, H), ("up", I, H), ("down", H, I)]
    out = {"workload": f"qwen2-7b mlp (gate, up, down) x {layers} layers, batch 1",
           "peak_gbs": hbm, "peak_source": f"{kind} hbm_gbs" + (" (MEASURED_PEAKS.json)" if kind == "measured" else
                                                                    " (6.65 TB/s, MEASURED_PEAKS.json absent)"),
           "timing": f"CUDA graph of one pass ({3 * layers} launches), {reps} replays, device time",
           "formats": {}}
    gen = torch.Generator(device=dev).manual_seed(24)
    stream = torch.cuda.Stream(device=dev)
    x_in = {k: torch.randn(k, generator=gen, device=dev) for k in (H, I)}
    host_sample = None
    for fmt in ("w4zp8", "w8", "f32"):
        sp, dense, ys, nbytes, dbytes = [], [], [], 0, 0
        for l in range(layers):
            for name, n, k in shapes:
                wf = torch.randn((n, k), generator=gen, device=dev) * 0.02
                if fmt == "f32":
                    qd, sd = wf, None
                else:
                    qd = torch.empty(n * k * BITS[fmt] // 8, dtype=torch.uint8, device=dev)
                    sd = torch.empty(n, dtype=torch.float32, device=dev)
                    plane.quantize_dev(fmt, wf, qd, sd)
                    del wf
                key = f"sp24b:{fmt}:{l}:{name}"
                sp.append((plane.register_sparse24_dev(key, fmt, n, k, qd, sd), k))
                dense.append((plane.register_dev(key + ":dense", fmt, n, k, qd, sd), k))
                ys.append(torch.empty(n, device=dev))
                nbytes += sp24_bytes(fmt, n, k)
                dbytes += gemv_bytes(n, k, 1, 32 if fmt == "f32" else BITS[fmt])
                if fmt == "w4zp8" and l == 0 and name == "gate":
                    host_sample = (n, k, qd.cpu().numpy(), sd.cpu().numpy())
                del qd, sd
        torch.cuda.synchronize()

        def timed(ws_):
            with torch.cuda.stream(stream):
                for (w, k), y in zip(ws_, ys):
                    plane.gemv_dev(w, x_in[k], y)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for (w, k), y in zip(ws_, ys):
                    plane.gemv_dev(w, x_in[k], y)
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize()
            with torch.cuda.stream(stream):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(reps):
                    graph.replay()
                e1.record()
            torch.cuda.synchronize()
            plane.stream_sync(stream)
            del graph
            return e0.elapsed_time(e1) / reps

        ms = timed(sp)
        ms_dense = timed(dense)
        per_launch_us = ms * 1e3 / len(sp)
        gbs = nbytes / (ms * 1e-3) / 1e9
        out["formats"][fmt] = {
            "us_per_pass": round(ms * 1e3, 1), "us_per_launch": round(per_launch_us, 2),
            "bytes_per_pass": nbytes, "achieved_gbs": round(gbs, 1), "frac": round(gbs / hbm, 4),
            "dense_us_per_pass": round(ms_dense * 1e3, 1), "dense_bytes_per_pass": dbytes,
            "speedup_vs_dense": round(ms_dense / ms, 3)}
        for (w, _), (d, _) in zip(sp, dense):
            plane.evict(w.key)
            plane.evict(d.key)
        del sp, dense, ys
    if host_sample is not None:
        n, k, q, s = host_sample
        x = np.random.Generator(np.random.PCG64(3)).standard_normal(k, dtype=np.float32)
        threads = oracle.max_threads()
        oracle.sparse_matvec_2_4("w4zp8", x, q, s, n, threads=threads)
        reps_c, t0 = 0, time.perf_counter()
        while reps_c < 3 or time.perf_counter() - t0 < 4.0:
            oracle.sparse_matvec_2_4("w4zp8", x, q, s, n, threads=threads)
            reps_c += 1
        dt = (time.perf_counter() - t0) / reps_c
        gpu_us = out["formats"]["w4zp8"]["us_per_launch"]
        out["cpu_baseline"] = {"us_per_launch": round(dt * 1e6, 1), "cores": threads, "kind": "port",
                               "sample": f"one w4zp8 gate matrix ({n} x {k}) x {reps_c} reps: C restatement of "
                                         "sparse_matvec_mul_2_4_tensor_into (cpu_engine.rs:1532-1640), "
                                         "OpenMP over rows",
                               "gpu_over_cpu": round(dt * 1e6 / gpu_us, 1)}
    return out


# ------------------------------------------------------------------ MoE (config 5)
def moe_bench(plane, dev, tokens=256, experts=64, top_k=8, hidden=3584, inter=2560, reps=10, cpu_tokens=8):
    """the MoE expert MLP of `tokens` decode tokens, 64
    SwiGLU experts (hidden 3584, intermediate 2560) in log4 from ~N(0,0.02),
    top-8 routing from softmax of seeded N(0,1) logits, one GPU.  One call =
    routing, gather, grouped gate+up GEMM, SiLU*up, grouped down GEMM,
    combine (bramha_cuda_moe_mlp_dev), timed with CUDA events over `reps`
    calls.  Algorithmic bytes = the distinct experts touched x 3*H*I/2 (+ their
    scales) + x, logits and out."""
    import torch
    import oracle
    hbm, kind = load_peaks()
    E, H, I, T, k = experts, hidden, inter, tokens, top_k
    gen = torch.Generator(device=dev).manual_seed(55)
    gu_q = torch.empty(E * 2 * I * H // 2, dtype=torch.uint8, device=dev)
    gu_s = torch.empty(E * 2 * I, dtype=torch.float32, device=dev)
    dn_q = torch.empty(E * H * I // 2, dtype=torch.uint8, device=dev)
    dn_s = torch.empty(E * H, dtype=torch.float32, device=dev)
    for e in range(E):
        wf = torch.randn((2 * I, H), generator=gen, device=dev) * 0.02
        plane.quantize_dev("log4", wf, gu_q[e * I * H:(e + 1) * I * H], gu_s[e * 2 * I:(e + 1) * 2 * I])
        wf = torch.randn((H, I), generator=gen, device=dev) * 0.02
        plane.quantize_dev("log4", wf, dn_q[e * H * I // 2:(e + 1) * H * I // 2], dn_s[e * H:(e + 1) * H])
    del wf
    gu = plane.register_dev("moeb:gate_up", "log4", E * 2 * I, H, gu_q, gu_s)
    dn = plane.register_dev("moeb:down", "log4", E * H, I, dn_q, dn_s)
    x = torch.randn((T, H), generator=gen, device=dev)
    lg = torch.randn((T, E), generator=gen, device=dev)
    out = torch.empty((T, H), device=dev)
    sel = torch.empty((T, k), dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for _ in range(3):
            plane.moe_mlp_dev(gu, dn, E, k, x, lg, out, sel)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            plane.moe_mlp_dev(gu, dn, E, k, x, lg, out, sel)
        e1.record()
    torch.cuda.synchronize()
    plane.stream_sync(stream)
    ms = e0.elapsed_time(e1) / reps
    touched = int(torch.unique(sel).numel())
    per_expert = 3 * H * I // 2 + 4 * (2 * I + H)
    nbytes = touched * per_expert + 4 * (2 * T * H + T * E)
    gbs = nbytes / (ms * 1e-3) / 1e9
    # end to end through the host-buffer call
    xh, lh = x.cpu().numpy(), lg.cpu().numpy()
    plane.moe_mlp(gu, dn, E, k, xh, lh)
    t0 = time.perf_counter()
    n_e2e = 5
    for _ in range(n_e2e):
        plane.moe_mlp(gu, dn, E, k, xh, lh)
    e2e_s = (time.perf_counter() - t0) / n_e2e
    res = {"workload": f"moe mlp: {T} tokens, {E} experts top-{k}, hidden {H}, intermediate {I}, log4, 1 GPU",
           "us_per_call": round(ms * 1e3, 1), "tokens_per_s": round(T / (ms * 1e-3), 1),
           "experts_touched": touched, "bytes_per_call": nbytes, "achieved_gbs": round(gbs, 1),
           "peak_gbs": hbm, "frac": round(gbs / hbm, 4),
           "peak_source": f"{kind} hbm_gbs" + (" (MEASURED_PEAKS.json)" if kind == "measured" else " (6.65 TB/s)"),
           "timing": f"CUDA events over {reps} calls of bramha_cuda_moe_mlp_dev (eager; scratch from the pool)",
           "e2e": {"tokens_per_s": round(T / e2e_s, 1), "api": "bramha_cuda_moe_mlp (host buffers, synchronous)",
                   "h2d_bytes": 4 * (T * H + T * E), "d2h_bytes": 4 * (T * H + T * k)}}
    # CPU: the oracle's restatement on a bounded sample of tokens, all host threads
    gq, gs, dq, ds = gu_q.cpu().numpy(), gu_s.cpu().numpy(), dn_q.cpu().numpy(), dn_s.cpu().numpy()
    # the oracle takes gate and up as separate stacks
    g4 = gq.reshape(E, 2, I * H // 2)
    s4 = gs.reshape(E, 2, I)
    gate = (np.ascontiguousarray(g4[:, 0]).reshape(-1), np.ascontiguousarray(s4[:, 0]).reshape(-1))
    up = (np.ascontiguousarray(g4[:, 1]).reshape(-1), np.ascontiguousarray(s4[:, 1]).reshape(-1))
    threads = oracle.max_threads()
    t0 = time.perf_counter()
    ref, _, _ = oracle.moe_mlp("log4", xh[:cpu_tokens], lh[:cpu_tokens], k, gate, up, (dq, ds), threads=threads)
    dt = time.perf_counter() - t0
    res["cpu_baseline"] = {"tokens_per_s": round(cpu_tokens / dt, 2), "cores": threads, "kind": "port",
                           "sample": f"{cpu_tokens} of the {T} tokens through the C restatement of run_mlp_into's "
                                     "MoE branch (cpu_engine.rs:1799-1989), OpenMP over tokens"}
    gpu_out = out.cpu().numpy()[:cpu_tokens]
    res["check_normwise_err_vs_cpu"] = float(np.max(np.abs(gpu_out - ref)) / np.max(np.abs(ref)))
    plane.evict(gu.key)
    plane.evict(dn.key)
    return res


# ------------------------------------------------------------------ decode step (config 2)
def decode_step_bench(plane, dev, prompt_len=512, new_tokens=128, fuse_norm=False):
    """a full Qwen2-0.5B-architecture decode step (24 layers,
    hidden 896, 14/2 heads of 64, SwiGLU 4864, RMSNorm 1e-6, RoPE 1e6, vocab
    151936) with random weights in log4, KV cache prefilled to `prompt_len` from
    uniform-random token ids (teacher forced), then `new_tokens` greedy tokens
    (repetition penalty 1.15, EOS stop disabled).  Each token is one replay of
    the step's CUDA graph; tokens/s from CUDA events over the greedy tokens.
    gemv_share = device time of the step's GEMV launches alone (their own graph)
    / the step's time."""
    import torch
    from bramha_b200 import DecodeConfig, DecodeLayer, DecodeModel

    cfg = DecodeConfig()
    gen = torch.Generator(device=dev).manual_seed(2024)
    qd, kvd, H, I, V = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim, cfg.hidden, cfg.intermediate, cfg.vocab
    keys = []

    def lin(name, n, k):
        wf = torch.randn((n, k), generator=gen, device=dev) * 0.02
        qb = torch.empty(n * k // 2, dtype=torch.uint8, device=dev)
        sb = torch.empty(n, dtype=torch.float32, device=dev)
        plane.quantize_dev("log4", wf, qb, sb)
        w = plane.register_dev(f"c2:{name}", "log4", n, k, qb, sb)
        keys.append(w.key)
        return w

    vec = lambda n, mean, std: torch.randn(n, generator=gen, device=dev) * std + mean
    layers = [DecodeLayer(vec(H, 1, 0.1), lin(f"{i}.q", qd, H), lin(f"{i}.k", kvd, H), lin(f"{i}.v", kvd, H),
                          vec(qd, 0, 0.1), vec(kvd, 0, 0.1), vec(kvd, 0, 0.1), lin(f"{i}.o", H, qd), vec(H, 1, 0.1),
                          lin(f"{i}.g", I, H), lin(f"{i}.u", I, H), lin(f"{i}.d", H, I)) for i in range(cfg.layers)]
    embed = torch.randn((V, H), generator=gen, device=dev)
    dm = DecodeModel(plane, cfg, layers, embed, vec(H, 1, 0.1), lin("lm", V, H),
                     max_ctx=prompt_len + new_tokens, max_generated=new_tokens, fuse_norm=fuse_norm)
    dm.capture()
    prompt = torch.randint(0, V, (prompt_len,), generator=torch.Generator().manual_seed(7)).tolist()
    dm.reset()
    e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    with torch.cuda.stream(dm.stream):
        e[0].record()
        for tok in prompt[:-1]:
            dm.set_token(tok)
            dm.step(greedy=False)
        e[1].record()
        dm.set_token(prompt[-1])
        e[2].record()
        for _ in range(new_tokens):
            dm.step(greedy=True)
        e[3].record()
    dm.sync()
    ms_tok = e[2].elapsed_time(e[3]) / new_tokens
    prefill_ms = e[0].elapsed_time(e[1]) / (prompt_len - 1)
    toks = dm.generated_tokens()
    # the step's GEMV launches alone, in their own graph
    gg = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gg, stream=dm.stream):
        for lw in dm.layers:
            plane.gemv_multi_dev([lw.q, lw.k, lw.v], dm.h, [dm.q, dm.k, dm.v], stream=dm.stream)
            plane.gemv_multi_dev([lw.o], dm.attn, [dm.o], stream=dm.stream)
            plane.gemv_multi_dev([lw.gate, lw.up], dm.h, [dm.g, dm.u], stream=dm.stream)
            plane.gemv_swiglu_dev(lw.down, dm.g, dm.u, dm.d, stream=dm.stream)
        plane.gemv_multi_dev([dm.lm_head], dm.h, [dm.logits], stream=dm.stream)
    reps = 20
    with torch.cuda.stream(dm.stream):
        gg.replay()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            gg.replay()
        b.record()
    dm.sync()
    gemv_ms = a.elapsed_time(b) / reps
    del gg
    dm.release()
    out = {"workload": f"qwen2-0.5b decode step ({cfg.layers} layers, log4 linears, f32 norms/biases/embedding), "
                       f"KV prefilled to {prompt_len} from uniform-random ids, {new_tokens} greedy tokens",
           "tokens_per_s": round(1e3 / ms_tok, 1), "ms_per_token": round(ms_tok, 4),
           "prefill_ms_per_token": round(prefill_ms, 4), "gemv_ms_per_token": round(gemv_ms, 4),
           "gemv_share": round(gemv_ms / ms_tok, 3), "kernel_launches_per_token": dm.kernel_launches_per_step(),
           "cuda_graph": True, "distinct_generated": len(set(toks)),
           "data": "synthetic: weights N(0,0.02) packed on the device, norms 1+N(0,0.1), biases N(0,0.1), "
                   "embedding N(0,1)"}
    for k in keys:
        plane.evict(k)
    del dm, layers, embed
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------ our arm
def run_ours(args, ws, rank, local):
    import torch
    import torch.distributed as dist
    from bramha_b200 import CudaComputePlane

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=120))
    plane = CudaComputePlane(local)
    fmt, B, bits = args.fmt, args.batch, BITS[args.fmt]
    sp = None
    if ws > 1:
        # column-shard group: a large linear's output rows split across the ranks; the
        # GEMV epilogue stores each rank's rows into every rank's copy over NVLink
        from bramha_b200 import ShardedPlane
        sp = ShardedPlane(plane, arena_bytes=64 << 20)
    shard_min = int(args.shard_min_mb * (1 << 20))

    # ---- weights: each linear generated whole (N(0,0.02), the same seed on every
    # rank), packed on the device; with N > 1 each rank keeps its rows
    gen = torch.Generator(device=dev)
    layers = []  # per layer: list of (group, [Weight], x, [y], None)
    step_bytes = 0
    t_setup = time.time()
    for li in range(args.layers + 1):
        groups = GROUPS if li < args.layers else [("lm_head", [("lm_head", V)], H)]
        entry = []
        for gname, parts, k in groups:
            wts, ys = [], []
            sharded = sp is not None and sum(n * k * bits // 8 for _, n in parts) >= shard_min
            for p, n in parts:
                gen.manual_seed(1_000_003 * li + sum(map(ord, p)))
                wf = torch.randn((n, k), generator=gen, device=dev, dtype=torch.float32).mul_(0.02)
                qd = torch.empty(n * k * bits // 8, dtype=torch.uint8, device=dev)
                sd = torch.empty(n, dtype=torch.float32, device=dev)
                plane.quantize_dev(fmt, wf, qd, sd)
                del wf
                if not sharded:
                    w = plane.register_dev(f"L{li}.{p}", fmt, n, k, qd, sd)
                    ys.append(torch.empty((B, n), dtype=torch.float32, device=dev))
                else:
                    w = sp.register_dev(f"L{li}.{p}", fmt, n, k, qd, sd)
                    ys.append(sp.empty((B, n)))  # the full output, in the symmetric arena
                del qd, sd
                wts.append(w)
                step_bytes += gemv_bytes(n, k, B, bits)  # whole-job algorithmic bytes
            gen.manual_seed(7 + li * 13 + len(entry))
            x = torch.randn((B, k), generator=gen, device=dev, dtype=torch.float32)
            entry.append((gname, wts, x, ys, sharded))
        layers.append(entry)
    torch.cuda.synchronize()
    setup_s = time.time() - t_setup
    launches_per_step = sum(len(e) for e in layers)

    stream = torch.cuda.Stream(device=dev)
    # the step is one GEMV chain (bramha_cuda_gemv_chain_dev); with N > 1 a run of
    # sharded GEMVs is followed by a wait for every rank's rows before an unsharded
    # GEMV (its input may be their output), and the step ends when all have landed
    flat = [(wts, x, ys, shd) for entry in layers for _, wts, x, ys, shd in entry]
    segments = []  # [(ops, ends with a sharded op)]
    for wts, x, ys, shd in flat:
        if not segments or (segments[-1][1] and not shd):
            segments.append(([], shd))
        segments[-1][0].append((wts, x, ys))
        segments[-1] = (segments[-1][0], shd)
    n_sharded = sum(1 for *_, shd in flat if shd)

    def step():
        for ops, ends_sharded in segments:
            plane.gemv_chain_dev(ops, B, stream)
            if ends_sharded:
                sp.sync(stream)

    # ---- capture one step (GEMVs and, on several GPUs, the NCCL all-gathers) in a
    # CUDA graph; replay it K times
    with torch.cuda.stream(stream):
        step()  # warm the launch path (occupancy queries, NCCL communicators) before capture
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier(device_ids=[local])
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    torch.cuda.synchronize()

    def run_step():
        if graph is not None:
            graph.replay()
        else:
            step()

    def barrier():
        if ws > 1:
            dist.barrier(device_ids=[local])

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            run_step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    with clocks:
        with torch.cuda.stream(stream):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                run_step()
            e1.record()
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    if ws > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = step_bytes / (ms * 1e-3) / 1e9

    # ---- spread: the same K-step region timed `repeats` more times
    rep_ms = []
    for _ in range(args.repeats):
        barrier()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            r0.record()
            for _ in range(args.steps):
                run_step()
            r1.record()
        torch.cuda.synchronize()
        v = r0.elapsed_time(r1) / args.steps
        if ws > 1:
            t = torch.tensor([v], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            v = float(t.item())
        rep_ms.append(v)
    spread = None
    if rep_ms:
        spread = {"repeats": len(rep_ms), "steps_each": args.steps,
                  "ms_per_step_median": round(statistics.median(rep_ms), 4),
                  "ms_per_step_min": round(min(rep_ms), 4), "ms_per_step_max": round(max(rep_ms), 4),
                  "value_median": round(step_bytes / (statistics.median(rep_ms) * 1e-3) / 1e9, 2)}

    # ---- per-launch durations: each group's launches (e.g. the 28 gate|up GEMVs)
    # captured in their own CUDA graph and replayed, so host launch latency is
    # not part of the measurement; mean device time per launch
    groups, group_sharded = {}, {}
    for entry in layers:
        for gname, wts, x, ys, shd in entry:
            groups.setdefault(gname, []).append((wts, x, ys))
            group_sharded[gname] = shd
    per = {}
    reps = 5
    for gname, items in groups.items():
        gg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gg, stream=stream):
            plane.gemv_chain_dev(items, B, stream)
            if group_sharded[gname]:
                sp.sync(stream)
        gg.replay()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a_.record()
            for _ in range(reps):
                gg.replay()
            b_.record()
        torch.cuda.synchronize()
        per[gname] = [a_.elapsed_time(b_) * 1e3 / (reps * len(items))] * len(items)
        del gg
    def shard(n, g):  # this rank's rows [lo, hi) of an n-row linear of group g
        return (n * rank // ws, n * (rank + 1) // ws) if group_sharded[g] else (0, n)

    group_bytes = {}  # this rank's algorithmic bytes per launch of each group
    for gname, parts, k in GROUPS + [("lm_head", [("lm_head", V)], H)]:
        group_bytes[gname] = sum(gemv_bytes(shard(n, gname)[1] - shard(n, gname)[0], k, B, bits) for _, n in parts)
    per_linear = {g: {"launches_per_step": len(v), "us_mean": round(sum(v) / len(v), 2),
                      "gbs": round(group_bytes[g] / (sum(v) / len(v) * 1e-6) / 1e9, 1),
                      "share": round(sum(v) / sum(sum(u) for u in per.values()), 3)} for g, v in per.items()}
    dom = max(per_linear, key=lambda g: per_linear[g]["share"])
    peak, peak_kind = load_peaks()
    achieved = per_linear[dom]["gbs"]
    traffic = None
    tpath = os.path.join(ROOT, "profiles", f"traffic_{fmt}_b{B}.json")
    if os.path.exists(tpath):
        try:
            traffic = json.load(open(tpath)).get(dom)
        except Exception:
            traffic = None

    # ---- e2e: the public host-buffer call for the whole step: one
    # bramha_cuda_host_chain_run per step (pinned host inputs copied in, the
    # 113 launches, every output copied back, one wait)
    h2d = d2h = 0
    host_ops = []
    for entry in layers:
        for gname, wts, x, ys, _ in entry:
            xh = torch.empty((B, x.shape[1]), dtype=torch.float32, pin_memory=True)
            xh.copy_(x.cpu())
            yhs = [torch.empty((B, w.n_full), dtype=torch.float32, pin_memory=True) for w in wts]
            host_ops.append((wts, xh, yhs))
            h2d += xh.numel() * 4
            d2h += sum(y.numel() * 4 for y in yhs)

    host_chain = plane.prepare_chain(host_ops, B)  # bound once (bramha_cuda_host_chain_create), as a host program would

    def e2e_step():
        host_chain.run()  # N > 1: every rank's host buffers receive the full outputs

    e2e_steps = max(2, min(args.steps, 10))
    e2e_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    if ws > 1:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_val = step_bytes / e2e_s / 1e9

    prefill = None
    if rank == 0 and ws == 1 and not args.no_prefill:
        prefill = prefill_bench(plane, dev, m=args.prefill_m)
    decode_step = None
    if rank == 0 and ws == 1 and not args.no_decode_step:
        decode_step = decode_step_bench(plane, dev)
    moe = None
    if rank == 0 and ws == 1 and not args.no_moe:
        moe = moe_bench(plane, dev, tokens=args.moe_tokens)
    sparse24 = None
    if rank == 0 and ws == 1 and not args.no_sparse:
        sparse24 = sparse24_bench(plane, dev, layers=args.sparse_layers)

    batches = None
    if rank == 0 and ws == 1 and B == 1 and not args.no_batch_lines:
        batches = batch_lines(plane, dev, layers, fmt)

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample(fmt, B)

    if rank == 0:
        tok_bytes = step_bytes
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None,
            "dtype": "e5m2 x e4m3 -> f32 (tcgen05 kind::f8f6f4)" if fmt == "log4" else "s8/u8 x s8 -> s32 (tcgen05 kind::i8)",
            "data": "synthetic (seeded N(0,0.02) weights packed on device, N(0,1) activations)",
            "config": {"workload": f"qwen2-7b linears ({args.layers} layers + lm_head), {fmt}, batch {B} decode GEMV",
                       "batch": B, "fmt": fmt, "hidden": H, "intermediate": I, "vocab": V, "layers": args.layers,
                       "parallelism": f"column-shard x{ws} of the linears >= {args.shard_min_mb:g} MB "
                                      f"({n_sharded} of {len(flat)} launches; the rest whole on every rank): each "
                                      "sharded GEMV's epilogue stores its rows into every rank's output over NVLink "
                                      "(no collective library)" if ws > 1 else "single GPU",
                       "l2": f"no flush: {step_bytes / 1e9:.2f} GB of packed weights per step >> 126 MB L2",
                       "cuda_graph": graph is not None,
                       "gemv_kernel": "tc_gemv_kernel: tile-major weights streamed by 2 bulk-copy producers, "
                                      "8-bit tcgen05 MMAs from 4 issuer threads, activations as 8-bit terms"},
            "tokens_per_s": round(B * 1e3 / ms, 2),
            "gpu_launches": launches_per_step * args.steps,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic, "kernel": f"gemv_kernel<{fmt}> ({dom})",
                         "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)" if peak_kind == "measured"
                         else "fallback 6.65 TB/s"},
            "frac_of_peak_step": round(value / peak, 4),
            "per_linear": per_linear,
            "clocks": clocks.summary(),
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "bramha_cuda_host_chain_run (the step's host-buffer GEMV chain bound once; pinned "
                           "host buffers; copies and launches replayed as one CUDA graph, the copies overlapping "
                           "the launches; synchronous), one call per step",
                    "tokens_per_s": round(B / e2e_s, 2)},
            "spread": spread,
            "cpu_baseline": cpu,
            "batch_lines": batches,
            "prefill": prefill,
            "decode_step": decode_step,
            "sparse24": sparse24,
            "moe": moe,
            "setup_s": round(setup_s, 1),
        }
        print(json.dumps(line), flush=True)
    del graph
    if ws > 1:
        torch.cuda.synchronize()
        dist.barrier(device_ids=[local])  # no rank reads or writes a peer's arena any more
        plane.close()
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--fmt", choices=list(BITS), default="log4")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--shard-min-mb", type=float, default=128.0,
                    help="N > 1: column-shard the linears with at least this many MB of packed weights")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--repeats", type=int, default=5, help="extra timed K-step regions for the spread")
    ap.add_argument("--no-batch-lines", action="store_true", help="skip the batch 8 / 64 measurement")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-3 prefill GEMM measurement")
    ap.add_argument("--no-decode-step", action="store_true", help="skip the config-2 decode-step measurement")
    ap.add_argument("--layers", type=int, default=LAYERS, help="decoder layers (smaller = profiling case)")
    ap.add_argument("--prefill-only", action="store_true",
                    help="run only the config-3 prefill GEMM measurement (profiling case) and print its JSON")
    ap.add_argument("--prefill-m", type=int, default=2048, help="tokens of the prefill GEMM measurement")
    ap.add_argument("--no-sparse", action="store_true", help="skip the 2:4 sparse GEMV measurement")
    ap.add_argument("--sparse-only", action="store_true",
                    help="run only the 2:4 sparse GEMV measurement (profiling case) and print its JSON")
    ap.add_argument("--sparse-layers", type=int, default=4, help="layers of the 2:4 measurement")
    ap.add_argument("--no-moe", action="store_true", help="skip the config-5 MoE measurement")
    ap.add_argument("--moe-only", action="store_true", help="run only the config-5 MoE measurement and print its JSON")
    ap.add_argument("--moe-tokens", type=int, default=256, help="tokens of the MoE measurement")
    ap.add_argument("--decode-only", action="store_true",
                    help="run only the config-2 decode-step measurement (profiling case) and print its JSON")
    args = ap.parse_args()
    if args.decode_only:
        import torch
        from bramha_b200 import CudaComputePlane
        torch.cuda.set_device(0)
        plane = CudaComputePlane(0)
        print(json.dumps({"decode_step": decode_step_bench(plane, torch.device("cuda", 0))}))
        plane.close()
        return
    if args.moe_only:
        import torch
        from bramha_b200 import CudaComputePlane
        torch.cuda.set_device(0)
        plane = CudaComputePlane(0)
        print(json.dumps({"moe": moe_bench(plane, torch.device("cuda", 0), tokens=args.moe_tokens)}))
        plane.close()
        return
    if args.sparse_only:
        import torch
        from bramha_b200 import CudaComputePlane
        torch.cuda.set_device(0)
        plane = CudaComputePlane(0)
        print(json.dumps({"sparse24": sparse24_bench(plane, torch.device("cuda", 0), layers=args.sparse_layers)}))
        plane.close()
        return
    if args.prefill_only:
        import torch
        from bramha_b200 import CudaComputePlane
        torch.cuda.set_device(0)
        plane = CudaComputePlane(0)
        print(json.dumps({"prefill": prefill_bench(plane, torch.device("cuda", 0), m=args.prefill_m)}))
        plane.close()
        return
    ws, rank, local = dist_setup(args)
    if args.impl == "reference":
        run_reference(args, ws, rank)
    else:
        run_ours(args, ws, rank, local)


if __name__ == "__main__":
    main()
