#!/usr/bin/env python
"""Benchmark of the g4w4 hot path on B200 (one JSON line on rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W]
                  [--workload serve|decode|ple|gemv|attn|attn_rows|head|gemm] [--impl g4|reference]

Workloads (the benchmark configurations; inputs are seeded synthetic data with the configs'
shapes and value distributions -- the reference publishes no dataset):
  serve (default) config 5: 256 sequences with 4096-token contexts split over the GPUs
        as independent replicas, one greedy decode step of all of them per step (one
        CUDA graph per GPU), token ids all-gathered with NCCL.  Metric: decode tok/s.
  decode config 4: batch 1, 2048-token prompt (prefill through the tcgen05 GEMM), then
        greedy decode steps (one CUDA graph per token).
  ple   config 2: PLE W4 gather-dequant of 4096 token ids from the [262144, 8960]
        table into bf16 [4096, 35, 256].  A step is one gather of a fresh id batch.
  gemv  config 1: W4A16 decode GEMV, x [1,1536], W [6144,1536]; a step is one call,
        rotating over 64 weight copies (340 MB > L2).
  attn  decode attention, 8 q heads / 1 KV head, hd 256, one sequence at keylen 4096.
  attn_rows  the serving step's batched decode attention: --batch sequences (256) at
        position 4096, a global layer or (--sliding) a 512-key window.
  head  the serving step's fused LM head: --batch rows (256) against the tied bf16
        table [262144, 1536], softcap 30 and the greedy pick in the epilogue.
  gemm  config 3: the W4A16 GEMM sweep, M in {16,128,512,2048} x (K,N) in
        {(1536,6144), (6144,1536), (1536,262144)}.
Timing: W warm-up steps, then K steps captured in one CUDA graph and timed with
CUDA events on the launching stream between barriers; max over ranks.
--impl reference times the CPU restatement of the reference's TFJS path (the
reference itself is JavaScript and cannot run here) on the host cores.
"""
from __future__ import annotations

import argparse
import ctypes as C
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}

# dram__bytes_read.sum + dram__bytes_write.sum per launch from the committed ncu captures
# (profiles/).  Writes that are still in L2 when a kernel ends are not counted by ncu.
TRAFFIC = {
    "ple_gather_kernel": 20_566_272 + 15_701_760,  # T = 4096 (profiles/ple_gather_kernel__config2_*)
    "gemv_w4a16_kernel": 5_336_576,                # config 1 (profiles/gemv_w4a16_kernel__config1_*)
    "attn_decode_kernel": 4_221_696,               # one sequence at keylen 4096 (profiles/attn_decode_kernel__dram_bytes_*)
}


def gemm_traffic(M: int, K: int, N: int) -> int:
    """DRAM bytes of one W4A16 GEMM launch: packed weights + scales + X once each.  Checked
    against the capture at M=2048, K=1536, N=6144 (11,650,560 B measured, 11,599,872 B by this
    formula; profiles/gemm_w4_tmem_kernel__config3_*); scaled by formula to other shapes."""
    return N * K // 2 + N * (K // 32) * 2 + M * K * 2


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {**PEAKS_FALLBACK, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ----------------------------------------------------------------- clocks ---
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        self.proc.wait()
        sms, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": mx,
                "samples": len(sms), "reasons": sorted(reasons)}


# ------------------------------------------------------------ distributed ---
class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None

    def init(self, use_cuda: bool):
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist
            if use_cuda:
                torch.cuda.set_device(self.local)
            dist.init_process_group("nccl" if use_cuda else "gloo", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local) if use_cuda else None)
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device="cuda" if torch.cuda.is_available() else "cpu")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


def time_graph(torch, ctx, launch, K, W, dist: Dist):
    """Warm up W launches eagerly, capture K launches in a CUDA graph, replay it once
    between barriers and return the device time (ms) of the K launches."""
    for i in range(W):
        launch(i)
    ctx.sync()
    stream = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    old = ctx.stream
    with torch.cuda.stream(stream):
        ctx.set_stream(stream)
        with torch.cuda.graph(g, stream=stream):
            for i in range(K):
                launch(W + i)
    ctx.set_stream(old)
    g.replay()  # untimed replay: uploads the graph
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        start.record(stream)
        g.replay()
        end.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    ms = start.elapsed_time(end)
    del g
    return dist.max(ms)


def time_e2e(torch, dist, step, n):
    """Device time (ms, max over ranks) of one end-to-end step through the public API:
    `step(i)` copies its inputs in from pinned host memory, runs, and copies the result out."""
    for i in range(2):
        step(i)
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(n):
        step(i)
    e.record()
    torch.cuda.synchronize()
    dist.barrier()
    return dist.max(s.elapsed_time(e)) / n


# ----------------------------------------------------------------- workloads
def ple_setup(torch, rt, ctx, n_batches, T=4096, vocab=262144, width=8960, seed=0):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randint(-7, 8, (vocab, width // 2, 2), device="cuda", dtype=torch.int16, generator=gen)
    nib = (q & 0xF).to(torch.uint8)
    packed = (nib[..., 0] | (nib[..., 1] << 4)).contiguous()
    del q, nib
    sc = torch.randn((vocab, width // 32), device="cuda", generator=gen).abs_().mul_(0.05).to(torch.bfloat16)
    tab = rt.PleW4Table(ctx, packed, sc)
    del packed, sc
    torch.cuda.empty_cache()
    ids = torch.randint(0, vocab, (n_batches, T), device="cuda", dtype=torch.int32, generator=gen)
    outs = [torch.empty((T, width), dtype=torch.bfloat16, device="cuda") for _ in range(3)]
    return tab, ids, outs


PLE_BYTES = 4096 * (4480 + 560) + 4096 * 4 + 4096 * 8960 * 2   # 94,060,544 B per call
GEMV_BYTES = 6144 * 1536 // 2 + 6144 * 1536 // 32 * 2 + 1536 * 2 + 6144 * 2   # 5,323,776 B per call
ATTN_BYTES = 4096 * 256 * 2 * 2 + 2 * 8 * 256 * 2   # K and V at keylen 4096, q and out: 4,202,496 B


def run_ple(args, torch, rt, ctx, dist, peaks):
    lib = importlib.import_module("gemma4-js_b200._lib").load()
    K, W = args.steps, args.warmup
    tab, ids, outs = ple_setup(torch, rt, ctx, K + W, vocab=args.vocab)
    T = 4096

    def launch(i):
        st = lib.g4_ple_gather(ctx.handle, tab.handle, C.c_void_p(ids[i].data_ptr()), T, 1,
                               C.c_void_p(outs[i % 3].data_ptr()), 1)
        if st:
            raise RuntimeError(lib.g4_last_error_string())

    n0 = rt.launch_count()
    clk = ClockSampler(dist.local)
    clk.start()
    ms = time_graph(torch, ctx, launch, K, W, dist)
    clocks = clk.stop()
    launches = rt.launch_count() - n0 - W
    ctx.check_device()
    per_launch_s = ms / 1e3 / K
    gbs = PLE_BYTES / per_launch_s / 1e9
    value = gbs * dist.world

    # e2e through the public API: pinned host ids -> device, gather, bf16 rows -> pinned host
    hid = [torch.randint(0, args.vocab, (T,), dtype=torch.int32).pin_memory() for _ in range(2)]
    dev_ids = torch.empty(T, dtype=torch.int32, device="cuda")
    hout = torch.empty((T, 8960), dtype=torch.bfloat16).pin_memory()
    e2e_steps = max(3, min(K, 20))
    for i in range(2):
        dev_ids.copy_(hid[i], non_blocking=True)
        tab.rows_to_gpu(dev_ids, out=outs[0])
        hout.copy_(outs[0], non_blocking=True)
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(e2e_steps):
        dev_ids.copy_(hid[i % 2], non_blocking=True)
        tab.rows_to_gpu(dev_ids, out=outs[0])
        hout.copy_(outs[0], non_blocking=True)
    e.record()
    torch.cuda.synchronize()
    dist.barrier()
    e2e_ms = dist.max(s.elapsed_time(e)) / e2e_steps
    e2e = {"value": round(PLE_BYTES / (e2e_ms / 1e3) / 1e9 * dist.world, 2), "unit": "GB/s",
           "h2d_bytes_per_step": T * 4, "d2h_bytes_per_step": T * 8960 * 2}
    peak = peaks["hbm_gbs"]
    line = {
        "metric": "PLE W4 gather-dequant throughput (algorithmic bytes)", "value": round(value, 2), "unit": "GB/s",
        "n_gpus": dist.world, "steps": K, "warmup": W, "ms_per_step": round(ms / K, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic (seeded int4 table, uniform ids)",
        "config": {"workload": "config2_ple_gather", "tokens_per_step_per_gpu": T, "table": [args.vocab, 8960],
                   "out": "bf16 [4096,35,256]",
                   "l2": "fresh random ids each step over a 1.32 GB table; 3 rotating 73 MB outputs (> 126 MB L2)"},
        "roofline": {"bound": "hbm", "kernel": "ple_gather_kernel", "achieved": round(gbs, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(gbs / peak, 4), "peak_source": peaks["source"],
                     "traffic": TRAFFIC["ple_gather_kernel"], "bytes_per_launch": PLE_BYTES},
        "e2e": e2e, "gpu_launches": launches, "clocks": clocks,
    }
    if dist.rank == 0 and dist.world == 1 and not getattr(args, "no_cpu", False):
        line["cpu_baseline"] = cpu_ple(sample_s=args.cpu_seconds, threads=1)
    return line


def run_gemv(args, torch, rt, ctx, dist, peaks):
    lib = importlib.import_module("gemma4-js_b200._lib").load()
    K, W = args.steps, args.warmup
    ctx.set_pdl(not args.no_pdl)  # back-to-back linears overlap as they do inside a decode step
    Kd, N, copies = 1536, 6144, args.copies or 64
    gen = torch.Generator(device="cuda").manual_seed(0)
    lins = []
    for c in range(copies):
        packed = torch.randint(-2**31, 2**31 - 1, (N, Kd // 8), device="cuda", dtype=torch.int32, generator=gen)
        sc = torch.randn((N, Kd // 32), device="cuda", generator=gen).abs_().mul_(0.02).to(torch.bfloat16)
        lins.append(rt.W4Linear(ctx, packed, sc))
    x = torch.randn((1, Kd), device="cuda", generator=gen).to(torch.bfloat16)
    ys = [torch.empty((1, N), dtype=torch.bfloat16, device="cuda") for _ in range(4)]

    def launch(i):
        st = lib.g4_linear_w4a16_impl(ctx.handle, lins[i % copies].handle, C.c_void_p(x.data_ptr()), 1,
                                      C.c_void_p(ys[i % 4].data_ptr()), 1, 1)
        if st:
            raise RuntimeError(lib.g4_last_error_string())

    n0 = rt.launch_count()
    clk = ClockSampler(dist.local)
    clk.start()
    ms = time_graph(torch, ctx, launch, K, W, dist)
    clocks = clk.stop()
    launches = rt.launch_count() - n0 - W
    byts = GEMV_BYTES
    per = ms / 1e3 / K
    gbs = byts / per / 1e9
    peak = peaks["hbm_gbs"]
    # e2e: x from pinned host memory, y back to pinned host memory, every call
    hx = x.cpu().pin_memory()
    hy = torch.empty((1, N), dtype=torch.bfloat16).pin_memory()

    def e2e_step(i):
        x.copy_(hx, non_blocking=True)
        launch(i)
        hy.copy_(ys[i % 4], non_blocking=True)

    e2e_ms = time_e2e(torch, dist, e2e_step, max(3, min(K, 50)))
    e2e = {"value": round(GEMV_BYTES / (e2e_ms / 1e3) / 1e9 * dist.world, 2), "unit": "GB/s",
           "h2d_bytes_per_step": Kd * 2, "d2h_bytes_per_step": N * 2}
    del lins
    torch.cuda.empty_cache()
    wide = gemv_wide(torch, rt, ctx, lib, peak)
    sweep = gemv_sweep(torch, rt, ctx, lib, peak, steps=max(K, 20))
    return {
        "metric": "W4A16 decode GEMV throughput (algorithmic bytes)", "value": round(gbs * dist.world, 2),
        "unit": "GB/s", "n_gpus": dist.world, "steps": K, "warmup": W, "ms_per_step": round(ms / K, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded)", "config": {"workload": "config1_gemv", "M": 1, "K": Kd, "N": N,
                                                  "l2": "64 rotating weight copies (340 MB > 126 MB L2)",
                                                  "pdl": not args.no_pdl},
        "roofline": {"bound": "hbm", "kernel": "gemv_w4a16_kernel", "achieved": round(gbs, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(gbs / peak, 4), "peak_source": peaks["source"],
                     "traffic": TRAFFIC["gemv_w4a16_kernel"], "bytes_per_launch": byts},
        "gpu_launches": launches, "clocks": clocks, "us_per_call": round(per * 1e6, 3), "e2e": e2e,
        "wide_gemv": wide, "decode_shape_sweep": sweep,
    }


GEMV_SWEEP = [(1536, 2048), (1536, 4096), (1536, 256), (1536, 512), (1536, 8960), (2048, 1536), (4096, 1536),
              (1536, 12288), (12288, 1536), (256, 1536)]


def gemv_sweep(torch, rt, ctx, lib, peak, steps=20):
    """The same GEMV at the model's decode shapes (K, N), M = 1, back to back in a CUDA
    graph over enough weight copies that each rotation exceeds L2 (>= 256 MB)."""
    out = []
    gen = torch.Generator(device="cuda").manual_seed(2)
    for Kd, N in GEMV_SWEEP:
        byts = N * Kd // 2 + N * Kd // 32 * 2 + Kd * 2 + N * 2
        copies = max(2, -(-(256 << 20) // byts))
        packed = torch.randint(-2**31, 2**31 - 1, (N, Kd // 8), device="cuda", dtype=torch.int32, generator=gen)
        sc = torch.randn((N, Kd // 32), device="cuda", generator=gen).abs_().mul_(0.02).to(torch.bfloat16)
        lins = [rt.W4Linear(ctx, packed, sc) for _ in range(copies)]  # the same bits, distinct buffers
        x = torch.randn((1, Kd), device="cuda", generator=gen).to(torch.bfloat16)
        y = torch.empty((1, N), dtype=torch.bfloat16, device="cuda")

        def launch(i, lins=lins, x=x, y=y):
            st = lib.g4_linear_w4a16_impl(ctx.handle, lins[i % len(lins)].handle, C.c_void_p(x.data_ptr()), 1,
                                          C.c_void_p(y.data_ptr()), 1, 1)
            if st:
                raise RuntimeError(lib.g4_last_error_string())

        ms = time_graph(torch, ctx, launch, steps, 3, Dist())
        per = ms / 1e3 / steps
        out.append({"K": Kd, "N": N, "us_per_call": round(per * 1e6, 2), "achieved_gbs": round(byts / per / 1e9, 1),
                    "frac": round(byts / per / 1e9 / peak, 4)})
        for L in lins:
            L.close()
        del lins, packed, sc
        torch.cuda.empty_cache()
    return out


def gemv_wide(torch, rt, ctx, lib, peak, N=262144, Kd=1536, reps=10):
    """The same GEMV kernel where streaming dominates its fixed latency: one token
    through a W4A16 linear of the tied-head shape (N = 262144, 226 MB of nibbles and
    scales, larger than L2), back to back in a CUDA graph."""
    gen = torch.Generator(device="cuda").manual_seed(1)
    packed = torch.randint(-2**31, 2**31 - 1, (N, Kd // 8), device="cuda", dtype=torch.int32, generator=gen)
    sc = torch.randn((N, Kd // 32), device="cuda", generator=gen).abs_().mul_(0.02).to(torch.bfloat16)
    lin = rt.W4Linear(ctx, packed, sc)
    del packed, sc
    x = torch.randn((1, Kd), device="cuda", generator=gen).to(torch.bfloat16)
    y = torch.empty((1, N), dtype=torch.bfloat16, device="cuda")

    def launch(i):
        st = lib.g4_linear_w4a16_impl(ctx.handle, lin.handle, C.c_void_p(x.data_ptr()), 1, C.c_void_p(y.data_ptr()), 1, 1)
        if st:
            raise RuntimeError(lib.g4_last_error_string())

    one = Dist()  # this GPU alone
    ms = time_graph(torch, ctx, launch, reps, 3, one)
    byts = N * Kd // 2 + N * Kd // 32 * 2 + Kd * 2 + N * 2
    per = ms / 1e3 / reps
    gbs = byts / per / 1e9
    lin.close()
    return {"N": N, "K": Kd, "M": 1, "bytes_per_call": byts, "us_per_call": round(per * 1e6, 2),
            "achieved_gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
            "note": "latency-free regime of gemv_w4a16_kernel; the headline line is the config-1 shape"}


def run_attn(args, torch, rt, ctx, dist, peaks):
    K, W = args.steps, args.warmup
    hd, keylen = 256, 4096
    copies = args.copies or 40  # 40 x 8 MB of K/V = 320 MB > L2
    gen = torch.Generator(device="cuda").manual_seed(0)
    caches = []
    for c in range(copies):
        kv = rt.KVCache(ctx, hd, keylen)
        kv.append(torch.randn((keylen, hd), device="cuda", generator=gen).to(torch.bfloat16),
                  torch.randn((keylen, hd), device="cuda", generator=gen).to(torch.bfloat16), keylen, 0)
        caches.append(kv)
    q = (torch.randn((1, 8, hd), device="cuda", generator=gen) * 0.1).to(torch.bfloat16)
    out = torch.empty((1, 8, hd), dtype=torch.bfloat16, device="cuda")
    ops = rt.GPUOps(ctx)

    def launch(i):
        ops.attention(q, caches[i % copies], 1, 8, hd, keylen, keylen - 1, False, 512, out=out)

    n0 = rt.launch_count()
    clk = ClockSampler(dist.local)
    clk.start()
    ms = time_graph(torch, ctx, launch, K, W, dist)
    clocks = clk.stop()
    launches = rt.launch_count() - n0 - W
    byts = ATTN_BYTES
    per = ms / 1e3 / K
    gbs = byts / per / 1e9
    peak = peaks["hbm_gbs"]
    hq = q.cpu().pin_memory()
    ho = torch.empty((1, 8, hd), dtype=torch.bfloat16).pin_memory()

    def e2e_step(i):
        q.copy_(hq, non_blocking=True)
        launch(i)
        ho.copy_(out, non_blocking=True)

    e2e_ms = time_e2e(torch, dist, e2e_step, max(3, min(K, 50)))
    e2e = {"value": round(ATTN_BYTES / (e2e_ms / 1e3) / 1e9 * dist.world, 2), "unit": "GB/s",
           "h2d_bytes_per_step": 8 * hd * 2, "d2h_bytes_per_step": 8 * hd * 2}
    return {
        "metric": "GQA decode attention throughput (algorithmic bytes)", "value": round(gbs * dist.world, 2),
        "unit": "GB/s", "n_gpus": dist.world, "steps": K, "warmup": W, "ms_per_step": round(ms / K, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded)", "config": {"workload": "decode_attention_global", "keylen": keylen, "hd": hd,
                                                  "heads": 8, "l2": "40 rotating KV caches (320 MB > L2)"},
        "roofline": {"bound": "hbm", "kernel": "attn_decode_kernel", "achieved": round(gbs, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(gbs / peak, 4), "peak_source": peaks["source"],
                     "traffic": TRAFFIC["attn_decode_kernel"], "bytes_per_launch": byts},
        "gpu_launches": launches, "clocks": clocks, "us_per_call": round(per * 1e6, 3), "e2e": e2e,
    }


def run_attn_rows(args, torch, rt, ctx, dist, peaks):
    """Batched decode attention as in the config 5 step: one query row for each of
    --batch sequences at position 4096 (device-side positions), global (4097 keys) or,
    with --sliding, the 512-key window of a sliding layer."""
    lib = importlib.import_module("gemma4-js_b200._lib")
    K, W = args.steps, args.warmup
    B, hd, pos = args.batch, 256, 4096
    stride = pos + 8
    sliding = bool(args.sliding)
    ctx.set_pdl(True)
    cache = rt.KVCache(ctx, hd, B * stride)
    gen = torch.Generator(device="cuda").manual_seed(0)
    for s in range(B):  # K ~ N(0, 0.3^2), V ~ N(0, 1): the scale of normed keys and values
        k = (torch.randn((stride, hd), device="cuda", generator=gen) * 0.3).to(torch.bfloat16)
        v = torch.randn((stride, hd), device="cuda", generator=gen).to(torch.bfloat16)
        cache.append(k, v, stride, s * stride)
    seq_pos = torch.full((B,), pos, dtype=torch.int32, device="cuda")
    q = (torch.randn((B, 8, hd), device="cuda", generator=gen) * 0.3).to(torch.bfloat16)
    out = torch.empty_like(q)
    rmap = lib.G4Rows(seq_pos.data_ptr(), 0, 1, 0, lib.G4_ROWS_HISTORY_READY)

    def launch(i):
        lib.call("g4_attention_rows", ctx.handle, C.c_void_p(q.data_ptr()), cache.handle, B, 8, hd, C.byref(rmap),
                 stride, int(sliding), 512, C.c_void_p(out.data_ptr()))

    n0 = rt.launch_count()
    clk = ClockSampler(dist.local)
    clk.start()
    ms = time_graph(torch, ctx, launch, K, W, dist)
    clocks = clk.stop()
    launches = rt.launch_count() - n0 - W
    ctx.check_device()
    keys = 512 if sliding else pos + 1
    byts = B * keys * hd * 2 * 2 + 2 * B * 8 * hd * 2
    per = ms / 1e3 / K
    gbs = byts / per / 1e9
    peak = peaks["hbm_gbs"]
    hq = q.cpu().pin_memory()
    ho = torch.empty_like(hq).pin_memory()

    def e2e_step(i):
        q.copy_(hq, non_blocking=True)
        launch(i)
        ho.copy_(out, non_blocking=True)

    e2e_ms = time_e2e(torch, dist, e2e_step, max(3, min(K, 50)))
    return {
        "metric": "batched decode attention throughput (algorithmic bytes)", "value": round(gbs * dist.world, 2),
        "unit": "GB/s", "n_gpus": dist.world, "steps": K, "warmup": W, "ms_per_step": round(ms / K, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
        "config": {"workload": "decode_attention_rows_" + ("sliding" if sliding else "global"), "batch": B,
                   "keys": keys, "hd": hd, "heads": 8,
                   "l2": f"{byts / 2**20:.0f} MB of K/V per launch" + (" (> L2)" if byts > 126e6 else " (L2-resident)")},
        "roofline": {"bound": "hbm", "kernel": "attn_decode_kernel", "achieved": round(gbs, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(gbs / peak, 4), "peak_source": peaks["source"], "traffic": None,
                     "bytes_per_launch": byts},
        "e2e": {"value": round(byts / (e2e_ms / 1e3) / 1e9 * dist.world, 2), "unit": "GB/s",
                "h2d_bytes_per_step": B * 8 * hd * 2, "d2h_bytes_per_step": B * 8 * hd * 2},
        "gpu_launches": launches, "clocks": clocks, "us_per_call": round(per * 1e6, 3),
    }


def run_head(args, torch, rt, ctx, dist, peaks):
    """The fused LM head of the config 5 step: logits of --batch rows against the tied
    bf16 table [262144, 1536] on tcgen05, softcap 30 and the greedy pick in the epilogue
    (g4_dense_argmax)."""
    lib = importlib.import_module("gemma4-js_b200._lib")
    model = importlib.import_module("gemma4-js_b200.model")
    K, W = args.steps, args.warmup
    M, V, Kd = args.batch, 262144, 1536
    ctx.set_pdl(True)
    gen = torch.Generator(device="cuda").manual_seed(0)
    E = (torch.randn((V, Kd), device="cuda", generator=gen) * 0.05).to(torch.bfloat16)
    head = model.Dense(ctx, E)
    del E
    x = torch.randn((M, Kd), device="cuda", generator=gen).to(torch.bfloat16)
    ids = torch.empty(M, dtype=torch.int32, device="cuda")
    vals = torch.empty(M, dtype=torch.float32, device="cuda")

    def launch(i):
        lib.call("g4_dense_argmax", ctx.handle, head.handle, C.c_void_p(x.data_ptr()), M, C.c_float(30.0),
                 C.c_void_p(ids.data_ptr()), C.c_void_p(vals.data_ptr()))

    n0 = rt.launch_count()
    clk = ClockSampler(dist.local)
    clk.start()
    ms = time_graph(torch, ctx, launch, K, W, dist)
    clocks = clk.stop()
    launches = rt.launch_count() - n0 - W
    ctx.check_device()
    per = ms / 1e3 / K
    flops = 2.0 * M * V * Kd
    tf = flops / per / 1e12
    hx = x.cpu().pin_memory()
    hid = torch.empty(M, dtype=torch.int32).pin_memory()

    def e2e_step(i):
        x.copy_(hx, non_blocking=True)
        launch(i)
        hid.copy_(ids, non_blocking=True)

    e2e_ms = time_e2e(torch, dist, e2e_step, max(3, min(K, 50)))
    return {
        "metric": "fused LM head (logits + softcap + greedy pick) TFLOP/s", "value": round(tf * dist.world, 1),
        "unit": "TFLOP/s", "n_gpus": dist.world, "steps": K, "warmup": W, "ms_per_step": round(ms / K, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
        "config": {"workload": "lm_head_argmax", "M": M, "vocab": V, "K": Kd,
                   "l2": "805 MB bf16 table per launch (> L2)",
                   "hbm_gbs": round(V * Kd * 2 / per / 1e9, 1)},
        "roofline": {"bound": "tensor", "kernel": "head_argmax_kernel", "achieved": round(tf, 1),
                     "peak": peaks["bf16_tflops"], "unit": "TFLOP/s", "frac": round(tf / peaks["bf16_tflops"], 4),
                     "peak_source": peaks["source"], "traffic": None, "flops_per_launch": flops},
        "e2e": {"value": round(flops / (e2e_ms / 1e3) / 1e12 * dist.world, 1), "unit": "TFLOP/s",
                "h2d_bytes_per_step": M * Kd * 2, "d2h_bytes_per_step": M * 4},
        "gpu_launches": launches, "clocks": clocks, "us_per_call": round(per * 1e6, 3),
    }


def run_gemm(args, torch, rt, ctx, dist, peaks):
    """benchmark config 3: M in {16,128,512,2048} x (K,N) in {(1536,6144), (6144,1536), (1536,262144)}."""
    lib = importlib.import_module("gemma4-js_b200._lib").load()
    K_steps, W = args.steps, args.warmup
    ctx.set_pdl(True)  # back-to-back launches overlap as they do inside a decode step
    gen = torch.Generator(device="cuda").manual_seed(0)
    points, clk = [], ClockSampler(dist.local)
    n0 = rt.launch_count()
    clk.start()
    tot_flop, tot_s = 0.0, 0.0
    e2e = None
    shapes = [(1536, 6144), (6144, 1536), (1536, 262144)]
    ms_list = (16, 128, 512, 2048)
    if args.gemm_shapes:  # "M1,M2:KxN,KxN" e.g. "128,256:1536x2560,6144x1536"
        mpart, spart = args.gemm_shapes.split(":")
        ms_list = tuple(int(m) for m in mpart.split(","))
        shapes = [tuple(int(v) for v in sh.split("x")) for sh in spart.split(",")]
    for (Kd, N) in shapes:
        wbytes = N * Kd // 2 + N * Kd // 16
        copies = max(1, min(32, (256 << 20) // wbytes + 1))   # > 126 MB of weights per rotation
        lins = []
        for c in range(copies):
            packed = torch.randint(-2**31, 2**31 - 1, (N, Kd // 8), device="cuda", dtype=torch.int32, generator=gen)
            sc = torch.randn((N, Kd // 32), device="cuda", generator=gen).abs_().mul_(0.02).to(torch.bfloat16)
            lins.append(rt.W4Linear(ctx, packed, sc))
            del packed, sc
        for M in ms_list:
            x = torch.randn((M, Kd), device="cuda", generator=gen).to(torch.bfloat16)
            y = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")

            def launch(i, M=M, x=x, y=y):
                st = lib.g4_linear_w4a16_impl(ctx.handle, lins[i % copies].handle, C.c_void_p(x.data_ptr()), M,
                                              C.c_void_p(y.data_ptr()), 1, args.gemm_impl)
                if st:
                    raise RuntimeError(lib.g4_last_error_string())

            steps = max(3, min(K_steps, 20 if N > 100000 else K_steps))
            ms = time_graph(torch, ctx, launch, steps, W, dist)
            per = ms / 1e3 / steps
            flop = 2.0 * M * Kd * N
            byts = wbytes + 2 * M * Kd + 2 * M * N
            ideal = max(flop / (peaks["bf16_tflops"] * 1e12), byts / (peaks["hbm_gbs"] * 1e9))
            points.append({"M": M, "K": Kd, "N": N, "us": round(per * 1e6, 2), "tflops": round(flop / per / 1e12, 1),
                           "gbs": round(byts / per / 1e9, 1), "frac_of_roofline": round(ideal / per, 3),
                           "kernel": {1: "gemv", 2: "tcgen05"}.get(args.gemm_impl, "gemv" if M <= 16 else "tcgen05")})
            if M >= 512:
                tot_flop += flop
                tot_s += per
            if (M, Kd, N) == (2048, 1536, 6144) and e2e is None:
                hx = x.cpu().pin_memory()
                hy = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()

                def e2e_step(i, x=x, y=y, hx=hx, hy=hy, launch=launch):
                    x.copy_(hx, non_blocking=True)
                    launch(i)
                    hy.copy_(y, non_blocking=True)

                e2e_ms = time_e2e(torch, dist, e2e_step, max(3, min(K_steps, 10)))
                e2e = {"value": round(flop / (e2e_ms / 1e3) / 1e12 * dist.world, 2), "unit": "TFLOP/s",
                       "h2d_bytes_per_step": M * Kd * 2, "d2h_bytes_per_step": M * N * 2,
                       "point": "M=2048, K=1536, N=6144 (x in from and y out to pinned host memory)"}
            del x, y
        del lins
        torch.cuda.empty_cache()
    clocks = clk.stop()
    ctx.check_device()
    tf = tot_flop / tot_s / 1e12 if tot_s > 0 else 0.0
    peak = peaks["bf16_tflops"]
    best = max(points, key=lambda p: p["tflops"])
    tf = tf if tot_s > 0 else best["tflops"]
    return {
        "metric": "W4A16 prefill GEMM TFLOP/s (config 3, M >= 512 aggregate)", "value": round(tf * dist.world, 2),
        "unit": "TFLOP/s", "n_gpus": dist.world, "steps": K_steps, "warmup": W,
        "ms_per_step": round(tot_s * 1e3, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded)",
        "config": {"workload": "config3_gemm_sweep", "l2": "rotating weight copies (> 256 MB per rotation)"},
        "roofline": {"bound": "tensor", "kernel": "gemm_w4a16_tcgen05_kernel", "achieved": round(best["tflops"], 1),
                     "peak": peak, "unit": "TFLOP/s", "frac": round(best["tflops"] / peak, 4),
                     "peak_source": peaks["source"], "traffic": gemm_traffic(best["M"], best["K"], best["N"]),
                     "traffic_basis": "ncu DRAM bytes at M=2048 K=1536 N=6144 scaled by the weight + X bytes",
                     "point": best},
        "sweep": points, "gpu_launches": rt.launch_count() - n0, "clocks": clocks, "e2e": e2e,
    }


def _decode_model(torch, rt, ctx, batch, max_seq, max_rows, seed=0):
    model = importlib.import_module("gemma4-js_b200.model")
    cfg = model.ModelConfig()
    w = model.random_weights_device(cfg, seed=seed)
    m = model.Gemma4Model(ctx, cfg, w, max_batch=batch, max_seq=max_seq, max_rows=max_rows)
    del w
    torch.cuda.empty_cache()
    return cfg, m


def _attn_roofline(torch, ctx, m, B, peaks, reps=20):
    """Times the dominant kernel (decode attention over a global layer's cache) alone
    with CUDA events on its launching stream, using the model's live caches."""
    lib = importlib.import_module("gemma4-js_b200._lib")
    Ly = next(L for L in m.layers if L["spec"]["full"] and not L["spec"]["shared"])
    hd = Ly["spec"]["hd"]
    rmap = lib.G4Rows(m.seq_pos.data_ptr(), 0, 1, 0)
    q = (torch.randn((B, 8, hd), device="cuda") * 0.3).to(torch.bfloat16)
    out = torch.empty_like(q)

    def launch():
        lib.call("g4_attention_rows", ctx.handle, C.c_void_p(q.data_ptr()), Ly["kv"].handle, B, 8, hd,
                 C.byref(rmap), m.max_seq, 0, 512, C.c_void_p(out.data_ptr()))

    launch()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        launch()
    e.record()
    torch.cuda.synchronize()
    per = s.elapsed_time(e) / 1e3 / reps
    keylen = int(m.seq_pos[:B].max().item()) + 1
    byts = B * keylen * hd * 2 * 2 + 2 * B * 8 * hd * 2
    gbs = byts / per / 1e9
    return {"bound": "hbm", "kernel": "attn_decode_kernel (+ combine when keys are split), global layer", "achieved": round(gbs, 1),
            "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4),
            "peak_source": peaks["source"],
            "traffic": int(TRAFFIC["attn_decode_kernel"] * B * keylen / 4096),
            "traffic_basis": "ncu DRAM bytes of one sequence at keylen 4096, times the sequences and keys of this launch",
            "bytes_per_launch": byts, "us_per_launch": round(per * 1e6, 2)}


SERVE_METRIC = "batched greedy decode throughput (config 5)"


def serve_config(world: int) -> dict:
    """The config object of the config-5 line, the same for both arms."""
    return {"workload": "config5_serving", "model": "gemma4-e2b-shaped (35L, hidden 1536, MLP 6144, 8q/1kv, hd 256)",
            "global_batch": 256, "batch_per_gpu": 256 // world, "seq_len": 4096, "new_tokens_per_step": 1,
            "parallelism": f"replicas x{world}, NCCL all-gather of token ids",
            "l2": "per step 1.5 GB of weights + KV of 256 x 4096 tokens (>> 126 MB L2)"}


def _serve_step_bytes(m, B: int, pos: int) -> dict:
    """Algorithmic HBM bytes of one decode step of B sequences at position `pos`: every
    W4A16 weight once (nibbles + scales), the tied bf16 head once, the embedding and PLE
    rows of the B tokens, each layer's K/V reads (window-limited on sliding layers) and
    the new K/V rows."""
    cfg = m.cfg
    w4 = sum(L[n].in_dim * L[n].out_dim * 9 // 16 for L in m.layers for n in ("qkv", "o", "gu", "down", "pg", "pp"))
    w4 += m.top.in_dim * m.top.out_dim * 9 // 16
    head = cfg.vocab * cfg.hidden * 2
    rows = B * (cfg.hidden * 2 + 5040)
    kv = 0
    for L in m.layers:
        s = L["spec"]
        keys = pos + 1 if s["full"] else min(pos + 1, cfg.window)
        kv += B * keys * s["hd"] * 4
        if not s["shared"]:
            kv += B * s["hd"] * 4
    return {"w4": w4, "head": head, "rows": rows, "kv": kv, "total": w4 + head + rows + kv}


def _step_linears(m, B: int):
    """(issue, flops, traffic) of every W4A16 linear of one decode step, in step order: per
    layer q/k/v, o, gate/up + GeGLU, down, PLE gate, PLE projection; then the per-layer
    model projection of the next step's inputs."""
    lib = importlib.import_module("gemma4-js_b200._lib")
    b, h = m.buf, m.ctx.handle
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    out = []
    for L in m.layers:
        for name, x in (("qkv", b["x"]), ("o", b["attn"]), ("gu", b["x"]), ("down", b["act"]), ("pg", b["x"]),
                        ("pp", b["pa"])):
            lin = L[name]
            if name == "gu":
                def issue(lin=lin, x=x):
                    lib.call("g4_linear_w4a16_geglu", h, lin.handle, P(x), B, P(b["act"]))
            else:
                def issue(lin=lin, x=x):
                    pl = lib.G4Planes()
                    lib.call("g4_linear_w4a16_planes", h, lin.handle, P(x), B, C.byref(pl))
            out.append((issue, 2.0 * B * lin.in_dim * lin.out_dim, gemm_traffic(B, lin.in_dim, lin.out_dim)))

    def top():
        lib.call("g4_linear_w4a16", h, m.top.handle, P(b["x"]), B, P(b["proj"]), 0)
    out.append((top, 2.0 * B * m.top.in_dim * m.top.out_dim, gemm_traffic(B, m.top.in_dim, m.top.out_dim)))
    return out


def _gemm_family_roofline(torch, ctx, m, B, peaks, reps=10):
    """The step's dominant kernel family by launch-list share: every W4A16 linear of one
    decode step (gemm_w4_tmem_kernel, plain and GeGLU instances, at M = B), issued back to
    back in step order with programmatic dependent launch, captured in a CUDA graph and
    timed with CUDA events on its launching stream.  The row-wise operators and the
    attention that sit between them inside the real step are left out, so this is the
    linears' own rate, not their in-step latency."""
    calls = _step_linears(m, B)
    flops = sum(f for _, f, _ in calls)
    traffic = sum(t for _, _, t in calls)
    for fn, _, _ in calls:  # eager warm-up: sizes the workspace, sets kernel attributes
        fn()
    ctx.sync()
    stream = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    old = ctx.stream
    n0 = importlib.import_module("gemma4-js_b200.runtime").launch_count()
    with torch.cuda.stream(stream):
        ctx.set_stream(stream)
        with torch.cuda.graph(g, stream=stream):
            for fn, _, _ in calls:
                fn()
    ctx.set_stream(old)
    launches = importlib.import_module("gemma4-js_b200.runtime").launch_count() - n0
    with torch.cuda.stream(stream):
        g.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        s.record(stream)
        for _ in range(reps):
            g.replay()
        e.record(stream)
    torch.cuda.synchronize()
    per = s.elapsed_time(e) / 1e3 / reps
    del g
    tf = flops / per / 1e12
    return {"bound": "tensor", "kernel": "gemm_w4_tmem_kernel: the step's W4A16 linears (6 per layer x 35 + the PLE "
                                        "model projection), back to back",
            "achieved": round(tf, 1), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
            "frac": round(tf / peaks["bf16_tflops"], 4), "peak_source": peaks["source"],
            "traffic": traffic,
            "traffic_basis": "per launch packed weights + scales + X once (ncu DRAM bytes at M=2048 K=1536 N=6144 "
                             "match this to 0.4%), summed over the step's linears",
            "flops_per_step": flops, "launches_per_step": launches, "us_per_step": round(per * 1e6, 1),
            "us_per_launch": round(per * 1e6 / max(launches, 1), 2)}


def run_serve(args, torch, rt, ctx, dist, peaks):
    """benchmark config 5: 256 sequences with 4096-token contexts, greedy decode; the batch
    is split across the GPUs as independent replicas; token ids all-gathered with NCCL."""
    K, W = args.steps, args.warmup
    B_total, ctx_len = 256, 4096
    if B_total % dist.world:
        raise SystemExit(f"256 sequences do not split over {dist.world} GPUs")
    B = B_total // dist.world
    max_seq = ctx_len + max(256, W + K + 2)
    cfg, m = _decode_model(torch, rt, ctx, B, max_seq, B)
    m.fill_kv_random(ctx_len, seed=dist.rank)
    g = torch.Generator(device="cuda").manual_seed(1000 + dist.rank)
    m.buf["next"][:B] = torch.randint(0, cfg.vocab, (B,), device="cuda", generator=g, dtype=torch.int32)
    m.capture_decode(batch=B)
    serving = importlib.import_module("gemma4-js_b200.serving")
    tg = serving.TokenGather(dist.pg, B_total, "cuda")
    gathered = tg.out

    def step():
        tg.gather(m.replay_decode())

    n0 = rt.launch_count()
    for _ in range(W):
        step()
    torch.cuda.synchronize()
    clk = ClockSampler(dist.local)
    clk.start()
    dist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(K):
        step()
    e.record()
    torch.cuda.synchronize()
    dist.barrier()
    clocks = clk.stop()
    ms = dist.max(s.elapsed_time(e))
    graph_nodes = rt.launch_count() - n0   # kernels launched eagerly (capture counts once)
    ctx.check_device()
    tok_s = B_total * K / (ms / 1e3)
    # e2e: ids in from pinned host memory, gathered ids out to pinned host memory, every step
    h_in = torch.randint(0, cfg.vocab, (B,), dtype=torch.int32).pin_memory()
    h_out = torch.empty(B_total, dtype=torch.int32).pin_memory()
    e2e_steps = max(3, min(K, 16))
    dist.barrier()
    torch.cuda.synchronize()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for _ in range(e2e_steps):
        m.buf["next"][:B].copy_(h_in, non_blocking=True)
        step()
        h_out.copy_(gathered, non_blocking=True)
    e2.record()
    torch.cuda.synchronize()
    e2e_ms = dist.max(s2.elapsed_time(e2)) / e2e_steps
    roof_attn = _attn_roofline(torch, ctx, m, B, peaks)
    roof_gemm = _gemm_family_roofline(torch, ctx, m, B, peaks)
    # per-GPU step: the slowest rank's step time and the algorithmic bytes of its batch
    sb = _serve_step_bytes(m, B, ctx_len + W + K // 2)
    step_s = ms / K / 1e3
    line = {
        "metric": SERVE_METRIC, "value": round(tok_s, 1), "unit": "tok/s",
        "n_gpus": dist.world, "steps": K, "warmup": W, "ms_per_step": round(ms / K, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init W4A16 weights, random bf16 K/V for the 4096-token contexts, random ids)",
        "config": serve_config(dist.world),
        "roofline": roof_gemm,
        "roofline_attention": roof_attn,
        "step_frac": round(sb["total"] / step_s / 1e9 / peaks["hbm_gbs"], 4),
        "per_gpu": {"batch": B, "step_ms": round(ms / K, 4), "tok_s": round(B / step_s, 1),
                    "step_bytes": sb, "step_hbm_gbs": round(sb["total"] / step_s / 1e9, 1),
                    "step_frac_basis": "algorithmic bytes per step (weights, head, rows, K/V) / ms_per_step / HBM peak"},
        "e2e": {"value": round(B_total / (e2e_ms / 1e3), 1), "unit": "tok/s", "h2d_bytes_per_step": B * 4,
                "d2h_bytes_per_step": B_total * 4},
        "gpu_launches": _graph_kernel_count(m) * K, "launches_per_step": _graph_kernel_count(m), "clocks": clocks,
    }
    if dist.rank == 0 and dist.world == 1:
        line["cpu_baseline"] = cpu_decode(batch=1, ctx_len=ctx_len)
    m.close()
    del m
    torch.cuda.empty_cache()
    if dist.world == 1 and not args.no_extras:
        line.update(_extras(args, torch, rt, ctx, dist, peaks))
    return line


def _extras(args, torch, rt, ctx, dist, peaks) -> dict:
    """The other north_star numbers in the same run (one GPU): config 1 GEMV, config 3
    GEMM sweep, config 2 PLE gather and config 4 batch-1 decode, each with its own value,
    roofline fraction, clocks and step time."""
    import copy

    def sub(fn, **kw):
        a = copy.copy(args)
        a.no_cpu = True
        for k, v in kw.items():
            setattr(a, k, v)
        try:
            ln = fn(a, torch, rt, ctx, dist, peaks)
        except Exception as ex:  # report, keep the headline line
            return {"error": f"{type(ex).__name__}: {ex}"}
        keep = ("metric", "value", "unit", "ms_per_step", "steps", "warmup", "roofline", "clocks", "e2e", "config",
                "us_per_call", "gpu_launches")
        out = {k: ln[k] for k in keep if k in ln}
        for k in ("sweep", "decode_shape_sweep", "wide_gemv", "persistent_decoder", "launches_per_step"):
            if k in ln:
                out[k] = ln[k]
        torch.cuda.empty_cache()
        return out

    ctx.set_pdl(True)
    return {"gemv": sub(run_gemv, steps=200, copies=0, no_pdl=False),
            "gemm": sub(run_gemm, steps=20, gemm_shapes="", gemm_impl=0),
            "ple": sub(run_ple, steps=50, vocab=262144),
            "decode": sub(run_decode, steps=128)}


def _graph_kernel_count(m):
    """Kernels of this library per captured decode step (counted while capturing)."""
    return getattr(m, "graph_kernels", 0)


def run_decode(args, torch, rt, ctx, dist, peaks):
    """benchmark config 4: batch 1, 2048-token random prompt, then greedy decode."""
    K, W = args.steps, args.warmup
    prompt_len = 2048
    cfg, m = _decode_model(torch, rt, ctx, 1, prompt_len + 2 * (W + K) + 64, prompt_len)
    ids = np.random.default_rng(dist.rank).integers(0, cfg.vocab, prompt_len)
    torch.cuda.synchronize()
    s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    first = m.prefill(0, ids)
    e0.record()
    torch.cuda.synchronize()
    prefill_ms = s0.elapsed_time(e0)
    m.buf["next"][0] = first
    m.capture_decode(batch=1)
    for _ in range(W):
        m.replay_decode()
    clk = ClockSampler(dist.local)
    clk.start()
    dist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(K):
        m.replay_decode()
    e.record()
    torch.cuda.synchronize()
    dist.barrier()
    clocks = clk.stop()
    ms = dist.max(s.elapsed_time(e))
    ctx.check_device()
    h_in = torch.tensor([first], dtype=torch.int32).pin_memory()
    h_out = torch.empty(1, dtype=torch.int32).pin_memory()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    n2 = max(3, min(K, 16))
    for _ in range(n2):
        m.buf["next"][:1].copy_(h_in, non_blocking=True)
        nxt = m.replay_decode()
        h_out.copy_(nxt, non_blocking=True)
    e2.record()
    torch.cuda.synchronize()
    e2e_ms = dist.max(s2.elapsed_time(e2)) / n2
    op_launches = _graph_kernel_count(m)
    persistent = _persistent_decode(torch, m, dist, K, W)
    w4_bytes = sum(L[n].in_dim * L[n].out_dim * 9 // 16 for L in m.layers for n in ("qkv", "o", "gu", "down", "pg", "pp"))
    per_tok = w4_bytes + m.top.in_dim * m.top.out_dim * 9 // 16 + cfg.vocab * cfg.hidden * 2
    tok_s = K / (ms / 1e3) * dist.world
    gbs = per_tok / (ms / 1e3 / K) / 1e9
    line = {
        "metric": "greedy decode throughput, batch 1 (config 4)", "value": round(tok_s, 1), "unit": "tok/s",
        "n_gpus": dist.world, "steps": K, "warmup": W, "ms_per_step": round(ms / K, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights, random prompt)",
        "config": {"workload": "config4_decode_b1", "prompt": prompt_len, "prefill_ms": round(prefill_ms, 2),
                   "l2": "1.5 GB of weights per token (>> L2)",
                   "decode_kernel": "operator path: one CUDA graph of PDL-chained kernels"},
        "roofline": {"bound": "hbm", "kernel": "whole decode step (weights + head bytes per token)",
                     "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(gbs / peaks["hbm_gbs"], 4), "peak_source": peaks["source"], "traffic": None,
                     "bytes_per_launch": per_tok},
        "e2e": {"value": round(1 / (e2e_ms / 1e3), 1), "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4},
        "gpu_launches": op_launches * K, "launches_per_step": op_launches, "clocks": clocks,
    }
    if persistent:
        persistent["achieved_gbs"] = round(per_tok / (persistent["ms_per_step"] / 1e3) / 1e9, 1)
        persistent["frac"] = round(persistent["achieved_gbs"] / peaks["hbm_gbs"], 4)
        line["persistent_decoder"] = persistent
    if dist.rank == 0 and dist.world == 1 and not getattr(args, "no_cpu", False):
        line["cpu_baseline"] = cpu_decode(batch=1, ctx_len=prompt_len)
    return line


def _persistent_decode(torch, m, dist, K, W):
    """The same decode measured through the persistent g4_decoder (one cooperative launch per
    token, opt-in): the step time over K graph replays after W warm-ups, then one eager step
    with the all-CTA timeline.  Runs after the operator path's timed region on the same
    sequence; None when the model's shapes are outside the decoder's range."""
    m.persistent, m._dec = True, None
    if m.decoder() is None:
        m.persistent = False
        return None
    m.capture_decode(batch=1)
    for _ in range(W):
        m.replay_decode()
    dist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(K):
        m.replay_decode()
    e.record()
    torch.cuda.synchronize()
    dist.barrier()
    ms = dist.max(s.elapsed_time(e)) / K
    m.ctx.check_device()
    out = {"kernel": "decode_step_kernel: the whole token in one cooperative launch (148 CTAs, grid barriers)",
           "ms_per_step": round(ms, 4), "value": round(1e3 / ms * dist.world, 1), "unit": "tok/s",
           "launches_per_step": _graph_kernel_count(m)}
    out["timeline"] = _decoder_timeline(torch, m)
    return out


def _decoder_timeline(torch, m):
    """One eager persistent step with every CTA's globaltimer stamps on, summarised per phase
    kind and averaged over the layers (us, medians over the CTAs): for each grid barrier the
    arrival skew (last - first CTA) and its own latency (median pass - last arrival); for each
    linear the wait for its weights and its compute; the attention tile's stages (CTAs with a
    tile); and each row-wise operator.  Taken after the timed region (it advances the sequence)."""
    lib = importlib.import_module("gemma4-js_b200._lib")
    dec = m.decoder()
    Lc = m.cfg.layers
    per = 1 + 2 + 39 * Lc + 2 + 1
    G = torch.cuda.get_device_properties(m.ctx.device).multi_processor_count
    buf = torch.zeros((G, per), dtype=torch.int64, device=m.ctx.torch_device)
    lib.call("g4_decoder_set_timeline", dec.handle, C.c_void_p(buf.data_ptr()), per)
    m.decode_step(batch=1)
    torch.cuda.synchronize()
    lib.call("g4_decoder_set_timeline", dec.handle, None, 0)
    m.ctx.check_device()
    t = buf.cpu().numpy().astype(np.float64) / 1e3
    t = t - t[:, 0].min()
    acc = {}
    state = {"i": 1, "prev": t[:, 0]}

    def add(key, val):
        acc.setdefault(key, []).append(float(val))

    def lin(name):
        i, prev = state["i"], state["prev"]
        add(f"linear_{name}.weights_wait_us", np.median(t[:, i] - prev))
        add(f"linear_{name}.compute_us", np.median(t[:, i + 1] - t[:, i]))
        state["i"], state["prev"] = i + 2, t[:, i + 1]

    def bar(name):
        i = state["i"]
        arrive, passed = t[:, i], t[:, i + 1]
        add(f"barrier_{name}.skew_us", arrive.max() - arrive.min())
        add(f"barrier_{name}.latency_us", np.median(passed) - arrive.max())
        state["i"], state["prev"] = i + 2, passed

    def op(name):
        i, prev = state["i"], state["prev"]
        add(f"op_{name}_us", np.median(t[:, i] - prev))
        state["i"], state["prev"] = i + 1, t[:, i]

    def attention():
        i, prev = state["i"], state["prev"]
        a = t[:, i:i + 4]
        busy = (a[:, 3] - a[:, 0]) > 0
        if busy.any():
            add("attention_tile.q_ready_us", np.median(a[busy, 1] - a[busy, 0]))
            add("attention_tile.kv_wait_us", np.median(a[busy, 2] - a[busy, 1]))
            add("attention_tile.attend_us", np.median(a[busy, 3] - a[busy, 2]))
            add("attention_tile.ctas", busy.sum())
            tot = np.where(busy, a[:, 3] - prev, -1.0)
            c = int(np.argmax(tot))
            add("attention_tile.slowest_us", tot[c])
            add("attention_tile.slowest_q_us", a[c, 1] - a[c, 0])
            add("attention_tile.slowest_kv_us", a[c, 2] - a[c, 1])
            add("attention_tile.slowest_attend_us", a[c, 3] - a[c, 2])
            add("attention_tile.slowest_start_us", a[c, 0] - prev[c])
            add("attention_tile.slowest_is_last_tile", float(c == int(busy.sum()) - 1))
        state["i"], state["prev"] = i + 4, a[:, 3]

    lin("top")
    for _ in range(Lc):
        lin("qkv"), bar("qkv"), attention(), bar("attention"), op("combine"), bar("combine"), op("load_attn")
        lin("o"), bar("o"), op("post_norm_add_o")
        lin("gate_up"), bar("gate_up"), op("load_act")
        lin("down"), bar("down"), op("post_norm_add_down")
        lin("ple_gate"), bar("ple_gate"), op("ple_mix_gelu")
        lin("ple_proj"), bar("ple_proj"), op("post_norm_add_ple")
    i = state["i"]
    head_arrive = t[:, i]
    out = {"total_us": round(float(np.median(t[:, per - 1])), 1), "ctas": G, "barriers": 8 * Lc + 1,
           "head_us": round(float(np.median(head_arrive - state["prev"])), 1)}
    for k, v in acc.items():
        group, _, field = k.partition(".")
        if field:
            out.setdefault(group, {})[field] = round(float(np.mean(v)), 2)
        else:
            out[group] = round(float(np.mean(v)), 2)
    return out


def native_oracle():
    """The oracle's C restatement built for this host's CPU (-march=native)."""
    oracle = importlib.import_module("oracle")
    import platform
    out = REPO / "_build" / f"oracle_native_{platform.node() or 'host'}.so"
    return oracle, oracle.lib(oracle.build(out, march="native"))


def cpu_ple(sample_s: float, threads: int, vocab_sample: int = 8192):
    """Times the restated LocalPleW4ShardReader.readRows on 4096-id batches over a
    host table of `vocab_sample` rows with the config's distributions."""
    import numpy as np
    oracle, L = native_oracle()
    rng = np.random.default_rng(0)
    q = rng.integers(-7, 8, size=(vocab_sample, 8960), dtype=np.int8)
    nib = (q.astype(np.int16) & 0xF).astype(np.uint8)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
    scales = oracle.f32_to_bf16_bits(np.abs(rng.normal(0, 0.05, (vocab_sample, 280))).astype(np.float32))
    ids = rng.integers(0, vocab_sample, 4096).astype(np.int32)
    oracle.ple_read_rows(packed, scales, ids[:64], bf16=True, nthreads=threads, L=L)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < sample_s:
        oracle.ple_read_rows(packed, scales, ids, bf16=True, nthreads=threads, L=L)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(PLE_BYTES * n / dt / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": "port", "cpu": _cpu_model(),
            "sample": f"{n} x 4096-id gathers (bf16 out) over a {vocab_sample}-row host table, {dt:.1f} s",
            "calls_per_s": round(n / dt, 4)}


class CpuDecode:
    """One greedy decode step of the restated TFJS path on the host: every linear of the 35
    layers dequantised on each call and multiplied in f32 (official-quantized-linear.js:82-128),
    attention over the context per layer (window 512 on 4 of 5 layers), the f32 tied head
    over 262144 rows (a BLAS matmul)."""

    SHAPES = {"qkv": (2560, 1536), "o": (1536, 2048), "gu": (12288, 1536), "down": (1536, 6144), "pg": (256, 1536),
              "pp": (1536, 256), "top": (8960, 1536)}

    def __init__(self, ctx_len: int, threads: int, layers: int = 35):
        import numpy as np
        self.np = np
        self.oracle, self.L = native_oracle()
        self.ctx_len, self.threads, self.layers = ctx_len, threads, layers
        rng = np.random.default_rng(0)
        self.W = {}
        for k, (n, kk) in self.SHAPES.items():
            self.W[k] = (rng.integers(0, 2**32, size=(n, kk // 8), dtype=np.uint64).astype(np.uint32).view(np.int32),
                         self.oracle.f32_to_bf16_bits(np.abs(rng.normal(0, 0.02, (n, kk // 32))).astype(np.float32)))
        self.head = rng.standard_normal((262144, 1536)).astype(np.float32) * 0.05
        self.kc = rng.standard_normal((ctx_len + 1, 256)).astype(np.float32)
        self.rng = rng

    def step(self, batch: int) -> float:
        """Runs one decode step for `batch` sequences; returns its wall time in seconds."""
        np, o, L = self.np, self.oracle, self.L
        q = self.rng.standard_normal((batch, 8, 256)).astype(np.float32)
        x = {k: self.rng.standard_normal((batch, kk)).astype(np.float32) for k, (n, kk) in self.SHAPES.items()}
        t0 = time.perf_counter()
        o.linear_w4a16(x["top"], *self.W["top"], nthreads=self.threads, L=L)
        for layer in range(self.layers):
            for k in ("qkv", "o", "gu", "down", "pg", "pp"):
                o.linear_w4a16(x[k], *self.W[k], nthreads=self.threads, L=L)
            full = (layer + 1) % 5 == 0
            keys = self.ctx_len + 1 if full else min(self.ctx_len + 1, 512)
            for b in range(batch):
                o.attention(q[b:b + 1], self.kc[:keys], self.kc[:keys], keys - 1, not full, 512)
        logits = x["top"][:, :1536] @ self.head.T
        dt = time.perf_counter() - t0
        del logits
        return dt


class CpuServeStep:
    """One greedy decode step of a whole batch on the host, as the reference's TFJS path
    computes a batch: each linear's weight dequantised to f32 once per call
    (official-quantized-linear.js:100-111, here all rows at once on the host threads) and
    multiplied by the batch's activations with tf.matMul(x, W^T) (:113-117, a BLAS sgemm
    here); attention per sequence over its own context, window 512 on 4 of 5 layers
    (official-w4a16-layer0.js:30-62: Q.K^T, softmax, P.V as batched BLAS); the f32 tied
    head over 262144 rows with the softcap and the greedy pick (gemma4-webgpu.js:413-480).
    Every sequence has its own K/V rows; the 35 layers cycle over one set of per-shape
    weights and one global-length K/V set, so host memory stays ~6 GB."""

    SHAPES = CpuDecode.SHAPES

    def __init__(self, batch: int, ctx_len: int, threads: int, layers: int = 35):
        self.oracle, self.L = native_oracle()
        self.batch, self.ctx_len, self.threads, self.layers = batch, ctx_len, threads, layers
        rng = np.random.default_rng(0)
        self.W, self.deq, self.x = {}, {}, {}
        for k, (n, kk) in self.SHAPES.items():
            self.W[k] = (rng.integers(0, 2**32, size=(n, kk // 8), dtype=np.uint64).astype(np.uint32).view(np.int32),
                         self.oracle.f32_to_bf16_bits(np.abs(rng.normal(0, 0.02, (n, kk // 32))).astype(np.float32)))
            self.deq[k] = np.empty((n, kk), np.float32)
            self.x[k] = rng.standard_normal((batch, kk), dtype=np.float32)
        # large operands tiled from one seeded 16 MB block (values do not change the cost)
        blk = rng.standard_normal(1 << 22, dtype=np.float32)
        self.head = self._tiled(blk, (262144, 1536), 0.05)
        keys = ctx_len + 1
        self.kc = self._tiled(blk[::-1], (batch, keys, 256), 0.3)
        self.vc = self._tiled(blk, (batch, keys, 256), 1.0)
        self.q = rng.standard_normal((batch, 8, 256), dtype=np.float32)
        from concurrent.futures import ThreadPoolExecutor
        self.pool = ThreadPoolExecutor(max_workers=threads)

    @staticmethod
    def _tiled(blk, shape, scale):
        n = int(np.prod(shape))
        out = np.empty(n, np.float32)
        for i in range(0, n, blk.size):
            j = min(n, i + blk.size)
            np.multiply(blk[:j - i], np.float32(scale), out=out[i:j])
        return out.reshape(shape)

    def _linear(self, k):
        self.oracle.dequant_w4a16_par(*self.W[k], out=self.deq[k], nthreads=self.threads, L=self.L)
        return self.x[k] @ self.deq[k].T

    def _attention_seqs(self, lo, hi, keys):
        out = np.empty((hi - lo, 8, 256), np.float32)
        for b in range(lo, hi):
            logits = self.q[b] @ self.kc[b, -keys:].T
            logits -= logits.max(-1, keepdims=True)
            p = np.exp(logits)
            p /= p.sum(-1, keepdims=True)
            out[b - lo] = p @ self.vc[b, -keys:]
        return out

    def _attention(self, keys):
        """Sequences split over the host threads, one single-threaded BLAS call per product."""
        from threadpoolctl import threadpool_limits
        n, B = self.threads, self.batch
        with threadpool_limits(1):
            parts = list(self.pool.map(lambda t: self._attention_seqs(B * t // n, B * (t + 1) // n, keys), range(n)))
        return np.concatenate(parts)

    def step(self) -> float:
        """Runs one decode step of the batch; returns its wall time in seconds."""
        t0 = time.perf_counter()
        self._linear("top")
        for layer in range(self.layers):
            full = (layer + 1) % 5 == 0
            self._linear("qkv")
            self._attention(self.ctx_len + 1 if full else min(self.ctx_len + 1, 512))
            for k in ("o", "gu", "down", "pg", "pp"):
                self._linear(k)
        logits = self.x["top"][:, :1536] @ self.head.T
        np.argmax(np.tanh(logits / np.float32(30.0)) * np.float32(30.0), axis=1)
        return time.perf_counter() - t0


def cpu_decode(batch: int, ctx_len: int, threads: int = 1, model_layers: int = 35):
    """The cpu_baseline object: one decode step of CpuDecode on `threads` host threads."""
    dt = CpuDecode(ctx_len, threads, model_layers).step(batch)
    return {"value": round(batch / dt, 5), "unit": "tok/s", "cores": threads, "kind": "port", "cpu": _cpu_model(),
            "sample": f"one decode step of {batch} sequence(s) at context {ctx_len}: {model_layers} layers x 6 W4A16 linears "
                      f"(dequantised per call) + attention + f32 tied head, {dt:.1f} s"}


def _cpu_model() -> str:
    """The host CPU's model name (first /proc/cpuinfo entry) and its logical core count."""
    name = "unknown"
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                name = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return f"{name} ({os.cpu_count()} logical cores)"


def _reference_line(args, dist, metric, value, unit, ms, config, dtype, sample, threads, hib=True, scaling="weak"):
    return {"impl": "reference", "metric": metric, "value": value, "unit": unit, "n_gpus": dist.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": hib,
            "scaling": scaling, "vs_baseline": None, "dtype": dtype, "data": "synthetic (seeded)", "config": config,
            "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": "port", "cpu": _cpu_model(), "sample": sample},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_reference(args, dist):
    """Reference arm: the CPU restatement of the TFJS path (the oracle port; the JS
    reference itself has no runtime in this image), all host threads, rank 0 only, on
    a bounded sample of the same workload per step."""
    threads = os.cpu_count() or 1
    K, W = args.steps, args.warmup
    import numpy as np
    if args.workload == "serve":
        # a step: one greedy decode step of the whole 256-sequence batch at context 4096,
        # the GPU arm's config
        m = CpuServeStep(256, 4096, threads)
        for _ in range(W):
            m.step()
        dt = sum(m.step() for _ in range(K))
        v = round(256 * K / dt, 4)
        return _reference_line(args, dist, SERVE_METRIC, v, "tok/s", dt / K * 1e3, serve_config(dist.world), "f32",
                               f"{K} decode steps of all 256 sequences at context 4096: 35 layers x 6 W4A16 linears "
                               f"dequantised once per call and multiplied as one f32 GEMM over the batch, attention "
                               f"per sequence, f32 tied head + softcap + argmax", threads,
                               scaling="strong")
    if args.workload == "decode":
        # a step: one greedy decode step of one sequence at the 2048-token prompt
        m = CpuDecode(2048, threads)
        for _ in range(W):
            m.step(1)
        dt = sum(m.step(1) for _ in range(K))
        v = round(K / dt, 5)
        config = {"workload": "config4_decode_b1", "prompt": 2048, "l2": "1.5 GB of weights per token (>> L2)"}
        return _reference_line(args, dist, "greedy decode throughput, batch 1 (config 4)", v, "tok/s", dt / K * 1e3,
                               config, "f32", f"{K} decode steps of 1 sequence at context 2048 (35 layers x 6 W4A16 "
                                              f"linears dequantised per call, attention, f32 tied head)", threads)
    oracle, L = native_oracle()
    rng = np.random.default_rng(0)
    if args.workload in ("gemv", "gemm"):
        Kd, N, M = (1536, 6144, 1) if args.workload == "gemv" else (1536, 6144, 512)
        packed = rng.integers(0, 2**32, size=(N, Kd // 8), dtype=np.uint64).astype(np.uint32).view(np.int32)
        scales = oracle.f32_to_bf16_bits(np.abs(rng.normal(0, 0.02, (N, Kd // 32))).astype(np.float32))
        x = rng.standard_normal((M, Kd)).astype(np.float32)
        for _ in range(W):
            oracle.linear_w4a16(x, packed, scales, nthreads=threads, L=L)
        t0 = time.perf_counter()
        for _ in range(K):
            oracle.linear_w4a16(x, packed, scales, nthreads=threads, L=L)
        dt = time.perf_counter() - t0
        if args.workload == "gemv":
            v = round(GEMV_BYTES * K / dt / 1e9, 4)
            return _reference_line(args, dist, "W4A16 decode GEMV throughput (algorithmic bytes)", v, "GB/s",
                                   dt / K * 1e3, {"workload": "config1_gemv", "M": 1, "K": Kd, "N": N}, "f32",
                                   f"{K} calls of the dequantise-then-matmul linear (official-quantized-linear.js:82-128)",
                                   threads)
        v = round(2.0 * M * N * Kd * K / dt / 1e12, 5)
        return _reference_line(args, dist, "W4A16 prefill GEMM throughput (config 3 sweep)", v, "TFLOP/s",
                               dt / K * 1e3, {"workload": "config3_gemm", "sample": f"M={M} K={Kd} N={N}"}, "f32",
                               f"{K} calls at M={M}, (K, N) = ({Kd}, {N}), one point of the config 3 sweep", threads)
    if args.workload == "attn_rows":
        # a step: the attention of a bounded sample of the batch's sequences (the same
        # per-sequence work as the GPU launch), reported as algorithmic GB/s
        hd, pos, n = 256, 4096, 4
        keys = 512 if args.sliding else pos + 1
        kc = rng.standard_normal((pos + 1, hd)).astype(np.float32)
        vc = rng.standard_normal((pos + 1, hd)).astype(np.float32)
        q = rng.standard_normal((1, 8, hd)).astype(np.float32)
        for _ in range(W):
            oracle.attention(q, kc, vc, pos, bool(args.sliding), 512)
        t0 = time.perf_counter()
        for _ in range(K * n):
            oracle.attention(q, kc, vc, pos, bool(args.sliding), 512)
        dt = time.perf_counter() - t0
        byts = keys * hd * 2 * 2 + 2 * 8 * hd * 2
        v = round(byts * K * n / dt / 1e9, 4)
        return _reference_line(args, dist, "batched decode attention throughput (algorithmic bytes)", v, "GB/s",
                               dt / K * 1e3, {"workload": "decode_attention_rows_" + ("sliding" if args.sliding
                                                                                      else "global"),
                                              "batch": args.batch, "keys": keys, "hd": hd, "heads": 8}, "f32",
                               f"{n} of the {args.batch} sequences per step, one thread", 1)
    if args.workload == "head":
        # a step: logits + softcap + greedy pick of one row against a bounded vocabulary
        # sample (the f32 tied head of the CPU decode), reported as TFLOP/s
        Kd, vs = 1536, 16384
        E = (rng.standard_normal((vs, Kd)) * 0.05).astype(np.float32)
        x = rng.standard_normal((1, Kd)).astype(np.float32)
        for _ in range(W):
            np.argmax(np.tanh((x @ E.T) / 30.0) * 30.0)
        t0 = time.perf_counter()
        for _ in range(K):
            np.argmax(np.tanh((x @ E.T) / 30.0) * 30.0)
        dt = time.perf_counter() - t0
        v = round(2.0 * vs * Kd * K / dt / 1e12, 6)
        return _reference_line(args, dist, "fused LM head (logits + softcap + greedy pick) TFLOP/s", v, "TFLOP/s",
                               dt / K * 1e3, {"workload": "lm_head_argmax", "M": args.batch, "vocab": 262144,
                                              "K": Kd}, "f32",
                               f"{K} rows against a {vs}-row sample of the table (numpy, host BLAS threads)",
                               threads)
    if args.workload == "attn":
        keylen, hd = 4096, 256
        kc = rng.standard_normal((keylen, hd)).astype(np.float32)
        vc = rng.standard_normal((keylen, hd)).astype(np.float32)
        q = rng.standard_normal((1, 8, hd)).astype(np.float32)
        for _ in range(W):
            oracle.attention(q, kc, vc, keylen - 1, False, 512)
        t0 = time.perf_counter()
        for _ in range(K):
            oracle.attention(q, kc, vc, keylen - 1, False, 512)
        dt = time.perf_counter() - t0
        v = round(ATTN_BYTES * K / dt / 1e9, 4)
        return _reference_line(args, dist, "GQA decode attention throughput (algorithmic bytes)", v, "GB/s",
                               dt / K * 1e3, {"workload": "decode_attention_global", "keylen": keylen, "hd": hd,
                                              "heads": 8}, "f32", f"{K} global-attention decode calls, one thread",
                               1)
    vs = 8192
    q = rng.integers(-7, 8, size=(vs, 8960), dtype=np.int8)
    nib = (q.astype(np.int16) & 0xF).astype(np.uint8)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
    scales = oracle.f32_to_bf16_bits(np.abs(rng.normal(0, 0.05, (vs, 280))).astype(np.float32))
    batches = [rng.integers(0, vs, 4096).astype(np.int32) for _ in range(K + W)]
    for i in range(W):
        oracle.ple_read_rows(packed, scales, batches[i], bf16=True, nthreads=threads, L=L)
    t0 = time.perf_counter()
    for i in range(K):
        oracle.ple_read_rows(packed, scales, batches[W + i], bf16=True, nthreads=threads, L=L)
    dt = time.perf_counter() - t0
    v = PLE_BYTES * K / dt / 1e9
    return {"impl": "reference", "metric": "PLE W4 gather-dequant throughput (algorithmic bytes)",
            "value": round(v, 3), "unit": "GB/s", "n_gpus": dist.world, "steps": K, "warmup": W,
            "ms_per_step": round(dt / K * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8", "data": "synthetic (seeded int4 table, uniform ids)",
            "config": {"workload": "config2_ple_gather", "tokens_per_step_per_gpu": 4096},
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": "port", "cpu": _cpu_model(),
                             "sample": f"{K} x 4096-id gathers over an {vs}-row host table (C restatement of "
                                       f"ple-w4-shard-reader.js:65-104; the JS reference has no runtime here)"},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="serve",
                    choices=["ple", "gemv", "attn", "attn_rows", "head", "gemm", "decode", "serve"])
    ap.add_argument("--batch", type=int, default=256, help="attn_rows / head: rows (sequences)")
    ap.add_argument("--sliding", action="store_true", help="attn_rows: the 512-key window of a sliding layer")
    ap.add_argument("--impl", default="g4", choices=["g4", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--vocab", type=int, default=262144, help="ple: table rows (smaller for ncu captures)")
    ap.add_argument("--copies", type=int, default=0, help="gemv/attn: rotating weight / KV copies")
    ap.add_argument("--gemm-shapes", default="", help='gemm: "M1,M2:KxN,KxN" instead of the config 3 sweep')
    ap.add_argument("--gemm-impl", type=int, default=0, help="gemm: 0 auto, 1 GEMV, 2 tcgen05")
    ap.add_argument("--no-pdl", action="store_true", help="gemv: launch without programmatic dependent launch")
    ap.add_argument("--no-extras", action="store_true",
                    help="serve: skip the config 1-4 sub-measurements that the 1-GPU line carries")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep stdout to the one JSON line
    dist = Dist()
    if args.impl == "reference":
        if dist.rank == 0:
            print(json.dumps(run_reference(args, dist)), flush=True)
        return
    import torch
    dist.init(use_cuda=True)
    torch.cuda.set_device(dist.local)
    rt = importlib.import_module("gemma4-js_b200.runtime")
    ctx = rt.Context(dist.local)
    peaks = load_peaks()
    fn = {"ple": run_ple, "gemv": run_gemv, "attn": run_attn, "attn_rows": run_attn_rows, "head": run_head,
          "gemm": run_gemm, "decode": run_decode, "serve": run_serve}[args.workload]
    line = fn(args, torch, rt, ctx, dist, peaks)
    if dist.rank == 0:
        print(json.dumps(line), flush=True)
    ctx.sync()
    dist.close()


if __name__ == "__main__":
    main()
