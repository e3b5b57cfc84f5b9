#!/usr/bin/env python
"""Decode throughput of the CUDA TextEngine on B200.

One step = one TextEngine.generateBatch call over the workload: every row's window is encoded
(prefill) and then ``steps`` tokens are decoded greedily for every row. The default workload is
the batch-256 decode of a V4096 / d512 / 6-layer / 8-head / FFN2048 / window-512 padded decoder
(256-token prompts, 256 new tokens per row, fp32 weights and cache); with N GPUs each rank decodes
its own 256 rows (batch-sharded, no collective on the data path: weak scaling).

Prints one JSON line (rank 0). ``--impl reference`` times the CPU restatement of the reference
(full-window recompute per step, as TextEngine does) on the host cores instead.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

DEFAULT_WORKLOAD = "v4096-d512-l6-w512-b256-greedy"
BATCH1_WORKLOAD = "v8192-d768-l12-w1024-b1-greedy-bf16w"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="cuda", choices=["cuda", "reference"])
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batch1", action="store_true")
    ap.add_argument("--rows", type=int, default=0, help="override the workload's rows per GPU")
    ap.add_argument("--new-tokens", type=int, default=0, help="override tokens decoded per row")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        p = json.loads(path.read_text())
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, sm_max, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                sm_max = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": sm_max,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_baseline(workload, weights_path, threads=None, budget_s=15.0):
    """The reference's algorithm on the host cores: every step re-runs Module.forward over the
    full [rows, window] batch (TextEngine.generateBatch, TextEngine.java:232-254) with gemm.rs
    numerics, on a bounded sample of the workload's rows and steps."""
    from basalt_b200 import left_pad, synthetic_prompts
    from oracle import oracle as orc

    if threads:
        orc.set_threads(threads)
    m = workload.model
    oracle = orc.OracleEngine(orc.FAMILY_PADDED_DECODER, m.vocabulary, m.window, m.dimension,
                              m.layers, m.heads, m.hidden)
    oracle.load(weights_path)
    rows = min(4, workload.rows)
    prompts = synthetic_prompts(workload.prompt_seed, rows, workload.prompt, m.vocabulary)
    ctx = left_pad(prompts, m.window, m.vocabulary)
    t0 = time.perf_counter()
    oracle.generate_batch(ctx, 1)
    one = time.perf_counter() - t0
    steps = int(max(1, min(workload.steps, budget_s / max(one, 1e-3))))
    t0 = time.perf_counter()
    oracle.generate_batch(ctx, steps)
    elapsed = time.perf_counter() - t0
    line = {"value": rows * steps / elapsed, "unit": "tokens/s", "cores": orc.threads(),
            "kind": "port",
            "sample": f"{rows} rows x {steps} greedy steps of {workload.name}, full-window "
                      f"recompute per step ({elapsed:.1f} s)"}
    # The same model decoded the way a cached CPU engine would (one token per row per step over a
    # per-row KV cache), one row per host thread; decode rate from two runs that differ only in
    # the number of steps, so the token-by-token prefill cancels.
    crows = max(1, min(orc.threads(), workload.rows))
    cprompts = synthetic_prompts(workload.prompt_seed, crows, workload.prompt, m.vocabulary)
    cctx = left_pad(cprompts, m.window, m.vocabulary)
    t0 = time.perf_counter()
    oracle.generate_batch_cached(cctx, 1)
    base = time.perf_counter() - t0
    extra = int(max(1, min(workload.steps - 1, 64)))
    t0 = time.perf_counter()
    oracle.generate_batch_cached(cctx, 1 + extra)
    longer = time.perf_counter() - t0
    line["cached"] = {"value": crows * extra / max(1e-9, longer - base), "unit": "tokens/s",
                      "sample": f"{crows} rows x {extra} greedy steps over a per-row KV cache "
                                f"({base:.1f} s and {longer:.1f} s runs)"}
    return line


# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of a kernel class, from one
# ncu capture of the named workload (the commands are kept with the profile summaries):
# "gemm_step": mean over the 25 projection launches of one lane's decode step (at ~258 cached
# keys); "gemm": mean over the four prefill projections of one layer (M = 65 536 tokens).
NCU_TRAFFIC = {
    ("v4096-d512-l6-w512-b256-greedy", "gemm_step"): 7.64e6,
    ("v4096-d512-l6-w512-b256-greedy", "gemm"): 0.956e9,
}


def profile_summary(engine, run):
    """Per-kernel device time of one call of `run`, CUDA events around every launch."""
    import torch

    engine.profile(True)
    engine.profile_reset()
    run()
    torch.cuda.synchronize()
    prof = engine.profile_read()
    engine.profile(False)
    total_ms = sum(v["ms"] for v in prof.values()) or 1.0
    kernels = {n: {"launches": v["launches"], "ms": round(v["ms"], 3),
                   "share": round(v["ms"] / total_ms, 4),
                   "GB/s": round(v["bytes"] / (v["ms"] / 1000.0) / 1e9, 1) if v["ms"] else None,
                   "TFLOP/s": round(v["flops"] / (v["ms"] / 1000.0) / 1e12, 2) if v["ms"] else None}
               for n, v in sorted(prof.items(), key=lambda kv: -kv[1]["ms"])}
    return prof, kernels


def batch1(local, steps, warmup):
    """Single-stream latency: batch 1, 512-token prompt, 512 greedy tokens (bf16 weights)."""
    import torch

    from basalt_b200 import (Basalt, TextEngine, config, left_pad, synthetic_prompts,
                             write_synthetic_weights)

    w = config(BATCH1_WORKLOAD)
    m = w.model
    with tempfile.TemporaryDirectory() as tmp:
        path = Path(tmp) / "w.bin"
        write_synthetic_weights(m, path, w.weight_seed)
        engine = TextEngine.of(Basalt.create(local), m, m.vocabulary, m.window)
        engine.load(path)
    ctx = left_pad(synthetic_prompts(w.prompt_seed, 1, w.prompt, m.vocabulary), m.window,
                   m.vocabulary)
    stream = torch.cuda.ExternalStream(engine.cuda_stream(), device=torch.device("cuda", local))
    d_ctx = torch.from_numpy(ctx).to(f"cuda:{local}")
    d_tok = torch.empty((1, w.steps), dtype=torch.int32, device=f"cuda:{local}")
    d_one = torch.empty((1, 1), dtype=torch.int32, device=f"cuda:{local}")

    def call(n, out):
        engine.generate_device(d_ctx.data_ptr(), 1, ctx.shape[1], n, out.data_ptr())

    for _ in range(warmup):
        call(w.steps, d_tok)
        call(1, d_one)
    torch.cuda.synchronize()

    def timed(n, out, reps):
        # Median of separately timed calls: the per-token figure is a difference of two call
        # times, so one slow call would otherwise move it a lot.
        times = []
        for _ in range(max(3, reps)):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            call(n, out)
            b.record(stream)
            b.synchronize()
            times.append(a.elapsed_time(b))
        return float(np.median(times))

    full_ms = timed(w.steps, d_tok, steps)
    prefill_ms = timed(1, d_one, steps)
    per_token_ms = (full_ms - prefill_ms) / (w.steps - 1)
    prof, kernels = profile_summary(engine, lambda: call(w.steps, d_tok))
    hbm, _, src = measured_peaks()

    def gbs(entry):
        return entry["bytes"] / (entry["ms"] / 1000.0) / 1e9 if entry and entry["ms"] else None

    step_gbs = gbs(prof.get("decode_step"))
    # The same decode on the kernel-per-operation path (the fused step switched off), for the
    # GEMV and attention kernels' own bandwidth.
    os.environ["BST_FUSED_DECODE"] = "0"
    try:
        unfused_ms = timed(w.steps, d_tok, max(1, steps // 2))
        uprof, ukernels = profile_summary(engine, lambda: call(w.steps, d_tok))
    finally:
        del os.environ["BST_FUSED_DECODE"]
    gemv_gbs = gbs(uprof.get("gemv"))
    attn_gbs = gbs(uprof.get("attn_decode"))
    engine.close()
    return {"workload": w.name, "tokens_per_s": w.steps / (full_ms / 1000.0),
            "ms_per_call": full_ms, "prefill_ms": prefill_ms,
            "decode_ms_per_token": per_token_ms,
            "decode_step_GBps": step_gbs, "decode_step_frac": step_gbs / hbm if step_gbs else None,
            "kernels": kernels,
            "per_operation_path": {
                "decode_ms_per_token": (unfused_ms - prefill_ms) / (w.steps - 1),
                "gemv_GBps": gemv_gbs, "gemv_frac": gemv_gbs / hbm if gemv_gbs else None,
                "attn_decode_GBps": attn_gbs,
                "attn_decode_frac": attn_gbs / hbm if attn_gbs else None,
                "kernels": ukernels},
            "peak_source": src}


def other_configs(local, reps=3):
    """The other workloads of the scope table, timed on the device: C1 and C2 as per-call latency
    (L2-resident models), C3 with bf16 weights as decode tokens/s."""
    import torch

    from basalt_b200 import (Basalt, TextEngine, config, left_pad, synthetic_prompts,
                             write_synthetic_weights)

    from dataclasses import replace

    out = {}
    for name in ("v96-d128-l2-w64-b1-greedy", "v96-d256-l4-w128-b32-greedy",
                 "v96-d256-l4-w128-b32-sampled", "v4096-d512-l6-w512-b256-greedy-bf16w",
                 "v8192-d768-l12-w1024-n8192-sampled-bf16w"):
        w = config(name)
        if w.rows > 4096:
            # 8192 sequences in waves of max_rows: 64 of the 512 tokens per row keep the call short
            w = replace(w, steps=64)
        m = w.model
        with tempfile.TemporaryDirectory() as tmp:
            path = Path(tmp) / "w.bin"
            write_synthetic_weights(m, path, w.weight_seed)
            engine = TextEngine.of(Basalt.create(local), m, m.vocabulary, m.window)
            engine.load(path)
        ctx = left_pad(synthetic_prompts(w.prompt_seed, w.rows, w.prompt, m.vocabulary), m.window,
                       m.vocabulary)
        stream = torch.cuda.ExternalStream(engine.cuda_stream(), device=torch.device("cuda", local))
        d_ctx = torch.from_numpy(ctx).to(f"cuda:{local}")
        d_tok = torch.empty((w.rows, w.steps), dtype=torch.int32, device=f"cuda:{local}")
        d_one = torch.empty((w.rows, 1), dtype=torch.int32, device=f"cuda:{local}")

        def call(n, dst):
            if w.mode == "sample":
                engine.seed(w.sample_seed)
                engine.sample_device(d_ctx.data_ptr(), w.rows, ctx.shape[1], n, w.temperature,
                                     w.k, dst.data_ptr())
            else:
                engine.generate_device(d_ctx.data_ptr(), w.rows, ctx.shape[1], n, dst.data_ptr())

        def timed(n, dst):
            # Median of separately timed calls: the decode figure is a difference of two call
            # times, so one slow call would otherwise move it a lot.
            times = []
            for _ in range(reps):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                call(n, dst)
                b.record(stream)
                b.synchronize()
                times.append(a.elapsed_time(b))
            return float(np.median(times))

        call(w.steps, d_tok)
        call(1, d_one)
        torch.cuda.synchronize()
        full_ms = timed(w.steps, d_tok)
        first_ms = timed(1, d_one)
        decode_ms = (full_ms - first_ms) / max(1, w.steps - 1)
        out[name] = {"rows": w.rows, "new_tokens": w.steps, "ms_per_call": full_ms,
                     "prefill_ms": first_ms, "decode_ms_per_step": decode_ms,
                     "tokens_per_s": w.rows * w.steps / (full_ms / 1000.0),
                     "decode_tokens_per_s": w.rows / (decode_ms / 1000.0) if decode_ms > 0 else None}
        engine.close()
    return out


def run_reference(args, rank, world):
    from basalt_b200 import config, write_synthetic_weights

    if rank != 0:
        return
    workload = config(args.workload)
    with tempfile.TemporaryDirectory() as tmp:
        path = Path(tmp) / "w.bin"
        write_synthetic_weights(workload.model, path, workload.weight_seed)
        values = []
        base = None
        for i in range(args.warmup + args.steps):
            base = cpu_baseline(workload, path, budget_s=max(2.0, 60.0 / (args.steps + args.warmup)))
            if i >= args.warmup:
                values.append(base["value"])
    value = float(np.median(values))
    line = {
        "impl": "reference", "metric": "decode tokens/s", "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * workload.rows * workload.steps / value,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": workload.name, "global_batch": workload.rows * args.gpus,
                   "seq_len": workload.model.window},
        "cpu_baseline": {**base, "value": value},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch

    from basalt_b200 import (Basalt, TextEngine, config, left_pad, synthetic_prompts,
                             write_synthetic_weights)

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    workload = config(args.workload)
    if args.rows or args.new_tokens:
        from dataclasses import replace

        workload = replace(workload, rows=args.rows or workload.rows,
                           steps=args.new_tokens or workload.steps)
    m = workload.model
    tmp = tempfile.TemporaryDirectory()
    wpath = Path(tmp.name) / "w.bin"
    write_synthetic_weights(m, wpath, workload.weight_seed)
    engine = TextEngine.of(Basalt.create(local), m, m.vocabulary, m.window)
    engine.load(wpath)

    # This rank's contiguous shard of one seeded draw of rows x world prompts (weak scaling:
    # `rows` per GPU). Sampling workloads start the shard's generator where the unsharded run
    # would be at its first row.
    from basalt_b200.sharding import shard_rng_state, shard_rows

    first, R = shard_rows(workload.rows * world, world, rank)
    prompts = synthetic_prompts(workload.prompt_seed, workload.rows * world, workload.prompt,
                                m.vocabulary)
    ctx = left_pad(prompts[first:first + R], m.window, m.vocabulary)
    steps = workload.steps
    if workload.mode == "sample":
        engine.rng_state = shard_rng_state(workload.sample_seed, steps, first)

    stream = torch.cuda.ExternalStream(engine.cuda_stream(), device=torch.device("cuda", local))
    d_ctx = torch.from_numpy(ctx).to(f"cuda:{local}")
    d_tok = torch.empty((R, steps), dtype=torch.int32, device=f"cuda:{local}")
    torch.cuda.synchronize()

    def device_step():
        engine.generate_device(d_ctx.data_ptr(), R, ctx.shape[1], steps, d_tok.data_ptr())

    for _ in range(args.warmup):
        device_step()
    torch.cuda.synchronize()

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    launches0 = engine.stats()["launches"]
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(local) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            device_step()
        stop.record(stream)
        stop.synchronize()
    barrier()
    launches = engine.stats()["launches"] - launches0
    ms = start.elapsed_time(stop)
    if dist:
        t = torch.tensor([ms], device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    tokens_per_step = R * steps * world
    value = tokens_per_step * args.steps / (ms / 1000.0)

    # End to end through the C ABI with host buffers: pinned contexts in, tokens out, every step.
    h_ctx = torch.from_numpy(ctx).pin_memory()
    h_tok = torch.empty((R, steps), dtype=torch.int32).pin_memory()
    from basalt_b200 import _lib

    lib = _lib.load()

    def host_step():
        code = lib.bst_generate(engine.handle, ctypes.cast(h_ctx.data_ptr(), _lib._i32p), R,
                                ctx.shape[1], steps, ctypes.cast(h_tok.data_ptr(), _lib._i32p),
                                _lib.TOKEN_SINK(0), None)
        if code:
            raise RuntimeError(_lib.last_error(engine.handle))

    host_step()
    barrier()
    e2e_start = torch.cuda.Event(enable_timing=True)
    e2e_stop = torch.cuda.Event(enable_timing=True)
    e2e_start.record(stream)
    for _ in range(args.steps):
        host_step()
    e2e_stop.record(stream)
    e2e_stop.synchronize()
    barrier()
    e2e_ms = e2e_start.elapsed_time(e2e_stop)
    if dist:
        t = torch.tensor([e2e_ms], device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = tokens_per_step * args.steps / (e2e_ms / 1000.0)

    # Prefill alone (one decoded token) vs the whole call: decode-only throughput.
    d_one = torch.empty((R, 1), dtype=torch.int32, device=f"cuda:{local}")
    engine.generate_device(d_ctx.data_ptr(), R, ctx.shape[1], 1, d_one.data_ptr())
    torch.cuda.synchronize()
    one_ms = []
    for _ in range(3):  # median of separately timed calls
        one_start = torch.cuda.Event(enable_timing=True)
        one_stop = torch.cuda.Event(enable_timing=True)
        one_start.record(stream)
        engine.generate_device(d_ctx.data_ptr(), R, ctx.shape[1], 1, d_one.data_ptr())
        one_stop.record(stream)
        one_stop.synchronize()
        one_ms.append(one_start.elapsed_time(one_stop))
    prefill_ms = float(np.median(one_ms))
    step_ms = ms / args.steps
    decode_tps = R * (steps - 1) / max(1e-9, (step_ms - prefill_ms) / 1000.0)

    # The decode step as a whole against HBM: every weight once plus the K/V every row reads
    # (mean cache length over the call), per decode step.
    kvb = 2 if m.kv_dtype == "bf16" else 4
    wbytes = 2 if m.weight_dtype == "bf16" else 4
    params = m.layers * (4 * m.dimension ** 2 + 2 * m.dimension * m.hidden) + m.vocabulary * m.dimension
    mean_len = min(m.window, workload.prompt + (steps + 1) / 2.0)
    step_bytes = R * m.layers * 2 * m.dimension * kvb * mean_len + params * wbytes
    step_s = max(1e-12, (step_ms - prefill_ms) / 1000.0 / max(1, steps - 1))
    hbm_peak, _, _ = measured_peaks()
    step_hbm = {"achieved": step_bytes / step_s / 1e9, "peak": hbm_peak, "unit": "GB/s",
                "frac": step_bytes / step_s / 1e9 / hbm_peak, "bytes_per_step": step_bytes,
                "mean_cache_len": mean_len}

    # Per-kernel device time with CUDA events around each launch (one instrumented step).
    prof, kernels = profile_summary(engine, device_step)
    top = max(prof.items(), key=lambda kv: kv[1]["ms"])
    name, k = top
    hbm, bf16, peak_src = measured_peaks()

    def tensor_roofline(cls, k):
        per_launch_s = k["ms"] / 1000.0 / k["launches"]
        achieved = k["flops"] / k["launches"] / per_launch_s / 1e12
        # fp32 weights run as 3xTF32 (three tf32 passes, tf32 at half the bf16 rate); bf16
        # weights as two bf16 passes: the ceiling for useful flops is the bf16 peak over that.
        passes, rate = (2, 1.0) if m.weight_dtype == "bf16" else (3, 0.5)
        useful_peak = bf16 * rate / passes
        return {"bound": "tensor", "achieved": achieved, "peak": bf16, "unit": "TFLOP/s",
                "frac": achieved / bf16, "traffic": None, "kernel": cls, "peak_source": peak_src,
                "tensor_passes": passes, "useful_flops_peak": useful_peak,
                "useful_frac": achieved / useful_peak}

    def hbm_roofline(cls, k):
        per_launch_s = k["ms"] / 1000.0 / k["launches"]
        achieved = k["bytes"] / k["launches"] / per_launch_s / 1e9
        return {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "traffic": None, "kernel": cls, "peak_source": peak_src}

    # Prefill GEMMs ("gemm", M = prompt tokens) are tensor-bound; the decode step's GEMMs
    # ("gemm_step", M = 128 rows per lane) stream their weights once per step: HBM / latency.
    roofline = tensor_roofline(name, k) if name == "gemm" else hbm_roofline(name, k)
    roofline["traffic"] = NCU_TRAFFIC.get((workload.name, name))

    line = {
        "metric": "decode tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16" if m.weight_dtype == "bf16" else "f32",
        "data": "synthetic: N(0,0.02) weights from java.util.Random(0), prompts from "
                f"java.util.Random({workload.prompt_seed}).nextInt({m.vocabulary})",
        "config": {"workload": workload.name, "model": f"padded decoder V{m.vocabulary} "
                   f"d{m.dimension} L{m.layers} H{m.heads} F{m.hidden} W{m.window}",
                   "global_batch": R * world, "seq_len": m.window, "prompt": workload.prompt,
                   "new_tokens": steps, "parallelism": f"batch-sharded x{world}",
                   "weights": m.weight_dtype, "kv_cache": m.kv_dtype,
                   "l2": "inputs larger than L2 (KV cache > 1 GB per GPU)"},
        "prefill_ms": prefill_ms, "decode_tokens_per_s": decode_tps * world,
        "decode_step_hbm": step_hbm,
        "e2e": {"value": e2e_value, "unit": "tokens/s",
                "h2d_bytes_per_step": int(ctx.nbytes), "d2h_bytes_per_step": int(R * steps * 4)},
        "gpu_launches": int(launches),
        "roofline": roofline,
        "roofline_prefill_gemm": (
            {**tensor_roofline("gemm", prof["gemm"]),
             "traffic": NCU_TRAFFIC.get((workload.name, "gemm"))} if "gemm" in prof else None),
        "kernels": kernels,
        "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_batch1:
        line["batch1"] = batch1(local, max(1, args.steps), max(1, args.warmup))
        line["configs"] = other_configs(local)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(workload, wpath)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    engine.close()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
