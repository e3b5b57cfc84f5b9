#!/usr/bin/env python
"""Decode throughput of the CUDA TextEngine on B200.

One step = one TextEngine.generateBatch call over the workload: every row's window is encoded
(prefill) and then ``steps`` tokens are decoded greedily for every row. The default workload is
the batch-256 decode of a V4096 / d512 / 6-layer / 8-head / FFN2048 / window-512 padded decoder
(256-token prompts, 256 new tokens per row, fp32 weights and cache); with N GPUs each rank decodes
its own 256 rows (batch-sharded, no collective on the data path: weak scaling). The same line
carries the 8192-sequence sampled workload split over the N ranks (strong scaling, key ``c5``).

Prints one JSON line (rank 0). ``--impl reference`` times the CPU restatement of the reference
(full-window recompute per step, as TextEngine does) on the host cores instead; that arm never
loads the CUDA library.

Ranks talk through a gloo process group only (start/stop barriers and the maximum of the ranks'
device times); nothing on the data path crosses GPUs.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

DEFAULT_WORKLOAD = "v4096-d512-l6-w512-b256-greedy"
BATCH1_WORKLOAD = "v8192-d768-l12-w1024-b1-greedy-bf16w"
SCALING_WORKLOAD = "v8192-d768-l12-w1024-n8192-sampled-bf16w"

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one decode step of the named
# workload from one ncu capture of its launches at 258 cached keys per row (summarised in the
# profiles directory): the kernels other than attention move a fixed amount per step (weights,
# split-K partials, activations), the attention kernels a fixed amount per (row, cached key), so
# the step's traffic at the call's mean cache length is fixed + per_row_key * rows * length.
NCU_STEP_TRAFFIC = {
    # Per 128-row lane and layer: QKV 6.84 MB, O 2.65, fix-ups 1.35 + 4.24 + 4.49, FFN1 8.94,
    # FFN2 10.51 (39.02 MB); 12 lane-layers plus the head's 17.33 MB. Attention: 138.02 MB for
    # 128 rows x 258 keys per layer, 4 179 B per (row, key, layer).
    "v4096-d512-l6-w512-b256-greedy": {"fixed": 12 * 39.02e6 + 17.33e6,
                                       "per_row_key": 6 * 138.02e6 / (128 * 258)},
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="cuda", choices=["cuda", "reference"])
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batch1", action="store_true")
    ap.add_argument("--no-scaling", action="store_true", help="skip the 8192-sequence workload")
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


def workload_of(args):
    from dataclasses import replace

    from basalt_b200.configs import config

    workload = config(args.workload)
    if args.rows or args.new_tokens:
        workload = replace(workload, rows=args.rows or workload.rows,
                           steps=args.new_tokens or workload.steps)
    return workload


def config_line(workload, rows_per_rank, world):
    """The ``config`` object both arms print (the reference arm times the same workload)."""
    m = workload.model
    return {"workload": workload.name,
            "model": f"padded decoder V{m.vocabulary} d{m.dimension} L{m.layers} H{m.heads} "
                     f"F{m.hidden} W{m.window}",
            "global_batch": rows_per_rank * world, "seq_len": m.window,
            "prompt": workload.prompt, "new_tokens": workload.steps,
            "parallelism": f"batch-sharded x{world}", "weights": m.weight_dtype,
            "kv_cache": m.kv_dtype, "l2": "inputs larger than L2 (KV cache > 1 GB per GPU)"}


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


# ---------------------------------------------------------------------------------------------
# CPU side: the oracle (the reference's algorithm restated in C++), never the CUDA library.
# ---------------------------------------------------------------------------------------------
def oracle_engine(workload, weights_path):
    from oracle import oracle as orc

    m = workload.model
    engine = orc.OracleEngine(orc.FAMILY_PADDED_DECODER, m.vocabulary, m.window, m.dimension,
                              m.layers, m.heads, m.hidden)
    engine.load(weights_path)
    return engine


def cpu_sample(engine, workload, rows, steps):
    """Times TextEngine.generateBatch's algorithm (TextEngine.java:232-254: every step re-runs
    Module.forward over the full [rows, window] batch, gemm.rs numerics) on `rows` rows of the
    workload for `steps` steps. Returns (tokens/s, seconds)."""
    from oracle import oracle as orc

    m = workload.model
    prompts = orc.synthetic_prompts(workload.prompt_seed, rows, workload.prompt, m.vocabulary)
    ctx = orc.left_pad(prompts, m.window, m.vocabulary)
    t0 = time.perf_counter()
    engine.generate_batch(ctx, steps)
    elapsed = time.perf_counter() - t0
    return rows * steps / elapsed, elapsed


def cpu_baseline(workload, weights_path, budget_s=15.0):
    """The reference's algorithm on the host cores, on a bounded sample of the workload's rows and
    steps (``value``), plus the same model decoded the way a KV-cached CPU engine would
    (``cached``)."""
    from oracle import oracle as orc

    engine = oracle_engine(workload, weights_path)
    m = workload.model
    rows = min(4, workload.rows)
    _, one = cpu_sample(engine, workload, rows, 1)
    steps = int(max(1, min(workload.steps, budget_s / max(one, 1e-3))))
    value, elapsed = cpu_sample(engine, workload, rows, steps)
    line = {"value": value, "unit": "tokens/s", "cores": orc.threads(), "kind": "port",
            "sample": f"{rows} rows x {steps} greedy steps of {workload.name}, full-window "
                      f"recompute per step ({elapsed:.1f} s)"}
    # One row per host thread over a per-row KV cache; decode rate from two runs that differ only
    # in the number of steps, so the token-by-token prefill cancels.
    crows = max(1, min(orc.threads(), workload.rows))
    cctx = orc.left_pad(orc.synthetic_prompts(workload.prompt_seed, crows, workload.prompt,
                                              m.vocabulary), m.window, m.vocabulary)
    t0 = time.perf_counter()
    engine.generate_batch_cached(cctx, 1)
    base = time.perf_counter() - t0
    extra = int(max(1, min(workload.steps - 1, 64)))
    t0 = time.perf_counter()
    engine.generate_batch_cached(cctx, 1 + extra)
    longer = time.perf_counter() - t0
    line["cached"] = {"value": crows * extra / max(1e-9, longer - base), "unit": "tokens/s",
                      "sample": f"{crows} rows x {extra} greedy steps over a per-row KV cache "
                                f"({base:.1f} s and {longer:.1f} s runs)"}
    return line


def run_reference(args, rank, world):
    """The reference arm: the reference's CPU algorithm (the oracle) on this box's host cores, on
    the GPU arm's workload, metric and config. Each step is one measured sample of 4 rows decoded
    for a few full-window-recompute steps; nothing is extrapolated. Rank 0 alone runs."""
    if rank != 0:
        return
    from oracle import oracle as orc

    workload = workload_of(args)
    m = workload.model
    with tempfile.TemporaryDirectory() as tmp:
        path = Path(tmp) / "w.bin"
        orc.write_synthetic_weights(m, path, workload.weight_seed)
        engine = oracle_engine(workload, path)
    rows = min(4, workload.rows)
    _, one = cpu_sample(engine, workload, rows, 1)
    # Steps per sample so that warm-up plus timed samples take about 90 s of host time.
    per_sample_s = 90.0 / max(1, args.steps + args.warmup)
    steps = int(max(1, min(workload.steps, per_sample_s / max(one, 1e-3))))
    values, seconds = [], []
    for i in range(args.warmup + args.steps):
        value, elapsed = cpu_sample(engine, workload, rows, steps)
        if i >= args.warmup:
            values.append(value)
            seconds.append(elapsed)
    value = float(np.median(values))
    sample = (f"{rows} rows x {steps} greedy steps of {workload.name} per step, full-window "
              f"recompute per decoded token (TextEngine.generateBatch), median of {args.steps} "
              f"samples")
    line = {
        "impl": "reference", "metric": "decode tokens/s", "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * float(np.mean(seconds)),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: N(0,0.02) weights from java.util.Random(0), prompts from "
                f"java.util.Random({workload.prompt_seed}).nextInt({m.vocabulary})",
        "config": config_line(workload, workload.rows, world),
        "extrapolated": False,
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": orc.threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------
# GPU side.
# ---------------------------------------------------------------------------------------------
_WEIGHTS = {}


def weights_file(model, seed, tmpdir):
    """One synthetic weight file per (architecture, dtype, seed) for the whole run."""
    from basalt_b200 import write_synthetic_weights

    key = (model.family, model.vocabulary, model.window, model.dimension, model.layers,
           model.heads, model.hidden, model.weight_dtype, seed)
    if key not in _WEIGHTS:
        path = Path(tmpdir) / f"w{len(_WEIGHTS)}.bin"
        write_synthetic_weights(model, path, seed)
        _WEIGHTS[key] = path
    return _WEIGHTS[key]


def open_engine(local, model, seed, tmpdir):
    from basalt_b200 import Basalt, TextEngine

    engine = TextEngine.of(Basalt.create(local), model, model.vocabulary, model.window)
    engine.load(weights_file(model, seed, tmpdir))
    return engine


def event_time(stream, fn, reps):
    """Median of `reps` separately timed calls of fn (CUDA events on the engine's stream)."""
    import torch

    times = []
    for _ in range(max(1, reps)):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        b.synchronize()
        times.append(a.elapsed_time(b))
    return float(np.median(times))


def prefill_roofline(m, rows, prompt, prefill_ms):
    """The prefill call (one decoded token) against the tensor peak: the projections' useful flops
    (2 M N K over every layer, plus the head on each row's last position); fp32 weights run as
    3xTF32 (three tf32 passes at half the bf16 rate), bf16 weights as two bf16 passes."""
    _, bf16_peak, peak_src = measured_peaks()
    tokens = rows * prompt
    d, F = m.dimension, m.hidden
    flops = 2.0 * tokens * m.layers * (4 * d * d + 2 * d * F) + 2.0 * rows * d * m.vocabulary
    passes, rate = (2, 1.0) if m.weight_dtype == "bf16" else (3, 0.5)
    achieved = flops / (prefill_ms / 1000.0) / 1e12
    return {"bound": "tensor", "achieved": achieved, "peak": bf16_peak, "unit": "TFLOP/s",
            "frac": achieved / bf16_peak, "tensor_passes": passes,
            "useful_flops_peak": bf16_peak * rate / passes,
            "useful_frac": achieved / (bf16_peak * rate / passes), "tokens": tokens,
            "note": "whole prefill call (projections, attention, LayerNorms) against the "
                    "projections' flops", "peak_source": peak_src}


def batch1(local, steps, warmup, tmpdir):
    """Single-stream latency: batch 1, 512-token prompt, 512 greedy tokens (bf16 weights)."""
    import torch

    from basalt_b200 import config, left_pad, synthetic_prompts

    w = config(BATCH1_WORKLOAD)
    m = w.model
    engine = open_engine(local, m, w.weight_seed, tmpdir)
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
    # The per-token figure is a difference of two call times: medians of separate calls.
    full_ms = event_time(stream, lambda: call(w.steps, d_tok), max(3, steps))
    prefill_ms = event_time(stream, lambda: call(1, d_one), max(3, steps))
    per_token_ms = (full_ms - prefill_ms) / (w.steps - 1)
    hbm, _, src = measured_peaks()
    # Algorithmic bytes of one decode step: every weight once, the cache each row reads (mean
    # length over the call) and the logits row.
    wb = 2 if m.weight_dtype == "bf16" else 4
    kvb = 2 if m.kv_dtype == "bf16" else 4
    params = m.layers * (4 * m.dimension ** 2 + 2 * m.dimension * m.hidden) + \
        m.vocabulary * m.dimension
    mean_len = w.prompt + (w.steps + 1) / 2.0
    step_bytes = params * wb + m.layers * 2 * m.dimension * kvb * mean_len + m.vocabulary * 4
    achieved = step_bytes / (per_token_ms / 1000.0) / 1e9
    # The same decode on the kernel-per-operation path (the fused step switched off).
    os.environ["BST_FUSED_DECODE"] = "0"
    try:
        call(w.steps, d_tok)
        unfused_ms = event_time(stream, lambda: call(w.steps, d_tok), max(1, steps // 2))
    finally:
        del os.environ["BST_FUSED_DECODE"]
    engine.close()
    return {"workload": w.name, "tokens_per_s": w.steps / (full_ms / 1000.0),
            "ms_per_call": full_ms, "prefill_ms": prefill_ms,
            "decode_ms_per_token": per_token_ms,
            "decode_step": {"kernel": "k_decode_step (one cooperative launch per token)",
                            "bytes_per_step": step_bytes, "achieved": achieved,
                            "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                            "peak_source": src},
            "per_operation_path": {"decode_ms_per_token": (unfused_ms - prefill_ms) /
                                   (w.steps - 1)}}


def other_configs(local, tmpdir, reps=3):
    """The other workloads of the scope table, timed on the device: C1 and C2 as per-call latency
    (L2-resident models), C3 with bf16 weights as decode tokens/s."""
    import torch

    from basalt_b200 import config, left_pad, synthetic_prompts

    out = {}
    for name in ("v96-d128-l2-w64-b1-greedy", "v96-d256-l4-w128-b32-greedy",
                 "v96-d256-l4-w128-b32-sampled", "v4096-d512-l6-w512-b256-greedy-bf16w"):
        w = config(name)
        m = w.model
        engine = open_engine(local, m, w.weight_seed, tmpdir)
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

        call(w.steps, d_tok)
        call(1, d_one)
        torch.cuda.synchronize()
        full_ms = event_time(stream, lambda: call(w.steps, d_tok), reps)
        first_ms = event_time(stream, lambda: call(1, d_one), reps)
        decode_ms = (full_ms - first_ms) / max(1, w.steps - 1)
        out[name] = {"rows": w.rows, "new_tokens": w.steps, "ms_per_call": full_ms,
                     "prefill_ms": first_ms, "decode_ms_per_step": decode_ms,
                     "tokens_per_s": w.rows * w.steps / (full_ms / 1000.0),
                     "decode_tokens_per_s": w.rows / (decode_ms / 1000.0) if decode_ms > 0 else None}
        if w.rows * w.prompt >= 4096:
            out[name]["roofline_prefill"] = prefill_roofline(m, w.rows, w.prompt, first_ms)
        engine.close()
    return out


def scaling_workload(local, rank, world, barrier, max_over_ranks, tmpdir):
    """The 8192-sequence streamSampled workload (T = 1.0, seed 9, 128-token prompts, 512 tokens,
    bf16 weights) split into contiguous row blocks over the ranks (strong scaling). Each rank's
    generator starts where one engine seeded once would be at its first row, so the ranks together
    draw exactly the unsharded run's tokens. One timed call per rank after a short warm-up call."""
    import torch

    from basalt_b200 import config, left_pad, synthetic_prompts
    from basalt_b200.sharding import shard_rng_state, shard_rows

    w = config(SCALING_WORKLOAD)
    m = w.model
    first, R = shard_rows(w.rows, world, rank)
    engine = open_engine(local, m, w.weight_seed, tmpdir)
    prompts = synthetic_prompts(w.prompt_seed, w.rows, w.prompt, m.vocabulary)
    ctx = left_pad(prompts[first:first + R], m.window, m.vocabulary)
    stream = torch.cuda.ExternalStream(engine.cuda_stream(), device=torch.device("cuda", local))
    d_ctx = torch.from_numpy(ctx).to(f"cuda:{local}")
    d_tok = torch.empty((R, w.steps), dtype=torch.int32, device=f"cuda:{local}")

    def call(steps):
        engine.rng_state = shard_rng_state(w.sample_seed, steps, first)
        engine.sample_device(d_ctx.data_ptr(), R, ctx.shape[1], steps, w.temperature, w.k,
                             d_tok.data_ptr())

    call(8)
    torch.cuda.synchronize()
    barrier()
    ms = event_time(stream, lambda: call(w.steps), 1)
    barrier()
    per_rank = max_over_ranks(ms, gather=True)
    engine.close()
    slowest = max(per_rank)
    return {"workload": w.name, "sequences": w.rows, "rows_per_rank": R, "new_tokens": w.steps,
            "scaling": "strong", "n_gpus": world, "ms": slowest,
            "tokens_per_s": w.rows * w.steps / (slowest / 1000.0),
            "per_rank_ms": per_rank, "spread": slowest / min(per_rank)}


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch

    from basalt_b200 import _lib, left_pad, synthetic_prompts

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()

    def max_over_ranks(value, gather=False):
        if not dist:
            return [value] if gather else value
        if gather:
            out = [None] * world
            dist.all_gather_object(out, value)
            return out
        t = torch.tensor([value], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    tmp = tempfile.TemporaryDirectory()
    workload = workload_of(args)
    m = workload.model
    engine = open_engine(local, m, workload.weight_seed, tmp.name)

    # This rank's contiguous shard of one seeded draw of rows x world prompts (weak scaling:
    # `rows` per GPU).
    from basalt_b200.sharding import shard_rows

    first, R = shard_rows(workload.rows * world, world, rank)
    prompts = synthetic_prompts(workload.prompt_seed, workload.rows * world, workload.prompt,
                                m.vocabulary)
    ctx = left_pad(prompts[first:first + R], m.window, m.vocabulary)
    steps = workload.steps

    stream = torch.cuda.ExternalStream(engine.cuda_stream(), device=torch.device("cuda", local))
    d_ctx = torch.from_numpy(ctx).to(f"cuda:{local}")
    d_tok = torch.empty((R, steps), dtype=torch.int32, device=f"cuda:{local}")
    torch.cuda.synchronize()

    def device_step():
        engine.generate_device(d_ctx.data_ptr(), R, ctx.shape[1], steps, d_tok.data_ptr())

    for _ in range(args.warmup):
        device_step()
    barrier()

    launches0 = engine.stats()["launches"]
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            device_step()
        stop.record(stream)
        stop.synchronize()
    barrier()
    launches = engine.stats()["launches"] - launches0
    ms = max_over_ranks(start.elapsed_time(stop))
    tokens_per_step = R * steps * world
    value = tokens_per_step * args.steps / (ms / 1000.0)

    # End to end through the C ABI with host buffers: pinned contexts in, tokens out, every step.
    h_ctx = torch.from_numpy(ctx).pin_memory()
    h_tok = torch.empty((R, steps), dtype=torch.int32).pin_memory()
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
    e2e_ms = max_over_ranks(e2e_start.elapsed_time(e2e_stop))
    e2e_value = tokens_per_step * args.steps / (e2e_ms / 1000.0)

    # Prefill alone (one decoded token) against the whole call: the decode steps' share.
    d_one = torch.empty((R, 1), dtype=torch.int32, device=f"cuda:{local}")
    engine.generate_device(d_ctx.data_ptr(), R, ctx.shape[1], 1, d_one.data_ptr())
    torch.cuda.synchronize()
    prefill_ms = event_time(
        stream, lambda: engine.generate_device(d_ctx.data_ptr(), R, ctx.shape[1], 1,
                                               d_one.data_ptr()), 3)
    step_ms = ms / args.steps
    decode_ms = (step_ms - prefill_ms) / max(1, steps - 1)
    decode_tps = R / max(1e-12, decode_ms / 1000.0)

    # Roofline of the decode step, timed by CUDA events on the engine's stream over the timed
    # calls: one step is one CUDA graph (every layer's projections, attention, fix-ups and the
    # selection) replayed per token. Algorithmic bytes: every weight once plus the K/V each row
    # reads at the call's mean cache length.
    hbm_peak, bf16_peak, peak_src = measured_peaks()
    kvb = 2 if m.kv_dtype == "bf16" else 4
    wbytes = 2 if m.weight_dtype == "bf16" else 4
    params = m.layers * (4 * m.dimension ** 2 + 2 * m.dimension * m.hidden) + \
        m.vocabulary * m.dimension
    mean_len = min(m.window, workload.prompt + (steps + 1) / 2.0)
    kv_bytes = R * m.layers * 2 * m.dimension * kvb * mean_len
    step_bytes = kv_bytes + params * wbytes
    achieved = step_bytes / max(1e-12, decode_ms / 1000.0) / 1e9
    traffic = NCU_STEP_TRAFFIC.get(workload.name)
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                "frac": achieved / hbm_peak,
                "traffic": (traffic["fixed"] + traffic["per_row_key"] * R * mean_len)
                if traffic and R == 256 else None,
                "kernel": "decode step (CUDA graph of the step's kernels)",
                "algorithmic_bytes": step_bytes, "ms": decode_ms, "peak_source": peak_src}
    prefill_roof = prefill_roofline(m, R, workload.prompt, prefill_ms)

    line = {
        "metric": "decode tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16" if m.weight_dtype == "bf16" else "f32",
        "data": "synthetic: N(0,0.02) weights from java.util.Random(0), prompts from "
                f"java.util.Random({workload.prompt_seed}).nextInt({m.vocabulary})",
        "config": config_line(workload, R, world),
        "prefill_ms": prefill_ms, "decode_tokens_per_s": decode_tps * world,
        "e2e": {"value": e2e_value, "unit": "tokens/s",
                "h2d_bytes_per_step": int(ctx.nbytes), "d2h_bytes_per_step": int(R * steps * 4)},
        "gpu_launches": int(launches),
        "roofline": roofline,
        "roofline_prefill": prefill_roof,
        "clocks": clocks.summary(),
    }
    engine.close()
    if not args.no_scaling:
        line["c5"] = scaling_workload(local, rank, world, barrier, max_over_ranks, tmp.name)
    if rank == 0 and world == 1 and not args.no_batch1:
        line["batch1"] = batch1(local, max(1, args.steps), max(1, args.warmup), tmp.name)
        line["configs"] = other_configs(local, tmp.name)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(workload, weights_file(m, workload.weight_seed,
                                                                   tmp.name))
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
