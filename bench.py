#!/usr/bin/env python3
"""Benchmark of the B200 absorbed-MLA decode-attention path (one JSON line on rank 0).

A step is one attention task (K1 prologue + K2 split-KV attention + K3 merge/W_UV)
over one batch, with the latent cache resident in HBM. Metric: KV GB/s, the latent
cache bytes a step must read (sum_b (T_b + 1) * 1152) over its device time; the line
also gives µs per layer-step and the HBM roofline fraction of the attention kernel.

    python bench.py [--workload config5a] [--steps K] [--warmup W]
    torchrun --nproc-per-node N bench.py --gpus N ...     # by-request shards, weak scaling
    python bench.py --impl reference ...                  # the CPU oracle on the host cores
"""
from __future__ import annotations

import argparse
import ctypes
import importlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

fleet = importlib.import_module("fleet-mi300x_b200")
workloads = importlib.import_module("fleet-mi300x_b200.workloads")
native = importlib.import_module("fleet-mi300x_b200.native")

METRIC = "MLA decode attn KV GB/s"
FALLBACK_HBM_GBS = 6650.0


def measured_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback 6.65 TB/s"


def ncu_traffic(workload: str) -> float | None:
    """Per-launch DRAM bytes of the attention kernel from the committed ncu summary."""
    p = ROOT / "profiles" / f"attention_{workload}_ncu.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1].strip())
    return None


# ---------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.3)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------- set-up
def build_workload(name: str, dev: torch.device, rank: int):
    wl = workloads.WORKLOADS[name]
    lengths = wl.seq_lens()
    cfg = fleet.ModelConfig()
    lw = workloads.make_layer_weights(wl.seed)
    w = fleet.LayerWeights(*(t.to(dev) for t in (lw.q_proj, lw.kv_a_proj_with_mqa, lw.kv_a_layernorm,
                                                   lw.kv_b_proj, lw.o_proj)))
    cos, sin = fleet.device_rope_tables(cfg, max(lengths) + 8, dev)
    cache = fleet.PagedLatentCache.for_lengths(lengths, permute=wl.permute, zero=False,
                                               generator=torch.Generator().manual_seed(wl.seed + rank), device=dev)
    workloads.fill_pool_random(cache.pages, wl.seed + 1000 * rank)
    x_n = workloads.make_hidden(wl.seed + 1, len(lengths)).to(dev)
    runner = fleet.MlaDecodeAttention(cfg, w, cos, sin)
    q, kv_a = runner.project(x_n)
    q, kv_a = q.contiguous(), kv_a.contiguous()
    return wl, lengths, runner, cache, x_n, q, kv_a


def time_loop(fn, steps: int, stream: torch.cuda.Stream) -> float:
    """Device ms per call, CUDA events on the launching stream."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) / steps


L2_BYTES = 126e6


class StepTimer:
    """CUDA-event timing of repeated calls on the launching stream. When a step reads
    less than 4x L2 of cache rows, 256 MB are written between timed calls (outside the
    timed events, one event pair per call) so that no call finds the previous one's
    rows in L2; a ~50 us spin follows the flush, so that the call's launches are queued
    before its start event fires and the events hold device time only."""

    def __init__(self, stream: torch.cuda.Stream, kv_bytes: int, device):
        self.stream = stream
        self.flush = (torch.empty(256 << 20, dtype=torch.uint8, device=device)
                      if kv_bytes < 4 * L2_BYTES else None)
        self.kv_bytes = kv_bytes

    def __call__(self, fn, steps: int) -> float:
        if self.flush is None:
            return time_loop(fn, steps, self.stream)
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        torch.cuda.synchronize()
        for a, b in evs:
            self.flush.zero_()
            torch.cuda._sleep(100_000)
            a.record(self.stream)
            fn()
            b.record(self.stream)
        evs[-1][1].synchronize()
        return sum(a.elapsed_time(b) for a, b in evs) / steps

    def describe(self) -> str:
        if self.flush is None:
            return "no flush: each step reads %.0f MB of cache rows, > 4x the 126 MB L2" % (self.kv_bytes / 1e6)
        return ("L2 flushed: 256 MB written before every timed step, outside its CUDA events "
                "(the step reads %.1f MB of cache rows)" % (self.kv_bytes / 1e6))


def cpu_oracle_sample(name: str, budget_s: float, faithful: bool) -> dict:
    """Times the CPU oracle on a bounded sample of the workload's requests."""
    from oracle import mla_oracle as O
    wl = workloads.WORKLOADS[name]
    lengths = wl.seq_lens()
    cfg = O.Config()
    lw = workloads.make_layer_weights(wl.seed)
    f = lambda t: t.float().numpy()
    w = O.Weights(f(lw.q_proj), f(lw.kv_a_proj_with_mqa), f(lw.kv_a_layernorm), f(lw.kv_b_proj))
    x_n = workloads.make_hidden(wl.seed + 1, min(len(lengths), 64)).float().numpy()
    rng = np.random.default_rng(wl.seed)
    attend = O.attend_rows if faithful else O.attend_rows_fast
    cos, sin = cfg.cos_sin(max(lengths) + 8)
    done_bytes, done_req, t_total = 0, 0, 0.0
    i = 0
    while t_total < budget_s and done_req < 64 * len(lengths):
        b = i % len(lengths)
        T = lengths[b]
        rows = O.bf16_round(rng.standard_normal((T, 576), dtype=np.float32))
        q, kv_a = O.project(cfg, w, x_n[b % len(x_n)])
        t0 = time.perf_counter()
        row = O.kv_post(cfg, w, kv_a, T, cos, sin)
        allr = np.concatenate([rows, row[None]], 0)
        attend(cfg, w, q, allr, T, cos, sin)
        t_total += time.perf_counter() - t0
        done_bytes += (T + 1) * 1152
        done_req += 1
        i += 1
    try:
        from threadpoolctl import threadpool_info
        cores = max([x.get("num_threads", 1) for x in threadpool_info()] or [1])
    except Exception:
        cores = os.cpu_count() or 1
    return {"value": done_bytes / t_total / 1e9, "unit": "GB/s", "cores": int(cores), "kind": "port",
            "sample": f"{done_req} requests of {name} ({done_bytes / 1e6:.1f} MB of cache rows), "
                      f"{'per-head loop (reference_decode.py:245-254)' if faithful else 'all-heads vectorised'} "
                      f"NumPy/BLAS, {t_total:.2f} s",
            "seconds": t_total}


# ---------------------------------------------------------------------------- arms
def run_reference_arm(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    steps_out = []
    per_step_budget = max(0.5, min(6.0, 120.0 / max(1, args.steps + args.warmup)))
    for _ in range(args.warmup):
        cpu_oracle_sample(args.workload, per_step_budget / 4, faithful=True)
    info = None
    for _ in range(args.steps):
        info = cpu_oracle_sample(args.workload, per_step_budget, faithful=True)
        steps_out.append(info)
    total_s = sum(s["seconds"] for s in steps_out)
    total_b = sum(s["value"] * s["seconds"] * 1e9 for s in steps_out)
    value = total_b / total_s / 1e9
    wl = workloads.WORKLOADS[args.workload]
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total_s / max(1, args.steps),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded)",
        "config": {"workload": args.workload, "batch_per_gpu": wl.batch, "parallelism": "cpu-host"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": info["cores"], "kind": "port",
                         "sample": info["sample"] + " per step"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_gpu_arm(args, rank: int, world: int, local_rank: int) -> None:
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
    dist = None
    if world > 1:
        import torch.distributed as dist
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    if args.workload == "config5b" and world > 1:
        run_sequence_sharded(args, rank, world, local_rank, dev, dist)
        return

    wl, lengths, runner, cache, x_n, q, kv_a = build_workload(args.workload, dev, rank)
    B = len(lengths)
    out = torch.empty(B, 2048, dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev)
    step = lambda: runner.attend(q, kv_a, cache, out)
    if args.sweep_splits:
        run_split_sweep(args, runner, cache, q, kv_a, lengths, stream)
        return

    # warm-up (also JIT-free: the library is prebuilt)
    for _ in range(max(3, args.warmup)):
        step()
    runner.check_errors()
    kv_b = workloads.kv_bytes(lengths)
    timer = StepTimer(stream, kv_b, dev)

    # The product's step for a decode loop: K1-K3 captured once as a CUDA graph
    # (DecodeGraph, PDL edges between the kernels) and replayed; it must reproduce
    # the eager step bit for bit before it is timed.
    out_g = torch.empty_like(out)
    graph = fleet.DecodeGraph(runner, cache, inputs="qkv", q=q, kv_a=kv_a, out=out_g)
    for _ in range(max(3, args.warmup)):
        graph.replay()
    step()
    torch.cuda.synchronize()
    if not torch.equal(out_g, out):
        raise RuntimeError("graph step output differs from the eager step")
    runner.check_errors()

    # ---- timed region: K steps of the whole task, inputs resident
    clocks = ClockSampler(local_rank)
    with clocks:
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        ms = timer(graph.replay, args.steps)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        ms_eager = timer(step, args.steps)
    ms_max = ms
    if dist:
        t = torch.tensor([ms, ms_eager], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max, ms_eager = float(t[0].item()), float(t[1].item())
    runner.check_errors()

    tot_b = workloads.total_bytes(lengths)
    value = world * kv_b / (ms_max * 1e-3) / 1e9

    # ---- stage timings: the attention kernel alone (roofline) and the other two
    p = runner.params(q, kv_a, cache, out)
    sptr = ctypes.c_void_p(stream.cuda_stream)
    lib = runner.lib
    native.check(lib.mla_prologue(ctypes.byref(p), sptr), "prologue")
    k1_ms = timer(lambda: lib.mla_prologue(ctypes.byref(p), sptr), max(5, args.steps))
    k2_ms = timer(lambda: lib.mla_attention(ctypes.byref(p), sptr), max(5, args.steps))
    k3_ms = timer(lambda: lib.mla_merge_uv(ctypes.byref(p), sptr), max(5, args.steps))
    peak, peak_src = measured_peak()
    k2_gbs = kv_b / (k2_ms * 1e-3) / 1e9
    traffic = ncu_traffic(args.workload)

    # ---- the q | kv_a projection (K0, the step before the task) and o_proj + residual
    # (K5, the step after), decode batches only; both weights fit in L2, so L2 is flushed
    # before every timed call
    projection = None
    if B <= native.MAX_PROJECT_BATCH:
        ptimer = StepTimer(stream, 0, dev)
        runner.attend_x(x_n, cache, out, stage="project")
        k0_ms = ptimer(lambda: runner.attend_x(x_n, cache, out, stage="project"), max(5, args.steps))
        w_bytes = runner.w_qkv.numel() * 2
        projection = {"kernel": "k0_project", "weight_bytes": w_bytes, "k0_us": round(k0_ms * 1e3, 2),
                      "k0_gbs": round(w_bytes / (k0_ms * 1e-3) / 1e9, 1),
                      "k0_frac_of_peak": round(w_bytes / (k0_ms * 1e-3) / 1e9 / peak, 4),
                      "l2": "flushed: 256 MB written before every timed call, outside its CUDA events"}
        h = torch.randn(B, 2048, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).to(dev)
        h2 = torch.empty_like(h)
        po = runner.params(None, None, cache, out, x_n=x_n, residual=h, h_out=h2)
        native.check(lib.mla_o_proj(ctypes.byref(po), sptr), "o_proj")
        k5_ms = ptimer(lambda: lib.mla_o_proj(ctypes.byref(po), sptr), max(5, args.steps))
        wo_bytes = runner.w_o.numel() * 2
        projection["o_proj"] = {"kernel": "k_weight_stream<16, residual>", "weight_bytes": wo_bytes,
                                "k5_us": round(k5_ms * 1e3, 2),
                                "k5_gbs": round(wo_bytes / (k5_ms * 1e-3) / 1e9, 1),
                                "k5_frac_of_peak": round(wo_bytes / (k5_ms * 1e-3) / 1e9 / peak, 4)}

    # ---- e2e through the public API: pinned host x_n -> device, the task, R(out) -> host,
    # every step. HostPipeline (graph.py) replays the step as a CUDA graph and overlaps the
    # copies of neighbouring steps with its compute. Workloads that fit in 4x L2 are timed
    # one step at a time after an L2 flush instead (latency from the input copy to the
    # output copy), since a pipeline would re-read the cache from L2.
    x_host = x_n.cpu().pin_memory()
    pipe = fleet.HostPipeline(runner, cache)
    first = pipe.submit(x_host)
    pipe.wait()
    want = runner(x_n, cache).float().cpu()
    if (first.float() - want).abs().max() > 1e-2 * want.abs().max():
        raise RuntimeError("pipelined step output differs from the eager call")
    for _ in range(3):
        pipe.submit(x_host)
    pipe.wait()
    if dist:
        dist.barrier()
    if timer.flush is None:
        e2e_mode = "pipelined: input copy of step k+1 and output copy of step k-1 overlap step k's compute"
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record(pipe.compute)
        pipe.h2d.wait_event(start)
        for _ in range(args.steps):
            pipe.submit(x_host)
        end.record(pipe.d2h)
        pipe.wait()
        e2e_ms = start.elapsed_time(end) / args.steps
    else:
        # latency-bound configs: one graph per step holding the input copy, the step and
        # the output copy on one stream (HostStepGraph), checked against the eager call
        e2e_mode = ("per-step latency: one CUDA graph of input copy (pinned host -> device), step, output "
                    "copy (device -> pinned host); L2 flushed before every step")
        hsg = fleet.HostStepGraph(runner, cache)
        hsg.x_host.copy_(x_host)
        hsg.replay()
        torch.cuda.synchronize()
        if (hsg.out_host.float() - want).abs().max() > 1e-2 * want.abs().max():
            raise RuntimeError("host-step graph output differs from the eager call")
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        torch.cuda.synchronize()
        for a, b in evs:
            timer.flush.zero_()
            torch.cuda._sleep(100_000)
            a.record(stream)
            hsg.replay()
            b.record(stream)
        torch.cuda.synchronize()
        e2e_ms = sum(a.elapsed_time(b) for a, b in evs) / args.steps
    if dist:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * kv_b / (e2e_ms * 1e-3) / 1e9

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_oracle_sample(args.workload, args.cpu_seconds, faithful=False)
        cpu.pop("seconds", None)

    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    us = ms_max * 1e3
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) latents, N(0,0.02) weights)",
        "config": {"workload": args.workload, "batch_per_gpu": B, "context": (lengths[0] if len(set(lengths)) == 1
                                                                            else [min(lengths), max(lengths)]),
                   "page_size": 64, "block_table": "permuted" if wl.permute else "contiguous",
                   "parallelism": f"by-request x{world}" if world > 1 else "single GPU",
                   "kv_bytes_per_gpu_step": kv_b, "l2": timer.describe(),
                   "step": "K1-K3 replayed as one CUDA graph (DecodeGraph); eager_ms_per_step is the same "
                           "step launched through the C ABI call by call"},
        "us_per_layer_step": round(us, 3),
        "eager_ms_per_step": round(ms_eager, 5),
        "kv_frac_of_hbm_peak": round(value / world / peak, 4),
        "attn_tokens_per_s_27_layers": round(world * B / (27 * us * 1e-6), 1),
        "stages_us": {"prologue": round(k1_ms * 1e3, 2), "attention": round(k2_ms * 1e3, 2),
                      "merge_uv": round(k3_ms * 1e3, 2)},
        "roofline": {"bound": "hbm", "kernel": "k2_attention_mma", "achieved": round(k2_gbs, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(k2_gbs / peak, 4), "traffic": traffic,
                     "algorithmic_bytes_per_launch": kv_b, "peak_source": peak_src},
        "cpu_baseline": cpu,
        "projection": projection,
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "ms_per_step": round(e2e_ms, 5),
                "h2d_bytes_per_step": int(x_n.numel() * 2), "d2h_bytes_per_step": int(out.numel() * 2),
                "path": ("HostPipeline (double-buffered graphs, copies on their own streams)" if timer.flush is None
                         else "HostStepGraph (one graph: copy in, step, copy out)") +
                        ": pinned x_n H2D, the step (q|kv_a projection: K0 for <= 64 requests, else cuBLAS; "
                        "K1-K3), R(out) D2H", "mode": e2e_mode},
        "gpu_launches": native.load_library().mla_launches_per_step() * args.steps,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def run_sequence_sharded(args, rank: int, world: int, local_rank: int, dev: torch.device, dist) -> None:
    """Config 5b across `world` GPUs: one 131,072-token sequence split by page-aligned KV
    ranges; per step K1+K2+K3 on each range and the fixed-order combine of the 8.4 KB
    partials (distributed.py). --exchange peer (default): K3 stores the partials into
    every rank's exchange buffer over NVLink and K4 combines, one library call per
    step; --exchange nccl: an NCCL all-gather and mla_combine_shards. Total work is
    fixed: strong scaling."""
    dmod = importlib.import_module("fleet-mi300x_b200.distributed")
    wl = workloads.WORKLOADS["config5b"]
    T = wl.seq_lens()[0]
    cfg = fleet.ModelConfig()
    lw = workloads.make_layer_weights(wl.seed)
    w = fleet.LayerWeights(*(t.to(dev) for t in (lw.q_proj, lw.kv_a_proj_with_mqa, lw.kv_a_layernorm,
                                                   lw.kv_b_proj)))
    cos, sin = fleet.device_rope_tables(cfg, T + 8, dev)
    a, b = dmod.sequence_shards(T, world)[rank]
    last = rank == world - 1
    cache = fleet.PagedLatentCache.for_lengths([b - a], extra_tokens=1 if last else 0, permute=True, zero=False,
                                               generator=torch.Generator().manual_seed(wl.seed + rank), device=dev)
    workloads.fill_pool_random(cache.pages, wl.seed + 1000 * rank)
    runner = fleet.MlaDecodeAttention(cfg, w, cos, sin)
    x_n = workloads.make_hidden(wl.seed + 1, 1).to(dev)
    q, kv_a = (t.contiguous() for t in runner.project(x_n))
    pos = torch.tensor([T], dtype=torch.int32, device=dev)
    local = torch.empty(1, 16, native.SHARD_STRIDE, dtype=torch.float32, device=dev)
    parts = torch.empty(world, 1, 16, native.SHARD_STRIDE, dtype=torch.float32, device=dev)
    out = torch.empty(1, 2048, dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev)
    ex = dmod.ExchangeBuffers.create(rank, world, max_batch=1) if args.exchange == "peer" else None

    def step():
        if ex is not None:
            runner.attend(q, kv_a, cache, out, rope_pos=pos, new_row=last, exchange=ex)
            return
        runner.attend(q, kv_a, cache, rope_pos=pos, shard_out=local, new_row=last)
        dist.all_gather_into_tensor(parts, local)
        fleet.combine_shards(parts, out)

    for _ in range(max(3, args.warmup)):
        step()
    runner.check_errors()
    kv_b = workloads.kv_bytes([T])
    timer = StepTimer(stream, kv_b // world, dev)
    clocks = ClockSampler(local_rank)
    with clocks:
        dist.barrier()
        torch.cuda.synchronize()
        ms = timer(step, args.steps)
        torch.cuda.synchronize()
        dist.barrier()
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    runner.check_errors()

    # ---- stage timings (each stage repeated alone on every rank at once; max over
    # ranks). A K3 repeated without its K4 rewrites the same slot and flags, which the
    # next whole step's K4 then reads, so the exchange protocol stays in step.
    def stage(name):
        if name == "combine" and ex is None:
            return lambda: fleet.combine_shards(parts, out)
        if name == "all_gather":
            return lambda: dist.all_gather_into_tensor(parts, local)
        if name == "k1_k2_k3":
            return lambda: [runner.attend(q, kv_a, cache, out if ex is not None else None, st, rope_pos=pos,
                                          shard_out=None if ex is not None else local, new_row=last, exchange=ex)
                            for st in ("prologue", "attention", "merge")]
        return lambda: runner.attend(q, kv_a, cache, out if ex is not None else None, name, rope_pos=pos,
                                     shard_out=None if ex is not None else local, new_row=last, exchange=ex)
    names = ["prologue", "attention", "merge", "k1_k2_k3"] + ([] if ex is not None else ["all_gather", "combine"])
    stage_ms = []
    for name in names:
        dist.barrier()
        torch.cuda.synchronize()
        stage_ms.append(timer(stage(name), max(5, args.steps // 2)))
    if ex is not None:  # the same step with the exchange as K3 + K4 instead of the fused K3
        names.append("step_k3_k4_split")
        runner.flags |= native.FLAG_EXCHANGE_SPLIT
        dist.barrier()
        torch.cuda.synchronize()
        stage_ms.append(timer(step, max(5, args.steps // 2)))
        runner.flags &= ~native.FLAG_EXCHANGE_SPLIT
    step()  # a whole step last: the peer protocol's step counter advances again
    torch.cuda.synchronize()
    runner.check_errors()
    t = torch.tensor(stage_ms, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    stages_us = {n: round(float(v) * 1e3, 2) for n, v in zip(names, t.tolist())}
    peak, _ = measured_peak()
    torch.cuda.synchronize()
    dist.barrier()
    if ex is not None:
        ex.close()
    dist.barrier()
    dist.destroy_process_group()
    if rank != 0:
        return
    value = kv_b / (ms_max * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max, 5), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) latents, N(0,0.02) weights)",
        "config": {"workload": "config5b", "batch": 1, "context": T, "page_size": 64,
                   "parallelism": (f"sequence-sharded x{world}: page-aligned KV ranges, " +
                                   (f"peer exchange of {16 * native.SHARD_STRIDE * 4} B partials per GPU (K3 stores "
                                    "into every rank's buffer over NVLink, K4 waits on flags and combines; no NCCL "
                                    "in the step)" if ex is not None else
                                    f"NCCL all-gather of {16 * native.SHARD_STRIDE * 4} B partials per GPU, "
                                    "fixed-order combine")),
                   "kv_bytes_per_step": kv_b, "kv_bytes_per_gpu": kv_b // world,
                   "l2": timer.describe()},
        "us_per_layer_step": round(ms_max * 1e3, 3),
        "kv_frac_of_hbm_peak_per_gpu": round(value / world / peak, 4),
        "gpu_launches": (native.load_library().mla_launches_per_step() + 1) * args.steps,
        "exchange": args.exchange,
        "stages_us": stages_us,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def run_split_sweep(args, runner, cache, q, kv_a, lengths, stream) -> None:
    """Split-count sweep (one GPU): the whole step, K2 alone and the LSE merge + W_UV (K3)
    alone at each CTA count of the split-KV plan. Every output is checked against the
    default plan's (one CTA per SM) before it is timed. Prints one JSON line."""
    kv_b = workloads.kv_bytes(lengths)
    B = len(lengths)
    lib = runner.lib
    sptr = ctypes.c_void_p(stream.cuda_stream)
    timer = StepTimer(stream, kv_b, q.device)
    runner.num_ctas = 0
    ref = runner.attend(q, kv_a, cache).float()
    rows = []
    for n in args.sweep_splits:
        runner.num_ctas = n
        out = torch.empty(B, 2048, dtype=torch.bfloat16, device=q.device)
        for _ in range(max(3, args.warmup)):
            runner.attend(q, kv_a, cache, out)
        runner.check_errors()
        rel = float(((out.float() - ref).abs().max() / ref.abs().max()).item())
        if rel > 1e-2:
            raise RuntimeError(f"split count {n}: output differs from the default plan's (max rel {rel:.3e})")
        step_ms = timer(lambda: runner.attend(q, kv_a, cache, out), args.steps)
        p = runner.params(q, kv_a, cache, out)
        k2_ms = timer(lambda: lib.mla_attention(ctypes.byref(p), sptr), args.steps)
        k3_ms = timer(lambda: lib.mla_merge_uv(ctypes.byref(p), sptr), args.steps)
        ctas, slots = ctypes.c_int32(), ctypes.c_int32()
        native.check(lib.mla_plan_info(ctypes.byref(p), ctypes.byref(ctas), ctypes.byref(slots)), "plan_info")
        # a request's tiles are cut at CTA boundaries: at most (ctas + B - 1) segments in all
        rows.append({"num_ctas": ctas.value, "partials_per_request_max_avg": round((ctas.value + B - 1) / B, 2),
                     "step_us": round(step_ms * 1e3, 2), "attention_us": round(k2_ms * 1e3, 2),
                     "merge_uv_us": round(k3_ms * 1e3, 2), "kv_gbs": round(kv_b / (step_ms * 1e-3) / 1e9, 1),
                     "max_rel_vs_default": rel})
    runner.num_ctas = 0
    print(json.dumps({"sweep": "split count", "workload": args.workload, "batch": B, "l2": timer.describe(),
                      "kv_bytes": kv_b, "rows": rows}), flush=True)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="config5a", choices=sorted(workloads.WORKLOADS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="CPU baseline sample: seconds of oracle work on the host cores (about 10-30 s)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="config5b on N > 1 GPUs: how the shard partials move (peer memory or NCCL)")
    ap.add_argument("--sweep-splits", type=lambda v: [int(x) for x in v.split(",")], default=None,
                    help="comma-separated CTA counts of the split plan, e.g. 1,2,4,8,16,32,64,148; "
                         "prints a sweep line instead of the bench line (one GPU)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
    else:
        run_gpu_arm(args, rank, world, local_rank)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
