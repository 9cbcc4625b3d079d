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


def host_threads() -> int:
    """Host threads this process may run on (its CPU affinity), whatever OMP_NUM_THREADS says."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def use_all_host_threads() -> int:
    """Give torch and NumPy's BLAS every host thread of this process. torchrun exports
    OMP_NUM_THREADS=1 to its ranks, which would leave the CPU legs on one core."""
    n = host_threads()
    torch.set_num_threads(n)
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(limits=n)
    except Exception:
        pass
    return n


class CpuSample:
    """The CPU oracle on a bounded sample of a workload's requests (the cpu_baseline leg
    and the reference arm). Inputs are prepared once, outside any timing: the layer's
    weights, q / kv_a of up to 64 requests and the cache rows of up to 4 distinct
    requests (seeded N(0, 1) bf16 latents, reused round-robin), so that the timed work is
    the task itself: the new row (kv_post) and the attention over the request's rows.
    `faithful` runs the per-head loop of reference_decode.py:245-254 (oracle.attend_rows),
    otherwise the all-heads vectorised form (oracle.attend_rows_fast)."""

    def __init__(self, name: str):
        from oracle import mla_oracle as O
        self.O = O
        self.name = name
        self.wl = workloads.WORKLOADS[name]
        self.lengths = self.wl.seq_lens()
        self.cfg = O.Config()
        lw = workloads.make_layer_weights(self.wl.seed)
        f = lambda t: t.float().numpy()
        self.w = O.Weights(f(lw.q_proj), f(lw.kv_a_proj_with_mqa), f(lw.kv_a_layernorm), f(lw.kv_b_proj))
        self.cos, self.sin = self.cfg.cos_sin(max(self.lengths) + 8)
        x_n = workloads.make_hidden(self.wl.seed + 1, min(len(self.lengths), 64)).float().numpy()
        self.qkv = [O.project(self.cfg, self.w, x) for x in x_n]
        rng = np.random.default_rng(self.wl.seed)
        self.rows = {}
        for b in range(min(len(self.lengths), 4)):
            T = self.lengths[b]
            if T not in self.rows:
                self.rows[T] = O.bf16_round(rng.standard_normal((T + 1, 576), dtype=np.float32))
        self.i = 0

    def run(self, budget_s: float, faithful: bool, max_requests: int | None = None) -> dict:
        O = self.O
        attend = O.attend_rows if faithful else O.attend_rows_fast
        done_bytes, done_req, t_total = 0, 0, 0.0
        limit = max_requests or 64 * len(self.lengths)
        while t_total < budget_s and done_req < limit:
            b = self.i % len(self.lengths)
            T = self.lengths[b]
            allr = self.rows.get(T)
            if allr is None:  # a ragged length without prepared rows: the nearest prepared one
                T = min(self.rows, key=lambda t: abs(t - T))
                allr = self.rows[T]
            q, kv_a = self.qkv[b % len(self.qkv)]
            t0 = time.perf_counter()
            allr[T] = O.kv_post(self.cfg, self.w, kv_a, T, self.cos, self.sin)
            attend(self.cfg, self.w, q, allr, T, self.cos, self.sin)
            t_total += time.perf_counter() - t0
            done_bytes += (T + 1) * 1152
            done_req += 1
            self.i += 1
        return {"value": done_bytes / t_total / 1e9, "unit": "GB/s", "cores": host_threads(), "kind": "port",
                "sample": f"{done_req} requests of {self.name} ({done_bytes / 1e6:.1f} MB of cache rows), "
                          f"{'per-head loop (reference_decode.py:245-254)' if faithful else 'all-heads vectorised'} "
                          f"NumPy/BLAS on {host_threads()} host threads, {t_total:.2f} s",
                "seconds": t_total, "bytes": done_bytes, "requests": done_req}


def check_sequence_sharded(inp: dict) -> dict:
    """The CPU leg's check of the sequence-sharded step: its combined R(out) against the
    oracle (all-heads form of reference_decode.py:239-254) over all rows of the sequence."""
    from oracle import mla_oracle as O
    wl = workloads.WORKLOADS["config5b"]
    lw = workloads.make_layer_weights(wl.seed)
    f = lambda t: t.float().numpy()
    w = O.Weights(f(lw.q_proj), f(lw.kv_a_proj_with_mqa), f(lw.kv_a_layernorm), f(lw.kv_b_proj))
    cfg = O.Config()
    T = inp["T"]
    cos, sin = cfg.cos_sin(T + 8)
    new_row = O.kv_post(cfg, w, inp["kv_a"][0], T, cos, sin)
    want = O.attend_rows_fast(cfg, w, inp["q"].reshape(16, 192), np.concatenate([inp["rows"], new_row[None]]), T,
                              cos, sin)
    got = inp["out"][0]
    rel = float(np.max(np.abs(got - want)) / np.max(np.abs(want)))
    cs = float(got @ want / (np.linalg.norm(got) * np.linalg.norm(want) + 1e-30))
    return {"oracle": f"oracle.attend_rows_fast over all {T + 1} rows", "max_rel_vs_oracle": rel, "cos": cs,
            "bar": 2e-2, "ok": bool(rel <= 2e-2)}


def cpu_oracle_sample(name: str, budget_s: float, faithful: bool) -> dict:
    """Times the CPU oracle on a bounded sample of the workload's requests (all host threads)."""
    use_all_host_threads()
    return CpuSample(name).run(budget_s, faithful)


# ---------------------------------------------------------------------------- arms
REFERENCE_TIMED_S = 100.0  # seconds of oracle work in the reference arm's timed steps, all of them together


def run_reference_arm(args, rank: int, world: int) -> None:
    """The reference's own algorithm for this path on the host cores: the oracle's
    per-head loop, which restates reference_decode.py:245-254 and is pinned to the
    reference's outputs (the reference itself is pure Python and cannot be installed
    or shipped here). Rank 0 only. Each step is a bounded sample of the same workload;
    the timed steps hold about REFERENCE_TIMED_S seconds of work together, so the arm
    ends within a few minutes whatever --steps is."""
    if rank != 0:
        return
    threads = use_all_host_threads()
    t_start = time.perf_counter()
    sample = CpuSample(args.workload)
    per_step = max(0.3, min(6.0, REFERENCE_TIMED_S / max(1, args.steps)))
    for _ in range(args.warmup):
        sample.run(min(0.5, per_step), faithful=True)
    steps_out = [sample.run(per_step, faithful=True) for _ in range(args.steps)]
    total_s = sum(s["seconds"] for s in steps_out)
    total_b = sum(s["bytes"] for s in steps_out)
    n_req = sum(s["requests"] for s in steps_out)
    value = total_b / total_s / 1e9
    wl = workloads.WORKLOADS[args.workload]
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total_s / max(1, args.steps),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded)",
        "config": {"workload": args.workload, "batch_per_gpu": wl.batch, "parallelism": "cpu-host"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{n_req} requests of {args.workload} over {args.steps} steps of about "
                                   f"{per_step:.1f} s each, per-head loop (reference_decode.py:245-254) "
                                   f"NumPy/BLAS on {threads} host threads; wall {time.perf_counter() - t_start:.0f} s"},
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
    # (K5, the step after): a weight stream up to 64 requests, a tcgen05 GEMM beyond;
    # cuBLAS on the same operands beside them. L2 flushed before every timed call.
    ptimer = StepTimer(stream, 0, dev)
    runner.attend_x(x_n, cache, out, stage="project")
    k0_ms = ptimer(lambda: runner.attend_x(x_n, cache, out, stage="project", check=False), max(5, args.steps))
    cublas_ms = ptimer(lambda: runner.project(x_n), max(5, args.steps))
    w_bytes = runner.w_qkv.numel() * 2
    gemm = B > native.MAX_PROJECT_BATCH
    flops = 2 * B * runner.w_qkv.shape[0] * runner.w_qkv.shape[1]
    bf16_peak = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()).get("bf16_tflops") \
        if (ROOT / "MEASURED_PEAKS.json").exists() else 1590.0
    projection = {"kernel": "k_project_tc (tcgen05 GEMM, 128 x 64 tiles over all of K)" if gemm else
                  "k_weight_stream<32> (m16n8k16 weight stream)",
                  "batch": B, "weight_bytes": w_bytes, "k0_us": round(k0_ms * 1e3, 2),
                  "cublas_us_same_operands": round(cublas_ms * 1e3, 2),
                  "k0_gbs": round(w_bytes / (k0_ms * 1e-3) / 1e9, 1),
                  "k0_frac_of_hbm_peak": round(w_bytes / (k0_ms * 1e-3) / 1e9 / peak, 4),
                  "k0_tflops": round(flops / (k0_ms * 1e-3) / 1e12, 1),
                  "k0_frac_of_bf16_peak": round(flops / (k0_ms * 1e-3) / 1e12 / bf16_peak, 4),
                  "l2": "flushed: 256 MB written before every timed call, outside its CUDA events"}
    h = torch.randn(B, 2048, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).to(dev)
    h2 = torch.empty_like(h)
    po = runner.params(None, None, cache, out, x_n=x_n, residual=h, h_out=h2)
    native.check(lib.mla_o_proj(ctypes.byref(po), sptr), "o_proj")
    k5_ms = ptimer(lambda: lib.mla_o_proj(ctypes.byref(po), sptr), max(5, args.steps))
    wo_bytes = runner.w_o.numel() * 2
    projection["o_proj"] = {"kernel": "k_project_tc<residual>" if gemm else "k_weight_stream<16, residual>",
                            "weight_bytes": wo_bytes, "k5_us": round(k5_ms * 1e3, 2),
                            "k5_gbs": round(wo_bytes / (k5_ms * 1e-3) / 1e9, 1),
                            "k5_frac_of_hbm_peak": round(wo_bytes / (k5_ms * 1e-3) / 1e9 / peak, 4)}

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

    # ---- the sequence-sharded variant (config 5b) in the same processes at N > 1; the other
    # configurations on this GPU at N = 1
    seq = None
    if world > 1 and not args.no_extra:
        seq = sequence_sharded_block(args, rank, world, dev, dist)
    others = stack = None
    if world == 1 and not args.no_extra:
        peak0, _ = measured_peak()
        oclocks = ClockSampler(local_rank)
        with oclocks:
            others = {n: other_config_summary(n, dev, max(10, args.steps), peak0)
                      for n in ("config1", "config3", "config4", "config5b") if n != args.workload}
            for n in others:
                others[n]["stack"] = stack_summary(n, dev, max(10, args.steps), peak0)
                torch.cuda.empty_cache()
            stack = stack_summary(args.workload, dev, max(5, args.steps // 2), peak0)
            torch.cuda.empty_cache()
        others["clocks"] = oclocks.summary()

    seq_inp = seq.pop("_check_inputs") if seq is not None else None
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    # CPU leg, rank 0 alone once the other ranks have left (a rank waiting in a collective
    # would compete for the host cores): the CPU baseline, and the oracle's check of the
    # sequence-sharded output
    cpu = None
    if not args.no_cpu_baseline:
        cpu = cpu_oracle_sample(args.workload, args.cpu_seconds, faithful=False)
        for k in ("seconds", "bytes", "requests"):
            cpu.pop(k, None)
    if seq_inp is not None:
        seq["check"] = check_sequence_sharded(seq_inp)
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
                        ": pinned x_n H2D, the step (q|kv_a projection: the library's weight stream for <= 64 "
                        "requests, else cuBLAS, measured faster than the library's tcgen05 GEMM here; K1-K3), "
                        "R(out) D2H", "mode": e2e_mode},
        "gpu_launches": native.load_library().mla_launches_per_step() * args.steps,
        "clocks": clocks.summary(),
    }
    if seq is not None:
        line["sequence_sharded"] = seq
    if others is not None:
        line["stack"] = stack
        line["other_configs"] = others
    print(json.dumps(line), flush=True)


def sequence_sharded_block(args, rank: int, world: int, dev: torch.device, dist, exchange: str = "peer") -> dict:
    """Config 5b across `world` GPUs, in the processes of the current run: one sequence of
    131,072 cached rows split by page-aligned KV ranges (distributed.sequence_shards); per
    step K1-K3 on each range and the fixed-order combine of the 8.4 KB shard partials.
    exchange="peer": K3 stores the partials into every rank's exchange buffer over NVLink
    and combines them itself where its grid is resident at once (else K4 does), one
    library call per step; "nccl": an NCCL all-gather and mla_combine_shards.

    Every rank draws the same 131,072 rows (one seeded generator), so the same rows are
    also timed unsharded on each rank's own GPU (the N = 1 step, a CUDA graph of K1-K3):
    strong-scaling efficiency = t(1) / (N t(N)), both measured in this run, max over
    ranks. The combined output is compared with the one-GPU step's; rank 0 keeps the
    inputs so that its CPU leg checks it against the oracle over all rows. Total work is
    fixed: strong scaling. Collective: every rank calls this."""
    dmod = importlib.import_module("fleet-mi300x_b200.distributed")
    wl = workloads.WORKLOADS["config5b"]
    T = wl.seq_lens()[0]
    cfg = fleet.ModelConfig()
    lw = workloads.make_layer_weights(wl.seed)
    w = fleet.LayerWeights(*(t.to(dev) for t in (lw.q_proj, lw.kv_a_proj_with_mqa, lw.kv_a_layernorm,
                                                   lw.kv_b_proj)))
    cos, sin = fleet.device_rope_tables(cfg, T + 8, dev)
    rows = torch.randn(T, 576, generator=torch.Generator(device=dev).manual_seed(wl.seed), device=dev)
    rows = rows.to(torch.bfloat16)
    runner = fleet.MlaDecodeAttention(cfg, w, cos, sin)
    x_n = workloads.make_hidden(wl.seed + 1, 1).to(dev)
    q, kv_a = (t.contiguous() for t in runner.project(x_n))
    if dist is not None:  # every shard must use the same q / kv_a bits
        dist.broadcast(q, 0)
        dist.broadcast(kv_a, 0)
    pos = torch.tensor([T], dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    kv_b = workloads.kv_bytes([T])
    steps = max(5, args.steps)

    # ---- N = 1 on this rank's own GPU: the whole sequence, the same rows
    full = fleet.PagedLatentCache.for_lengths([T], permute=True, zero=False,
                                              generator=torch.Generator().manual_seed(wl.seed), device=dev)
    full.write_rows(0, 0, rows)
    one = torch.empty(1, 2048, dtype=torch.bfloat16, device=dev)
    g1 = fleet.DecodeGraph(runner, full, inputs="qkv", q=q, kv_a=kv_a, out=one)
    for _ in range(max(3, args.warmup)):
        g1.replay()
    g1.synchronize()
    t1_timer = StepTimer(stream, kv_b, dev)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    t1_ms = t1_timer(g1.replay, steps)
    g1.synchronize()
    del g1

    # ---- N shards
    a, b = dmod.sequence_shards(T, world)[rank]
    last = rank == world - 1
    cache = fleet.PagedLatentCache.for_lengths([b - a], extra_tokens=1 if last else 0, permute=True, zero=False,
                                               generator=torch.Generator().manual_seed(wl.seed + rank), device=dev)
    cache.write_rows(0, 0, rows[a:b])
    out = torch.empty(1, 2048, dtype=torch.bfloat16, device=dev)
    local = torch.empty(1, 16, native.SHARD_STRIDE, dtype=torch.float32, device=dev)
    parts = torch.empty(world, 1, 16, native.SHARD_STRIDE, dtype=torch.float32, device=dev)
    ex = None
    if exchange == "peer":
        ex = (dmod.ExchangeBuffers.create(rank, world, max_batch=1) if dist is not None
              else dmod.ExchangeBuffers.local(1, max_batch=1)[0])

    def step():
        if ex is not None:
            runner.attend(q, kv_a, cache, out, rope_pos=pos, new_row=last, exchange=ex)
            return
        runner.attend(q, kv_a, cache, rope_pos=pos, shard_out=local, new_row=last)
        if dist is not None:
            dist.all_gather_into_tensor(parts, local)
            fleet.combine_shards(parts, out)
        else:
            fleet.combine_shards(local[None], out)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    runner.check_errors()
    timer = StepTimer(stream, kv_b // world, dev)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    tn_ms = timer(step, steps)
    torch.cuda.synchronize()
    runner.check_errors()

    # ---- stage times (each stage repeated alone on every rank at once). A K3 repeated
    # without the combine rewrites the same lines, which the next whole step reads again,
    # so the exchange protocol stays in step.
    def stage(name):
        so = None if ex is not None else local
        o = out if ex is not None else None
        return lambda: runner.attend(q, kv_a, cache, o, name, rope_pos=pos, shard_out=so, new_row=last, exchange=ex)
    names = ["prologue", "attention", "merge"]
    stage_ms = []
    for name in names:
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        stage_ms.append(timer(stage(name), max(5, steps // 2)))
    if ex is not None:  # the same step with the exchange as K3 + K4 instead of the fused K3
        names.append("step_k3_k4_split")
        runner.flags |= native.FLAG_EXCHANGE_SPLIT
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        stage_ms.append(timer(step, max(5, steps // 2)))
        runner.flags &= ~native.FLAG_EXCHANGE_SPLIT
    step()  # a whole step last: the exchange's step counter advances on every rank
    torch.cuda.synchronize()
    runner.check_errors()

    # ---- the same in a 27-layer decode step (LayerStackGraph): every layer its own rows,
    # whole on one GPU and sharded over the N, the shards of all layers sharing the
    # exchange buffers (one protocol step per layer)
    layers = STACK_LAYERS
    stack_one = stack_n = None
    g_rows = torch.Generator(device=dev).manual_seed(wl.seed + 17)
    full_l, shard_l = [], []
    for l in range(layers):
        rl = torch.randn(T, 576, generator=g_rows, device=dev).to(torch.bfloat16)
        c1 = fleet.PagedLatentCache.for_lengths([T], permute=True, zero=False,
                                                generator=torch.Generator().manual_seed(l), device=dev)
        c1.write_rows(0, 0, rl)
        cn = fleet.PagedLatentCache.for_lengths([b - a], extra_tokens=1 if last else 0, permute=True, zero=False,
                                                generator=torch.Generator().manual_seed(l + 100 * rank), device=dev)
        cn.write_rows(0, 0, rl[a:b])
        full_l.append(c1)
        shard_l.append(cn)
        del rl
    st1 = fleet.LayerStackGraph([runner] * layers, full_l, mode="slice", q=[q] * layers, kv_a=[kv_a] * layers)
    kw = dict(rope_pos=pos, new_row=last)
    if ex is not None:
        kw["exchange"] = ex
    if dist is not None:
        dist.barrier()
    stn = fleet.LayerStackGraph([runner] * layers, shard_l, mode="slice", q=[q] * layers, kv_a=[kv_a] * layers,
                                attend_kw=kw) if ex is not None else None
    stimer = StepTimer(stream, layers * kv_b // world, dev)
    for _ in range(3):
        st1.replay()
    st1.synchronize()
    stack_one = stimer(st1.replay, max(5, steps // 2)) / layers
    st1.synchronize()
    if stn is not None:
        for _ in range(3):
            stn.replay()
        stn.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        stack_n = stimer(stn.replay, max(5, steps // 2)) / layers
        stn.synchronize()
    del st1, stn
    torch.cuda.synchronize()

    t = torch.tensor([t1_ms, tn_ms, stack_one, stack_n or 0.0] + stage_ms, device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    t1_ms, tn_ms, stack_one, stack_n, *stage_ms = t.tolist()

    # ---- the combined output against the one-GPU step on the same rows; rank 0 keeps the
    # inputs for the oracle check of its CPU leg (check_sequence_sharded)
    rel1 = float((out.float() - one.float()).abs().max() / one.float().abs().max())
    check_inputs = None
    if rank == 0:
        check_inputs = {"q": q.float().cpu().numpy(), "kv_a": kv_a.float().cpu().numpy(),
                        "rows": rows.float().cpu().numpy(), "out": out.float().cpu().numpy(), "T": T}
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    if ex is not None:
        ex.close()
    if dist is not None:
        dist.barrier()
    peak, _ = measured_peak()
    how = (f"peer exchange of {16 * native.SHARD_STRIDE * 4} B partials per GPU: K3 stores them into every rank's "
           "buffer over NVLink (64-bit stores tagged with the step) and combines them where its grid is resident "
           "at once, else K4 does; no collective library in the step" if ex is not None else
           f"NCCL all-gather of {16 * native.SHARD_STRIDE * 4} B partials per GPU, then mla_combine_shards")
    return {
        "workload": "config5b", "context": T, "n_gpus": world, "exchange": exchange, "how": how,
        "us_per_layer_step": round(tn_ms * 1e3, 3), "kv_gbs": round(kv_b / (tn_ms * 1e-3) / 1e9, 1),
        "kv_frac_of_hbm_peak_per_gpu": round(kv_b / world / (tn_ms * 1e-3) / 1e9 / peak, 4),
        "one_gpu_us_per_layer_step": round(t1_ms * 1e3, 3),
        "strong_scaling_efficiency": round(t1_ms / (world * tn_ms), 4),
        "speedup_vs_one_gpu": round(t1_ms / tn_ms, 3),
        "stages_us": {n: round(v * 1e3, 2) for n, v in zip(names, stage_ms)},
        "kv_bytes_per_step": kv_b, "kv_bytes_per_gpu": kv_b // world,
        "l2": timer.describe(), "timing": "device time per step, CUDA events, max over ranks",
        "max_rel_vs_one_gpu": rel1, "check": None, "_check_inputs": check_inputs,
        "stack": None if ex is None else {
            "layers": layers, "us_per_layer_step": round(stack_n * 1e3, 3),
            "one_gpu_us_per_layer_step": round(stack_one * 1e3, 3),
            "speedup_vs_one_gpu": round(stack_one / stack_n, 3),
            "strong_scaling_efficiency": round(stack_one / (world * stack_n), 4),
            "kv_frac_of_hbm_peak_per_gpu": round(kv_b / world / (stack_n * 1e-3) / 1e9 / peak, 4),
            "what": "27 layers in one CUDA graph (LayerStackGraph), each layer its own 131,072 rows; on N GPUs "
                    "each rank its shard of every layer, one exchange buffer set for all layers"},
    }


def run_sequence_sharded(args, rank: int, world: int, local_rank: int, dev: torch.device, dist) -> None:
    """`--workload config5b` under torchrun: the sequence-sharded step alone, as its own
    bench line (strong scaling)."""
    clocks = ClockSampler(local_rank)
    with clocks:
        blk = sequence_sharded_block(args, rank, world, dev, dist, exchange=args.exchange)
    inp = blk.pop("_check_inputs")
    dist.barrier()
    dist.destroy_process_group()
    if rank != 0:
        return
    # CPU leg, rank 0 alone: the oracle's check of the combined output, and the CPU baseline
    blk["check"] = check_sequence_sharded(inp)
    cpu = None
    if not args.no_cpu_baseline:
        cpu = cpu_oracle_sample("config5b", args.cpu_seconds, faithful=False)
        for k in ("seconds", "bytes", "requests"):
            cpu.pop(k, None)
    us = blk["us_per_layer_step"]
    line = {
        "metric": METRIC, "value": blk["kv_gbs"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(us * 1e-3, 6), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) latents, N(0,0.02) weights)",
        "config": {"workload": "config5b", "batch": 1, "context": blk["context"], "page_size": 64,
                   "parallelism": f"sequence-sharded x{world}: page-aligned KV ranges, {blk['how']}",
                   "kv_bytes_per_step": blk["kv_bytes_per_step"], "kv_bytes_per_gpu": blk["kv_bytes_per_gpu"],
                   "l2": blk["l2"]},
        "us_per_layer_step": us,
        "kv_frac_of_hbm_peak_per_gpu": blk["kv_frac_of_hbm_peak_per_gpu"],
        "gpu_launches": (native.load_library().mla_launches_per_step() + 1) * args.steps,
        "sequence_sharded": blk,
        "cpu_baseline": cpu,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


STACK_LAYERS = 27  # DeepSeek-V2-Lite's decoder layers


def stack_summary(name: str, dev: torch.device, steps: int, peak: float, layers: int = STACK_LAYERS) -> dict:
    """The attention slice of `layers` layers as one CUDA graph (LayerStackGraph, slice
    mode): each layer has its own weights (seeded per layer) and its own cache with the
    workload's shape, as in a decoder, so the step reads layers x the KV bytes. Device time
    per step / layers = µs per layer-step inside a multi-layer decode step, the unit of the
    reference's per-layer figure (measured inside its all-layers persistent kernel). L2 is
    flushed before every timed step if the stack reads less than 4x L2."""
    wl = workloads.WORKLOADS[name]
    lengths = wl.seq_lens()
    cfg = fleet.ModelConfig()
    cos, sin = fleet.device_rope_tables(cfg, max(lengths) + 8, dev)
    x_n = workloads.make_hidden(wl.seed + 1, len(lengths)).to(dev)
    runners, caches, qs, kvs = [], [], [], []
    for l in range(layers):
        lw = workloads.make_layer_weights(wl.seed + 1000 * (l + 1))
        w = fleet.LayerWeights(*(t.to(dev) for t in (lw.q_proj, lw.kv_a_proj_with_mqa, lw.kv_a_layernorm,
                                                       lw.kv_b_proj)))
        r = fleet.MlaDecodeAttention(cfg, w, cos, sin)
        c = fleet.PagedLatentCache.for_lengths(lengths, permute=wl.permute, zero=False,
                                               generator=torch.Generator().manual_seed(wl.seed + l), device=dev)
        workloads.fill_pool_random(c.pages, wl.seed + 7919 * (l + 1))
        q, kv_a = (t.contiguous() for t in r.project(x_n))
        runners.append(r)
        caches.append(c)
        qs.append(q)
        kvs.append(kv_a)
    stack = fleet.LayerStackGraph(runners, caches, mode="slice", q=qs, kv_a=kvs)
    for _ in range(3):
        stack.replay()
    stack.synchronize()
    kv_b = workloads.kv_bytes(lengths)
    weights = layers * (2 * 16 * 128 * 512 * 2)
    timer = StepTimer(torch.cuda.current_stream(dev), layers * kv_b + weights, dev)
    ms = timer(stack.replay, steps)
    stack.synchronize()
    us = ms * 1e3 / layers
    return {"layers": layers, "us_per_layer_step": round(us, 3), "kv_gbs": round(kv_b / (us * 1e-6) / 1e9, 1),
            "kv_frac_of_hbm_peak": round(kv_b / (us * 1e-6) / 1e9 / peak, 4),
            "step_us": round(ms * 1e3, 2),
            "l2": "flushed before every timed step" if timer.flush is not None else "no flush (> 4x L2 per step)"}


def other_config_summary(name: str, dev: torch.device, steps: int, peak: float) -> dict:
    """One of the other benchmark configurations on this GPU, for the headline line's
    `other_configs`: the graph step (K1-K3, CUDA graph) after an L2 flush (if the step reads
    less than 4x L2) and device time per kernel, each kernel alone after a flush."""
    wl, lengths, runner, cache, x_n, q, kv_a = build_workload(name, dev, 0)
    B = len(lengths)
    stream = torch.cuda.current_stream(dev)
    kv_b = workloads.kv_bytes(lengths)
    out = torch.empty(B, 2048, dtype=torch.bfloat16, device=dev)
    for _ in range(3):
        runner.attend(q, kv_a, cache, out)
    out_g = torch.empty_like(out)
    graph = fleet.DecodeGraph(runner, cache, inputs="qkv", q=q, kv_a=kv_a, out=out_g)
    for _ in range(3):
        graph.replay()
    runner.attend(q, kv_a, cache, out)
    torch.cuda.synchronize()
    if not torch.equal(out_g, out):
        raise RuntimeError(f"{name}: graph step output differs from the eager step")
    runner.check_errors()
    timer = StepTimer(stream, kv_b, dev)
    ms = timer(graph.replay, steps)
    p = runner.params(q, kv_a, cache, out)
    sptr = ctypes.c_void_p(stream.cuda_stream)
    lib = runner.lib
    k1 = timer(lambda: lib.mla_prologue(ctypes.byref(p), sptr), steps)
    k2 = timer(lambda: lib.mla_attention(ctypes.byref(p), sptr), steps)
    k3 = timer(lambda: lib.mla_merge_uv(ctypes.byref(p), sptr), steps)
    torch.cuda.synchronize()
    runner.check_errors()
    gbs = kv_b / (ms * 1e-3) / 1e9
    return {"batch": B, "context": lengths[0] if len(set(lengths)) == 1 else [min(lengths), max(lengths)],
            "us_per_layer_step": round(ms * 1e3, 2), "kv_gbs": round(gbs, 1),
            "kv_frac_of_hbm_peak": round(gbs / peak, 4), "kv_bytes": kv_b,
            "stages_us": {"prologue": round(k1 * 1e3, 2), "attention": round(k2 * 1e3, 2),
                          "merge_uv": round(k3 * 1e3, 2)},
            "attention_frac_of_hbm_peak": round(kv_b / (k2 * 1e-3) / 1e9 / peak, 4),
            "l2": "flushed before every timed call" if timer.flush is not None else "no flush (> 4x L2 per step)"}


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
    ap.add_argument("--no-extra", action="store_true",
                    help="headline only: skip other_configs (N = 1) and the sequence-sharded block (N > 1)")
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
