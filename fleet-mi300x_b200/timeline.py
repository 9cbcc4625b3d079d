"""Kernel timeline of one decode step, from the trace build of the library.

`python fleet-mi300x_b200/build.py --trace` builds libmla_decode_trace.so, whose kernels
stamp `%globaltimer` per CTA at entry, after `griddepcontrol.wait` and at exit (the last
warp to return), record the SM id, and set two kernel-specific marks:

    K1: mark1 = absorb MMAs stored, mark2 = per-request work (q_pe RoPE, new row) done
    K3: mark1 = cluster form: this CTA's folds published (before waiting for the other
        ranks' pushes); plain form: W_UV staged; mark2 = o_c of the block complete

`python -m fleet-mi300x_b200.timeline config5b` (from the repository root, on a GPU)
replays one workload's step as a CUDA graph with the L2 flushed before each replay and
prints, per kernel, the first/median/last of each stamp in microseconds from the step's
first kernel entry. The trace library is loaded through MLA_DECODE_LIB; the stamps cost
a few global stores per CTA, so step times here run slightly above the bench's.
"""
from __future__ import annotations

import ctypes
import json
import os
import sys
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
TRACE_LIB = PKG / "libmla_decode_trace.so"
NAMES = ["K1", "K2", "K3", "K4", "K0/K5"]
KERNELS, CTAS, EVENTS = 5, 512, 6  # the trace build's [kernel][CTA][event] array


def read(lib) -> np.ndarray:
    """The stamps of the kernels run since the last read, [kernel][CTA][event] int64
    (events: entry, after wait, exit, SM id + 1, mark1, mark2; 0 = not stamped)."""
    buf = (ctypes.c_ulonglong * (KERNELS * CTAS * EVENTS))()
    if lib.mla_timeline_read(buf, KERNELS * CTAS * EVENTS) != 0:
        raise RuntimeError("mla_timeline_read failed")
    return np.frombuffer(buf, dtype=np.uint64).reshape(KERNELS, CTAS, EVENTS).astype(np.int64)


def summarize(t: np.ndarray) -> dict:
    """Per kernel: CTA count and [first, median, last] of each stamp, in us from the
    earliest entry of any kernel."""
    entries = t[:, :, 0][t[:, :, 0] > 0]
    if not entries.size:
        return {}
    base = int(entries.min())
    out = {}
    for k in range(KERNELS):
        m = t[k, :, 0] > 0
        if not m.any():
            continue
        d = {"ctas": int(m.sum())}
        for ev, name in ((0, "entry"), (1, "waited"), (2, "exit"), (4, "mark1"), (5, "mark2")):
            v = t[k, m, ev]
            v = v[v > 0] - base
            if v.size:
                d[name] = [round(float(v.min()) / 1e3, 2), round(float(np.median(v)) / 1e3, 2),
                           round(float(v.max()) / 1e3, 2)]
        out[NAMES[k]] = d
    return out


def main(argv: list[str]) -> int:
    name = argv[0] if argv else "config5b"
    os.environ["MLA_DECODE_LIB"] = str(TRACE_LIB)
    import importlib
    import torch
    fleet = importlib.import_module("fleet-mi300x_b200")
    native = importlib.import_module("fleet-mi300x_b200.native")
    workloads = importlib.import_module("fleet-mi300x_b200.workloads")
    lib = native.load_library()
    lib.mla_timeline_read.argtypes = [ctypes.c_void_p, ctypes.c_uint64]
    lib.mla_timeline_read.restype = ctypes.c_int
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    wl = workloads.WORKLOADS[name]
    lengths = wl.seq_lens()
    cfg = fleet.ModelConfig()
    lw = workloads.make_layer_weights(wl.seed)
    w = fleet.LayerWeights(*(x.to(dev) for x in (lw.q_proj, lw.kv_a_proj_with_mqa, lw.kv_a_layernorm, lw.kv_b_proj)))
    cos, sin = fleet.device_rope_tables(cfg, max(lengths) + 8, dev)
    cache = fleet.PagedLatentCache.for_lengths(lengths, permute=wl.permute, zero=False,
                                               generator=torch.Generator().manual_seed(wl.seed), device=dev)
    workloads.fill_pool_random(cache.pages, wl.seed)
    runner = fleet.MlaDecodeAttention(cfg, w, cos, sin)
    q, kv_a = (x.contiguous() for x in runner.project(workloads.make_hidden(wl.seed + 1, len(lengths)).to(dev)))
    out = torch.empty(len(lengths), 2048, dtype=torch.bfloat16, device=dev)
    graph = fleet.DecodeGraph(runner, cache, inputs="qkv", q=q, kv_a=kv_a, out=out)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(5):
        graph.replay()
    torch.cuda.synchronize()
    for _ in range(3):
        flush.zero_()
        torch.cuda._sleep(100_000)
        torch.cuda.synchronize()
        read(lib)
        graph.replay()
        torch.cuda.synchronize()
        print(json.dumps({"workload": name, **summarize(read(lib))}))
    runner.check_errors()
    return 0


if __name__ == "__main__":
    raise SystemExit(main(sys.argv[1:]))
