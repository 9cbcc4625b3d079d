"""mla_decode_step_static: the decode step with the library's own static workspace.

Its output must equal mla_decode_step's (caller-allocated workspace, same kernels,
same split plan) bit for bit, on two calls in a row, and a call must not change the
device's free memory or torch's allocation count. The file name makes pytest collect
it last, so it runs both after every other GPU test in one process and alone.
"""
import ctypes
import gc
import importlib

import pytest
import torch

from mla_testlib import fleet, workloads

pytestmark = pytest.mark.gpu
native = importlib.import_module("fleet-mi300x_b200.native")

LENS = [0, 37, 64, 130, 511, 1000, 2048, 4095]


def _setup(dev):
    cfg = fleet.ModelConfig()
    cos, sin = fleet.rope_tables(cfg, 4160)
    lw = workloads.make_layer_weights(11)
    runner = fleet.MlaDecodeAttention(
        cfg, fleet.LayerWeights(*(t.to(dev) for t in (lw.q_proj, lw.kv_a_proj_with_mqa, lw.kv_a_layernorm,
                                                       lw.kv_b_proj))),
        torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev))
    g = torch.Generator().manual_seed(12)
    cache = fleet.PagedLatentCache.for_lengths(LENS, spare_pages=3, generator=g, device=dev)
    cache.pages.copy_(torch.randn(cache.pages.shape, generator=g).to(torch.bfloat16))
    q = torch.randn(len(LENS), 3072, generator=g).to(torch.bfloat16).to(dev)
    kv_a = torch.randn(len(LENS), 576, generator=g).to(torch.bfloat16).to(dev)
    return runner, cache, q, kv_a


def test_static_step_equals_decode_step_on_two_calls(cuda_device):
    runner, cache, q, kv_a = _setup(cuda_device)
    want = runner.attend(q, kv_a, cache)  # mla_decode_step with a torch-allocated workspace
    runner.check_errors()
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    for call in range(2):
        out = torch.full_like(want, float("nan"))
        p = runner.params(q, kv_a, cache, out)
        p.workspace, p.workspace_bytes = None, 0  # ignored by the static entry point
        # earlier tests' garbage must not be freed inside the measured window
        gc.collect()
        gc.disable()
        try:
            torch.cuda.synchronize(cuda_device)
            free0, _ = torch.cuda.mem_get_info(cuda_device)
            alloc0 = torch.cuda.memory_allocated(cuda_device)
            native.check(runner.lib.mla_decode_step_static(ctypes.byref(p), stream), "mla_decode_step_static", p)
            torch.cuda.synchronize(cuda_device)
            alloc1 = torch.cuda.memory_allocated(cuda_device)
            free1, _ = torch.cuda.mem_get_info(cuda_device)
        finally:
            gc.enable()
        runner.check_errors()
        assert torch.equal(out, want), f"call {call}: static-scratch output differs from mla_decode_step's"
        assert alloc1 == alloc0
        if call == 1:  # the first call may load the library's device image, which holds the scratch
            assert free1 == free0, "the static step allocated device memory"


def test_static_step_refuses_batches_beyond_its_scratch(cuda_device):
    runner, cache, q, kv_a = _setup(cuda_device)
    out = torch.zeros(len(LENS), 2048, dtype=torch.bfloat16, device=cuda_device)
    p = runner.params(q, kv_a, cache, out)
    p.batch = 600  # needs 35.6 MB of workspace at 148 CTAs; the static scratch holds 32 MiB
    p.num_ctas = 148
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    assert runner.lib.mla_decode_step_static(ctypes.byref(p), stream) == -8  # MLA_E_LIMIT, nothing launched
    torch.cuda.synchronize(cuda_device)
    assert not out.any()
