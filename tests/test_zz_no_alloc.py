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


def _static_call(runner, p, dev):
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    p.workspace, p.workspace_bytes = None, 0  # ignored by the static entry point
    native.check(runner.lib.mla_decode_step_static(ctypes.byref(p), stream), "mla_decode_step_static", p)
    torch.cuda.synchronize(dev)
    runner.check_errors()


def test_static_step_with_projection_and_o_proj(cuda_device):
    """The whole attention block from the static scratch: K0 projects q | kv_a from x_n
    into the scratch's qkv region, K1-K3 attend, K5 applies o_proj and the residual.
    Bit for bit equal to mla_decode_step with a caller workspace, on two calls in a row."""
    runner, cache, _, _ = _setup(cuda_device)
    lw = workloads.make_layer_weights(11)
    runner.w_o = lw.o_proj.to(cuda_device).contiguous()
    B = len(LENS)
    g = torch.Generator().manual_seed(13)
    x_n = workloads.make_hidden(14, B).to(cuda_device)
    h = torch.randn(B, 2048, generator=g).to(torch.bfloat16).to(cuda_device)
    out_w, h_w = torch.empty(B, 2048, dtype=torch.bfloat16, device=cuda_device), torch.empty_like(h)
    p = runner.params(None, None, cache, out_w, x_n=x_n, residual=h, h_out=h_w)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    native.check(runner.lib.mla_decode_step(ctypes.byref(p), stream), "mla_decode_step", p)
    torch.cuda.synchronize(cuda_device)
    runner.check_errors()
    for call in range(2):
        out_s, h_s = torch.full_like(out_w, float("nan")), torch.full_like(h, float("nan"))
        _static_call(runner, runner.params(None, None, cache, out_s, x_n=x_n, residual=h, h_out=h_s), cuda_device)
        assert torch.equal(out_s, out_w), f"call {call}: R(out) differs"
        assert torch.equal(h_s, h_w), f"call {call}: the new hidden state differs"


def test_static_step_at_the_default_plan_limit(cuda_device):
    """463 requests, the largest batch whose workspace fits the 32 MiB scratch at the
    default 296 split-KV CTAs (464 is refused): equal to mla_decode_step bit for bit."""
    B = 463
    runner, _, _, _ = _setup(cuda_device)
    lens = [int(x) for x in torch.randint(0, 200, (B,), generator=torch.Generator().manual_seed(15))]
    g = torch.Generator().manual_seed(16)
    cache = fleet.PagedLatentCache.for_lengths(lens, generator=g, device=cuda_device)
    cache.pages.copy_(torch.randn(cache.pages.shape, generator=g).to(torch.bfloat16))
    q = torch.randn(B, 3072, generator=g).to(torch.bfloat16).to(cuda_device)
    kv_a = torch.randn(B, 576, generator=g).to(torch.bfloat16).to(cuda_device)
    assert runner.workspace_bytes(B) <= native.STATIC_SCRATCH_BYTES < runner.workspace_bytes(B + 1)
    want = runner.attend(q, kv_a, cache).clone()
    runner.check_errors()
    for call in range(2):
        out = torch.full_like(want, float("nan"))
        _static_call(runner, runner.params(q, kv_a, cache, out), cuda_device)
        assert torch.equal(out, want), f"call {call}: static-scratch output differs at {B} requests"
    p = runner.params(q, kv_a, cache, out)
    p.batch = B + 1
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    assert runner.lib.mla_decode_step_static(ctypes.byref(p), stream) == -8  # MLA_E_LIMIT, before any launch


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
