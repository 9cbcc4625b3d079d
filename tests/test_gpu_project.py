"""K0, the in-library q | kv_a projection (reference_decode.py:225-231): q = R(W_q x_n),
kv_a = R(W_kv_a x_n), and the whole x_n -> R(out) slice through the C ABI
(MlaDecodeParams.x_n). Up to 64 requests K0 streams the weight (m16n8k16); beyond, it is
a tcgen05 GEMM with the K quarters of a tile in a 4-CTA cluster (65, 100, 256 and 300
requests: a partial second M tile, two M tiles, a second row of clusters)."""
import ctypes
import importlib

import numpy as np
import pytest
import torch

from mla_testlib import COS_MIN, REL_TIGHT, O, fleet, oracle_weights, rel_cos, workloads

pytestmark = pytest.mark.gpu
native = importlib.import_module("fleet-mi300x_b200.native")


def _a256(x):
    return (x + 255) // 256 * 256


def qkv_offset(batch, ctas):
    off = _a256((batch + 1) * 4)
    off = _a256(off + 16 + ctas * 32)  # the split plan: header and one 32-byte entry per CTA
    off = _a256(off + batch * 16 * 576 * 2)
    off = _a256(off + (ctas + batch) * 16 * 2 * 4)
    return _a256(off + (ctas + batch) * 16 * 512 * 4)


def _setup(dev, B, seed=40):
    cfg = fleet.ModelConfig()
    cos, sin = fleet.device_rope_tables(cfg, 600, dev)
    lw = workloads.make_layer_weights(seed)
    runner = fleet.MlaDecodeAttention(cfg, fleet.LayerWeights(
        *(t.to(dev) for t in (lw.q_proj, lw.kv_a_proj_with_mqa, lw.kv_a_layernorm, lw.kv_b_proj))), cos, sin)
    g = torch.Generator().manual_seed(seed + 1)
    lens = [int(x) for x in torch.randint(0, 500, (B,), generator=g)]
    cache = fleet.PagedLatentCache.for_lengths(lens, spare_pages=1, generator=g, device=dev)
    cache.pages.copy_(torch.randn(cache.pages.shape, generator=g).to(torch.bfloat16))
    x = torch.randn(B, 2048, generator=g).to(torch.bfloat16).to(dev)
    return runner, cache, x, lw, lens


@pytest.mark.parametrize("B", [1, 5, 16, 17, 64, 65, 100, 256, 300])
def test_projection_matches_oracle(cuda_device, B):
    runner, cache, x, lw, _ = _setup(cuda_device, B)
    runner.attend_x(x, cache, stage="project")
    torch.cuda.synchronize()
    p = runner._step_p
    ctas = ctypes.c_int32()
    native.check(runner.lib.mla_plan_info(ctypes.byref(p), ctypes.byref(ctas), None), "plan_info")
    off = qkv_offset(B, ctas.value)
    got = runner._ws[off: off + B * 3648 * 2].view(torch.bfloat16).view(B, 3648).float().cpu().numpy()
    again = runner.attend_x(x, cache, stage="project")
    torch.cuda.synchronize()
    got2 = runner._ws[off: off + B * 3648 * 2].view(torch.bfloat16).view(B, 3648).float().cpu().numpy()
    np.testing.assert_array_equal(got, got2)  # fixed summation order: the same bits every call
    w = oracle_weights(lw)
    W = np.concatenate([w.q_proj, w.kv_a_proj_with_mqa])
    xs = x.float().cpu().numpy()
    cfg = O.Config()
    for b in range(B):
        q, kv_a = O.project(cfg, w, xs[b])
        want = np.concatenate([q.reshape(-1), kv_a])
        diff = np.abs(got[b] - want)
        # two fp32 summation orders of a 2048-term dot product differ by at most
        # (K - 1) 2^-24 sum|w x|; after that, each side rounds to bf16 (one step)
        terms = np.abs(W) @ np.abs(xs[b])
        bound = 2.0 ** -7 * np.maximum(np.abs(want), np.abs(got[b])) + 2047 * 2.0 ** -24 * terms
        worst = int(np.argmax(diff - bound))
        assert np.all(diff <= bound), (f"request {b} row {worst}: got {got[b][worst]}, oracle {want[worst]}, "
                                       f"sum|w x| {terms[worst]}")
        assert np.count_nonzero(diff) <= 0.02 * want.size, f"request {b}: {np.count_nonzero(diff)} rounding differences"


@pytest.mark.parametrize("B", [1, 7, 64, 200])
def test_slice_from_x_matches_oracle_and_cublas_path(cuda_device, B):
    runner, cache, x, lw, lens = _setup(cuda_device, B, seed=50)
    cache_b = fleet.PagedLatentCache(cache.n_pages, B, cache.max_blocks, device=cuda_device)
    cache_b.pages.copy_(cache.pages); cache_b.block_table.copy_(cache.block_table); cache_b.seq_lens.copy_(cache.seq_lens)
    rows = [cache.read_rows(b, 0, lens[b]).float().cpu().numpy() for b in range(B)]
    got = runner.attend_x(x, cache).float().cpu().numpy()
    q, kv_a = runner.project(x)
    via_cublas = runner.attend(q, kv_a, cache_b).float().cpu().numpy()
    runner.check_errors()
    rel, cs = rel_cos(got, via_cublas)
    assert rel <= 1e-2 and cs >= 0.99999, (rel, cs)
    cfg, w = O.Config(), oracle_weights(lw)
    cos, sin = cfg.cos_sin(600)
    for b in range(min(B, 4)):
        flat = np.zeros((lens[b] + 1, 576), np.float32)
        flat[:lens[b]] = rows[b]
        want = O.attention_task(cfg, w, x[b].float().cpu().numpy(), flat, lens[b], cos, sin)
        rel, cs = rel_cos(got[b], want)
        assert rel <= REL_TIGHT and cs >= COS_MIN, (b, rel, cs)


def test_projection_refusals(cuda_device):
    runner, cache, x, _, _ = _setup(cuda_device, 2, seed=60)
    out = torch.zeros(2, 2048, dtype=torch.bfloat16, device=cuda_device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    p = runner.params(None, None, cache, out, x_n=x)
    bad = native.MlaDecodeParams.from_buffer_copy(p)
    bad.x_stride = 2050  # not a multiple of 8 elements
    assert runner.lib.mla_decode_step(ctypes.byref(bad), stream) == -3
    bad = native.MlaDecodeParams.from_buffer_copy(p)
    bad.q = x.data_ptr()  # q given together with x_n
    assert runner.lib.mla_decode_step(ctypes.byref(bad), stream) == -1
    torch.cuda.synchronize()
    assert not out.any()
