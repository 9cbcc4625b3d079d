"""K5, o_proj with the layer's residual add (reference_decode.py:256, 300): the whole
attention half of a decoder layer, x_n -> h' = R(h + R(W_o R(out))), as one library call."""
import ctypes
import importlib

import numpy as np
import pytest
import torch

from mla_testlib import O, fleet, oracle_weights, rel_cos, workloads

pytestmark = pytest.mark.gpu
native = importlib.import_module("fleet-mi300x_b200.native")
BF = torch.bfloat16


def _setup(dev, B, seed):
    cfg = fleet.ModelConfig()
    cos, sin = fleet.device_rope_tables(cfg, 600, dev)
    lw = workloads.make_layer_weights(seed)
    g = torch.Generator().manual_seed(seed + 1)
    w_o = (torch.randn(2048, 2048, generator=g) * 0.02).to(BF)
    runner = fleet.MlaDecodeAttention(cfg, fleet.LayerWeights(
        *(t.to(dev) for t in (lw.q_proj, lw.kv_a_proj_with_mqa, lw.kv_a_layernorm, lw.kv_b_proj)), o_proj=w_o.to(dev)),
        cos, sin)
    lens = [int(x) for x in torch.randint(0, 500, (B,), generator=g)]
    cache = fleet.PagedLatentCache.for_lengths(lens, spare_pages=1, generator=g, device=dev)
    cache.pages.copy_(torch.randn(cache.pages.shape, generator=g).to(BF))
    x = torch.randn(B, 2048, generator=g).to(BF).to(dev)
    h = torch.randn(B, 2048, generator=g).to(BF).to(dev)
    return runner, cache, x, h, lw, w_o, lens


@pytest.mark.parametrize("B", [1, 9, 64, 65, 256])  # 65, 256: the tcgen05 GEMM form of K5
def test_o_proj_residual_matches_numpy_on_the_same_out(cuda_device, B):
    """K5 through the C ABI (mla_o_proj): the weight stream up to 64 requests, the tcgen05
    GEMM beyond, on R(out) of a library step, against NumPy's fp32 GEMV + roundings."""
    runner, cache, x, h, _, w_o, _ = _setup(cuda_device, B, 70)
    out = runner.attend_x(x, cache)
    h_new = torch.empty_like(h)
    p = runner.params(None, None, cache, out, x_n=x, residual=h, h_out=h_new)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    native.check(runner.lib.mla_o_proj(ctypes.byref(p), stream), "mla_o_proj", p)
    runner.check_errors()
    cfg = O.Config()
    W = w_o.float().numpy()
    o_np, h_np, got = out.float().cpu().numpy(), h.float().cpu().numpy(), h_new.float().cpu().numpy()
    for b in range(B):
        want = O.o_proj_residual(cfg, W, o_np[b], h_np[b])
        # R(W_o out) may differ by the fp32 summation order, (K - 1) 2^-24 sum|w o|, and then
        # by one bf16 step of that intermediate (reference_decode.py:256 rounds it); the
        # residual add rounds once more (one step of the result; where h and the product
        # nearly cancel, the intermediate's step is the larger one)
        slack = 2047 * 2.0 ** -24 * (np.abs(W) @ np.abs(o_np[b]))
        inter = np.abs(W @ o_np[b])
        bound = 2.0 ** -7 * inter + 2.0 ** -6 * np.maximum(np.abs(want), np.abs(got[b])) + slack
        worst = int(np.argmax(np.abs(got[b] - want) - bound))
        assert np.all(np.abs(got[b] - want) <= bound), (b, worst, got[b][worst], want[worst])
        assert np.count_nonzero(got[b] != want) <= 0.02 * want.size


def test_attention_block_matches_oracle(cuda_device):
    B = 5
    runner, cache, x, h, lw, w_o, lens = _setup(cuda_device, B, 80)
    rows = [cache.read_rows(b, 0, lens[b]).float().cpu().numpy() for b in range(B)]
    out = torch.empty(B, 2048, dtype=BF, device=cuda_device)
    h_new = runner.attention_block(x, cache, h, out=out).float().cpu().numpy()
    runner.check_errors()
    out = out.float().cpu().numpy()
    cfg, w = O.Config(), oracle_weights(lw)
    cos, sin = cfg.cos_sin(600)
    W = w_o.float().numpy()
    for b in range(B):
        flat = np.zeros((lens[b] + 1, 576), np.float32)
        flat[:lens[b]] = rows[b]
        attn = O.attention_task(cfg, w, x[b].float().cpu().numpy(), flat, lens[b], cos, sin)
        hb = h[b].float().cpu().numpy()
        rel, cs = rel_cos(out[b], attn)  # R(out), the slice itself: the usual bar
        assert rel <= 1e-2 and cs >= 0.9999, (b, rel, cs)
        # the attention half's contribution h' - h: h' is rounded to bf16 at |h'| ~ 1-4
        # (steps of 2^-7 .. 2^-6), noise of a few percent of the contribution's RMS, so
        # compare direction and mean error (K5's own arithmetic is checked tightly above)
        want = O.o_proj_residual(cfg, W, attn, hb)
        d, dw = h_new[b] - hb, want - hb
        _, cs = rel_cos(d, dw)
        assert cs >= 0.999 and np.mean(np.abs(d - dw)) <= 0.05 * np.mean(np.abs(dw)), (b, cs)


def test_attention_block_in_place_and_refusals(cuda_device):
    runner, cache, x, h, _, _, _ = _setup(cuda_device, 3, 90)
    h_copy = h.clone()
    ref = runner.attention_block(x, cache, h_copy, h_out=torch.empty_like(h))
    got = runner.attention_block(x, cache, h, h_out=h)  # residual updated in place
    assert torch.equal(got, ref) and got.data_ptr() == h.data_ptr()
    out = torch.empty(3, 2048, dtype=BF, device=cuda_device)
    p = runner.params(None, None, cache, out, x_n=x, residual=h, h_out=h)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    bad = native.MlaDecodeParams.from_buffer_copy(p)
    bad.out_stride = 2052  # K5 reads out through TMA: a multiple of 8 elements
    assert runner.lib.mla_decode_step(ctypes.byref(bad), stream) == -3
    bad = native.MlaDecodeParams.from_buffer_copy(p)
    bad.residual = None
    assert runner.lib.mla_decode_step(ctypes.byref(bad), stream) == -1
