"""The one-kernel step (MLA_FLAG_FUSED_STEP, MlaDecodeAttention(fused_step=True)):
prologue, split-KV attention and merge + W_UV of one request in one launch.

Checked against the oracle (oracle.attend_rows_fast, the reference's arithmetic,
reference_decode.py:224-254) at lengths across page and half-page boundaries up to
config 5b's 131,072 rows, against the three-kernel path, bit for bit against itself
(repeated calls, a CUDA-graph replay, the library's static scratch), as one shard of a
sequence-sharded step (gathered partials and the peer exchange, ranks emulated on one
GPU), and for the errors and refusals of the flag.
"""
import ctypes

import numpy as np
import pytest
import torch

from mla_testlib import COS_MIN, REL_TIGHT, REL_TOL, O, fleet, oracle_weights, rel_cos, workloads

pytestmark = pytest.mark.gpu
BF = torch.bfloat16
native = fleet.native
dist_mod = __import__("importlib").import_module("fleet-mi300x_b200.distributed")


def _assert_close(got, want, what):
    rel, cs = rel_cos(got, want)
    assert rel <= REL_TOL, f"{what}: max rel {rel:.3e} above the 2e-2 bar (cos {cs:.6f})"
    assert rel <= REL_TIGHT and cs >= COS_MIN, f"{what}: max rel {rel:.3e}, cos {cs:.7f}"
    return rel


def _setup(dev, T, seed=11, permute=True):
    """One request with T cached rows of N(0, 1) latents on permuted pages; q / kv_a from
    the oracle's projection of a seeded hidden state; runners with and without the flag."""
    cfg = O.Config()
    cos, sin = cfg.cos_sin(T + 8)
    lw = workloads.make_layer_weights(seed)
    w = oracle_weights(lw)
    cache = fleet.PagedLatentCache.for_lengths([T], permute=permute, zero=False, spare_pages=2,
                                               generator=torch.Generator().manual_seed(seed), device=dev)
    workloads.fill_pool_random(cache.pages, seed)
    x_n = workloads.make_hidden(seed + 1, 1).float().numpy()[0]
    qn, kvn = O.project(cfg, w, x_n)
    wd = fleet.LayerWeights(*(t.to(dev) for t in (lw.q_proj, lw.kv_a_proj_with_mqa, lw.kv_a_layernorm,
                                                  lw.kv_b_proj, lw.o_proj)))
    cos_t, sin_t = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    fused = fleet.MlaDecodeAttention(fleet.ModelConfig(), wd, cos_t, sin_t, fused_step=True)
    plain = fleet.MlaDecodeAttention(fleet.ModelConfig(), wd, cos_t, sin_t)
    q = torch.from_numpy(qn.reshape(1, -1)).to(BF).to(dev)
    kv_a = torch.from_numpy(kvn[None]).to(BF).to(dev)
    return dict(cfg=cfg, cos=cos, sin=sin, w=w, cache=cache, qn=qn, kvn=kvn, q=q, kv_a=kv_a, fused=fused,
                plain=plain, T=T, lw=lw, wd=wd, cos_t=cos_t, sin_t=sin_t)


def _oracle(d):
    cfg, w, T, cache = d["cfg"], d["w"], d["T"], d["cache"]
    rows = cache.read_rows(0, 0, T).float().cpu().numpy() if T else np.zeros((0, 576), np.float32)
    new_row = O.kv_post(cfg, w, d["kvn"], T, d["cos"], d["sin"])
    return new_row, O.attend_rows_fast(cfg, w, d["qn"], np.concatenate([rows, new_row[None]]), T, d["cos"], d["sin"])


@pytest.mark.parametrize("T", [0, 1, 31, 32, 63, 64, 65, 1000, 1023, 4096, 40000, 131072])
def test_fused_vs_oracle_and_three_kernels(cuda_device, T):
    d = _setup(cuda_device, T)
    out = d["fused"].attend(d["q"], d["kv_a"], d["cache"])
    d["fused"].check_errors()
    new_row, want = _oracle(d)
    row = d["cache"].read_rows(0, T, 1)[0].float().cpu().numpy()
    np.testing.assert_allclose(row, new_row, rtol=1e-2, atol=1e-6, err_msg=f"appended row at {T}")
    rel = _assert_close(out[0].float().cpu().numpy(), want, f"fused T={T}")
    # the same request through K1-K3 (the appended row is rewritten identically)
    ref = d["plain"].attend(d["q"], d["kv_a"], d["cache"])
    d["plain"].check_errors()
    rel3, _ = rel_cos(out[0].float().cpu().numpy(), ref[0].float().cpu().numpy())
    assert rel3 <= 5e-3, f"T={T}: fused vs three kernels max rel {rel3:.3e}"
    # repeated calls: same bits (the counters were left zero, the fold order is fixed)
    for _ in range(2):
        again = d["fused"].attend(d["q"], d["kv_a"], d["cache"])
        d["fused"].check_errors()
        assert torch.equal(again, out), f"T={T}: a repeated fused step differs"
    print(f"fused T={T}: max rel {rel:.3e} vs oracle, {rel3:.3e} vs K1-K3")


def test_fused_block_and_graph(cuda_device):
    """The whole block from x_n (K0 weight stream + the one kernel + K5 o_proj and
    residual) against the three-kernel block, and a CUDA-graph replay of the fused step
    equal to the eager call bit for bit."""
    d = _setup(cuda_device, 5000)
    x_n = workloads.make_hidden(12, 1).to(cuda_device)
    res = workloads.make_hidden(13, 1).to(cuda_device)
    h_f = d["fused"].attention_block(x_n, d["cache"], res)
    d["fused"].check_errors()
    h_p = d["plain"].attention_block(x_n, d["cache"], res)
    d["plain"].check_errors()
    rel, cs = rel_cos(h_f.float().cpu().numpy(), h_p.float().cpu().numpy())
    assert rel <= 1e-2 and cs >= COS_MIN, f"fused block vs three kernels: max rel {rel:.3e}, cos {cs:.7f}"
    eager = d["fused"].attend(d["q"], d["kv_a"], d["cache"])
    graph = fleet.DecodeGraph(d["fused"], d["cache"], inputs="qkv", q=d["q"], kv_a=d["kv_a"])
    for _ in range(3):
        g = graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(g, eager), "graph replay of the fused step differs from the eager call"
    d["fused"].check_errors()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_sequence_shards(cuda_device, world):
    """One sequence split over `world` emulated ranks, each rank's step the one kernel:
    gathered partials (shard_out + mla_combine_shards) and the peer exchange (every rank's
    kernel stores its lines into every rank's buffer, then every rank's K4) give the same
    bits, and match the oracle over all rows."""
    T = 24000
    d = _setup(cuda_device, T, permute=False)
    dev = cuda_device
    rows = d["cache"].read_rows(0, 0, T)
    caches = []
    for r, (a, b) in enumerate(dist_mod.sequence_shards(T, world)):
        c = fleet.PagedLatentCache.for_lengths([b - a], extra_tokens=1 if r == world - 1 else 0, spare_pages=1,
                                               generator=torch.Generator().manual_seed(50 + r), device=dev)
        c.write_rows(0, 0, rows[a:b])
        caches.append(c)
    pos = torch.tensor([T], dtype=torch.int32, device=dev)
    runner = d["fused"]
    gathered = dist_mod.emulate_sequence_shards(runner, d["q"], d["kv_a"], caches, pos)
    runner.check_errors()
    ex = dist_mod.ExchangeBuffers.local(world, max_batch=1)
    try:
        for step in range(3):  # both parities of the exchange buffers, then the first again
            outs = dist_mod.emulate_exchange_step(runner, d["q"], d["kv_a"], caches, pos, ex)
            runner.check_errors()
            for r, o in enumerate(outs):
                assert torch.equal(o, gathered), f"world {world} step {step}: rank {r} differs from the gathered combine"
    finally:
        torch.cuda.synchronize()
        ex[0].close()
    new_row, want = _oracle(d)
    a, b = dist_mod.sequence_shards(T, world)[-1]
    dev_row = caches[-1].read_rows(0, b - a, 1)[0].float().cpu().numpy()
    np.testing.assert_allclose(dev_row, new_row, rtol=1e-2, atol=1e-6)
    # the oracle over the same rows (the unsharded cache's row T was never written: use the oracle's)
    rel = _assert_close(gathered[0].float().cpu().numpy(), want, f"fused over {world} ranks")
    print(f"fused x{world}: max rel {rel:.3e}")


def test_fused_errors_and_refusals(cuda_device):
    """A position past the RoPE tables records MLA_DEV_BAD_POSITION and writes zeros; a bad
    block-table entry records MLA_DEV_BAD_PAGE; the flag is refused for two requests, with
    the precision forms, and where the grid cannot hold the merge slices; the context keeps
    working (a good step after each)."""
    d = _setup(cuda_device, 700)
    runner, cache = d["fused"], d["cache"]
    good = runner.attend(d["q"], d["kv_a"], cache)
    runner.check_errors()
    # position past the tables
    saved = cache.seq_lens.clone()
    cache.seq_lens.fill_(d["cos_t"].shape[0] + 5)
    bad = runner.attend(d["q"], d["kv_a"], cache, check=False)
    torch.cuda.synchronize()
    with pytest.raises(native.MlaError) as e:
        runner.check_errors()
    assert e.value.code == 2
    assert not bad.float().abs().any(), "a request with a bad position must get zeros"
    cache.seq_lens.copy_(saved)
    # a bad page in the middle of the request
    bt = cache.block_table.clone()
    cache.block_table[0, 3] = cache.n_pages + 7
    runner.attend(d["q"], d["kv_a"], cache, check=False)
    torch.cuda.synchronize()
    with pytest.raises(native.MlaError) as e:
        runner.check_errors()
    assert e.value.code == 1
    cache.block_table.copy_(bt)
    again = runner.attend(d["q"], d["kv_a"], cache)
    runner.check_errors()
    assert torch.equal(again, good), "the step after the errors differs"
    # refusals
    lib = native.load_library()
    p = runner.params(d["q"], d["kv_a"], cache, torch.empty(1, 2048, dtype=BF, device=cuda_device))
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert p.flags & native.FLAG_FUSED_STEP
    for flags, ctas in ((native.FLAG_FUSED_STEP | native.FLAG_QC_HILO, 0), (native.FLAG_FUSED_STEP, 16)):
        p.flags, p.num_ctas = flags, ctas
        assert lib.mla_decode_step(ctypes.byref(p), stream) == -1
    p.flags, p.num_ctas = native.FLAG_FUSED_STEP, 0
    assert lib.mla_prologue(ctypes.byref(p), stream) == -1
    assert lib.mla_merge_uv(ctypes.byref(p), stream) == -1
    p.batch = 2
    assert lib.mla_decode_step(ctypes.byref(p), stream) == -1
    again = runner.attend(d["q"], d["kv_a"], cache)
    runner.check_errors()
    assert torch.equal(again, good)


def test_fused_static_scratch(cuda_device):
    """mla_decode_step_static with the flag (its counters live in the library's static
    scratch, zero at load): equal to mla_decode_step with the runner's workspace, twice."""
    d = _setup(cuda_device, 3000)
    runner, cache = d["fused"], d["cache"]
    lib = native.load_library()
    want = runner.attend(d["q"], d["kv_a"], cache)
    runner.check_errors()
    out = torch.empty(1, 2048, dtype=BF, device=cuda_device)
    p = runner.params(d["q"], d["kv_a"], cache, out)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(2):
        out.zero_()
        assert lib.mla_decode_step_static(ctypes.byref(p), stream) == 0
        torch.cuda.synchronize()
        runner.check_errors()
        assert torch.equal(out, want), "the static-scratch fused step differs"
