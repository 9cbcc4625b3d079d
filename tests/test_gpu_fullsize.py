"""Parity at the benchmark's full sizes: every request of the configurations the bench
times, through the C ABI, against the oracle (vectorised form, oracle.attend_rows_fast;
the reference's arithmetic, reference_decode.py:239-254).

  config 5a  256 requests x 4,096 cached rows, permuted 64-row pages, the default split
             plan (296 plan CTAs, pair-merged), K3 in 32-request blocks: the bench's
             headline step, eager and as the CUDA graph the bench replays
  config 4   8 x 32,768: all eight requests
  config 3   32 ragged requests in [512, 8192]: all of them
  config 5b  one sequence of 131,072 rows on one GPU, and sequence-sharded over 2, 4
             and 8 emulated ranks with the peer exchange (every rank's K1-K3, then every
             rank's K4, on one GPU; each rank's result must equal every other's)

Inputs are the bench's: the same seeds, latents and weights (workloads.WORKLOADS). The
oracle runs request by request on rows read back from the device cache; rows 0..T-1 are
untouched by the step, the appended row T is checked against the oracle's kv_post.
"""
import importlib

import numpy as np
import pytest
import torch

from mla_testlib import COS_MIN, REL_TIGHT, REL_TOL, O, fleet, oracle_weights, rel_cos, workloads

pytestmark = pytest.mark.gpu
BF = torch.bfloat16
dist_mod = importlib.import_module("fleet-mi300x_b200.distributed")


def _assert_close(got, want, what):
    rel, cs = rel_cos(got, want)
    assert rel <= REL_TOL, f"{what}: max rel {rel:.3e} above the 2e-2 bar (cos {cs:.6f})"
    assert rel <= REL_TIGHT and cs >= COS_MIN, f"{what}: max rel {rel:.3e}, cos {cs:.7f}"
    return rel


def _bench_inputs(name, dev):
    """The bench's workload (bench.build_workload): weights, permuted cache filled with
    N(0, 1) bf16 latents, x_n; q / kv_a from the oracle's projection of x_n."""
    wl = workloads.WORKLOADS[name]
    lengths = wl.seq_lens()
    cfg = O.Config()
    cos, sin = cfg.cos_sin(max(lengths) + 8)
    lw = workloads.make_layer_weights(wl.seed)
    w = oracle_weights(lw)
    cache = fleet.PagedLatentCache.for_lengths(lengths, permute=wl.permute, zero=False,
                                               generator=torch.Generator().manual_seed(wl.seed), device=dev)
    workloads.fill_pool_random(cache.pages, wl.seed)
    x_n = workloads.make_hidden(wl.seed + 1, len(lengths)).float().numpy()
    qs, kvs = zip(*(O.project(cfg, w, x) for x in x_n))
    q = np.stack([x.reshape(-1) for x in qs])
    kv_a = np.stack(kvs)
    runner = fleet.MlaDecodeAttention(fleet.ModelConfig(), fleet.LayerWeights(
        *(t.to(dev) for t in (lw.q_proj, lw.kv_a_proj_with_mqa, lw.kv_a_layernorm, lw.kv_b_proj))),
        torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev))
    return dict(cfg=cfg, cos=cos, sin=sin, w=w, cache=cache, q=q, kv_a=kv_a, lengths=lengths, runner=runner,
                q_t=torch.from_numpy(q).to(BF).to(dev), kv_a_t=torch.from_numpy(kv_a).to(BF).to(dev))


def _check_all_requests(d, got, what):
    """Every request against the oracle on the device's own rows; the appended row too."""
    cfg, w, cos, sin, cache = d["cfg"], d["w"], d["cos"], d["sin"], d["cache"]
    worst = 0.0
    for b, T in enumerate(d["lengths"]):
        rows = cache.read_rows(b, 0, T).float().cpu().numpy()
        new_row = O.kv_post(cfg, w, d["kv_a"][b], T, cos, sin)
        dev_row = cache.read_rows(b, T, 1)[0].float().cpu().numpy()
        np.testing.assert_allclose(dev_row, new_row, rtol=1e-2, atol=1e-6, err_msg=f"{what}: row {T} of request {b}")
        want = O.attend_rows_fast(cfg, w, d["q"][b].reshape(cfg.heads, cfg.q_head_dim),
                                  np.concatenate([rows, new_row[None]]), T, cos, sin)
        worst = max(worst, _assert_close(got[b], want, f"{what}: request {b} (T={T})"))
    return worst


def test_config5a_every_request_eager_and_graph(cuda_device):
    """The timed configuration: 256 x 4,096 with the default plan (296 plan CTAs, every CTA
    pair-merged: 33,024 half-page tiles, 544 -> 400 partials per head for K3) and K3's
    32-request blocks (B > 144).
    The bench replays the step as a CUDA graph; the graph's output must equal the eager
    call's bit for bit, and both must match the oracle on all 256 requests."""
    d = _bench_inputs("config5a", cuda_device)
    runner = d["runner"]
    out = runner.attend(d["q_t"], d["kv_a_t"], d["cache"])
    runner.check_errors()
    graph = fleet.DecodeGraph(runner, d["cache"], inputs="qkv", q=d["q_t"], kv_a=d["kv_a_t"])
    for _ in range(2):
        g = graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(g, out), "graph replay differs from the eager step"
    runner.check_errors()
    worst = _check_all_requests(d, out.float().cpu().numpy(), "config5a")
    print(f"config5a: 256 requests, worst max rel {worst:.3e}")


@pytest.mark.parametrize("name", ["config4", "config3"])
def test_every_request_vs_oracle(cuda_device, name):
    """Config 4 (8 x 32,768: 8,200 half-page tiles over 296 plan CTAs, pair-merged, 19
    partials per request) and config 3 (32 ragged requests, permuted pages): every request."""
    d = _bench_inputs(name, cuda_device)
    out = d["runner"].attend(d["q_t"], d["kv_a_t"], d["cache"])
    d["runner"].check_errors()
    worst = _check_all_requests(d, out.float().cpu().numpy(), name)
    print(f"{name}: {len(d['lengths'])} requests, worst max rel {worst:.3e}")


def test_config5b_one_gpu(cuda_device):
    """One sequence of 131,072 cached rows on one GPU: 4,097 half-page tiles over 296 plan CTAs, 148
    pair-merged partials per head, K3's 4-CTA cluster form."""
    d = _bench_inputs("config5b", cuda_device)
    out = d["runner"].attend(d["q_t"], d["kv_a_t"], d["cache"])
    d["runner"].check_errors()
    worst = _check_all_requests(d, out.float().cpu().numpy(), "config5b")
    print(f"config5b: worst max rel {worst:.3e}")


def test_one_request_of_524288_rows(cuda_device):
    """The longest sequence in the suite: 524,288 cached rows (604 MB, four times config 5b) on
    permuted pages, 16,385 half-page tiles over the default 296 plan CTAs (about 55 per CTA,
    pair-merged),
    K3's cluster form; the RoPE position and the appended row at 524,288."""
    T = 524288
    cfg = O.Config()
    cos, sin = cfg.cos_sin(T + 8)
    lw = workloads.make_layer_weights(9)
    w = oracle_weights(lw)
    dev = cuda_device
    cache = fleet.PagedLatentCache.for_lengths([T], permute=True, zero=False,
                                               generator=torch.Generator().manual_seed(9), device=dev)
    workloads.fill_pool_random(cache.pages, 9)
    x_n = workloads.make_hidden(10, 1).float().numpy()[0]
    qn, kvn = O.project(cfg, w, x_n)
    runner = fleet.MlaDecodeAttention(fleet.ModelConfig(), fleet.LayerWeights(
        *(t.to(dev) for t in (lw.q_proj, lw.kv_a_proj_with_mqa, lw.kv_a_layernorm, lw.kv_b_proj))),
        torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev))
    out = runner.attend(torch.from_numpy(qn.reshape(1, -1)).to(BF).to(dev), torch.from_numpy(kvn[None]).to(BF).to(dev),
                        cache)
    runner.check_errors()
    d = dict(cfg=cfg, w=w, cos=cos, sin=sin, cache=cache, q=qn.reshape(1, -1), kv_a=kvn[None], lengths=[T])
    worst = _check_all_requests(d, out.float().cpu().numpy(), "524,288 rows")
    print(f"524,288 rows: max rel {worst:.3e}")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_config5b_sequence_sharded_emulated(cuda_device, world):
    """Config 5b split over `world` ranks by page-aligned KV ranges (distributed.
    sequence_shards), with the peer exchange: every rank's K1-K3 (K3 stores its partial
    into every rank's exchange buffer), then every rank's K4 (waits for all lines, combines
    in rank order). All ranks' outputs are equal bit for bit, equal to the NCCL path's
    gathered combine, and match the oracle over all 131,073 rows."""
    wl = workloads.WORKLOADS["config5b"]
    T = wl.seq_lens()[0]
    cfg = O.Config()
    cos, sin = cfg.cos_sin(T + 8)
    lw = workloads.make_layer_weights(wl.seed)
    w = oracle_weights(lw)
    dev = cuda_device
    g = torch.Generator(device=dev).manual_seed(wl.seed)
    rows = torch.randn(T, 576, generator=g, device=dev).to(BF)
    caches = []
    for r, (a, b) in enumerate(dist_mod.sequence_shards(T, world)):
        c = fleet.PagedLatentCache.for_lengths([b - a], extra_tokens=1 if r == world - 1 else 0, spare_pages=1,
                                               generator=torch.Generator().manual_seed(wl.seed + r), device=dev)
        c.write_rows(0, 0, rows[a:b])
        caches.append(c)
    x_n = workloads.make_hidden(wl.seed + 1, 1).float().numpy()[0]
    qn, kvn = O.project(cfg, w, x_n)
    runner = fleet.MlaDecodeAttention(fleet.ModelConfig(), fleet.LayerWeights(
        *(t.to(dev) for t in (lw.q_proj, lw.kv_a_proj_with_mqa, lw.kv_a_layernorm, lw.kv_b_proj))),
        torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev))
    q = torch.from_numpy(qn.reshape(1, -1)).to(BF).to(dev)
    kv_a = torch.from_numpy(kvn[None]).to(BF).to(dev)
    pos = torch.tensor([T], dtype=torch.int32, device=dev)
    gathered = dist_mod.emulate_sequence_shards(runner, q, kv_a, caches, pos)
    ex = dist_mod.ExchangeBuffers.local(world, max_batch=1)
    try:
        for step in range(2):  # both parities of the exchange buffers
            outs = dist_mod.emulate_exchange_step(runner, q, kv_a, caches, pos, ex)
            runner.check_errors()
            for r, o in enumerate(outs):
                assert torch.equal(o, gathered), f"world {world} step {step}: rank {r} differs from the gathered combine"
    finally:
        torch.cuda.synchronize()
        ex[0].close()
    new_row = O.kv_post(cfg, w, kvn, T, cos, sin)
    a, b = dist_mod.sequence_shards(T, world)[-1]
    dev_row = caches[-1].read_rows(0, b - a, 1)[0].float().cpu().numpy()
    np.testing.assert_allclose(dev_row, new_row, rtol=1e-2, atol=1e-6)
    want = O.attend_rows_fast(cfg, w, qn, np.concatenate([rows.float().cpu().numpy(), new_row[None]]), T, cos, sin)
    rel = _assert_close(outs[0][0].float().cpu().numpy(), want, f"config5b over {world} ranks")
    print(f"config5b x{world}: max rel {rel:.3e}")
