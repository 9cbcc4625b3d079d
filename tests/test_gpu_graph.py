"""DecodeGraph: the captured step (with PDL edges between K1, K2 and K3) must give
bit-identical outputs and cache rows to the eager step, over a decode loop in which the
graph itself advances seq_lens."""
import pytest
import torch

from mla_testlib import fleet, workloads

pytestmark = pytest.mark.gpu
LENS = [0, 1, 63, 64, 100, 1000, 2047]


def _runner_and_cache(dev, seed=21):
    cfg = fleet.ModelConfig()
    cos, sin = fleet.device_rope_tables(cfg, 2200, dev)
    lw = workloads.make_layer_weights(seed)
    runner = fleet.MlaDecodeAttention(cfg, fleet.LayerWeights(
        *(t.to(dev) for t in (lw.q_proj, lw.kv_a_proj_with_mqa, lw.kv_a_layernorm, lw.kv_b_proj))), cos, sin)
    g = torch.Generator().manual_seed(seed)
    cache = fleet.PagedLatentCache.for_lengths(LENS, extra_tokens=8, spare_pages=2, generator=g, device=dev)
    cache.pages.copy_(torch.randn(cache.pages.shape, generator=g).to(torch.bfloat16))
    return runner, cache


def _clone(cache):
    c = fleet.PagedLatentCache(cache.n_pages, cache.batch, cache.max_blocks, device=cache.device)
    c.pages.copy_(cache.pages)
    c.block_table.copy_(cache.block_table)
    c.seq_lens.copy_(cache.seq_lens)
    return c


def test_graph_decode_loop_matches_eager(cuda_device):
    runner, cache_e = _runner_and_cache(cuda_device)
    cache_g = _clone(cache_e)
    graph = fleet.DecodeGraph(runner, cache_g, advance=True)
    g = torch.Generator().manual_seed(5)
    for step in range(4):
        x = torch.randn(len(LENS), 2048, generator=g).to(torch.bfloat16).to(cuda_device)
        want = runner(x, cache_e).clone()
        cache_e.advance()
        graph.x_n.copy_(x)
        got = graph.replay()
        torch.cuda.synchronize(cuda_device)
        runner.check_errors()
        assert torch.equal(got, want), f"step {step}: graph output differs from the eager step"
    assert torch.equal(cache_g.seq_lens, cache_e.seq_lens)
    assert torch.equal(cache_g.pages, cache_e.pages)


def test_graph_from_qkv_matches_eager(cuda_device):
    runner, cache = _runner_and_cache(cuda_device, seed=22)
    g = torch.Generator().manual_seed(6)
    q = torch.randn(len(LENS), 3072, generator=g).to(torch.bfloat16).to(cuda_device)
    kv_a = torch.randn(len(LENS), 576, generator=g).to(torch.bfloat16).to(cuda_device)
    want = runner.attend(q, kv_a, cache).clone()
    graph = fleet.DecodeGraph(runner, cache, inputs="qkv", q=q, kv_a=kv_a)
    for _ in range(3):
        got = graph.replay()
    torch.cuda.synchronize(cuda_device)
    runner.check_errors()
    assert torch.equal(got, want)


def test_host_pipeline_matches_eager_loop(cuda_device):
    runner, cache_e = _runner_and_cache(cuda_device, seed=23)
    cache_p = _clone(cache_e)
    pipe = fleet.HostPipeline(runner, cache_p, advance=True)
    g = torch.Generator().manual_seed(8)
    xs = [torch.randn(len(LENS), 2048, generator=g).to(torch.bfloat16).pin_memory() for _ in range(5)]
    got = []
    for k, x in enumerate(xs):
        got.append(pipe.submit(x))
        if k % 2 == 1:  # each host buffer is reused two steps later: read it before then
            pipe.wait()
            got[k - 1], got[k] = got[k - 1].clone(), got[k].clone()
    pipe.wait()
    got[-1] = got[-1].clone()
    for k, x in enumerate(xs):
        want = runner(x.to(cuda_device), cache_e).cpu()
        cache_e.advance()
        assert torch.equal(got[k], want), f"step {k}"
    runner.check_errors()
    assert torch.equal(cache_p.seq_lens, cache_e.seq_lens)
    assert torch.equal(cache_p.pages, cache_e.pages)


def test_host_step_graph_matches_eager_loop(cuda_device):
    """The one-graph host step (copy in, step, copy out): every replay copies the new
    host input and returns the eager step's output, and with advance=True the cache
    grows as the eager loop's does."""
    runner, cache_e = _runner_and_cache(cuda_device, seed=29)
    cache_h = _clone(cache_e)
    hsg = fleet.HostStepGraph(runner, cache_h, advance=True)
    g = torch.Generator().manual_seed(9)
    for k in range(4):
        x = torch.randn(len(LENS), 2048, generator=g).to(torch.bfloat16)
        hsg.x_host.copy_(x)
        got = hsg.replay()
        torch.cuda.synchronize(cuda_device)
        want = runner(x.to(cuda_device), cache_e).cpu()
        cache_e.advance()
        assert torch.equal(got, want), f"step {k}"
    runner.check_errors()
    assert torch.equal(cache_h.seq_lens, cache_e.seq_lens)
    assert torch.equal(cache_h.pages, cache_e.pages)


def _bad_entry(cache):
    """Point request 4's first logical page outside the pool (the kernels' bounds checks
    record MLA_DEV_BAD_PAGE and read page 0 instead; nothing faults)."""
    good = cache.block_table[4, 0].clone()
    cache.block_table[4, 0] = cache.n_pages + 7
    return good


def test_host_pipeline_raises_device_errors_without_check_errors(cuda_device):
    """A bad block-table entry in a pipelined decode loop surfaces as MlaError from the
    pipeline itself (wait(), or the next submit()), with no check_errors() call; once the
    table is repaired the loop runs on."""
    runner, cache = _runner_and_cache(cuda_device, seed=31)
    pipe = fleet.HostPipeline(runner, cache)
    x = torch.randn(len(LENS), 2048, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).pin_memory()
    pipe.submit(x)
    pipe.wait()
    good = _bad_entry(cache)
    pipe.submit(x)
    with pytest.raises(fleet.MlaError) as e:
        pipe.wait()
    assert e.value.code == 1
    cache.block_table[4, 0] = good
    pipe.submit(x)
    pipe.wait()  # the error was cleared when it was raised
    runner.check_errors()


def test_decode_graph_and_eager_calls_raise_device_errors(cuda_device):
    """The same through a replayed CUDA graph (raised by synchronize() or the next replay)
    and through the eager call (check='sync' raises at once; the default raises at the
    next call, without synchronising)."""
    runner, cache = _runner_and_cache(cuda_device, seed=32)
    graph = fleet.DecodeGraph(runner, cache)
    graph.replay()
    graph.synchronize()
    good = _bad_entry(cache)
    graph.replay()
    with pytest.raises(fleet.MlaError) as e:
        graph.synchronize()
    assert e.value.code == 1
    x = graph.x_n.clone()
    with pytest.raises(fleet.MlaError):
        runner(x, cache, check="sync")
    runner(x, cache)
    torch.cuda.synchronize(cuda_device)
    with pytest.raises(fleet.MlaError):
        runner(x, cache)  # raised before this call launches anything
    cache.block_table[4, 0] = good
    runner(x, cache, check="sync")
    graph.replay()
    graph.synchronize()
