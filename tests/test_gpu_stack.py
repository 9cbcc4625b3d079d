"""LayerStackGraph: a decode step over a stack of layers as one CUDA graph (the B200 form
of the reference's all-layers persistent loop, src/kernels/fleet_kernel.hip:938-1043).

Over two decode steps (the graph advances seq_lens itself), the replayed stack must give
the eager layer loop's outputs and cache rows bit for bit:
  slice mode  each layer's K1-K3 from its own q / kv_a over its own cache;
  block mode  the hidden state through input RMSNorm, K0-K5 (projection, attention, o_proj
              and the residual in the library) and a torch FFN with its residual, per layer.
"""
import pytest
import torch
import torch.nn.functional as F

from mla_testlib import fleet, workloads

pytestmark = pytest.mark.gpu
graph_mod = __import__("importlib").import_module("fleet-mi300x_b200.graph")
LENS = [0, 63, 64, 700, 2047]
LAYERS = 3


def _layers(dev, seed, with_o=False):
    cfg = fleet.ModelConfig()
    cos, sin = fleet.device_rope_tables(cfg, 2200, dev)
    runners, caches = [], []
    for l in range(LAYERS):
        lw = workloads.make_layer_weights(seed + l)
        ts = (lw.q_proj, lw.kv_a_proj_with_mqa, lw.kv_a_layernorm, lw.kv_b_proj) + ((lw.o_proj,) if with_o else ())
        runners.append(fleet.MlaDecodeAttention(cfg, fleet.LayerWeights(*(t.to(dev) for t in ts)), cos, sin))
        g = torch.Generator().manual_seed(seed + 100 + l)
        c = fleet.PagedLatentCache.for_lengths(LENS, extra_tokens=4, spare_pages=2, generator=g, device=dev)
        c.pages.copy_(torch.randn(c.pages.shape, generator=g).to(torch.bfloat16))
        caches.append(c)
    return runners, caches


def _clone(cache):
    c = fleet.PagedLatentCache(cache.n_pages, cache.batch, cache.max_blocks, device=cache.device)
    c.pages.copy_(cache.pages)
    c.block_table.copy_(cache.block_table)
    c.seq_lens.copy_(cache.seq_lens)
    return c


def test_stack_slice_mode_matches_eager_loop(cuda_device):
    runners, caches_g = _layers(cuda_device, seed=40)
    caches_e = [_clone(c) for c in caches_g]
    stack = fleet.LayerStackGraph(runners, caches_g, mode="slice", advance=True)
    g = torch.Generator().manual_seed(41)
    B = len(LENS)
    for step in range(2):
        qs = [torch.randn(B, 3072, generator=g).to(torch.bfloat16).to(cuda_device) for _ in range(LAYERS)]
        kvs = [torch.randn(B, 576, generator=g).to(torch.bfloat16).to(cuda_device) for _ in range(LAYERS)]
        want = []
        for l in range(LAYERS):
            want.append(runners[l].attend(qs[l], kvs[l], caches_e[l]).clone())
            caches_e[l].advance()
            stack.q[l].copy_(qs[l])
            stack.kv_a[l].copy_(kvs[l])
        stack.replay()
        stack.synchronize()
        for l in range(LAYERS):
            assert torch.equal(stack.out[l], want[l]), f"step {step} layer {l}"
    for ce, cg in zip(caches_e, caches_g):
        assert torch.equal(ce.seq_lens, cg.seq_lens)
        assert torch.equal(ce.pages, cg.pages)


def test_stack_block_mode_matches_eager_loop(cuda_device):
    runners, caches_g = _layers(cuda_device, seed=50, with_o=True)
    caches_e = [_clone(c) for c in caches_g]
    B, H = len(LENS), 2048
    g = torch.Generator().manual_seed(51)
    norms = [(1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).to(cuda_device) for _ in range(LAYERS)]
    ffn_w = [((torch.randn(2 * 512, H, generator=g) * 0.02).to(torch.bfloat16).to(cuda_device),
              (torch.randn(H, 512, generator=g) * 0.02).to(torch.bfloat16).to(cuda_device)) for _ in range(LAYERS)]

    def ffn(l, h):
        gate, up = F.linear(graph_mod.rms_norm_bf16(h, norms[l]), ffn_w[l][0]).chunk(2, dim=-1)
        h.add_(F.linear(F.silu(gate) * up, ffn_w[l][1]))

    h0 = torch.randn(B, H, generator=g).to(torch.bfloat16).to(cuda_device)
    stack = fleet.LayerStackGraph(runners, caches_g, mode="block", in_norms=norms, ffn=ffn, advance=True,
                                  h=h0.clone())
    h_e = h0.clone()
    for step in range(2):
        for l in range(LAYERS):
            x_n = graph_mod.rms_norm_bf16(h_e, norms[l])
            runners[l].attention_block(x_n, caches_e[l], h_e, h_out=h_e)
            ffn(l, h_e)
            caches_e[l].advance()
        stack.replay()
        stack.synchronize()
        assert torch.equal(stack.h, h_e), f"step {step}: hidden state differs from the eager loop"
    for ce, cg in zip(caches_e, caches_g):
        assert torch.equal(ce.pages, cg.pages)
