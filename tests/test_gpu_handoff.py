"""Prefill hand-off on the GPU (libmla_decode.so: mla_rows_to_pages): finished rows
scattered into pages exactly, raw kv_a rows turned into cache rows with the decode
step's arithmetic, the reference's cache file loaded into paged caches, a decode step
on top of a raw prefill, and bad positions / pages reported without a fault."""
import importlib

import numpy as np
import pytest
import torch

from mla_testlib import COS_MIN, REL_TIGHT, O, fleet, oracle_weights, rel_cos, workloads

pytestmark = pytest.mark.gpu
handoff = importlib.import_module("fleet-mi300x_b200.handoff")
BF = torch.bfloat16

LENS = [0, 1, 63, 64, 65, 300]
FIRST = [0, 5, 0, 64, 1, 0]


def _cache(dev, lens, first, seed):
    g = torch.Generator().manual_seed(seed)
    return fleet.PagedLatentCache.for_lengths([n + f for n, f in zip(lens, first)], extra_tokens=1, spare_pages=2,
                                              generator=g, device=dev)


def test_final_rows_scatter_exactly(cuda_device):
    cache = _cache(cuda_device, LENS, FIRST, 1)
    g = torch.Generator().manual_seed(2)
    rows = torch.randn(sum(LENS), 576, generator=g).to(BF)
    starts = np.concatenate([[0], np.cumsum(LENS)])
    before = cache.pages.float().cpu().numpy()
    handoff.rows_to_pages(cache, rows.to(cuda_device), starts, FIRST)
    want = before.copy()
    O.scatter_rows(want, cache.block_table.cpu().numpy(), rows.float().numpy(), starts, FIRST)
    assert np.array_equal(cache.pages.float().cpu().numpy(), want)


def test_raw_rows_match_oracle_kv_post(cuda_device):
    cfg, lw = fleet.ModelConfig(), workloads.make_layer_weights(7, norm="uniform")
    cos, sin = fleet.device_rope_tables(cfg, 512, cuda_device)
    cache = _cache(cuda_device, LENS, FIRST, 3)
    g = torch.Generator().manual_seed(4)
    raw = torch.randn(sum(LENS), 576, generator=g).to(BF)
    starts = np.concatenate([[0], np.cumsum(LENS)])
    handoff.rows_to_pages(cache, raw.to(cuda_device), starts, FIRST, raw=True,
                          norm_w=lw.kv_a_layernorm.to(cuda_device), cos=cos, sin=sin)
    ocfg, w = O.Config(), oracle_weights(lw)
    ocos, osin = ocfg.cos_sin(512)
    n_diff = n_all = 0
    for b, (n, f) in enumerate(zip(LENS, FIRST)):
        if n == 0:
            continue
        want = O.prefill_rows(ocfg, w, raw[starts[b]:starts[b + 1]].float().numpy(), f, ocos, osin)
        got = cache.read_rows(b, f, n).float().cpu().numpy()
        # the RMSNorm scale may differ by one fp32 ulp (sum order); an element on a bf16
        # rounding boundary then rounds the other way, in bf16(y) and again in
        # bf16(bf16(y) * gamma): at most two bf16 steps
        ratio = np.abs(got - want) / np.maximum(np.abs(want), 1e-30)
        worst = np.unravel_index(int(np.argmax(ratio)), ratio.shape)
        assert ratio.max() <= 2.0 ** -6, (f"request {b} row {worst[0]} col {worst[1]}: got {got[worst]}, "
                                          f"oracle {want[worst]}")
        n_diff += np.count_nonzero(got != want)
        n_all += got.size
    assert n_diff <= 0.002 * n_all, f"{n_diff} of {n_all} elements differ"


def test_decode_after_raw_prefill_matches_oracle(cuda_device):
    T = 700
    cfg, lw = fleet.ModelConfig(), workloads.make_layer_weights(8, norm="uniform")
    cos, sin = fleet.device_rope_tables(cfg, T + 8, cuda_device)
    w_dev = fleet.LayerWeights(*(t.to(cuda_device) for t in (lw.q_proj, lw.kv_a_proj_with_mqa, lw.kv_a_layernorm,
                                                              lw.kv_b_proj)))
    runner = fleet.MlaDecodeAttention(cfg, w_dev, cos, sin)
    cache = fleet.PagedLatentCache.for_lengths([T], spare_pages=1, generator=torch.Generator().manual_seed(9),
                                               device=cuda_device)
    g = torch.Generator().manual_seed(10)
    raw = torch.randn(T, 576, generator=g).to(BF)
    handoff.rows_to_pages(cache, raw.to(cuda_device), [0, T], raw=True, norm_w=w_dev.kv_a_layernorm, cos=cos, sin=sin)
    x = torch.randn(1, 2048, generator=g).to(BF)
    got = runner(x.to(cuda_device), cache)[0].float().cpu().numpy()
    runner.check_errors()
    ocfg, w = O.Config(), oracle_weights(lw)
    ocos, osin = ocfg.cos_sin(T + 8)
    flat = np.zeros((T + 1, 576), np.float32)
    flat[:T] = O.prefill_rows(ocfg, w, raw.float().numpy(), 0, ocos, osin)
    want = O.attention_task(ocfg, w, x[0].float().numpy(), flat, T, ocos, osin)
    rel, cs = rel_cos(got, want)
    assert rel <= REL_TIGHT and cs >= COS_MIN, (rel, cs)


def test_reference_cache_file_into_pages(cuda_device, tmp_path):
    layers, max_pos, S = 2, 200, 150
    g = torch.Generator().manual_seed(11)
    flat = torch.zeros(layers, max_pos, 576, dtype=BF)
    flat[:, :S] = torch.randn(layers, S, 576, generator=g).to(BF)
    path = tmp_path / "fleet_cache.bin"
    handoff.write_flat_cache(path, flat)
    caches = handoff.caches_from_flat(handoff.read_flat_cache(path, layers, max_pos), S, device=cuda_device,
                                      generator=torch.Generator().manual_seed(12))
    for l, c in enumerate(caches):
        assert int(c.seq_lens[0]) == S
        assert torch.equal(c.read_rows(0, 0, S).cpu(), flat[l, :S])


def test_bad_positions_and_pages_are_reported(cuda_device):
    cache = _cache(cuda_device, [10, 10], [0, 0], 13)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    rows = torch.ones(20, 576, dtype=BF, device=cuda_device)
    handoff.rows_to_pages(cache, rows, [0, 10, 20], [0, cache.max_blocks * 64 - 5], error_word=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 2  # MLA_DEV_BAD_POSITION; request 0's rows still landed
    assert torch.equal(cache.read_rows(0, 0, 10).cpu(), rows[:10].cpu())
    err.zero_()
    cache.block_table[1, 0] = cache.n_pages + 3
    handoff.rows_to_pages(cache, rows, [0, 10, 20], [0, 0], error_word=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 1  # MLA_DEV_BAD_PAGE
