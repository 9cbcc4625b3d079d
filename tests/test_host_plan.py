"""Host-side logic without a GPU: the split-KV plan arithmetic and the paged cache helpers.

The plan (fleet-mi300x_b200/csrc/mla_common.cuh: plan_begin / plan_cta_of, the cursor in
mla_attention.cu, the partial lookup in mla_merge.cu) is restated here in Python and
checked for exact coverage: every 64-token tile is owned by exactly one CTA, every
(CTA, request) segment gets its own partial slot c + b, and the merge finds exactly
the CTAs that wrote a request's partials.
"""
import importlib
import random

import pytest
import torch

fleet = importlib.import_module("fleet-mi300x_b200")
workloads = importlib.import_module("fleet-mi300x_b200.workloads")


def plan_begin(c, U, G):
    return c * U // G


def plan_cta_of(u, U, G):
    return ((u + 1) * G - 1) // U


def simulate(seq_lens, num_ctas):
    tiles = [(t + 1 + 63) // 64 for t in seq_lens]
    cum = [0]
    for n in tiles:
        cum.append(cum[-1] + n)
    U = cum[-1]
    G = min(num_ctas, U)
    owner = {}
    segments = []
    for c in range(G):
        u0, u1 = plan_begin(c, U, G), plan_begin(c + 1, U, G)
        assert u1 > u0, "every CTA with work gets at least one tile"
        for u in range(u0, u1):
            # upper_bound(cum[0..B], u) - 1
            b = max(i for i in range(len(tiles)) if cum[i] <= u)
            assert cum[b] <= u < cum[b + 1]
            assert u not in owner
            owner[u] = (c, b)
            if u == u0 or u == cum[b]:
                segments.append((c, b))
    assert sorted(owner) == list(range(U))
    slots = [c + b for c, b in segments]
    assert len(set(slots)) == len(slots), "partial slots are unique"
    assert max(slots) < num_ctas + len(tiles)
    for b in range(len(tiles)):
        c0, c1 = plan_cta_of(cum[b], U, G), plan_cta_of(cum[b + 1] - 1, U, G)
        writers = sorted(c for c, bb in segments if bb == b)
        assert writers == list(range(c0, c1 + 1)), (b, writers, c0, c1)
    return G, segments


@pytest.mark.parametrize("num_ctas", [1, 2, 3, 7, 148, 296, 4096])
def test_plan_edge_lengths(num_ctas):
    simulate([0, 1, 62, 63, 64, 65, 127, 128, 129, 200, 1000, 1023, 4095], num_ctas)


def test_plan_random():
    rng = random.Random(0)
    for _ in range(200):
        B = rng.randint(1, 40)
        lens = [rng.choice([0, 1, 63, 64, rng.randint(0, 5000)]) for _ in range(B)]
        simulate(lens, rng.choice([1, 2, 5, 17, 148, 300]))


def test_plan_baseline_configs():
    for name in ("config1", "config3", "config4"):
        simulate(workloads.WORKLOADS[name].seq_lens(), 148)
    # config 5a: 256 x 4097 rows -> 65 tiles each over 148 CTAs
    G, seg = simulate([4096] * 256, 148)
    assert G == 148 and len(seg) <= 148 + 256


def test_paged_cache_helpers_cpu():
    lengths = [0, 63, 64, 130]
    cache = fleet.PagedLatentCache.for_lengths(lengths, spare_pages=2, permute=True,
                                               generator=torch.Generator().manual_seed(0), device="cpu")
    assert cache.batch == 4 and cache.max_blocks == 3
    assert cache.seq_lens.tolist() == lengths
    used = [int(x) for b, n in enumerate(lengths) for x in cache.block_table[b, : (n + 1 + 63) // 64]]
    assert len(set(used)) == len(used), "no page is shared between requests"
    assert all(0 <= x < cache.n_pages for x in used)
    rows = torch.randn(130, 576).to(torch.bfloat16)
    cache.write_rows(3, 0, rows)
    assert torch.equal(cache.read_rows(3, 0, 130), rows)
    assert torch.equal(cache.read_rows(3, 64, 1)[0], rows[64])
    cache.advance()
    assert cache.seq_lens.tolist() == [n + 1 for n in lengths]


def test_byte_accounting():
    assert workloads.kv_bytes([1024]) == 1025 * 1152
    assert workloads.kv_bytes([4096] * 256) == 256 * 4097 * 1152
    # W_UK + W_UV = 4,194,304 B is part of the total
    assert workloads.total_bytes([1024]) - workloads.kv_bytes([1024]) == 4194304 + 3072 * 2 + 576 * 2 + 1152 + 4096


def test_model_config_refuses_other_shapes():
    cfg = fleet.ModelConfig(kv_lora_rank=256)
    with pytest.raises(ValueError):
        cfg.check_supported()
    fleet.ModelConfig().check_supported()


def test_no_cpu_path_without_cuda_tensors():
    lw = workloads.make_layer_weights(0)
    cfg = fleet.ModelConfig()
    cos, sin = fleet.rope_tables(cfg, 16)
    with pytest.raises(RuntimeError):
        fleet.MlaDecodeAttention(cfg, lw, torch.from_numpy(cos), torch.from_numpy(sin))


def test_row_stride_of_single_row_views():
    att = importlib.import_module("fleet-mi300x_b200.attention")
    import numpy as np
    v = torch.from_numpy(np.zeros(576, np.float32)[None])  # NumPy broadcast view: batch stride 0
    assert v.stride(0) == 0 and att._row_stride(v) == 576
    w = torch.zeros(4, 3648)[:, :3072]
    assert att._row_stride(w) == 3648
