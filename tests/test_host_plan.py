"""Host-side logic without a GPU: the split-KV plan arithmetic and the paged cache helpers.

The plan (fleet-mi300x_b200/csrc/mla_common.cuh: plan_begin / plan_cta_of, the cursor in
mla_attention.cu, the partial lookup in mla_merge.cu) is restated here in Python and
checked for exact coverage: every tile (UNIT rows: the default split-KV kernel's 32-row
half pages) is owned by exactly one CTA, every
(CTA, request) segment gets its own partial slot c + b, and the merge finds exactly
the CTAs that wrote a request's partials.
"""
import importlib
import random

import pytest
import torch

fleet = importlib.import_module("fleet-mi300x_b200")
workloads = importlib.import_module("fleet-mi300x_b200.workloads")


UNIT = 32  # mla_common.cuh:plan_unit_rows for the default split-KV kernel


def tiles_of(seq_lens, unit=UNIT):
    """plan_tiles: the cached rows plus the new one, in tiles of `unit` rows."""
    return [(t + 1 + unit - 1) // unit for t in seq_lens]


def plan_begin(c, U, G):
    return c * U // G


def plan_cta_of(u, U, G):
    return ((u + 1) * G - 1) // U


def simulate(seq_lens, num_ctas):
    tiles = tiles_of(seq_lens)
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
    simulate([0, 1, 30, 31, 32, 33, 62, 63, 64, 65, 127, 128, 129, 200, 1000, 1023, 4095], num_ctas)


def test_plan_random():
    rng = random.Random(0)
    for _ in range(200):
        B = rng.randint(1, 40)
        lens = [rng.choice([0, 1, 63, 64, rng.randint(0, 5000)]) for _ in range(B)]
        simulate(lens, rng.choice([1, 2, 5, 17, 148, 300]))


def test_plan_baseline_configs():
    for name in ("config1", "config3", "config4"):
        simulate(workloads.WORKLOADS[name].seq_lens(), 148)
    # config 5a: 256 x 4097 rows -> 129 half-page tiles each over 148 CTAs
    G, seg = simulate([4096] * 256, 148)
    assert G == 148 and len(seg) <= 148 + 256
    assert tiles_of([4096]) == [129] and tiles_of([4096], 64) == [65]


def k2_grid(num_ctas, sm_count):
    """mla_common.cuh:k2_grid."""
    two = (num_ctas + 1) // 2
    return num_ctas if num_ctas <= sm_count else max(two, sm_count)


def k2_pairs(num_ctas, sm_count):
    """mla_common.cuh:k2_pairs (default split-KV kernel)."""
    return num_ctas % 2 == 0 and 2 * k2_grid(num_ctas, sm_count) == num_ctas


def paired_slots(seq_lens, num_ctas):
    """The pair merge of mla_attention_mma.cu: plan CTAs 2k, 2k + 1 run in kernel CTA k;
    where their boundary falls inside a request, 2k + 1's first segment is merged into
    2k's last one. Returns, per request, the slots written, in tile order."""
    G, segments = simulate(seq_lens, num_ctas)
    tiles = tiles_of(seq_lens)
    cum = [0]
    for n in tiles:
        cum.append(cum[-1] + n)
    U = cum[-1]
    by_cta = {}
    for c, b in segments:
        by_cta.setdefault(c, []).append(b)
    written = {b: [] for b in range(len(tiles))}
    for c in range(G):
        for i, b in enumerate(by_cta[c]):
            mid = plan_begin(c, U, G)
            merged_away = c % 2 == 1 and i == 0 and cum[b] < mid  # group 1's first segment, request started before
            if not merged_away:
                written[b].append(c)
    return G, cum, written


def part_idx(c0, c1, paired):
    """mla_merge.cu:PartIdx over a request's plan CTAs [c0, c1]."""
    if not paired:
        return list(range(c0, c1 + 1))
    n = 1 + (c1 >> 1) - (c0 >> 1)
    return [c0 if e == 0 else 2 * ((c0 >> 1) + e) for e in range(n)]


@pytest.mark.parametrize("T,num_ctas,sms,expect", [
    (131071, 296, 148, True), (65535, 296, 148, True), (9440, 296, 148, True),  # 296 tiles: G = num_ctas
    (9439, 296, 148, False),  # 295 tiles: G < num_ctas
    (1023, 296, 148, False), (131071, 148, 148, False), (131071, 200, 148, False), (131071, 400, 148, True),
    (9000, 296, 148, False), (18880, 296, 148, True)])
def test_pair_merge_single_request(T, num_ctas, sms, expect):
    """One request: every boundary between 2k and 2k + 1 is inside it, so the slots are 0, 2, 4, ..."""
    G, cum, written = paired_slots([T], num_ctas)
    paired = k2_pairs(num_ctas, sms) and G == num_ctas
    assert paired == expect
    if paired:
        U = cum[-1]
        assert written[0] == part_idx(plan_cta_of(0, U, G), plan_cta_of(U - 1, U, G), True)
        assert written[0] == list(range(0, G, 2))


def test_pair_merge_random_batches():
    """Ragged batches (empty requests, requests inside one plan CTA, requests across many): the
    slots K3 enumerates with PartIdx are exactly those the pair-merged split-KV kernel writes,
    in tile order, and each written slot is unique."""
    rng = random.Random(7)
    for _ in range(300):
        B = rng.randint(1, 60)
        lens = [rng.choice([0, 1, 63, 64, 127, rng.randint(0, 3000), rng.randint(0, 40000)]) for _ in range(B)]
        num_ctas = rng.choice([2, 4, 16, 296, 400])
        G, cum, written = paired_slots(lens, num_ctas)
        if G != num_ctas:
            continue
        U = cum[-1]
        slots = []
        for b in range(B):
            if cum[b + 1] == cum[b]:
                assert written[b] == []
                continue
            c0, c1 = plan_cta_of(cum[b], U, G), plan_cta_of(cum[b + 1] - 1, U, G)
            assert written[b] == part_idx(c0, c1, True), (lens, num_ctas, b)
            slots += [c + b for c in written[b]]
        assert len(set(slots)) == len(slots)


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
