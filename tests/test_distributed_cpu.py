"""Multi-GPU host logic on CPU: shard plans and the sequence-sharded exchange protocol.

The protocol runs as two gloo ranks: each computes its range's partial with the
oracle, the partials are all-gathered, and every rank combines them in sequence
order. The result must equal unsharded attention over all rows.
"""
import importlib
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mla_testlib import O, rel_cos, workloads

dist_mod = importlib.import_module("fleet-mi300x_b200.distributed")


@pytest.mark.parametrize("cached,world", [(0, 1), (0, 4), (1, 2), (63, 2), (64, 2), (4095, 8), (131072, 8), (100, 4)])
def test_sequence_shards_cover_page_aligned(cached, world):
    r = dist_mod.sequence_shards(cached, world)
    assert len(r) == world
    assert r[0][0] == 0 and r[-1][1] == cached
    for (a, b), (c, d) in zip(r, r[1:]):
        assert b == c and a <= b
    for a, b in r[:-1]:
        assert a % 64 == 0 and b % 64 == 0
    sizes = [b - a for a, b in r]
    # balanced to within a page (the last range also attends the new row)
    assert max(sizes) - min(sizes) <= 64 + 1 or cached < 64 * world


def test_request_shard_balanced():
    lens = workloads.WORKLOADS["config3"].seq_lens()
    owners = [dist_mod.request_shard(lens, 4, r) for r in range(4)]
    assert sorted(b for o in owners for b in o) == list(range(len(lens)))
    loads = [sum(lens[b] + 1 for b in o) for o in owners]
    assert max(loads) - min(loads) <= max(lens) + 1


def _problem(T, seed=3):
    cfg = O.Config()
    cos, sin = cfg.cos_sin(T + 8)
    lw = workloads.make_layer_weights(seed, norm="uniform")
    w = O.Weights(*(t.float().numpy() for t in (lw.q_proj, lw.kv_a_proj_with_mqa, lw.kv_a_layernorm, lw.kv_b_proj)))
    rows = workloads.make_cache_rows(seed + 1, T, torch.from_numpy(cos), torch.from_numpy(sin)).float().numpy()
    x_n = workloads.make_hidden(seed + 2, 1).float().numpy()[0]
    q, kv_a = O.project(cfg, w, x_n)
    new_row = O.kv_post(cfg, w, kv_a, T, cos, sin)
    full = O.attend_rows(cfg, w, q, np.concatenate([rows, new_row[None]]), T, cos, sin)
    return cfg, w, q, rows, new_row, cos, sin, full


def _rank_partial(cfg, w, q, rows, new_row, cos, sin, T, world, rank):
    a, b = dist_mod.sequence_shards(T, world)[rank]
    mine = rows[a:b]
    if rank == world - 1:
        mine = np.concatenate([mine, new_row[None]])
    return O.attend_rows_partial(cfg, w, q, mine, T, cos, sin)


@pytest.mark.parametrize("T,world", [(1000, 3), (130, 4), (63, 2)])
def test_shard_combine_equals_full(T, world):
    cfg, w, q, rows, new_row, cos, sin, full = _problem(T)
    parts = [_rank_partial(cfg, w, q, rows, new_row, cos, sin, T, world, r) for r in range(world)]
    got = O.combine_partials(parts)
    rel, cs = rel_cos(got, full)
    assert rel <= 1e-2 and cs >= 0.99999, (rel, cs)


def _worker(rank, world, port, T, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, w, q, rows, new_row, cos, sin, full = _problem(T)
        y, m, L = _rank_partial(cfg, w, q, rows, new_row, cos, sin, T, world, rank)
        local = torch.zeros(16, 132, dtype=torch.float32)
        local[:, :128] = torch.from_numpy(y)
        local[:, 128] = torch.from_numpy(m)
        local[:, 129] = torch.from_numpy(L)
        gathered = [torch.zeros_like(local) for _ in range(world)]
        dist.all_gather(gathered, local)
        parts = [(g[:, :128].numpy(), g[:, 128].numpy(), g[:, 129].numpy()) for g in gathered]
        got = O.combine_partials(parts)
        rel, cs = rel_cos(got, full)
        result_q.put((rank, rel, cs, got.tobytes()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_gloo_two_ranks_sequence_sharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, T = 2, 700
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, T, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    for rank, rel, cs, _ in res:
        assert rel <= 1e-2 and cs >= 0.99999, (rank, rel, cs)
    assert res[0][3] == res[1][3], "every rank must hold the same combined output"


# ---------------------------------------------------------------- peer exchange (host side)
native = importlib.import_module("fleet-mi300x_b200.native")


def _align256(x):
    return (x + 255) // 256 * 256


@pytest.mark.parametrize("world,max_batch", [(1, 1), (2, 1), (8, 1), (3, 70), (8, 256), (2, 16), (2, 17)])
def test_exchange_buffer_size(world, max_batch):
    """mla_exchange_bytes (host arithmetic, no GPU): the step counter and two parities of
    [world][max_batch][16 heads][65] step-tagged 16-byte lines (64 lines of y pairs and
    one of m, L), each region 256-byte aligned."""
    want = 256 + _align256(2 * world * max_batch * 16 * 65 * 16)
    assert dist_mod.exchange_bytes(world, max_batch) == want


def test_exchange_buffer_size_refused():
    import ctypes
    lib = native.load_library()
    n = ctypes.c_uint64()
    assert lib.mla_exchange_bytes(0, 1, ctypes.byref(n)) == -1
    assert lib.mla_exchange_bytes(native.MAX_RANKS + 1, 1, ctypes.byref(n)) == -8
    assert lib.mla_exchange_bytes(2, 0, ctypes.byref(n)) == -1


def test_exchange_views_fill_params():
    ex = dist_mod.ExchangeBuffers([0x1000, 0x2000, 0x3000], 1, 3, 5, timeout_us=777)
    p = native.new_params()
    ex.apply(p)
    assert list(p.exchange)[:3] == [0x1000, 0x2000, 0x3000]
    assert all(v is None for v in list(p.exchange)[3:])
    assert (p.rank, p.world, p.exchange_batch, p.exchange_timeout_us) == (1, 3, 5, 777)
    with pytest.raises(ValueError):
        dist_mod.ExchangeBuffers([0] * 9, 0, 9, 1)
    with pytest.raises(ValueError):
        dist_mod.ExchangeBuffers([0, 0], 2, 2, 1)


def _handle_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        got = dist_mod.gather_handles(bytes([rank + 1]) * native.IPC_HANDLE_BYTES, world)
        q.put((rank, got))
    finally:
        dist.destroy_process_group()


def test_gloo_ranks_gather_ipc_handles():
    """The handle exchange of ExchangeBuffers.create: every rank ends with every
    rank's handle in rank order."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world = 3
    port = _free_port()
    procs = [ctx.Process(target=_handle_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = [bytes([r + 1]) * native.IPC_HANDLE_BYTES for r in range(world)]
    for rank, got in res:
        assert got == want, rank
