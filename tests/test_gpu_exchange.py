"""The peer-memory shard exchange on the GPU (libmla_decode.so: K3 in exchange mode,
K4 = mla_exchange_combine): K3 stores each shard's partial into every rank's exchange
buffer and raises flags there, K4 waits for the flags and combines in rank order.

On one device the ranks are emulated: every rank's K1-K3 run one after another, then
every rank's K4, so each K4 starts after all flags it waits for are set. The result
must equal the NCCL path's (local partials, gathered, mla_combine_shards) bit for bit,
since both fold the same fp32 partials in the same order. With two devices the ranks
run as processes, one per GPU, the buffers mapped through CUDA IPC.
"""
import datetime
import importlib
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from mla_testlib import COS_MIN, REL_TIGHT, O, fleet, oracle_weights, rel_cos, workloads

pytestmark = pytest.mark.gpu
dist_mod = importlib.import_module("fleet-mi300x_b200.distributed")
native = importlib.import_module("fleet-mi300x_b200.native")
BF = torch.bfloat16


def _runner(dev, seed=3, max_pos=8192):
    cfg = O.Config()
    cos, sin = cfg.cos_sin(max_pos)
    lw = workloads.make_layer_weights(seed, norm="uniform")
    runner = fleet.MlaDecodeAttention(fleet.ModelConfig(), fleet.LayerWeights(
        *(t.to(dev) for t in (lw.q_proj, lw.kv_a_proj_with_mqa, lw.kv_a_layernorm, lw.kv_b_proj))),
        torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev))
    return runner, lw, cfg, cos, sin


def _sharded_caches(lengths, world, dev, seed):
    """Random cache rows for each request, split into each rank's cache by
    sequence_shards (the last rank owns the new row)."""
    g = torch.Generator().manual_seed(seed)
    rows = [torch.randn(n, 576, generator=g).to(BF) for n in lengths]
    caches = []
    for r in range(world):
        ranges = [dist_mod.sequence_shards(n, world)[r] for n in lengths]
        c = fleet.PagedLatentCache.for_lengths([b - a for a, b in ranges], extra_tokens=1 if r == world - 1 else 0,
                                               spare_pages=1, generator=torch.Generator().manual_seed(seed + r),
                                               device=dev)
        for i, (a, b) in enumerate(ranges):
            if b > a:
                c.write_rows(i, 0, rows[i][a:b].to(dev))
        caches.append(c)
    return caches, rows


def _inputs(B, dev, seed):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, 3072, generator=g) * 0.5).to(BF).to(dev)
    kv_a = torch.randn(B, 576, generator=g).to(BF).to(dev)
    return q, kv_a


@pytest.mark.parametrize("lengths,world", [([5000], 3), ([130], 4), ([64], 2), ([4095], 8), ([300] * 5, 2),
                                           ([37 * i + 5 for i in range(70)], 3),
                                           ([411 * i + 7 for i in range(13)], 2),  # K3 in two blocks of 8
                                           ([40000], 2)])  # shards of 626 half-page tiles: pair-merged partials
def test_emulated_exchange_equals_gathered_combine(cuda_device, lengths, world):
    runner, *_ = _runner(cuda_device, max_pos=max(8192, max(lengths) + 8))
    B = len(lengths)
    caches, _ = _sharded_caches(lengths, world, cuda_device, seed=11)
    q, kv_a = _inputs(B, cuda_device, seed=12)
    pos = torch.tensor(lengths, dtype=torch.int32, device=cuda_device)
    want = dist_mod.emulate_sequence_shards(runner, q, kv_a, caches, pos)
    ex = dist_mod.ExchangeBuffers.local(world, max_batch=B + 3)
    try:
        for step in range(3):  # three steps: both parities of the buffers, then the first again
            outs = dist_mod.emulate_exchange_step(runner, q, kv_a, caches, pos, ex)
            runner.check_errors()
            for r, o in enumerate(outs):
                assert torch.equal(o, want), (step, r)
    finally:
        torch.cuda.synchronize()
        ex[0].close()


@pytest.mark.parametrize("T", [6000, 40000])  # 40000: each shard's split plan is pair-merged (k2_pairs)
def test_exchange_matches_oracle(cuda_device, T):
    world = 2
    runner, lw, cfg, cos, sin = _runner(cuda_device, seed=5, max_pos=max(8192, T + 8))
    w = oracle_weights(lw)
    rows = workloads.make_cache_rows(6, T, torch.from_numpy(cos), torch.from_numpy(sin))
    x_n = workloads.make_hidden(7, 1).float().numpy()[0]
    qn, kvn = O.project(cfg, w, x_n)
    new_row = O.kv_post(cfg, w, kvn, T, cos, sin)
    want = O.attend_rows(cfg, w, qn, np.concatenate([rows.float().numpy(), new_row[None]]), T, cos, sin)
    caches = []
    for r, (a, b) in enumerate(dist_mod.sequence_shards(T, world)):
        c = fleet.PagedLatentCache.for_lengths([b - a], extra_tokens=1 if r == world - 1 else 0, spare_pages=1,
                                               generator=torch.Generator().manual_seed(r), device=cuda_device)
        c.write_rows(0, 0, rows[a:b].to(cuda_device))
        caches.append(c)
    q = torch.from_numpy(qn.reshape(1, -1)).to(BF).to(cuda_device)
    kv_a = torch.from_numpy(kvn[None]).to(BF).to(cuda_device)
    pos = torch.tensor([T], dtype=torch.int32, device=cuda_device)
    ex = dist_mod.ExchangeBuffers.local(world, max_batch=1)
    try:
        outs = dist_mod.emulate_exchange_step(runner, q, kv_a, caches, pos, ex)
        runner.check_errors()
        rel, cs = rel_cos(outs[0][0].float().cpu().numpy(), want)
        assert rel <= REL_TIGHT and cs >= COS_MIN, (rel, cs)
        assert torch.equal(outs[0], outs[1])
    finally:
        torch.cuda.synchronize()
        ex[0].close()


@pytest.mark.parametrize("split", [False, True], ids=["fused", "split"])
@pytest.mark.parametrize("lengths", [[700, 1, 64, 4000], [int(x) for x in np.random.default_rng(5).integers(0, 300, 150)],
                                     [int(x) for x in np.random.default_rng(6).integers(0, 300, 300)]],
                         ids=["cluster-form", "b150-32-blocks", "b300-not-resident"])
def test_world1_exchange_step_equals_local_combine(cuda_device, lengths, split):
    """One shard, the whole step in one call: K3 fused with the combine where its grid
    is resident at once (4 requests: 64 cluster CTAs; 150: 80 CTAs of 32 requests),
    else, or with MLA_FLAG_EXCHANGE_SPLIT, K3 + K4 (300 requests: 160 CTAs). Either
    equals shard_out + mla_combine_shards bit for bit."""
    runner, *_ = _runner(cuda_device)
    if split:
        runner.flags |= native.FLAG_EXCHANGE_SPLIT
    caches, _ = _sharded_caches(lengths, 1, cuda_device, seed=21)
    q, kv_a = _inputs(len(lengths), cuda_device, seed=22)
    part = torch.empty(len(lengths), 16, native.SHARD_STRIDE, dtype=torch.float32, device=cuda_device)
    runner.attend(q, kv_a, caches[0], shard_out=part)
    want = fleet.combine_shards(part[None])
    ex = dist_mod.ExchangeBuffers.local(1, max_batch=len(lengths))
    try:
        for _ in range(3):
            got = runner.attend(q, kv_a, caches[0], exchange=ex[0])
            runner.check_errors()
            assert torch.equal(got, want)
    finally:
        torch.cuda.synchronize()
        ex[0].close()


def test_exchange_step_in_cuda_graph(cuda_device):
    """The emulated two-rank step captured once and replayed: the step counter lives in
    device memory, so every replay flips the parity by itself."""
    runner, *_ = _runner(cuda_device)
    lengths = [3000]
    caches, _ = _sharded_caches(lengths, 2, cuda_device, seed=31)
    q, kv_a = _inputs(1, cuda_device, seed=32)
    pos = torch.tensor(lengths, dtype=torch.int32, device=cuda_device)
    want = dist_mod.emulate_sequence_shards(runner, q, kv_a, caches, pos)
    ex = dist_mod.ExchangeBuffers.local(2, max_batch=1)
    try:
        side = torch.cuda.Stream(cuda_device)
        side.wait_stream(torch.cuda.current_stream(cuda_device))
        with torch.cuda.stream(side):
            outs = dist_mod.emulate_exchange_step(runner, q, kv_a, caches, pos, ex)
        torch.cuda.current_stream(cuda_device).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            outs = dist_mod.emulate_exchange_step(runner, q, kv_a, caches, pos, ex)
        for _ in range(3):
            for o in outs:
                o.zero_()
            g.replay()
            torch.cuda.synchronize()
            runner.check_errors()
            assert all(torch.equal(o, want) for o in outs)
    finally:
        torch.cuda.synchronize()
        ex[0].close()


@pytest.mark.parametrize("split", [False, True], ids=["fused", "split"])
def test_missing_peer_times_out_with_error(cuda_device, split):
    """Rank 1 never runs: rank 0's combine (the fused K3, or K4) waits for lines nothing
    writes, gives up after the limit, records MLA_DEV_PEER_TIMEOUT and writes zeros.
    The context stays usable."""
    runner, *_ = _runner(cuda_device)
    if split:
        runner.flags |= native.FLAG_EXCHANGE_SPLIT
    caches, _ = _sharded_caches([500], 2, cuda_device, seed=41)
    q, kv_a = _inputs(1, cuda_device, seed=42)
    pos = torch.tensor([500], dtype=torch.int32, device=cuda_device)
    ex = dist_mod.ExchangeBuffers.local(2, max_batch=1, timeout_us=20_000)
    try:
        out = torch.full((1, 2048), 1.0, dtype=BF, device=cuda_device)
        runner.attend(q, kv_a, caches[0], out, rope_pos=pos, new_row=False, exchange=ex[0])
        torch.cuda.synchronize()
        with pytest.raises(fleet.MlaError) as e:  # clears the device and the host error word
            runner.check_errors()
        assert e.value.code == 4  # MLA_DEV_PEER_TIMEOUT
        assert not out.float().abs().sum().item()
        # the device still runs work after the timed-out wait
        again = runner.attend(q, kv_a, caches[1], rope_pos=pos, new_row=True)
        torch.cuda.synchronize()
        runner.check_errors()
        assert torch.isfinite(again.float()).all()
    finally:
        torch.cuda.synchronize()
        ex[0].close()


def test_exchange_params_refused(cuda_device):
    runner, *_ = _runner(cuda_device)
    caches, _ = _sharded_caches([100, 100], 1, cuda_device, seed=51)
    q, kv_a = _inputs(2, cuda_device, seed=52)
    ex = dist_mod.ExchangeBuffers.local(2, max_batch=1)
    try:
        with pytest.raises(ValueError):  # batch above the buffers' size
            runner.attend(q, kv_a, caches[0], exchange=ex[0])
        p = runner.params(q, kv_a, caches[0], torch.empty(2, 2048, dtype=BF, device=cuda_device))
        ex[0].apply(p)
        p.exchange_batch = 2
        p.rank = 2  # outside the world
        s = torch.cuda.current_stream(cuda_device).cuda_stream
        import ctypes
        assert runner.lib.mla_decode_step(ctypes.byref(p), ctypes.c_void_p(s)) == -1
        p.rank, p.exchange_batch = 0, 1
        assert runner.lib.mla_decode_step(ctypes.byref(p), ctypes.c_void_p(s)) == -8  # batch 2 > 1
        p.exchange_batch = 2
        p.exchange[1] = p.exchange[1] + 8  # not 256-byte aligned
        assert runner.lib.mla_decode_step(ctypes.byref(p), ctypes.c_void_p(s)) == -3
    finally:
        torch.cuda.synchronize()
        ex[0].close()


def _peer_worker(rank, world, port, T, q_out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    ex = None
    try:
        runner, lw, cfg, cos, sin = _runner(dev, seed=5, max_pos=T + 8)
        caches, rows = _sharded_caches([T], world, dev, seed=61)
        q, kv_a = _inputs(1, dev, seed=62)
        pos = torch.tensor([T], dtype=torch.int32, device=dev)
        ex = dist_mod.ExchangeBuffers.create(rank, world, max_batch=1)
        step = dist_mod.SequenceShardedAttention(runner, rank, world, exchange=ex)
        runner.project = lambda x: (q, kv_a)
        x0 = torch.zeros(1, 2048, dtype=BF, device=dev)
        outs = [step.step(x0, caches[rank], pos).clone() for _ in range(3)]  # fused K3 (grid resident)
        runner.flags |= native.FLAG_EXCHANGE_SPLIT
        outs += [step.step(x0, caches[rank], pos).clone() for _ in range(2)]  # K3 + K4
        runner.flags &= ~native.FLAG_EXCHANGE_SPLIT
        outs += [step.step(x0, caches[rank], pos).clone()]  # and back: the step counter is shared
        torch.cuda.synchronize()
        runner.check_errors()
        # the same step on this GPU alone, all ranks emulated, gathered combine
        want = dist_mod.emulate_sequence_shards(runner, q, kv_a, caches, pos)
        same = all(torch.equal(o, want) for o in outs)
        dist.barrier()
        q_out.put((rank, same, outs[0].float().cpu().numpy()))
    except Exception as e:  # report instead of leaving the parent waiting on the queue
        q_out.put((rank, repr(e), None))
        raise
    finally:
        if ex is not None:
            torch.cuda.synchronize()
            dist.barrier()
            ex.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_exchange_gpus(world):
    """One process per GPU (2, and 4 or 8 where the box has them), buffers mapped through IPC."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    qq = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, 9000, qq)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([qq.get(timeout=300) for _ in range(world)], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=120)
    assert all(same is True for _, same, _ in res), [(r, s) for r, s, _ in res]
    assert all(p.exitcode == 0 for p in procs)
    assert all(np.array_equal(res[0][2], x[2]) for x in res[1:])
