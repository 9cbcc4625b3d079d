"""Parity of the B200 path (libmla_decode.so through its C ABI) with the oracle.

Golden cases compare against the reference's own outputs; paged/ragged batches and
the full-size configs compare against the oracle restatement on the same seeded
inputs. Bar: max relative error <= 2e-2 on the bf16 outputs (the north star's
tolerance), held here to REL_TIGHT with a cosine floor.
"""
import numpy as np
import pytest
import torch

from mla_testlib import COS_MIN, REL_TIGHT, REL_TOL, GoldenCase, O, fleet, oracle_weights, rel_cos, workloads

pytestmark = pytest.mark.gpu

BF = torch.bfloat16


def to_dev(lw, dev):
    return fleet.LayerWeights(*(t.to(dev) for t in (lw.q_proj, lw.kv_a_proj_with_mqa, lw.kv_a_layernorm,
                                                      lw.kv_b_proj)))


def assert_close(got, want, what, rel_tol=REL_TIGHT):
    rel, cs = rel_cos(got, want)
    assert rel <= REL_TOL, f"{what}: max rel {rel:.3e} above the 2e-2 bar (cos {cs:.6f})"
    assert rel <= rel_tol and cs >= COS_MIN, f"{what}: max rel {rel:.3e}, cos {cs:.7f}"
    return rel, cs


def golden_runner(case, dev, **kw):
    cfg = fleet.ModelConfig()
    cos = torch.from_numpy(case.cos).to(dev)
    sin = torch.from_numpy(case.sin).to(dev)
    cache = fleet.PagedLatentCache.for_lengths([case.T], extra_tokens=case.steps, spare_pages=2,
                                               generator=torch.Generator().manual_seed(1), device=dev)
    cache.write_rows(0, 0, case.rows.to(dev))
    return fleet.MlaDecodeAttention(cfg, to_dev(case.lw, dev), cos, sin, **kw), cache


KERNELS = [dict(kernel="mma"), dict(kernel="tcgen05"), dict(check_kernel=True)]
KERNEL_IDS = ["mma", "tcgen05", "check"]


@pytest.mark.parametrize("name", ["t37", "config1", "walk"])
@pytest.mark.parametrize("kw", KERNELS, ids=KERNEL_IDS)
def test_golden_from_reference_qkv(golden, cuda_device, name, kw):
    """Kernels fed the reference's own q / kv_a reproduce its R(out) and appended row."""
    case = GoldenCase(golden, name)
    runner, cache = golden_runner(case, cuda_device, **kw)
    for s in range(case.steps):
        q = torch.from_numpy(case.q[s]).to(BF)[None].to(cuda_device)
        kv_a = torch.from_numpy(case.kv_a[s]).to(BF)[None].to(cuda_device)
        out = runner.attend(q, kv_a, cache)
        runner.check_errors()
        assert_close(out[0].float().cpu().numpy(), case.out[s], f"{name} step {s}")
        row = cache.read_rows(0, case.T + s, 1)[0].float().cpu().numpy()
        # the appended row: RMSNorm/RoPE in fp32 with bf16 rounding; ties aside it is bit-exact
        mism = np.count_nonzero(row != case.new_rows[s])
        assert mism <= 2, f"{name} step {s}: {mism} appended-row elements differ"
        np.testing.assert_allclose(row, case.new_rows[s], rtol=1e-2, atol=1e-6)
        cache.advance()


@pytest.mark.parametrize("name", ["config1", "walk"])
def test_golden_from_hidden_state(golden, cuda_device, name):
    """The public call from x_n (cuBLAS projection + kernels) against the reference's R(out)."""
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
    case = GoldenCase(golden, name)
    runner, cache = golden_runner(case, cuda_device)
    for s in range(case.steps):
        x_n = torch.from_numpy(case.x_n[s]).to(BF).to(cuda_device)
        out = fleet.attention_absorbed(fleet.ModelConfig(), runner.w, x_n, cache, runner=runner)
        runner.check_errors()
        assert_close(out.float().cpu().numpy(), case.out[s], f"{name} step {s} from x_n")
        cache.advance()


def ragged_batch(dev, lengths, seed=5, normed=True, permute=True):
    """A paged batch with seeded rows and q/kv_a from the oracle's projection of seeded x_n."""
    cfg = O.Config()
    max_pos = max(lengths) + 8
    cos, sin = cfg.cos_sin(max_pos)
    lw = workloads.make_layer_weights(seed, norm="uniform")
    w = oracle_weights(lw)
    cache = fleet.PagedLatentCache.for_lengths(lengths, spare_pages=3, permute=permute,
                                               generator=torch.Generator().manual_seed(seed), device=dev)
    for b, n in enumerate(lengths):
        if n:
            cache.write_rows(b, 0, workloads.make_cache_rows(100 + b, n, torch.from_numpy(cos),
                                                             torch.from_numpy(sin), normed=normed))
    x_n = workloads.make_hidden(seed + 1, len(lengths)).float().numpy()
    qs, kvs = zip(*(O.project(cfg, w, x) for x in x_n))
    q = np.stack([x.reshape(-1) for x in qs])
    kv_a = np.stack(kvs)
    return dict(cfg=cfg, cos=cos, sin=sin, lw=lw, w=w, cache=cache, q=q, kv_a=kv_a, lengths=lengths)


def oracle_paged(bt, pages_np, d, requests=None, fast=False):
    seq = np.array(d["lengths"], np.int32)
    return O.attention_task_paged(d["cfg"], d["w"], d["q"], d["kv_a"], pages_np, bt, seq, d["cos"], d["sin"],
                                  fast=fast, requests=requests)


def run_gpu(d, dev, num_ctas=0, check_kernel=False, kernel="mma"):
    runner = fleet.MlaDecodeAttention(fleet.ModelConfig(), to_dev(d["lw"], dev), torch.from_numpy(d["cos"]).to(dev),
                                      torch.from_numpy(d["sin"]).to(dev), num_ctas=num_ctas,
                                      check_kernel=check_kernel, kernel=kernel)
    q = torch.from_numpy(d["q"]).to(BF).to(dev)
    kv_a = torch.from_numpy(d["kv_a"]).to(BF).to(dev)
    out = runner.attend(q, kv_a, d["cache"])
    runner.check_errors()
    return out.float().cpu().numpy()


# around the 64-row pages and the 32-row half pages (the default kernel's plan tiles)
EDGE_LENGTHS = [0, 1, 30, 31, 32, 33, 62, 63, 64, 65, 95, 96, 97, 127, 128, 129, 200, 1000, 1023, 4095]


@pytest.mark.parametrize("kernel", ["mma", "tcgen05"])
@pytest.mark.parametrize("num_ctas", [0, 1, 3, 7, 64, 500])
def test_ragged_paged_batch(cuda_device, num_ctas, kernel):
    """Edge lengths around page and half-page boundaries (0 cached rows = only the new token), a
    permuted block table, and split plans from 1 CTA to more CTAs than tiles."""
    d = ragged_batch(cuda_device, EDGE_LENGTHS)
    pages_np = d["cache"].pages.float().cpu().numpy()
    bt = d["cache"].block_table.cpu().numpy()
    want, rows = oracle_paged(bt, pages_np, d)
    got = run_gpu(d, cuda_device, num_ctas=num_ctas, kernel=kernel)
    for b in range(len(EDGE_LENGTHS)):
        assert_close(got[b], want[b], f"request {b} (T={EDGE_LENGTHS[b]}, ctas={num_ctas}, {kernel})")
    gpu_pages = d["cache"].pages.float().cpu().numpy()
    for b, n in enumerate(EDGE_LENGTHS):
        r = gpu_pages[bt[b][n // 64], n % 64]
        np.testing.assert_allclose(r, rows[b], rtol=1e-2, atol=1e-6)


@pytest.mark.parametrize("B", [64, 65, 150, 200, 300, 1000])
def test_large_batch_merge_blocks(cuda_device, B):
    """The batch thresholds of the plan and of K3's forms:
    - 64: the largest batch whose split-KV kernel and K3 derive the plan themselves before
      their waits; K3's cluster form in four 16-request blocks (256 CTAs, two waves);
    - 65: the plan from K1's per-CTA entries; K3's plain form in 16-request blocks;
    - 150-300: past one wave of 16-request blocks (16 heads x ceil(B/16) > 148 SMs), K3 runs
      in 32-request blocks, two m16 tiles on one staged W_UV[h]; partial last blocks (B = 150:
      22 requests, B = 200: 8) leave whole tiles empty;
    - 1000: 512 K3 CTAs in several waves, about three requests per plan CTA."""
    rng = np.random.default_rng(B)
    lengths = [int(x) for x in rng.integers(0, 400, size=B)]
    d = ragged_batch(cuda_device, lengths)
    pages_np = d["cache"].pages.float().cpu().numpy()
    bt = d["cache"].block_table.cpu().numpy()
    want, _ = oracle_paged(bt, pages_np, d, fast=True)
    got = run_gpu(d, cuda_device)
    for b in range(B):
        assert_close(got[b], want[b], f"request {b} of {B} (T={lengths[b]})")


@pytest.mark.parametrize("lengths", [[9440], [40000], [9000, 20, 12000, 0, 3000, 64, 8000, 1],
                                     [5000, 64, 1, 12000, 0, 700, 9000, 33, 2048, 65, 3000, 128],
                                     [127] * 40 + [30000] + [5] * 30],
                         ids=["one-296-tiles", "one-1251-tiles", "ragged-8", "ragged-12", "ragged-71"])
def test_pair_merge(cuda_device, lengths):
    """Plans of at least 296 tiles (32-row half pages) with the default 296 plan CTAs: each
    split-KV CTA runs two adjacent plan CTAs and, where their boundary falls inside a request,
    merges the two partials of that request in shared memory before K3 (k2_pairs). One request of exactly
    296 tiles (the last holding only the new row) merges at every CTA; ragged batches merge
    at some boundaries and not at others (empty requests, requests inside one plan CTA).
    Checked against the oracle, against plans that do not pair (148 CTAs, the check kernel),
    and for repeatable bits."""
    d = ragged_batch(cuda_device, lengths)
    pages_np = d["cache"].pages.float().cpu().numpy()
    bt = d["cache"].block_table.cpu().numpy()
    want, _ = oracle_paged(bt, pages_np, d, fast=True)
    got = run_gpu(d, cuda_device)
    np.testing.assert_array_equal(got, run_gpu(d, cuda_device))
    unpaired = run_gpu(d, cuda_device, num_ctas=148)
    ck = run_gpu(d, cuda_device, check_kernel=True)
    for b, T in enumerate(lengths):
        assert_close(got[b], want[b], f"request {b} (T={T}), paired")
        assert_close(unpaired[b], want[b], f"request {b} (T={T}), 148 CTAs")
        assert_close(got[b], ck[b], f"request {b} (T={T}), paired vs check kernel")


def test_tensor_core_kernels_vs_check_kernel(cuda_device):
    d = ragged_batch(cuda_device, EDGE_LENGTHS)
    a = run_gpu(d, cuda_device, num_ctas=5)
    t = run_gpu(d, cuda_device, num_ctas=5, kernel="tcgen05")
    b = run_gpu(d, cuda_device, num_ctas=5, check_kernel=True)
    for i in range(len(EDGE_LENGTHS)):
        assert_close(a[i], b[i], f"mma vs check, request {i}")
        assert_close(t[i], b[i], f"tcgen05 vs check, request {i}")


@pytest.mark.parametrize("kernel", ["mma", "tcgen05"])
def test_deterministic_and_page_permutation_invariant(cuda_device, kernel):
    lengths = [300, 5000, 77, 2048]
    d1 = ragged_batch(cuda_device, lengths, permute=True)
    o1 = run_gpu(d1, cuda_device, num_ctas=9, kernel=kernel)
    o1b = run_gpu(d1, cuda_device, num_ctas=9, kernel=kernel)
    np.testing.assert_array_equal(o1, o1b)  # same plan, same bits (no atomics, fixed merge order)
    d2 = ragged_batch(cuda_device, lengths, permute=False)
    o2 = run_gpu(d2, cuda_device, num_ctas=9, kernel=kernel)
    np.testing.assert_array_equal(o1, o2)   # physical page placement does not matter


def test_duplicate_requests_identical(cuda_device):
    d = ragged_batch(cuda_device, [700, 700])
    # make request 1 a copy of request 0 (same rows, same q/kv_a)
    d["cache"].write_rows(1, 0, d["cache"].read_rows(0, 0, 700))
    d["q"][1], d["kv_a"][1] = d["q"][0], d["kv_a"][0]
    o = run_gpu(d, cuda_device, num_ctas=1)
    np.testing.assert_array_equal(o[0], o[1])


def test_single_row_is_uv_of_new_row(cuda_device):
    """T = 0: softmax over one row is 1, so R(out) = R(W_UV c_new) per head."""
    d = ragged_batch(cuda_device, [0])
    got = run_gpu(d, cuda_device)[0]
    row = O.kv_post(d["cfg"], d["w"], d["kv_a"][0], 0, d["cos"], d["sin"])
    kvb = d["w"].kv_b_proj.reshape(16, 256, 512)
    want = O.bf16_round(np.einsum("hvl,l->hv", kvb[:, 128:], row[:512]).reshape(-1))
    assert_close(got, want, "single row")


def test_device_errors_are_reported(cuda_device):
    """A block-table entry outside the pool and a position outside the rope table are
    caught by the kernels' bounds checks, recorded in the error word, and do not fault."""
    d = ragged_batch(cuda_device, [100, 100])
    d["cache"].block_table[1, 0] = d["cache"].n_pages + 5
    runner = fleet.MlaDecodeAttention(fleet.ModelConfig(), to_dev(d["lw"], cuda_device),
                                      torch.from_numpy(d["cos"]).to(cuda_device),
                                      torch.from_numpy(d["sin"]).to(cuda_device))
    q = torch.from_numpy(d["q"]).to(BF).to(cuda_device)
    kv_a = torch.from_numpy(d["kv_a"]).to(BF).to(cuda_device)
    runner.attend(q, kv_a, d["cache"])
    with pytest.raises(fleet.MlaError) as e:
        runner.check_errors()
    assert e.value.code == 1
    # position beyond the rope table: recorded, that request's output is zero
    d2 = ragged_batch(cuda_device, [100, 100])
    d2["cache"].seq_lens[1] = d2["cos"].shape[0] + 10
    out = runner.attend(q, kv_a, d2["cache"])
    with pytest.raises(fleet.MlaError) as e:
        runner.check_errors()
    assert e.value.code == 2
    assert torch.count_nonzero(out[1]) == 0
    # the context stays usable
    d3 = ragged_batch(cuda_device, [100])
    run_gpu(d3, cuda_device)


@pytest.mark.parametrize("num_ctas", [0, 3, 7])
def test_requests_without_tiles_between_segments(cuda_device, num_ctas):
    """Requests whose position lies outside the RoPE table get no tiles in the split plan
    (zero output, MLA_DEV_BAD_POSITION). A warp group whose range runs from the request
    before such a request to the one after it skips it when it requests the next segment's
    query and row count ahead of time; the valid requests still match the oracle."""
    lengths = [3000, 100, 5000, 64, 2000]
    d = ragged_batch(cuda_device, lengths)
    pages_np = d["cache"].pages.float().cpu().numpy()
    bt = d["cache"].block_table.cpu().numpy()
    want, _ = oracle_paged(bt, pages_np, d, requests=[0, 2, 4], fast=True)
    for b in (1, 3):
        d["cache"].seq_lens[b] = d["cos"].shape[0] + 10
    runner = fleet.MlaDecodeAttention(fleet.ModelConfig(), to_dev(d["lw"], cuda_device),
                                      torch.from_numpy(d["cos"]).to(cuda_device),
                                      torch.from_numpy(d["sin"]).to(cuda_device), num_ctas=num_ctas)
    q = torch.from_numpy(d["q"]).to(BF).to(cuda_device)
    kv_a = torch.from_numpy(d["kv_a"]).to(BF).to(cuda_device)
    out = runner.attend(q, kv_a, d["cache"])
    with pytest.raises(fleet.MlaError) as e:
        runner.check_errors()
    assert e.value.code == 2
    got = out.float().cpu().numpy()
    for b in (1, 3):
        assert np.count_nonzero(got[b]) == 0
    for b in (0, 2, 4):
        assert_close(got[b], want[b], f"request {b} (T={lengths[b]}, ctas={num_ctas})")


@pytest.mark.parametrize("cfg_name,subset", [("config3", [0, 13, 31]), ("config4", [2])])
def test_full_size_config_subset(cuda_device, cfg_name, subset):
    """Configs 3 and 4 at full size: every request against the CUDA-core check
    kernel, a subset against the oracle (vectorised form)."""
    wl = workloads.WORKLOADS[cfg_name]
    lengths = wl.seq_lens()
    cfg = O.Config()
    cos, sin = cfg.cos_sin(max(lengths) + 8)
    lw = workloads.make_layer_weights(wl.seed)
    w = oracle_weights(lw)
    cache = fleet.PagedLatentCache.for_lengths(lengths, permute=True,
                                               generator=torch.Generator().manual_seed(wl.seed), device=cuda_device)
    workloads.fill_pool_random(cache.pages, wl.seed)
    x_n = workloads.make_hidden(wl.seed, len(lengths)).float().numpy()
    qs, kvs = zip(*(O.project(cfg, w, x) for x in x_n))
    d = dict(cfg=cfg, cos=cos, sin=sin, lw=lw, w=w, cache=cache, q=np.stack([x.reshape(-1) for x in qs]),
             kv_a=np.stack(kvs), lengths=lengths)
    pages_before = cache.pages.float().cpu().numpy()
    tc = run_gpu(d, cuda_device)
    t5 = run_gpu(d, cuda_device, kernel="tcgen05")
    ck = run_gpu(d, cuda_device, check_kernel=True)
    for b in range(len(lengths)):
        assert_close(tc[b], ck[b], f"{cfg_name} request {b}: mma vs check")
        assert_close(t5[b], ck[b], f"{cfg_name} request {b}: tcgen05 vs check")
    want, _ = oracle_paged(cache.block_table.cpu().numpy(), pages_before, d, requests=subset, fast=True)
    for b in subset:
        assert_close(tc[b], want[b], f"{cfg_name} request {b} vs oracle")


def _ulp_err(got, want):
    """|got - want| in units of the bf16 spacing at |want| (0 = the same bf16 value)."""
    w = np.abs(np.asarray(want, np.float64))
    spacing = np.exp2(np.floor(np.log2(np.maximum(w, 1e-30))) - 7)
    return np.abs(np.asarray(got, np.float64) - np.asarray(want, np.float64)) / spacing


@pytest.mark.parametrize("flags", [dict(qc_hilo=True), dict(p_hilo=True), dict(qc_hilo=True, p_hilo=True)],
                         ids=["qc", "p", "qc+p"])
def test_hilo_precision_forms(cuda_device, flags):
    """MLA_FLAG_QC_HILO / MLA_FLAG_P_HILO keep q_c and P as bf16 hi/lo pairs. Each must pass
    the parity bar, give repeatable bits, and bring R(out) no further from the oracle's fp32
    arithmetic than the default form; with both, nearly every output element is the
    oracle's bf16 value or its neighbour."""
    d = ragged_batch(cuda_device, EDGE_LENGTHS + [20000])
    pages_np = d["cache"].pages.float().cpu().numpy()
    bt = d["cache"].block_table.cpu().numpy()
    want, _ = oracle_paged(bt, pages_np, d, fast=True)
    runner = fleet.MlaDecodeAttention(fleet.ModelConfig(), to_dev(d["lw"], cuda_device),
                                      torch.from_numpy(d["cos"]).to(cuda_device),
                                      torch.from_numpy(d["sin"]).to(cuda_device), **flags)
    q = torch.from_numpy(d["q"]).to(BF).to(cuda_device)
    kv_a = torch.from_numpy(d["kv_a"]).to(BF).to(cuda_device)
    got = runner.attend(q, kv_a, d["cache"]).float().cpu().numpy()
    again = runner.attend(q, kv_a, d["cache"]).float().cpu().numpy()
    runner.check_errors()
    np.testing.assert_array_equal(got, again)
    base = run_gpu(d, cuda_device)
    for b in range(len(d["lengths"])):
        assert_close(got[b], want[b], f"request {b} (T={d['lengths'][b]}, {flags})")
    e_hilo, e_base = _ulp_err(got, want), _ulp_err(base, want)
    assert e_hilo.mean() <= e_base.mean(), (e_hilo.mean(), e_base.mean())
    if len(flags) == 2:
        assert np.mean(e_hilo <= 1.0) >= 0.995, f"{np.mean(e_hilo <= 1.0):.4f} of elements within one bf16 step"
    print(f"{flags}: mean ulp error {e_hilo.mean():.3f} (default {e_base.mean():.3f}), "
          f"within one step {np.mean(e_hilo <= 1.0):.4f} (default {np.mean(e_base <= 1.0):.4f})")


def test_hilo_flags_refused_with_other_kernels(cuda_device):
    with pytest.raises(ValueError):
        fleet.MlaDecodeAttention(fleet.ModelConfig(), to_dev(workloads.make_layer_weights(1), cuda_device),
                                 torch.zeros(8, 64, device=cuda_device), torch.zeros(8, 64, device=cuda_device),
                                 kernel="tcgen05", qc_hilo=True)
