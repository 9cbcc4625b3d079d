"""Pins the CPU oracle (oracle/mla_oracle.py) to the reference's own outputs.

The golden vectors were produced by importing the reference's reference_decode.py
(tests/golden/make_golden.py). These tests need no GPU.
"""
import numpy as np
import pytest
import torch

from mla_testlib import GoldenCase, O, fleet, rel_cos, workloads


def test_known_answers(golden):
    cfg = O.Config()
    # reference tests/test_absorbed_equivalence.py:128-137: 0.114721, mscale 1.260804
    assert cfg.softmax_scale == pytest.approx(float(golden["ka/softmax_scale"]), abs=1e-15)
    assert abs(cfg.softmax_scale - 0.114721) < 5e-7
    assert O.yarn_get_mscale(40.0, 0.707) == pytest.approx(float(golden["ka/mscale"]), abs=1e-15)
    assert abs(float(golden["ka/mscale"]) - 1.260804) < 5e-7
    assert fleet.ModelConfig().softmax_scale == pytest.approx(float(golden["ka/softmax_scale"]), abs=1e-15)


def test_bf16_round_exact(golden):
    np.testing.assert_array_equal(O.bf16_round(golden["ka/bf16_in"]), golden["ka/bf16_out"])
    t = torch.from_numpy(golden["ka/bf16_in"]).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(t, golden["ka/bf16_out"])  # torch's bf16 cast is the same rounding


def test_yarn_tables_exact(golden):
    pos = golden["ka/rope_positions"]
    cfg = O.Config()
    cos, sin = cfg.cos_sin(int(pos.max()) + 1)
    np.testing.assert_array_equal(cos[pos], golden["ka/cos"])
    np.testing.assert_array_equal(sin[pos], golden["ka/sin"])
    # the product's host-side table builder (fleet-mi300x_b200/config.py) is the same arithmetic
    pc, ps = fleet.rope_tables(fleet.ModelConfig(), int(pos.max()) + 1)
    np.testing.assert_array_equal(pc[pos], golden["ka/cos"])
    np.testing.assert_array_equal(ps[pos], golden["ka/sin"])


def test_rope_interleave(golden):
    cfg = O.Config()
    cos, sin = cfg.cos_sin(8)
    out = O.apply_rope(golden["ka/rope_x"], cos[5][None, :], sin[5][None, :])
    np.testing.assert_array_equal(out, golden["ka/rope_out"])
    # reference tests/test_absorbed_equivalence.py:103-125: differs from plain RoPE, keeps the norm
    x = golden["ka/rope_x"][:1]
    half = 32
    plain = x * cos[5] + np.concatenate([-x[:, half:], x[:, :half]], axis=-1) * sin[5]
    assert np.max(np.abs(out[:1] - plain)) > 1e-3
    assert abs(np.linalg.norm(out[:1]) / np.linalg.norm(x) - 1.0) < 1e-4


def test_tiny_config_walk(golden):
    """Tiny HF-comparison config, 12 tokens through an empty cache (cache accumulation)."""
    cfg = O.Config(hidden=64, heads=4, kv_lora_rank=16, qk_nope=16, qk_rope=8, v_head=16, rope_original_max=32)
    w = O.Weights(golden["tiny/q_proj"], golden["tiny/kv_a"], golden["tiny/kv_a_ln"], golden["tiny/kv_b"])
    S = golden["tiny/x_n"].shape[0]
    cos, sin = cfg.cos_sin(S)
    cache = np.zeros((S, 24), np.float32)
    for t in range(S):
        out = O.attention_task(cfg, w, golden["tiny/x_n"][t], cache, t, cos, sin)
        rel, cos_ = rel_cos(out, golden["tiny/out"][t])
        assert rel <= 1e-5 and cos_ >= 1 - 1e-9, (t, rel, cos_)
    np.testing.assert_allclose(cache, golden["tiny/cache"], rtol=0, atol=0)


@pytest.mark.parametrize("name", ["t37", "config1", "walk"])
def test_dsv2_cases(golden, name):
    case = GoldenCase(golden, name)
    cache = np.zeros((case.max_pos, 576), np.float32)
    cache[: case.T] = case.rows.float().numpy()
    for s in range(case.steps):
        pos = case.T + s
        # the projections, as the reference computes them
        q, kv_a = O.project(case.cfg, case.w, case.x_n[s])
        np.testing.assert_array_equal(q.reshape(-1), case.q[s])
        np.testing.assert_array_equal(kv_a, case.kv_a[s])
        out = O.attention_task(case.cfg, case.w, case.x_n[s], cache, pos, case.cos, case.sin)
        rel, cs = rel_cos(out, case.out[s])
        assert rel <= 1e-5 and cs >= 1 - 1e-9, (s, rel, cs)
        np.testing.assert_array_equal(cache[pos], case.new_rows[s])
        # the vectorised form used for big cases and the CPU baseline
        fast = O.attend_rows_fast(case.cfg, case.w, q, cache[: pos + 1], pos, case.cos, case.sin)
        rel_f, cs_f = rel_cos(fast, case.out[s])
        assert rel_f <= 1e-2 and cs_f >= 0.99999, (s, rel_f, cs_f)


def test_paged_oracle_matches_flat(golden):
    """The paged restatement on a permuted block table equals the flat reference walk."""
    case = GoldenCase(golden, "walk")
    P = 64
    n_pages = (case.max_pos + P - 1) // P + 3
    rng = np.random.default_rng(0)
    perm = rng.permutation(n_pages).astype(np.int32)
    pages = np.zeros((n_pages, P, 576), np.float32)
    bt = perm[None, : (case.max_pos + P - 1) // P]
    rows = case.rows.float().numpy()
    for t in range(case.T):
        pages[bt[0][t // P], t % P] = rows[t]
    for s in range(case.steps):
        seq = np.array([case.T + s], np.int32)
        out, new = O.attention_task_paged(case.cfg, case.w, case.q[s][None], case.kv_a[s][None], pages, bt,
                                          seq, case.cos, case.sin)
        rel, cs = rel_cos(out[0], case.out[s])
        assert rel <= 1e-5, rel
        np.testing.assert_array_equal(new[0], case.new_rows[s])


def test_absorbed_equals_naive():
    """reference tests/test_absorbed_equivalence.py:63-87 restated: folding W_UK/W_UV
    equals materialising K and V per head (fp32, S = 37)."""
    rng = np.random.default_rng(0)
    cfg = O.Config(bf16=False)
    S = 37
    q_nope = rng.standard_normal((16, 128), dtype=np.float32) * 0.05
    q_pe = rng.standard_normal((16, 64), dtype=np.float32) * 0.05
    c = rng.standard_normal((S, 512), dtype=np.float32) * 0.05
    k_pe = rng.standard_normal((S, 64), dtype=np.float32) * 0.05
    kv_b = rng.standard_normal((16 * 256, 512), dtype=np.float32) * 0.02
    naive = np.empty(16 * 128, np.float32)
    absorbed = np.empty(16 * 128, np.float32)
    for h in range(16):
        w_uk = kv_b[h * 256: h * 256 + 128]
        w_uv = kv_b[h * 256 + 128: h * 256 + 256]
        s = ((c @ w_uk.T) @ q_nope[h] + k_pe @ q_pe[h]) * cfg.softmax_scale
        naive[h * 128:(h + 1) * 128] = O.softmax(s) @ (c @ w_uv.T)
        s2 = (c @ (q_nope[h] @ w_uk) + k_pe @ q_pe[h]) * cfg.softmax_scale
        absorbed[h * 128:(h + 1) * 128] = w_uv @ (O.softmax(s2) @ c)
    rel, cs = rel_cos(absorbed, naive)
    assert rel <= 1e-5 and cs >= 1 - 1e-6


def test_workload_generators_deterministic():
    a = workloads.make_layer_weights(3)
    b = workloads.make_layer_weights(3)
    assert torch.equal(a.kv_b_proj, b.kv_b_proj) and torch.equal(a.q_proj, b.q_proj)
    w = workloads.WORKLOADS["config3"]
    assert w.seq_lens() == w.seq_lens()
    assert all(512 <= t <= 8192 for t in w.seq_lens()) and len(w.seq_lens()) == 32
    x = workloads.make_hidden(0, 2)
    rms = x.float().pow(2).mean(-1).sqrt()
    assert torch.all((rms - 1).abs() < 1e-2)
