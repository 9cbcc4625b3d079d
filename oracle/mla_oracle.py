"""TEST INFRASTRUCTURE — CPU oracle of the absorbed-MLA attention task. Not product code.

Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and
`--impl reference`) may import this module, and only as the checker / the timed CPU
baseline; the product path (fleet-mi300x_b200/) never calls it.

A NumPy restatement of the reference's attention task, split at the north-star
boundary: post-RMSNorm x_n in, R(out) before o_proj out. Each function cites the
reference lines it follows (paths relative to the cklxx/fleet-mi300x tree). The
restatement is pinned against golden vectors produced by the reference's own
`reference_decode.py` (tests/golden/make_golden.py, tests/test_oracle_golden.py).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np


# ------------------------------------------------------------------ primitives

def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest bf16 (ties to even) -> fp32 (src/host/reference_decode.py:37-48)."""
    x = np.array(x, dtype=np.float32)
    u = x.view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return r.astype(np.uint32).view(np.float32)


def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float, bf16: bool = False) -> np.ndarray:
    """DeepseekV2RMSNorm with HF's two bf16 roundings (reference_decode.py:51-65)."""
    x32 = x.astype(np.float32)
    var = np.mean(x32 * x32, axis=-1, keepdims=True)
    y = x32 * (1.0 / np.sqrt(var + eps))
    if bf16:
        y = bf16_round(y)
    out = y * weight.astype(np.float32)
    return bf16_round(out) if bf16 else out


def softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    """Max-subtracted softmax (reference_decode.py:72-75)."""
    m = np.max(x, axis=axis, keepdims=True)
    e = np.exp(x - m)
    return e / np.sum(e, axis=axis, keepdims=True)


def yarn_get_mscale(scale: float, mscale: float) -> float:
    """reference_decode.py:78-82."""
    if scale <= 1:
        return 1.0
    return 0.1 * mscale * math.log(scale) + 1.0


def yarn_find_correction_dim(num_rotations, dim, base, max_pos):
    """reference_decode.py:85-86."""
    return (dim * math.log(max_pos / (num_rotations * 2 * math.pi))) / (2 * math.log(base))


def yarn_find_correction_range(beta_fast, beta_slow, dim, base, max_pos):
    """reference_decode.py:89-92."""
    low = math.floor(yarn_find_correction_dim(beta_fast, dim, base, max_pos))
    high = math.ceil(yarn_find_correction_dim(beta_slow, dim, base, max_pos))
    return max(low, 0), min(high, dim - 1)


def yarn_linear_ramp_mask(low, high, dim):
    """reference_decode.py:95-99."""
    if low == high:
        high += 0.001
    linear = (np.arange(dim, dtype=np.float32) - low) / (high - low)
    return np.clip(linear, 0, 1)


def yarn_cos_sin(dim, seq_len, base, scale, original_max, beta_fast, beta_slow, mscale, mscale_all_dim):
    """YaRN cos/sin tables [seq_len, dim] (reference_decode.py:102-117)."""
    freq_extra = 1.0 / (base ** (np.arange(0, dim, 2, dtype=np.float32) / dim))
    freq_inter = 1.0 / (scale * base ** (np.arange(0, dim, 2, dtype=np.float32) / dim))
    low, high = yarn_find_correction_range(beta_fast, beta_slow, dim, base, original_max)
    inv_freq_mask = 1.0 - yarn_linear_ramp_mask(low, high, dim // 2)
    inv_freq = freq_inter * (1 - inv_freq_mask) + freq_extra * inv_freq_mask
    t = np.arange(seq_len, dtype=np.float32)
    freqs = np.outer(t, inv_freq)
    emb = np.concatenate([freqs, freqs], axis=-1)
    _mscale = yarn_get_mscale(scale, mscale) / yarn_get_mscale(scale, mscale_all_dim)
    return np.cos(emb) * _mscale, np.sin(emb) * _mscale


def rotate_half(x: np.ndarray) -> np.ndarray:
    """reference_decode.py:120-122."""
    half = x.shape[-1] // 2
    return np.concatenate([-x[..., half:], x[..., :half]], axis=-1)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """DeepseekV2 RoPE: interleave-transpose, then rotate_half (reference_decode.py:125-134)."""
    d = x.shape[-1]
    x = x.reshape(*x.shape[:-1], d // 2, 2).swapaxes(-1, -2).reshape(*x.shape[:-1], d)
    return x * cos + rotate_half(x) * sin


# ------------------------------------------------------------------ config / weights

@dataclass
class Config:
    """The fields of reference_decode.ModelConfig the attention task reads (:166-203)."""
    hidden: int = 2048
    heads: int = 16
    kv_lora_rank: int = 512
    qk_nope: int = 128
    qk_rope: int = 64
    v_head: int = 128
    rms_eps: float = 1e-6
    rope_theta: float = 1e4
    rope_factor: float = 40.0
    rope_original_max: int = 4096
    beta_fast: float = 32.0
    beta_slow: float = 1.0
    mscale: float = 0.707
    mscale_all_dim: float = 0.707
    bf16: bool = True

    def r(self, x):
        """R(): round where HF's bf16 modules round (reference_decode.py:189-191)."""
        return bf16_round(x) if self.bf16 else x

    @property
    def q_head_dim(self) -> int:
        return self.qk_nope + self.qk_rope

    @property
    def softmax_scale(self) -> float:
        """reference_decode.py:197-203."""
        s = self.q_head_dim ** -0.5
        if self.mscale_all_dim:
            m = yarn_get_mscale(self.rope_factor, self.mscale_all_dim)
            s = s * m * m
        return s

    def cos_sin(self, seq_len: int):
        return yarn_cos_sin(self.qk_rope, seq_len, self.rope_theta, self.rope_factor, self.rope_original_max,
                            self.beta_fast, self.beta_slow, self.mscale, self.mscale_all_dim)


@dataclass
class Weights:
    """fp32 arrays holding bf16 values (reference_decode.LayerWeights, :139-159)."""
    q_proj: np.ndarray              # [heads*q_head_dim, hidden]
    kv_a_proj_with_mqa: np.ndarray  # [kv_lora+qk_rope, hidden]
    kv_a_layernorm: np.ndarray      # [kv_lora]
    kv_b_proj: np.ndarray           # [heads*(qk_nope+v_head), kv_lora]


# ------------------------------------------------------------------ the task

def project(cfg: Config, w: Weights, x_n: np.ndarray):
    """q and kv_a of one token (reference_decode.py:225-231)."""
    q = cfg.r(w.q_proj @ x_n).reshape(cfg.heads, cfg.q_head_dim)
    kv_a = cfg.r(w.kv_a_proj_with_mqa @ x_n)
    return q, kv_a


def kv_post(cfg: Config, w: Weights, kv_a: np.ndarray, pos: int, cos, sin) -> np.ndarray:
    """The appended cache row: RMSNorm(c_new), RoPE(k_pe_new) (reference_decode.py:230-237)."""
    L = cfg.kv_lora_rank
    c_new = rms_norm(kv_a[:L], w.kv_a_layernorm, cfg.rms_eps, cfg.bf16)
    k_pe_new = cfg.r(apply_rope(kv_a[L:][None, :], cos[pos][None, :], sin[pos][None, :])[0])
    return np.concatenate([c_new, k_pe_new]).astype(np.float32)


def attend_rows(cfg: Config, w: Weights, q: np.ndarray, rows: np.ndarray, pos: int, cos, sin) -> np.ndarray:
    """Absorbed attention of one token over cache rows [S, 576] (reference_decode.py:235, 239-256).

    q: [heads, q_head_dim] (bf16-valued). Returns R(out) [heads*v_head] before o_proj.
    """
    H, Dk, Dv, L = cfg.heads, cfg.qk_nope, cfg.v_head, cfg.kv_lora_rank
    q_nope, q_pe = q[:, :Dk], q[:, Dk:]
    q_pe = cfg.r(apply_rope(q_pe, cos[pos][None, :], sin[pos][None, :]))
    c = rows[:, :L]
    k_pe = rows[:, L:]
    out = np.empty(H * Dv, dtype=np.float32)
    for h in range(H):
        base = h * (Dk + Dv)
        w_uk = w.kv_b_proj[base: base + Dk]
        w_uv = w.kv_b_proj[base + Dk: base + Dk + Dv]
        q_c = q_nope[h] @ w_uk
        s = (c @ q_c + k_pe @ q_pe[h]) * cfg.softmax_scale
        p = softmax(s)
        o_c = p @ c
        out[h * Dv:(h + 1) * Dv] = w_uv @ o_c
    return cfg.r(out)


def attention_task(cfg: Config, w: Weights, x_n: np.ndarray, cache: np.ndarray, pos: int, cos, sin) -> np.ndarray:
    """reference_decode.attention_absorbed (:210-256) from x_n (after :222) to R(out) (the
    argument of o_proj at :256). Appends this token's row to `cache` in place."""
    q, kv_a = project(cfg, w, x_n)
    cache[pos] = kv_post(cfg, w, kv_a, pos, cos, sin)
    return attend_rows(cfg, w, q, cache[: pos + 1], pos, cos, sin)


def attention_task_qkv(cfg: Config, w: Weights, q_flat: np.ndarray, kv_a: np.ndarray, rows: np.ndarray,
                       pos: int, cos, sin) -> tuple[np.ndarray, np.ndarray]:
    """The same task from given q [heads*q_head_dim] and kv_a [576] (bf16-valued) and the
    request's cached rows [pos, 576]: returns (R(out), appended row)."""
    row = kv_post(cfg, w, kv_a, pos, cos, sin)
    all_rows = np.concatenate([rows[:pos], row[None, :]], axis=0)
    q = q_flat.reshape(cfg.heads, cfg.q_head_dim)
    return attend_rows(cfg, w, q, all_rows, pos, cos, sin), row


# ------------------------------------------------------------------ batched / fast forms

def attend_rows_fast(cfg: Config, w: Weights, q: np.ndarray, rows: np.ndarray, pos: int, cos, sin) -> np.ndarray:
    """attend_rows with all heads at once (matrix products instead of the per-head
    loop). Same arithmetic, different summation order; used for large cases and as the
    timed CPU baseline."""
    H, Dk, Dv, L = cfg.heads, cfg.qk_nope, cfg.v_head, cfg.kv_lora_rank
    q_nope, q_pe = q[:, :Dk], q[:, Dk:]
    q_pe = cfg.r(apply_rope(q_pe, cos[pos][None, :], sin[pos][None, :]))
    kvb = w.kv_b_proj.reshape(H, Dk + Dv, L)
    q_c = np.einsum("hd,hdl->hl", q_nope, kvb[:, :Dk])                 # [H, L]
    qa = np.concatenate([q_c, q_pe], axis=1)                            # [H, 576]
    s = (rows @ qa.T) * cfg.softmax_scale                               # [S, H]
    s = s - s.max(axis=0, keepdims=True)
    e = np.exp(s)
    p = e / e.sum(axis=0, keepdims=True)
    o_c = p.T @ rows[:, :L]                                             # [H, L]
    out = np.einsum("hvl,hl->hv", kvb[:, Dk:], o_c).reshape(-1)
    return cfg.r(out.astype(np.float32))


def attention_task_paged(cfg: Config, w: Weights, q: np.ndarray, kv_a: np.ndarray, pages: np.ndarray,
                         block_table: np.ndarray, seq_lens: np.ndarray, cos, sin, *, fast: bool = False,
                         requests=None) -> tuple[np.ndarray, np.ndarray]:
    """The batched paged task: for every request b, append its row at seq_lens[b] in page
    block_table[b][pos // 64] (mutating `pages` [n_pages, 64, 576]) and attend over rows
    0..seq_lens[b]. q [B, heads*q_head_dim], kv_a [B, 576]. Returns (out [B, heads*v_head],
    rows appended [B, 576]). `requests` restricts the work to a subset of b (others are 0)."""
    B = q.shape[0]
    P = pages.shape[1]
    out = np.zeros((B, cfg.heads * cfg.v_head), dtype=np.float32)
    new_rows = np.zeros((B, cfg.kv_lora_rank + cfg.qk_rope), dtype=np.float32)
    attend = attend_rows_fast if fast else attend_rows
    for b in (range(B) if requests is None else requests):
        pos = int(seq_lens[b])
        row = kv_post(cfg, w, kv_a[b], pos, cos, sin)
        pages[block_table[b][pos // P], pos % P] = row
        n_blocks = pos // P + 1
        rows = pages[block_table[b][:n_blocks]].reshape(-1, pages.shape[2])[: pos + 1]
        out[b] = attend(cfg, w, q[b].reshape(cfg.heads, cfg.q_head_dim), rows, pos, cos, sin)
        new_rows[b] = row
    return out, new_rows


# ------------------------------------------------------------------ sequence shards (multi-GPU protocol)

def attend_rows_partial(cfg: Config, w: Weights, q: np.ndarray, rows: np.ndarray, pos: int, cos, sin):
    """One shard's contribution for one token: rows [S, 576] of the shard (S may be 0).
    Returns (y [H, Dv], m [H], L [H]) with m the log2-domain max of scaled scores,
    L = sum 2^(s - m) and y = W_UV (sum 2^(s - m) c) / L: the per-chunk (m, l, acc) of
    attention.h:230-351 with W_UV applied (it is linear), as exchanged between GPUs."""
    H, Dk, Dv, L = cfg.heads, cfg.qk_nope, cfg.v_head, cfg.kv_lora_rank
    if rows.shape[0] == 0:
        return np.zeros((H, Dv), np.float32), np.full(H, -np.inf, np.float32), np.zeros(H, np.float32)
    q_nope, q_pe = q[:, :Dk], q[:, Dk:]
    q_pe = cfg.r(apply_rope(q_pe, cos[pos][None, :], sin[pos][None, :]))
    kvb = w.kv_b_proj.reshape(H, Dk + Dv, L)
    q_c = np.einsum("hd,hdl->hl", q_nope, kvb[:, :Dk])
    qa = np.concatenate([q_c, q_pe], axis=1)
    s2 = (rows @ qa.T).astype(np.float64) * cfg.softmax_scale * np.log2(np.e)   # [S, H]
    m = s2.max(axis=0)
    e = np.exp2(s2 - m)
    Lsum = e.sum(axis=0)
    o_c = (e.T @ rows[:, :L]) / Lsum[:, None]
    y = np.einsum("hvl,hl->hv", kvb[:, Dk:], o_c)
    return y.astype(np.float32), m.astype(np.float32), Lsum.astype(np.float32)


def combine_partials(parts):
    """Fixed-order LSE combine of per-shard (y, m, L) into R(out) [H*Dv] (shard order)."""
    ms = np.stack([p[1] for p in parts]).astype(np.float64)       # [R, H]
    gm = ms.max(axis=0)
    acc = 0.0
    W = 0.0
    for y, m, Lr in parts:
        w = np.where(Lr > 0, Lr * np.exp2(m.astype(np.float64) - gm), 0.0)
        acc = acc + w[:, None] * y
        W = W + w
    return bf16_round((acc / W[:, None]).reshape(-1).astype(np.float32))


# ------------------------------------------------------------------ prefill hand-off

def flat_cache_file_bytes(rows_per_layer, max_pos: int) -> bytes:
    """The reference's prefill->decode cache file (src/host/kv_convert.py:124-139,
    write_fleet_cache_bin): raw bf16 [layers][max_pos][576] in C order, each layer's
    prefill rows at positions 0..S-1 and zeros after. rows_per_layer: fp32 arrays
    [S, 576] holding bf16 values."""
    layers = len(rows_per_layer)
    full = np.zeros((layers, max_pos, rows_per_layer[0].shape[1]), np.float32)
    for l, r in enumerate(rows_per_layer):
        full[l, : r.shape[0]] = r
    u = bf16_round(full).view(np.uint32) >> np.uint32(16)
    return u.astype(np.uint16).tobytes(order="C")


def scatter_rows(pages: np.ndarray, block_table: np.ndarray, rows: np.ndarray, row_start, first_pos=None) -> None:
    """Paged placement of request b's rows row_start[b]..row_start[b+1]-1 at positions
    first_pos[b] + i: position t is page block_table[b][t // 64], slot t % 64 (the
    paged layout that replaces the flat [max_pos][576] cache of
    src/runtime/fleet_types.h:106-111). pages: [n_pages, 64, 576], updated in place."""
    for b in range(len(row_start) - 1):
        p0 = 0 if first_pos is None else int(first_pos[b])
        for i in range(int(row_start[b]), int(row_start[b + 1])):
            t = p0 + i - int(row_start[b])
            pages[int(block_table[b][t // 64]), t % 64] = rows[i]


def prefill_rows(cfg: Config, w: Weights, kv_a_raw: np.ndarray, first_pos: int, cos, sin) -> np.ndarray:
    """Cache rows of a prefill's raw kv_a rows [S, 576] at positions first_pos + i: the
    decode step's row arithmetic (kv_post, reference_decode.py:230-237) per position,
    which is what kv_convert.build_fleet_cache (src/host/kv_convert.py:92-121) computes
    with HF's bf16 modules."""
    return np.stack([kv_post(cfg, w, kv_a_raw[i], first_pos + i, cos, sin) for i in range(kv_a_raw.shape[0])])


def o_proj_residual(cfg: Config, w_o: np.ndarray, out: np.ndarray, h: np.ndarray) -> np.ndarray:
    """The attention half's last two lines: R(W_o R(out)) (reference_decode.py:256),
    then the bf16 residual add x = R(x + attn) (:300). out: R(out) [heads*v_head],
    h: the layer input [hidden]; both bf16-valued."""
    return cfg.r(h + cfg.r(w_o @ out))
