"""Model configuration and the YaRN RoPE tables of the MLA attention task.

Mirrors the fields of the reference's `ModelConfig` (src/host/reference_decode.py:166-203)
that the attention task reads, and its YaRN table builder `yarn_cos_sin`
(reference_decode.py:78-117, itself HF's DeepseekV2YarnRotaryEmbedding,
reference/modeling_deepseek.py:262-328). The tables are computed once on the host
in float32 with the same operation order, then uploaded, as the reference's launcher
does (src/host/fleet_launch.hip:186-219).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np


@dataclass
class ModelConfig:
    """DeepSeek-V2-Lite attention dims (reference/dsv2lite_config.json)."""

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

    @property
    def q_head_dim(self) -> int:
        return self.qk_nope + self.qk_rope

    @property
    def softmax_scale(self) -> float:
        """q_head_dim**-0.5 * mscale(factor, mscale_all_dim)**2 (reference_decode.py:197-203)."""
        s = self.q_head_dim ** -0.5
        if self.mscale_all_dim:
            m = yarn_get_mscale(self.rope_factor, self.mscale_all_dim)
            s = s * m * m
        return s

    def check_supported(self) -> None:
        """The kernels are specialised for the DeepSeek-V2-Lite attention shape, like the
        reference's launcher (src/host/fleet_launch.hip:573-577)."""
        got = (self.heads, self.qk_nope, self.qk_rope, self.v_head, self.kv_lora_rank)
        if got != (16, 128, 64, 128, 512):
            raise ValueError(
                f"MLA decode kernels support heads/qk_nope/qk_rope/v_head/kv_lora = "
                f"16/128/64/128/512 only, got {got}")


def yarn_get_mscale(scale: float, mscale: float) -> float:
    """HF yarn_get_mscale (reference_decode.py:78-82): identity below scale 1."""
    if scale <= 1:
        return 1.0
    return 0.1 * mscale * math.log(scale) + 1.0


def _correction_dim(num_rotations: float, dim: int, base: float, max_pos: int) -> float:
    return (dim * math.log(max_pos / (num_rotations * 2 * math.pi))) / (2 * math.log(base))


def yarn_cos_sin(dim: int, seq_len: int, base: float, scale: float, original_max: int,
                 beta_fast: float, beta_slow: float, mscale: float,
                 mscale_all_dim: float) -> tuple[np.ndarray, np.ndarray]:
    """cos/sin tables [seq_len, dim] float32 (reference_decode.py:102-117).

    inv_freq blends the extrapolated and interpolated frequencies over the YaRN
    correction range; cos/sin carry mscale(scale, mscale)/mscale(scale, mscale_all_dim).
    """
    exps = np.arange(0, dim, 2, dtype=np.float32) / dim
    freq_extra = 1.0 / (base ** exps)
    freq_inter = 1.0 / (scale * base ** exps)
    low = max(math.floor(_correction_dim(beta_fast, dim, base, original_max)), 0)
    high = min(math.ceil(_correction_dim(beta_slow, dim, base, original_max)), dim - 1)
    if low == high:
        high += 0.001
    ramp = np.clip((np.arange(dim // 2, dtype=np.float32) - low) / (high - low), 0, 1)
    extra_mask = 1.0 - ramp
    inv_freq = freq_inter * (1 - extra_mask) + freq_extra * extra_mask
    t = np.arange(seq_len, dtype=np.float32)
    freqs = np.outer(t, inv_freq)
    emb = np.concatenate([freqs, freqs], axis=-1)
    m = yarn_get_mscale(scale, mscale) / yarn_get_mscale(scale, mscale_all_dim)
    return np.cos(emb) * m, np.sin(emb) * m


def rope_tables(cfg: ModelConfig, max_pos: int) -> tuple[np.ndarray, np.ndarray]:
    """YaRN tables for positions 0..max_pos-1 of this config."""
    return yarn_cos_sin(cfg.qk_rope, max_pos, cfg.rope_theta, cfg.rope_factor,
                        cfg.rope_original_max, cfg.beta_fast, cfg.beta_slow,
                        cfg.mscale, cfg.mscale_all_dim)
