"""Seeded synthetic inputs with the shapes and distributions of the benchmark configs.

There is no checkpoint or dataset: every config draws its weights, hidden states and
cache rows from torch generators seeded per config, so any machine with this
environment regenerates the same bytes.

  weights     W_q [3072, 2048], W_kv_a [576, 2048], kv_b [4096, 512] ~ N(0, 0.02), bf16
  x_n         N(0, 1) hidden state after RMSNorm (unit weight), bf16
  cache rows  c_kv = RMSNorm(N(0, 1)) rows, k_pe = RoPE(N(0, 1)) at the row's position, bf16
              (config 1); plain N(0, 1) latents for the large paged configs (3-5)
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .attention import LayerWeights
from .config import ModelConfig

CFG = ModelConfig()


@dataclass(frozen=True)
class Workload:
    name: str
    batch: int
    lengths: tuple[int, ...] | None  # cached rows per request (position of the new token)
    ctx_lo: int = 0                  # ragged: uniform in [ctx_lo, ctx_hi]
    ctx_hi: int = 0
    permute: bool = True
    normed_cache: bool = False
    seed: int = 0

    def seq_lens(self) -> list[int]:
        if self.lengths is not None:
            return list(self.lengths) if len(self.lengths) == self.batch else [self.lengths[0]] * self.batch
        g = torch.Generator().manual_seed(self.seed + 7)
        return torch.randint(self.ctx_lo, self.ctx_hi + 1, (self.batch,), generator=g).tolist()


WORKLOADS = {
    # config 1: single layer, batch 1, context 1024 (the reference's NumPy case)
    "config1": Workload("config1", 1, (1024,), permute=False, normed_cache=True, seed=0),
    # config 3: batched paged decode, B=32, ragged contexts U[512, 8192], permuted block table
    "config3": Workload("config3", 32, None, 512, 8192, permute=True, seed=3),
    # config 4: long-context split-KV, B=8 x 32768
    "config4": Workload("config4", 8, (32768,), permute=True, seed=4),
    # config 5a: B=256 x 4096, sharded by request at N > 1
    "config5a": Workload("config5a", 256, (4096,), permute=True, seed=5),
    # config 5b: one sequence of 131072 tokens, sharded by sequence at N > 1
    "config5b": Workload("config5b", 1, (131072,), permute=True, seed=6),
}


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16)


def make_layer_weights(seed: int, device="cpu", std: float = 0.02, norm: str = "ones") -> LayerWeights:
    """Random-init attention weights of one DeepSeek-V2-Lite layer (bf16)."""
    g = torch.Generator().manual_seed(seed)
    c = CFG
    q = torch.randn(c.heads * c.q_head_dim, c.hidden, generator=g) * std
    kva = torch.randn(c.kv_lora_rank + c.qk_rope, c.hidden, generator=g) * std
    kvb = torch.randn(c.heads * (c.qk_nope + c.v_head), c.kv_lora_rank, generator=g) * std
    if norm == "ones":
        gam = torch.ones(c.kv_lora_rank)
    else:
        gam = torch.rand(c.kv_lora_rank, generator=g) * 0.4 + 0.8
    wo = torch.randn(c.hidden, c.heads * c.v_head, generator=g) * std  # drawn last: the others keep their values
    return LayerWeights(_bf16(q).to(device), _bf16(kva).to(device), _bf16(gam).to(device), _bf16(kvb).to(device),
                        _bf16(wo).to(device))


def rms_normalise(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """bf16(bf16(x / rms(x)) * 1): RMSNorm with unit weight and HF's two roundings."""
    x = x.float()
    y = x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps)
    return _bf16(_bf16(y).float())


def make_hidden(seed: int, batch: int, device="cpu") -> torch.Tensor:
    """x_n [batch, hidden] bf16: N(0,1) after RMSNorm."""
    g = torch.Generator().manual_seed(seed)
    return rms_normalise(torch.randn(batch, CFG.hidden, generator=g)).to(device)


def rope_rows(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """DeepseekV2 interleaved RoPE of rows x [n, 64] with per-row cos/sin [n, 64] (fp32)."""
    n, d = x.shape
    xi = x.view(n, d // 2, 2).transpose(1, 2).reshape(n, d)
    rot = torch.cat([-xi[:, d // 2:], xi[:, : d // 2]], dim=1)
    return xi * cos + rot * sin


def make_cache_rows(seed: int, n: int, cos: torch.Tensor, sin: torch.Tensor, start: int = 0,
                    normed: bool = True, device="cpu") -> torch.Tensor:
    """Cache rows for positions start..start+n-1: [n, 576] bf16 (c_kv | roped k_pe)."""
    g = torch.Generator().manual_seed(seed)
    c = torch.randn(n, CFG.kv_lora_rank, generator=g)
    kp = torch.randn(n, CFG.qk_rope, generator=g)
    c = rms_normalise(c) if normed else _bf16(c)
    if normed:
        kp = _bf16(rope_rows(kp, cos[start:start + n].float().cpu(), sin[start:start + n].float().cpu()))
    else:
        kp = _bf16(kp)
    return torch.cat([c, kp], dim=1).to(device)


def fill_pool_random(pages: torch.Tensor, seed: int) -> None:
    """Fill a whole page pool with N(0,1) bf16 latents on its device (large configs)."""
    g = torch.Generator(device=pages.device).manual_seed(seed)
    flat = pages.view(-1)
    chunk = 1 << 26
    for i in range(0, flat.numel(), chunk):
        n = min(chunk, flat.numel() - i)
        flat[i:i + n] = torch.randn(n, generator=g, device=pages.device).to(torch.bfloat16)


def kv_bytes(seq_lens) -> int:
    """Algorithmic latent-cache bytes one step reads: sum_b (T_b + 1) * 576 * 2."""
    return int(sum((int(t) + 1) * 576 * 2 for t in seq_lens))


def total_bytes(seq_lens) -> int:
    """All bytes one step of K1..K3 must move at least: the cache rows, W_UK and W_UV
    (4,194,304 B), and per request q (3072 x 2) + kv_a (576 x 2) in, the new row
    (1152) and the output (2048 x 2) out."""
    B = len(seq_lens)
    return kv_bytes(seq_lens) + 2 * 16 * 128 * 512 * 2 + B * (3072 * 2 + 576 * 2 + 1152 + 2048 * 2)


def flops(seq_lens) -> int:
    """Reported FLOPs (not the bound): 34,816 per attended row + absorb and W_UV per request."""
    B = len(seq_lens)
    return int(sum((int(t) + 1) * 34816 for t in seq_lens) + B * 2 * 2 * 16 * 128 * 512)
