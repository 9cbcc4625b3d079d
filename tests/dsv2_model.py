"""A DeepSeek-V2-Lite-shaped decoder in plain torch with random-init weights: test
infrastructure for the 27-layer token-identity gate (config 2).

The attention task of each decode step is a plug-in (`attn(layer, x_n, pos) -> R(out)`);
everything around it is shared by the arms being compared: token embedding, RMSNorms,
o_proj, the dense FFN of layer 0, the MoE of layers 1-26 (64 routed experts, softmax
gate, top-6 without renormalisation, 2 shared experts), the final norm and lm_head.
Shapes are those of the reference's model config (reference/dsv2lite_config.json:
hidden 2048, 27 layers, intermediate 10944, moe_intermediate 1408, vocab 102400).

The prompt is prefilled once, for all arms, with a causal form of the absorbed-attention
arithmetic that oracle/mla_oracle.py states for one token (project, kv_post,
attend_rows <- src/host/reference_decode.py:225-256): the same bf16 rounding points,
fp32 scores and softmax. Its latent rows seed every arm's cache.
"""
from __future__ import annotations

from dataclasses import dataclass
from types import SimpleNamespace

import torch
import torch.nn.functional as F

BF = torch.bfloat16
HEADS, NOPE, ROPE, VH, LORA = 16, 128, 64, 128, 512


@dataclass
class Shape:
    hidden: int = 2048
    layers: int = 27
    vocab: int = 102400
    dense_ffn: int = 10944
    moe_ffn: int = 1408
    experts: int = 64
    top_k: int = 6
    shared: int = 2
    first_dense: int = 1
    eps: float = 1e-6
    std: float = 0.02


def rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm of a bf16 model: fp32 normalisation rounded to bf16, times the bf16 weight
    (rounded again) -- the two roundings of reference_decode.py:51-65."""
    x32 = x.float()
    y = x32 * (1.0 / torch.sqrt(x32.pow(2).mean(-1, keepdim=True) + eps))
    return w * y.to(BF)


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Interleaved RoPE (interleave-transpose, then rotate_half), reference_decode.py:120-134."""
    d = x.shape[-1]
    x = x.reshape(*x.shape[:-1], d // 2, 2).transpose(-1, -2).reshape(*x.shape[:-1], d)
    rot = torch.cat([-x[..., d // 2:], x[..., : d // 2]], dim=-1)
    return x * cos + rot * sin


def mlp(x: torch.Tensor, gate_up: torch.Tensor, down: torch.Tensor) -> torch.Tensor:
    g, u = F.linear(x, gate_up).chunk(2, dim=-1)
    return F.linear(F.silu(g) * u, down)


class Dsv2Lite:
    """Weights of every layer plus prefill / decode drivers. `attn_weights[l]` holds the
    attention weights of layer l (bf16 LayerWeights on `device`)."""

    def __init__(self, shape: Shape, seed: int, device, attn_weights, softmax_scale: float):
        self.shape, self.device, self.scale = shape, torch.device(device), softmax_scale
        g = torch.Generator(device=self.device).manual_seed(seed)

        def rnd(*s):
            return (torch.randn(*s, generator=g, device=self.device) * shape.std).to(BF)

        H = shape.hidden
        ones = lambda n: torch.ones(n, dtype=BF, device=self.device)
        self.embed = rnd(shape.vocab, H)
        self.lm_head = rnd(shape.vocab, H)
        self.final_norm = ones(H)
        self.layers = []
        for l in range(shape.layers):
            L = SimpleNamespace(in_norm=ones(H), post_norm=ones(H), attn=attn_weights[l], o_proj=rnd(H, HEADS * VH))
            if l < shape.first_dense:
                L.gate_up, L.down = rnd(2 * shape.dense_ffn, H), rnd(H, shape.dense_ffn)
            else:
                L.router = rnd(shape.experts, H)
                L.e_gate_up = torch.stack([rnd(2 * shape.moe_ffn, H) for _ in range(shape.experts)])
                L.e_down = torch.stack([rnd(H, shape.moe_ffn) for _ in range(shape.experts)])
                L.s_gate_up = rnd(2 * shape.shared * shape.moe_ffn, H)
                L.s_down = rnd(H, shape.shared * shape.moe_ffn)
            self.layers.append(L)

    # ------------------------------------------------------------------ shared parts
    def ffn(self, l: int, x: torch.Tensor) -> torch.Tensor:
        L = self.layers[l]
        if l < self.shape.first_dense:
            return mlp(x, L.gate_up, L.down)
        scores = F.linear(x.float(), L.router.float()).softmax(dim=-1)
        w, idx = scores.topk(self.shape.top_k, dim=-1)
        out = torch.zeros(x.shape[0], x.shape[1], dtype=torch.float32, device=x.device)
        for e in torch.unique(idx).tolist():
            tok, slot = (idx == e).nonzero(as_tuple=True)
            y = mlp(x[tok], L.e_gate_up[e], L.e_down[e])
            out.index_add_(0, tok, y.float() * w[tok, slot, None])
        return out.to(BF) + mlp(x, L.s_gate_up, L.s_down)

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        """fp32 logits (an fp32 product of the bf16 head): bf16 logits would tie often at
        this vocabulary size, which leaves greedy argmax to index order."""
        if not hasattr(self, "_lm_head32"):
            self._lm_head32 = self.lm_head.float()
        return F.linear(rms(h, self.final_norm, self.shape.eps).float(), self._lm_head32)

    # ------------------------------------------------------------------ prefill
    def prefill_attention(self, l: int, x_n: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
        """Causal absorbed attention of positions 0..T-1. Returns (R(out) [T, 2048] bf16,
        latent rows [T, 576] bf16 = RMSNorm(c) | RoPE(k_pe))."""
        A, T = self.layers[l].attn, x_n.shape[0]
        q = F.linear(x_n, A.q_proj).float().view(T, HEADS, NOPE + ROPE)
        kv_a = F.linear(x_n, A.kv_a_proj_with_mqa)
        c = rms(kv_a[:, :LORA], A.kv_a_layernorm, self.shape.eps)
        k_pe = rope(kv_a[:, LORA:].float(), cos, sin).to(BF)
        rows = torch.cat([c, k_pe], dim=-1)
        q_pe = rope(q[..., NOPE:], cos[:, None], sin[:, None]).to(BF).float()
        kv_b = A.kv_b_proj.float().view(HEADS, NOPE + VH, LORA)
        q_c = torch.einsum("thd,hdl->thl", q[..., :NOPE], kv_b[:, :NOPE])
        cf, kf = c.float(), k_pe.float()
        s = (torch.einsum("thl,sl->hts", q_c, cf) + torch.einsum("thr,sr->hts", q_pe, kf)) * self.scale
        s = s.masked_fill(torch.ones(T, T, dtype=torch.bool, device=s.device).triu(1), float("-inf"))
        o_c = torch.einsum("hts,sl->thl", s.softmax(dim=-1), cf)
        out = torch.einsum("thl,hvl->thv", o_c, kv_b[:, NOPE:]).reshape(T, HEADS * VH).to(BF)
        return out, rows

    def attend_one(self, l: int, x_n: torch.Tensor, rows: torch.Tensor, pos: int, cos: torch.Tensor,
                   sin: torch.Tensor):
        """Decode-step attention of one token at `pos` in plain torch (fp32 scores and
        softmax, bf16 projections), over rows[0..pos-1] plus its own new row, which it
        stores into rows[pos]. The same arithmetic as prefill_attention's last query."""
        A = self.layers[l].attn
        q = F.linear(x_n, A.q_proj).float().view(1, HEADS, NOPE + ROPE)
        kv_a = F.linear(x_n, A.kv_a_proj_with_mqa)
        c_new = rms(kv_a[:, :LORA], A.kv_a_layernorm, self.shape.eps)
        k_new = rope(kv_a[:, LORA:].float(), cos[pos:pos + 1], sin[pos:pos + 1]).to(BF)
        rows[pos] = torch.cat([c_new, k_new], dim=-1)[0]
        r = rows[: pos + 1].float()
        q_pe = rope(q[..., NOPE:], cos[pos:pos + 1, None], sin[pos:pos + 1, None]).to(BF).float()
        kv_b = A.kv_b_proj.float().view(HEADS, NOPE + VH, LORA)
        q_c = torch.einsum("thd,hdl->thl", q[..., :NOPE], kv_b[:, :NOPE])
        s = (torch.einsum("thl,sl->hts", q_c, r[:, :LORA]) + torch.einsum("thr,sr->hts", q_pe, r[:, LORA:]))
        o_c = torch.einsum("hts,sl->thl", (s * self.scale).softmax(dim=-1), r[:, :LORA])
        return torch.einsum("thl,hvl->thv", o_c, kv_b[:, NOPE:]).reshape(1, HEADS * VH).to(BF)

    def prefill(self, tokens: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
        """Positions 0..T-1 of `tokens`: (latent rows of every layer, last hidden state)."""
        T = tokens.shape[0]
        h = self.embed[tokens]
        rows = []
        for l, L in enumerate(self.layers):
            out, r = self.prefill_attention(l, rms(h, L.in_norm, self.shape.eps), cos[:T], sin[:T])
            rows.append(r)
            h = h + F.linear(out, L.o_proj)
            h = h + self.ffn(l, rms(h, L.post_norm, self.shape.eps))
        return rows, h[-1:]

    # ------------------------------------------------------------------ decode
    def decode(self, token: int, pos: int, attn) -> torch.Tensor:
        """One token at `pos`; attn(l, x_n [1, 2048] bf16, pos) -> R(out) [1, 2048] bf16 and
        appends the token's row to layer l's cache. Returns fp32 logits [vocab]."""
        h = self.embed[token].view(1, -1)
        for l, L in enumerate(self.layers):
            out = attn(l, rms(h, L.in_norm, self.shape.eps), pos)
            h = h + F.linear(out, L.o_proj)
            h = h + self.ffn(l, rms(h, L.post_norm, self.shape.eps))
        return self.logits(h)[0]
