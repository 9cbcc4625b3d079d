"""The config-2 model harness (tests/dsv2_model.py) on CPU, pinned to the oracle.

Prefill of T+1 tokens must agree with prefill of T tokens followed by one decode step
whose attention is the oracle's attention task (the reference's arithmetic): same
appended latent rows, same logits within the bf16 tolerance. This checks the causal
prefill arithmetic that seeds every arm's cache in the 27-layer token-identity test.
"""
import numpy as np
import torch

from dsv2_model import Dsv2Lite, Shape
from mla_testlib import O, fleet, oracle_weights, rel_cos, workloads

T = 40


def _model():
    shape = Shape(layers=2, vocab=512, dense_ffn=256, moe_ffn=64, experts=8, top_k=2, shared=1)
    lws = [workloads.make_layer_weights(300 + l, norm="uniform") for l in range(shape.layers)]
    return Dsv2Lite(shape, 5, "cpu", lws, fleet.ModelConfig().softmax_scale), lws


def test_prefill_is_causal_and_matches_oracle_decode():
    model, lws = _model()
    cfg = O.Config()
    cos, sin = cfg.cos_sin(64)
    cos_t, sin_t = torch.from_numpy(cos), torch.from_numpy(sin)
    tokens = torch.randint(0, model.shape.vocab, (T + 1,), generator=torch.Generator().manual_seed(6))
    rows_full, h_full = model.prefill(tokens, cos_t, sin_t)
    rows, _ = model.prefill(tokens[:T], cos_t, sin_t)
    for l in range(model.shape.layers):
        assert torch.equal(rows[l], rows_full[l][:T]), "prefill rows depend on later tokens"

    ws = [oracle_weights(lw) for lw in lws]
    caches = [np.zeros((T + 1, 576), np.float32) for _ in ws]
    for l, r in enumerate(rows):
        caches[l][:T] = r.float().numpy()

    def attn(l, x_n, pos):
        out = O.attention_task(cfg, ws[l], x_n.float().numpy()[0], caches[l], pos, cos, sin)
        return torch.from_numpy(out).to(torch.bfloat16)[None]

    logits = model.decode(int(tokens[T]), T, attn)
    for l in range(model.shape.layers):
        mism = np.count_nonzero(caches[l][T] != rows_full[l][T].float().numpy())
        assert mism <= 4, f"layer {l}: {mism} elements of the appended row differ from prefill's"
    rel, cs = rel_cos(logits.numpy(), model.logits(h_full)[0].numpy())
    assert rel <= 2e-2 and cs >= 0.9999, (rel, cs)
