"""GPU checks of the configuration-4 harness (a Llama-style decoder whose
attention is routed by patch.apply() to sunshape_sdpa): on a small model,
every decode step's routed attention equals softmax attention over the
cache's own dequantised keys and values, and the decode runs end to end."""

import math

import pytest
import torch

import gpu_ref as G

pytestmark = pytest.mark.gpu


def test_small_decoder_routes_attention_to_sunshape(cuda_ok):
    from sunshape_mlx_b200 import harness as H, patch
    from sunshape_mlx_b200.cache import HybridSunShapeKVCache

    cfg = H.DecoderConfig(n_layers=2, hidden=512, n_heads=4, n_kv_heads=2, ffn=1024, vocab=1000)
    model = H.Decoder(cfg, device="cuda", seed=3)
    g = torch.Generator(device="cuda").manual_seed(4)
    codecs = H.fit_layer_codecs(model, torch.randint(0, cfg.vocab, (1, 1024), generator=g, device="cuda"),
                                rows=2048, kmeans_iters=4)
    caches = H.make_caches(model, codecs)
    assert all(isinstance(c, HybridSunShapeKVCache) for c in caches)
    prompt = torch.randint(0, cfg.vocab, (2, 300), generator=g, device="cuda")
    seen = []
    real = patch.scaled_dot_product_attention

    def spy(q, k, v, cache, scale, mask, sinks=None):
        out = real(q, k, v, cache, scale, mask)
        want = G.attention(G.scaled_queries(q, scale), cache.keys.float(), cache.values.float())
        seen.append(G.rel_err(out, want))
        return out

    patch.apply()
    try:
        patch.scaled_dot_product_attention = spy
        ids = model.forward(prompt, caches, 0).argmax(-1, keepdim=True)
        for i in range(3):
            logits = model.forward(ids, caches, 300 + i)
            assert torch.isfinite(logits).all()
            ids = logits.argmax(-1, keepdim=True)
    finally:
        patch.scaled_dot_product_attention = real
        patch.revert()
    assert len(seen) == 3 * cfg.n_layers
    assert max(seen) < 2e-2, seen  # bf16 queries and output
    assert all(c.offset == 303 for c in caches)
