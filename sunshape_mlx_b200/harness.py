"""Llama-style decoder for the end-to-end configuration-4 benchmark.

The reference runs its caches inside mlx-lm models and swaps attention by
monkey-patching mlx-lm's ``scaled_dot_product_attention`` (patch.py:27-34,
59-74). mlx-lm does not exist here, so this module is the model side of that
setup: a Llama-architecture decoder (RMSNorm, grouped-query attention with
RoPE, SwiGLU MLP) whose attention calls go through
``patch.current_sdpa()``. After ``patch.apply()`` they reach
``sunshape_sdpa`` for layers that hold a SunShape cache, exactly as the
patched mlx-lm model would; otherwise dense attention runs.

Weights are random (no checkpoints are available); projections use cuBLAS
through ``torch`` matmuls. Prefill attention is dense over the uncompressed
keys and values of the prompt, whose keys and values then go into the
compressed caches (one ``append`` per layer); every decode step appends the
new token and attends over the compressed cache.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

from . import patch
from .cache import create_kv_cache
from .codec import SunShapeBlockCodec

__all__ = ["DecoderConfig", "Decoder", "fit_layer_codecs", "make_caches"]


@dataclass
class DecoderConfig:
    n_layers: int = 32
    hidden: int = 4096
    n_heads: int = 32
    n_kv_heads: int = 8
    ffn: int = 14336
    vocab: int = 128256
    rope_theta: float = 1.0e6
    norm_eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.hidden // self.n_heads


class Decoder:
    """Weights and forward pass; ``forward(ids, caches, pos)`` returns the
    last position's logits (B, vocab) in float32."""

    def __init__(self, cfg: DecoderConfig, device="cuda", dtype=torch.bfloat16, seed: int = 7):
        self.cfg, self.device, self.dtype = cfg, torch.device(device), dtype
        g = torch.Generator(device=self.device).manual_seed(seed)
        D, H, Hk, d = cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim

        def w(*shape):
            return (torch.randn(*shape, generator=g, device=self.device, dtype=torch.float32) * 0.02).to(dtype)

        self.embed = w(cfg.vocab, D)
        self.layers = []
        for _ in range(cfg.n_layers):
            self.layers.append({
                "wqkv": w(D, (H + 2 * Hk) * d), "wo": w(H * d, D),
                "w13": w(D, 2 * cfg.ffn), "w2": w(cfg.ffn, D),
                "n1": torch.ones(D, device=self.device, dtype=dtype),
                "n2": torch.ones(D, device=self.device, dtype=dtype),
            })
        self.norm = torch.ones(D, device=self.device, dtype=dtype)
        self.lm_head = w(D, cfg.vocab)
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, device=self.device, dtype=torch.float32) / d))
        self._inv_freq = inv

    # ------------------------------------------------------------ pieces
    def _rms(self, x, wgt):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.cfg.norm_eps)).to(x.dtype) * wgt

    def _rope(self, x, pos0: int):
        # x (B, h, T, d); rotate-half convention
        T, d = x.shape[2], x.shape[3]
        t = torch.arange(pos0, pos0 + T, device=x.device, dtype=torch.float32)
        ang = torch.outer(t, self._inv_freq)
        cos, sin = ang.cos(), ang.sin()
        x1, x2 = x[..., : d // 2].float(), x[..., d // 2:].float()
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1).to(x.dtype)

    def _qkv(self, h, layer, pos0):
        cfg = self.cfg
        B, T, _ = h.shape
        H, Hk, d = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        qkv = self._rms(h, layer["n1"]) @ layer["wqkv"]
        q = qkv[..., : H * d].view(B, T, H, d).transpose(1, 2)
        k = qkv[..., H * d:(H + Hk) * d].view(B, T, Hk, d).transpose(1, 2)
        v = qkv[..., (H + Hk) * d:].view(B, T, Hk, d).transpose(1, 2)
        return self._rope(q, pos0), self._rope(k, pos0).contiguous(), v.contiguous()

    def _mlp(self, h, layer):
        x = self._rms(h, layer["n2"]) @ layer["w13"]
        a, b = x.chunk(2, dim=-1)
        return (F.silu(a) * b) @ layer["w2"]

    # ------------------------------------------------------------ passes
    @torch.no_grad()
    def forward(self, ids: torch.Tensor, caches, pos0: int, collect=None) -> torch.Tensor:
        """ids (B, T). With T > 1 (prefill) attention is dense and causal over
        the prompt and the prompt's keys/values are appended to each layer's
        cache; with T == 1 (decode) the new token is appended and attention
        goes through the patched router. ``collect`` (a list) receives each
        layer's post-RoPE keys and values (calibration)."""
        cfg = self.cfg
        h = self.embed[ids]
        B, T, _ = h.shape
        scale = 1.0 / math.sqrt(cfg.head_dim)
        sdpa = patch.current_sdpa()
        for li, layer in enumerate(self.layers):
            q, k, v = self._qkv(h, layer, pos0)
            if collect is not None:
                collect.append((k, v))
            cache = caches[li] if caches is not None else None
            if T > 1 or cache is None:
                o = patch._dense_sdpa(q, k, v, scale, "causal" if T > 1 else None)
                if cache is not None:
                    cache.append(k, v)
            else:
                cache.append(k, v)
                o = sdpa(q, None, None, cache, scale, None)
            o = o.transpose(1, 2).reshape(B, T, cfg.n_heads * cfg.head_dim)
            h = h + o @ layer["wo"]
            h = h + self._mlp(h, layer)
        hl = self._rms(h[:, -1], self.norm)
        return (hl @ self.lm_head).float()


@torch.no_grad()
def fit_layer_codecs(model: Decoder, calib_ids: torch.Tensor, *, block_dim: int = 4,
                     n_centroids: int = 256, rows: int = 4096, kmeans_iters: int = 15, seed: int = 0):
    """Per-layer key and value codecs (block-VQ, ProfilePerm) fit on the
    activations of one dense pass over ``calib_ids``: each layer's post-RoPE
    keys and its values, ``rows`` rows sampled from (tokens x kv-heads); the
    keys' ProfilePerm calibration uses the same layer's keys as queries."""
    acts = []
    model.forward(calib_ids, None, 0, collect=acts)
    d = model.cfg.head_dim
    rng = np.random.default_rng(seed)
    out = []
    for li, (k, v) in enumerate(acts):
        kr = k.transpose(1, 2).reshape(-1, d).float()
        vr = v.transpose(1, 2).reshape(-1, d).float()
        pick = torch.as_tensor(rng.permutation(kr.shape[0])[:rows], device=kr.device)
        kc = SunShapeBlockCodec(head_dim=d, block_dim=block_dim, n_centroids=n_centroids,
                                device=model.device)
        kc.fit(kr[pick], kr[pick], kmeans_iters=kmeans_iters, seed=seed + li)
        vc = SunShapeBlockCodec(head_dim=d, block_dim=block_dim, n_centroids=n_centroids,
                                device=model.device)
        vc.fit(vr[pick], vr[pick], kmeans_iters=kmeans_iters, seed=seed + 1000 + li)
        out.append((kc, vc))
    return out


def make_caches(model: Decoder, codecs):
    """One hybrid cache per layer: block-VQ keys and block-VQ values
    (``value_backend="sunshape"``), no fp16 tail (buffer_size 0)."""
    return [create_kv_cache(kc, n_kv_heads=model.cfg.n_kv_heads, value_backend="sunshape",
                            value_bits=8, value_codec=vc, buffer_size=0)
            for kc, vc in codecs]
