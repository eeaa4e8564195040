"""Drop-in routing of attention calls to the SunShape kernels (patch.py of
the reference).

The reference monkey-patches mlx-lm's ``scaled_dot_product_attention``.
Here the same router is exposed as :func:`scaled_dot_product_attention`
(mlx-lm's signature: queries, keys, values, cache, scale, mask, sinks) and
``apply()`` installs it as the attention function of this package's model
code and, when ``transformers`` is importable, registers it in
``transformers.AttentionInterface`` under the name ``"sunshape"``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .attention import sunshape_sdpa
from .cache import HybridSunShapeKVCache, SunShapeKVCache

__all__ = ["apply", "revert", "is_patched", "scaled_dot_product_attention", "current_sdpa"]

_patched = False


def _dense_sdpa(queries, keys, values, scale, mask):
    hq, hkv = queries.shape[1], keys.shape[1]
    if hq != hkv:
        keys = keys.repeat_interleave(hq // hkv, dim=1)
        values = values.repeat_interleave(hq // hkv, dim=1)
    is_causal = isinstance(mask, str) and mask == "causal"
    attn_mask = None if isinstance(mask, str) or mask is None else mask
    return F.scaled_dot_product_attention(queries, keys.to(queries.dtype), values.to(queries.dtype),
                                          attn_mask=attn_mask, is_causal=is_causal and
                                          queries.shape[2] > 1, scale=scale)


def scaled_dot_product_attention(queries, keys, values, cache, scale, mask, sinks=None):
    """Router (patch.py:59-74): SunShape caches -> sunshape_sdpa, else dense SDPA."""
    if isinstance(cache, (SunShapeKVCache, HybridSunShapeKVCache)):
        return sunshape_sdpa(queries, cache, scale, mask)
    if sinks is not None:
        raise NotImplementedError("attention sinks are not supported by the dense path")
    return _dense_sdpa(queries, keys, values, scale, mask)


def _hf_attention(module, query, key, value, attention_mask, scaling=None, dropout=0.0, **kw):
    cache = kw.get("sunshape_cache")
    out = scaled_dot_product_attention(query, key, value, cache,
                                       scaling if scaling is not None else query.shape[-1] ** -0.5,
                                       attention_mask if attention_mask is not None else None)
    return out.transpose(1, 2).contiguous(), None


def current_sdpa():
    """The attention function model code should call."""
    return scaled_dot_product_attention if _patched else _dense_sdpa_router


def _dense_sdpa_router(queries, keys, values, cache, scale, mask, sinks=None):
    return _dense_sdpa(queries, keys, values, scale, mask)


def apply() -> None:
    """Activate routing (idempotent)."""
    global _patched
    if _patched:
        return
    try:
        from transformers import AttentionInterface  # type: ignore

        AttentionInterface.register("sunshape", _hf_attention)
    except Exception:  # transformers absent or without the registry
        pass
    _patched = True


def revert() -> None:
    global _patched
    _patched = False


def is_patched() -> bool:
    return _patched
