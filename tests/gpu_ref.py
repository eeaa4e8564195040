"""Plain-torch fp32/fp64 references used by the GPU parity tests (independent
of the CUDA library: gathers and matmuls only)."""

import math

import numpy as np
import torch


def dequant_codec_space(idx: torch.Tensor, cents: torch.Tensor) -> torch.Tensor:
    """(..., nb) uint8 -> (..., nb*bd) f32 by indexing the centroid tables."""
    nb, k, bd = cents.shape
    flat = idx.long()
    out = cents[torch.arange(nb, device=idx.device), flat]  # (..., nb, bd)
    return out.reshape(*idx.shape[:-1], nb * bd)


def scaled_queries(q: torch.Tensor, scale: float) -> torch.Tensor:
    """attention.py:208 semantics: q * scale in q's dtype."""
    if q.dtype == torch.float16:
        return (q.float() * float(np.float16(scale))).half().float()
    if q.dtype == torch.bfloat16:
        return (q.float() * float(torch.tensor(scale).bfloat16())).bfloat16().float()
    return q.float() * scale


def attention(qs: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal=False, mask=None,
              mask_bool=False) -> torch.Tensor:
    """qs (B,Hq,Tq,D) f32 scaled; k,v (B,Hkv,T,D); fp64 softmax."""
    B, Hq, Tq, D = qs.shape
    hkv = k.shape[1]
    rep = Hq // hkv
    kk = k.double().repeat_interleave(rep, dim=1)
    vv = v.double().repeat_interleave(rep, dim=1)
    s = qs.double() @ kk.transpose(-1, -2)
    T = k.shape[2]
    if causal:
        ok = (torch.arange(T - Tq, T, device=qs.device)[:, None] >=
              torch.arange(T, device=qs.device)[None, :])
        s = torch.where(ok, s, torch.tensor(float(np.finfo(np.float32).min), dtype=s.dtype, device=s.device))
    if mask is not None:
        if mask_bool:
            s = torch.where(mask.bool(), s, torch.tensor(float(np.finfo(np.float32).min), dtype=s.dtype, device=s.device))
        else:
            s = s + mask.double()
    w = torch.softmax(s, dim=-1)
    return (w @ vv).float()


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    """max |a-b| / max |b|."""
    return float((a.float() - b.float()).abs().max() / b.float().abs().max().clamp(min=1e-30))
