"""Split-KV decode across GPUs for very long single sequences.

Each rank holds a contiguous token range of the cache (``shard_range``) as a
normal SunShape cache. A decode step computes this rank's unnormalised
(o, m, l) rows with the fused kernel (``attention.decode_partials``), gathers
all ranks' rows with one all-gather (NCCL over NVLink on GPUs; any backend
works), and merges them with the log-sum-exp kernel (``ss_lse_merge``):
    m* = max_g m_g,  out = sum_g o_g e^{m_g - m*} / sum_g l_g e^{m_g - m*}.
The exchanged payload is (B * Hq * Tq) x (D + 2) floats per rank.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib as L

__all__ = ["shard_range", "all_gather_partials", "merge_partials", "splitkv_sdpa",
           "PreparedSplitKV"]


def shard_range(n_tokens: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [lo, hi) token range of `rank` (balanced to within one token)."""
    return (n_tokens * rank) // world, (n_tokens * (rank + 1)) // world


def all_gather_partials(part: torch.Tensor, group=None) -> torch.Tensor:
    """(rows, D+2) per rank -> (world, rows, D+2) on every rank."""
    world = dist.get_world_size(group)
    part = part.contiguous()
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world, *part.shape), dtype=part.dtype, device=part.device)
        dist.all_gather_into_tensor(out, part, group=group)
        return out
    bufs = [torch.empty_like(part) for _ in range(world)]
    dist.all_gather(bufs, part, group=group)
    return torch.stack(bufs)


def merge_partials(parts: torch.Tensor, out_shape, out_dtype, v_rot=None) -> torch.Tensor:
    """Log-sum-exp merge of gathered partials on the GPU (ss_lse_merge)."""
    L.require_cuda(parts)
    g, rows, rf = parts.shape
    d = rf - 2
    out = torch.empty(out_shape, dtype=out_dtype, device=parts.device)
    L.call("ss_lse_merge", L.ptr(parts.contiguous()), g, rows, d, L.ptr(v_rot), L.ptr(out),
           L.dtype_code(out_dtype), d, L.stream_ptr(parts.device))
    return out


def splitkv_sdpa(queries: torch.Tensor, shard_cache, scale: float, group=None) -> torch.Tensor:
    """Decode attention over a cache sharded by token range across the group."""
    from .attention import decode_partials

    part = decode_partials(queries, shard_cache, scale)
    parts = all_gather_partials(part, group)
    v_rot = None
    spec = shard_cache.attention_spec()
    if spec.get("v_rot") is not None:
        v_rot = spec["v_rot"].contiguous()
    return merge_partials(parts, queries.shape, queries.dtype, v_rot)


class PreparedSplitKV:
    """The split-KV decode step with everything built once (the argument
    block of this shard's fused decode, the gather and output buffers): each
    ``run()`` is one C call for this shard's (o, m, l) rows, one all-gather
    into a kept buffer and one C call for the log-sum-exp merge, so the host
    issues a step in microseconds. The shard cache must not be reallocated
    between calls; queries are read from ``q`` in place."""

    def __init__(self, q: torch.Tensor, shard_cache, scale: float, group=None):
        import ctypes as C

        from .attention import PreparedDecode

        B, Hq, Tq, D = q.shape
        self.group = group
        self.world = dist.get_world_size(group)
        self.part = torch.empty((B * Hq * Tq, D + 2), dtype=torch.float32, device=q.device)
        self.decode = PreparedDecode(q, shard_cache, scale, part_out=self.part)
        self.parts = torch.empty((self.world, *self.part.shape), dtype=torch.float32,
                                 device=q.device)
        self.out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
        vr = shard_cache.attention_spec().get("v_rot")
        self.v_rot = vr.contiguous() if vr is not None else None
        self._lib = L.load()
        self._merge_args = (C.c_void_p(self.parts.data_ptr()), self.world, self.part.shape[0], D,
                            L.ptr(self.v_rot), C.c_void_p(self.out.data_ptr()),
                            L.dtype_code(q.dtype), D)
        self.device = q.device

    def run_partials(self) -> torch.Tensor:
        return self.decode.run()

    def gather(self) -> None:
        if dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(self.parts, self.part, group=self.group)
        else:
            self.parts.copy_(all_gather_partials(self.part, self.group))

    def merge(self) -> torch.Tensor:
        L.check("ss_lse_merge", self._lib.ss_lse_merge(*self._merge_args, L.stream_ptr(self.device)))
        return self.out

    def run(self) -> torch.Tensor:
        self.run_partials()
        self.gather()
        return self.merge()
