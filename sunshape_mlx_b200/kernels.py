"""Kernel-level API (kernels.py of the reference), backed by the sm_100a C ABI.

Names and argument meanings follow the reference's wrappers so callers can
switch over; arrays are torch CUDA tensors (NumPy inputs are moved to the
current CUDA device). Where the reference returned ``None`` to request a CPU
fallback, these raise ``SunShapeCudaError`` instead.
"""

from __future__ import annotations

import numpy as np
import torch

from . import _lib as L

__all__ = [
    "pack_indices", "unpack_indices", "quantize_values", "dequantize_values",
    "quantize_scalar_to_indices", "block_vq_quantize_metal", "block_vq_score_metal",
    "fused_block_vq_attention", "fused_attention_metal", "fused_attention_causal_metal",
    "fused_attention_dequant_metal", "fused_attention_dequant_causal_metal",
    "get_kernel_stats", "reset_kernel_stats", "vq_assign", "vq_scores", "vq_dequant",
    "packed_dim", "decode_tile", "cuda_tensor",
]

# Every per-token array handed to the fused attention kernel must hold a
# whole number of these tiles per (batch, kv-head) pair.
decode_tile = 128


def cuda_tensor(x, dtype: torch.dtype | None = None, device=None) -> torch.Tensor:
    """Returns x as a contiguous CUDA tensor (copying host data over)."""
    if isinstance(x, torch.Tensor):
        t = x
    else:
        t = torch.as_tensor(np.asarray(x))
    if not t.is_cuda:
        t = t.to(device or torch.device("cuda", torch.cuda.current_device()))
    elif device is not None:
        t = t.to(device)
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t.contiguous()


def get_kernel_stats() -> dict[str, int]:
    """Dispatch counters per C entry point (kernels.py:45-47)."""
    return L.kernel_stats()


def reset_kernel_stats() -> None:
    """kernels.py:40-42."""
    L.reset_kernel_stats()


def packed_dim(d: int, bits: int) -> int:
    """uint32 words per packed row (value_codecs.py:90-101)."""
    if bits == 2:
        if d % 16:
            raise ValueError(f"head_dim must be divisible by 16 for 2-bit packing, got {d}")
        return d // 16
    if bits == 3:
        return (d + 9) // 10
    if bits == 4:
        if d % 8:
            raise ValueError(f"head_dim must be divisible by 8 for 4-bit packing, got {d}")
        return d // 8
    raise ValueError(f"Unsupported bits: {bits}")


# ------------------------------------------------------------------ codec kernels

def vq_assign(keys: torch.Tensor, centroids: torch.Tensor, *, perm: torch.Tensor | None = None,
              heavy: torch.Tensor | None = None, out_idx: torch.Tensor | None = None,
              out_pt: torch.Tensor | None = None, out_heavy: torch.Tensor | None = None,
              dist_mode: int = 0) -> torch.Tensor:
    """Nearest-centroid indices of every row of ``keys`` (..., d).

    keys may be a strided view with 2-level row layout (..., T, d); indices
    are written to ``out_idx`` (same leading shape, nb bytes per row).
    """
    L.poll_device_errors()
    L.require_cuda(keys, centroids)
    nb, k, bd = centroids.shape
    d = keys.shape[-1]
    if keys.stride(-1) != 1:
        keys = keys.contiguous()
    lead = keys.shape[:-1]
    if len(lead) == 0:
        raise ValueError("keys must have at least 2 dimensions")
    k3 = keys.reshape(-1, *keys.shape[-2:]) if keys.dim() > 2 else keys.unsqueeze(0)
    if keys.dim() > 3 and not _collapsible(keys):
        keys = keys.contiguous()
        k3 = keys.reshape(-1, *keys.shape[-2:])
    g, t = k3.shape[0], k3.shape[1]
    if out_idx is None:
        out_idx = torch.empty((*lead, nb), dtype=torch.uint8, device=keys.device)
    o3 = out_idx.reshape(-1, *out_idx.shape[-2:]) if out_idx.dim() > 2 else out_idx.unsqueeze(0)
    h3 = None
    if out_heavy is not None:
        h3 = out_heavy.reshape(-1, *out_heavy.shape[-2:]) if out_heavy.dim() > 2 else out_heavy.unsqueeze(0)
    L.call("ss_vq_assign", L.ptr(k3), L.dtype_code(keys.dtype), g, t, k3.stride(0), k3.stride(1),
           d, L.ptr(perm), L.ptr(centroids), bd, k, L.ptr(heavy), L.ptr(o3), o3.stride(0),
           o3.stride(1), L.ptr(h3), h3.stride(0) if h3 is not None else 0,
           h3.stride(1) if h3 is not None else 0, L.ptr(out_pt), dist_mode,
           L.stream_ptr(keys.device))
    return out_idx


def rotate_rows(x: torch.Tensor, m: torch.Tensor, out_dtype=torch.float32) -> torch.Tensor:
    """x (..., d) @ m (d, d) on the library's own kernel (fp32 fused
    multiply-adds in index order); used for the rotations on the data path."""
    L.require_cuda(x, m)
    d = x.shape[-1]
    xf = x.reshape(-1, d)
    if xf.dtype != torch.float32 or xf.stride(-1) != 1:
        xf = xf.float().contiguous()
    mm = m.to(torch.float32).contiguous()
    out = torch.empty((*x.shape[:-1], d), dtype=out_dtype, device=x.device)
    L.call("ss_rotate_rows", L.ptr(xf), xf.shape[0], d, xf.stride(0), L.ptr(mm), L.ptr(out),
           L.dtype_code(out_dtype), d, L.stream_ptr(x.device))
    return out


def set_assign_path(path: str = "auto") -> None:
    """Selects the assignment kernel process-wide: "auto", "simt" (CUDA cores)
    or "tensor" (tcgen05; raises for unsupported shapes). Results are identical."""
    L.call("ss_set_assign_path", {"auto": 0, "simt": 1, "tensor": 2}[path])


def assign_check(device=None) -> None:
    """Synchronizes and raises if a tensor-core assignment pipeline wait timed out."""
    L.call("ss_vq_assign_check", L.stream_ptr(device or torch.device("cuda")))


def _collapsible(t: torch.Tensor) -> bool:
    """True if all dims before the last two collapse into one strided dim."""
    lead = t.shape[:-2]
    st = t.stride()[:-2]
    for i in range(len(lead) - 1):
        if st[i] != st[i + 1] * lead[i + 1]:
            return False
    return True


def vq_scores(q_codec: torch.Tensor, centroids: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    """out[q, t] = sum_b <q_b, C[b, idx[t, b]]> for q already in codec space."""
    L.require_cuda(q_codec, centroids, idx)
    q = q_codec.to(torch.float32).contiguous()
    nb, k, bd = centroids.shape
    t = idx.shape[0]
    out = torch.empty((q.shape[0], t), dtype=torch.float32, device=q.device)
    L.call("ss_vq_scores", L.ptr(q), q.shape[0], q.shape[1], L.ptr(centroids), bd, k, L.ptr(idx),
           t, idx.stride(0), L.ptr(out), out.stride(0), L.stream_ptr(q.device))
    return out


def vq_dequant(idx: torch.Tensor, centroids: torch.Tensor, *, inv_perm: torch.Tensor | None = None,
               heavy: torch.Tensor | None = None, heavy_vals: torch.Tensor | None = None,
               out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Rows of concatenated centroids (+ heavy fp16 blocks), inverse-permuted."""
    L.require_cuda(idx, centroids)
    nb, k, bd = centroids.shape
    d = nb * bd
    lead = idx.shape[:-1]
    i3 = idx.reshape(-1, *idx.shape[-2:]) if idx.dim() > 2 else idx.unsqueeze(0)
    out = torch.empty((*lead, d), dtype=out_dtype, device=idx.device)
    o3 = out.reshape(-1, *out.shape[-2:]) if out.dim() > 2 else out.unsqueeze(0)
    h3 = None
    if heavy_vals is not None:
        h3 = heavy_vals.reshape(-1, *heavy_vals.shape[-2:]) if heavy_vals.dim() > 2 else heavy_vals.unsqueeze(0)
    L.call("ss_vq_dequant", L.ptr(i3), i3.shape[0], i3.shape[1], i3.stride(0), i3.stride(1),
           L.ptr(centroids), d, bd, k, L.ptr(inv_perm), L.ptr(heavy), L.ptr(h3),
           h3.stride(0) if h3 is not None else 0, h3.stride(1) if h3 is not None else 0,
           L.ptr(o3), L.dtype_code(out_dtype), o3.stride(0), o3.stride(1),
           L.stream_ptr(idx.device))
    return out


def block_vq_quantize_metal(keys_transformed, centroids, n_blocks: int, n_centroids: int,
                            block_dim: int, head_dim: int) -> torch.Tensor:
    """Vectorized block-VQ assignment (kernels.py:1037-1082): keys already in
    codec space, (N, head_dim) -> (N, n_blocks) uint8."""
    k = cuda_tensor(keys_transformed)
    c = cuda_tensor(centroids, torch.float32, k.device)
    if c.shape != (n_blocks, n_centroids, block_dim) or k.shape[-1] != head_dim:
        raise ValueError("block_vq_quantize_metal: shape mismatch")
    return vq_assign(k, c)


def block_vq_score_metal(qdots, indices, n_qh: int, T_kv: int, n_blocks: int,
                         n_centroids: int) -> torch.Tensor:
    """score[q, t] = sum_b qdots[q, b, indices[t, b]] (kernels.py:87-116)."""
    qd = cuda_tensor(qdots, torch.float32)
    idx = cuda_tensor(indices, torch.uint8, qd.device)
    if qd.shape != (n_qh, n_blocks, n_centroids) or idx.shape != (T_kv, n_blocks):
        raise ValueError("block_vq_score_metal: shape mismatch")
    out = torch.empty((n_qh, T_kv), dtype=torch.float32, device=qd.device)
    L.call("ss_vq_scores_lut", L.ptr(qd), n_qh, n_blocks, n_centroids, L.ptr(idx), T_kv,
           idx.stride(0), L.ptr(out), out.stride(0), L.stream_ptr(qd.device))
    return out


# ------------------------------------------------------------------ packing / values

def pack_indices(indices, bits: int) -> torch.Tensor:
    """kernels.py:1102-1137."""
    x = cuda_tensor(indices, torch.uint8)
    d = x.shape[-1]
    if bits == 2 and d % 16:
        raise ValueError(f"Last dim must be divisible by 16 for 2-bit, got {d}")
    if bits == 4 and d % 8:
        raise ValueError(f"Last dim must be divisible by 8 for 4-bit, got {d}")
    if bits not in (2, 3, 4):
        raise ValueError(f"Unsupported bits: {bits}")
    nw = packed_dim(d, bits)
    out = torch.empty((*x.shape[:-1], nw), dtype=torch.int32, device=x.device)
    rows = x.numel() // d if d else 0
    L.call("ss_pack_indices", L.ptr(x), rows, d, bits, L.ptr(out), L.stream_ptr(x.device))
    return out  # int32 storage holding the uint32 bit patterns


def unpack_indices(packed, D: int, bits: int) -> torch.Tensor:
    """kernels.py:1140-1163 (codes returned as uint8)."""
    p = cuda_tensor(packed)
    if p.dtype != torch.int32:
        p = p.view(torch.int32) if p.element_size() == 4 else p.to(torch.int32)
    if bits not in (2, 3, 4):
        raise ValueError(f"Unsupported bits: {bits}")
    rows = p.numel() // p.shape[-1] if p.shape[-1] else 0
    out = torch.empty((*p.shape[:-1], D), dtype=torch.uint8, device=p.device)
    L.call("ss_unpack_indices", L.ptr(p), rows, D, bits, L.ptr(out), L.stream_ptr(p.device))
    return out


def quantize_scalar_to_indices(values, boundaries, *, prefer_metal: bool = True):
    """kernels.py:473-507: (indices uint8, backend)."""
    v = cuda_tensor(values, torch.float32)
    b = cuda_tensor(boundaries, torch.float32, v.device)
    out = torch.empty(v.shape, dtype=torch.uint8, device=v.device)
    L.call("ss_scalar_quantize", L.ptr(v), v.numel(), L.ptr(b), b.numel(), L.ptr(out),
           L.stream_ptr(v.device))
    return out, "cuda"


def quantize_values(values, bits: int = 4, group_size: int = 64):
    """Asymmetric per-group min-max (kernels.py:1173-1228).
    Returns (packed words, scales f32, zeros f32, n_groups); packed words are
    int32 tensors holding the reference's uint32 bit patterns."""
    v = cuda_tensor(values)
    if v.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        v = v.float()
    d = v.shape[-1]
    if d % group_size:
        raise ValueError(f"head_dim {d} not divisible by group_size {group_size}")
    g = d // group_size
    lead = v.shape[:-1]
    rows = v.numel() // d if d else 0
    packed = torch.empty((*lead, packed_dim(d, bits)), dtype=torch.int32, device=v.device)
    scales = torch.empty((*lead, g), dtype=torch.float32, device=v.device)
    zeros = torch.empty((*lead, g), dtype=torch.float32, device=v.device)
    L.call("ss_value_encode_grouped", L.ptr(v), L.dtype_code(v.dtype), 1, rows, 0, d, d, bits,
           group_size, L.ptr(packed), 0, packed.shape[-1], L.ptr(scales), L.ptr(zeros), 0, g,
           L.stream_ptr(v.device))
    return packed, scales, zeros, g


def dequantize_values(packed, scales, zeros, D: int, bits: int = 4, group_size: int = 64,
                      out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """q * scale + zero (kernels.py:1231-1269)."""
    p = cuda_tensor(packed)
    if p.dtype != torch.int32:
        p = p.view(torch.int32) if p.element_size() == 4 else p.to(torch.int32)
    s = cuda_tensor(scales, torch.float32, p.device)
    z = cuda_tensor(zeros, torch.float32, p.device)
    g = D // group_size
    lead = p.shape[:-1]
    rows = p.numel() // p.shape[-1] if p.shape[-1] else 0
    lv = torch.arange(2 ** bits, dtype=torch.float32, device=p.device)
    out = torch.empty((*lead, D), dtype=out_dtype, device=p.device)
    L.call("ss_value_decode", L.ptr(p), 1, rows, 0, p.shape[-1], D, bits, group_size, L.ptr(lv),
           L.ptr(s), L.SS_F32, L.ptr(z), 0, g, None, L.ptr(out), L.dtype_code(out_dtype), 0, D,
           L.stream_ptr(p.device))
    return out


# ------------------------------------------------------------------ fused attention

def fused_block_vq_attention(qdots, indices, values, T_q: int, T_kv: int, n_blocks: int,
                             n_centroids: int, head_dim: int) -> torch.Tensor:
    """Gather-score + causal softmax + value product from a precomputed table
    (kernels.py:514-563): scores by the gather kernel, the rest by torch ops
    on the GPU (this helper is not on the decode hot path)."""
    s = block_vq_score_metal(qdots, indices, T_q, T_kv, n_blocks, n_centroids)
    v = cuda_tensor(values, torch.float32, s.device)
    if T_kv >= T_q:
        qpos = torch.arange(T_kv - T_q, T_kv, device=s.device)
        kpos = torch.arange(T_kv, device=s.device)
        s = torch.where(qpos[:, None] >= kpos[None, :], s, torch.finfo(torch.float32).min)
    w = torch.softmax(s.double(), dim=-1).float()
    return w @ v


def _pad_rows(x: torch.Tensor, rows: int) -> torch.Tensor:
    if x.shape[0] == rows:
        return x.contiguous()
    out = torch.zeros((rows, *x.shape[1:]), dtype=x.dtype, device=x.device)
    out[: x.shape[0]] = x
    return out


def _fused(queries, centroids, indices, values_f16=None, packed=None, scales=None, zeros=None,
           bits=0, group_size=0, causal=False, q_offset=0):
    from .attention import _run_decode  # local import: attention imports this module

    q = cuda_tensor(queries, torch.float32)
    n_qh, d = q.shape
    c = cuda_tensor(centroids, torch.float32, q.device)
    idx = cuda_tensor(indices, torch.uint8, q.device)
    t = idx.shape[0]
    if t == 0:
        return torch.zeros((n_qh, d), dtype=torch.float32, device=q.device)
    if causal and q_offset != t - n_qh:
        raise NotImplementedError("causal fused attention supports q_offset = T_kv - n_qh only")
    cap = -(-t // decode_tile) * decode_tile
    spec = dict(idx=_pad_rows(idx, cap)[None, None], cap=cap, tc=t)
    if values_f16 is not None:
        spec["v"] = _pad_rows(cuda_tensor(values_f16, torch.float16, q.device), cap)[None, None]
    else:
        spec["vq"] = _pad_rows(cuda_tensor(packed, torch.int32, q.device), cap)[None, None]
        spec["vs"] = _pad_rows(cuda_tensor(scales, torch.float32, q.device), cap)[None, None]
        spec["vz"] = _pad_rows(cuda_tensor(zeros, torch.float32, q.device), cap)[None, None]
        spec["bits"], spec["group"] = bits, group_size
        spec["levels"] = [float(i) for i in range(2 ** bits)]
    out = torch.empty((1, n_qh, 1, d), dtype=torch.float32, device=q.device)
    # rows of `queries` are query positions of one head: map them to tq
    _run_decode(q.view(1, 1, n_qh, d), centroids=c, perm=None, scale=1.0, spec=spec,
                causal=causal, out=out.view(1, 1, n_qh, d))
    return out.view(n_qh, d)


def fused_attention_metal(queries, centroids, indices, values, n_qh: int, T_kv: int,
                          n_blocks: int, n_centroids: int, head_dim: int) -> torch.Tensor:
    """Fused online-softmax block-VQ attention (kernels.py:233-291): queries
    (n_qh, D) pre-scaled and in codec space; values are consumed as fp16."""
    return _fused(queries, centroids, indices, values_f16=values)


def fused_attention_causal_metal(queries, centroids, indices, values, n_qh: int, T_kv: int,
                                 n_blocks: int, n_centroids: int, head_dim: int,
                                 q_offset: int = 0) -> torch.Tensor:
    """Causal variant (kernels.py:388-446): row i sees keys <= q_offset + i."""
    return _fused(queries, centroids, indices, values_f16=values, causal=True, q_offset=q_offset)


def fused_attention_dequant_metal(queries, centroids, indices, packed_values, scales, zeros,
                                  n_qh: int, T_kv: int, n_blocks: int, n_centroids: int,
                                  head_dim: int, bits: int, group_size: int) -> torch.Tensor:
    """Fused attention over grouped-quantized values (kernels.py:697-765)."""
    return _fused(queries, centroids, indices, packed=packed_values, scales=scales, zeros=zeros,
                  bits=bits, group_size=group_size)


def fused_attention_dequant_causal_metal(queries, centroids, indices, packed_values, scales,
                                         zeros, n_qh: int, T_kv: int, n_blocks: int,
                                         n_centroids: int, head_dim: int, bits: int,
                                         group_size: int, q_offset: int = 0) -> torch.Tensor:
    """Causal variant of the fused dequant attention (kernels.py:870-928)."""
    return _fused(queries, centroids, indices, packed=packed_values, scales=scales, zeros=zeros,
                  bits=bits, group_size=group_size, causal=True, q_offset=q_offset)
