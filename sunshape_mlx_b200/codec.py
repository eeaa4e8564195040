"""SunShape block-VQ key codec on the GPU (codec.py of the reference).

State (centroids, permutation, masks, rotation) lives on a CUDA device.
quantize / dequantize / attention_scores and the k-means assignment and
update steps of ``fit`` run as sm_100a kernels through the C ABI; the small
calibration statistics (ProfilePerm, kurtosis mask, k-means initialisation)
are host-side control flow exactly as in the reference.
"""

from __future__ import annotations

import math
from typing import NamedTuple

import numpy as np
import torch

from . import kernels as K
from .rotation import (
    _matmul_f32,
    apply_permutation,
    covariance_block_permutation,
    generate_rotation_matrix,
    invert_permutation,
    mixed_precision_block_mask,
)

__all__ = ["SunShapeQuantized", "SunShapeBlockCodec", "_kmeans", "PERM_MODES"]

PERM_MODES = ("profileperm_baseline", "profileperm_localmetric_dsq", "profileperm_mixed_precision")
_MODES = PERM_MODES + ("rotated",)


class SunShapeQuantized(NamedTuple):
    """Quantized keys (codec.py:38-45): indices (N, n_blocks) uint8 on the GPU;
    passthrough_values (N, n_blocks, block_dim) f32 for mixed precision."""
    indices: torch.Tensor
    head_dim: int
    block_dim: int
    n_blocks: int
    passthrough_blocks: torch.Tensor | None = None
    passthrough_values: torch.Tensor | None = None


def _default_device():
    if not torch.cuda.is_available():
        raise RuntimeError("SunShape B200 needs a CUDA device (there is no CPU fallback)")
    return torch.device("cuda", torch.cuda.current_device())


def _kmeans_init(data_np_rows: int, n_centroids: int, seed: int) -> np.ndarray:
    """RandomState(seed).permutation(N)[:K] (codec.py:79-82)."""
    return np.random.RandomState(seed).permutation(data_np_rows)[:n_centroids]


def _kmeans(data, n_centroids: int, n_iters: int = 25, seed: int = 0) -> torch.Tensor:
    """Lloyd k-means of rows (codec.py:53-103) on the GPU: assignment by the
    block-VQ kernel in the reference's expanded-distance form, update by the
    in-order accumulation kernel."""
    x = K.cuda_tensor(data, torch.float32)
    n, d = x.shape
    if n <= n_centroids:
        out = torch.zeros((n_centroids, d), dtype=torch.float32, device=x.device)
        out[:n] = x
        return out
    cents = x[torch.as_tensor(_kmeans_init(n, n_centroids, seed), device=x.device)].clone()
    return _kmeans_blocks(x, cents[None], n_iters)[0]


def _kmeans_blocks(x: torch.Tensor, cents: torch.Tensor, n_iters: int,
                   skip: torch.Tensor | None = None) -> torch.Tensor:
    """Runs Lloyd iterations for all blocks at once. x (N, nb*bd) f32,
    cents (nb, K, bd) f32. Blocks flagged in ``skip`` keep their centroids."""
    from . import _lib as L

    nb, k, bd = cents.shape
    n = x.shape[0]
    assign = torch.empty((n, nb), dtype=torch.uint8, device=x.device)
    other = torch.empty_like(cents)
    cur = cents.contiguous().clone()
    for _ in range(n_iters):
        K.vq_assign(x, cur, out_idx=assign, dist_mode=1)
        L.call("ss_kmeans_update", L.ptr(x), n, nb, bd, L.ptr(assign), L.ptr(cur), L.ptr(other),
               k, L.stream_ptr(x.device))
        cur, other = other, cur
    if skip is not None and bool(skip.any()):
        cur[skip] = cents[skip]
    return cur


class SunShapeBlockCodec:
    """SunShape block vector-quantization codec (codec.py:217-637).

    Modes: ``profileperm_baseline``, ``profileperm_mixed_precision``,
    ``rotated`` (and ``profileperm_localmetric_dsq`` for state loading and
    quantize/scores with identity metric; its fit-time DSQ metric is not
    part of this build).
    """

    def __init__(self, head_dim: int, block_dim: int = 8, n_centroids: int = 256, c: float = 5.0,
                 n_refine_dsq: int = 3, mode: str = "profileperm_baseline",
                 use_rotation: bool = False, rotation_seed: int = 0, device=None,
                 n_heavy: int | None = None):
        if head_dim % block_dim != 0:
            raise ValueError("head_dim must be divisible by block_dim")
        if n_centroids > 256:
            raise ValueError("this build stores uint8 indices: n_centroids must be <= 256")
        self.device = torch.device(device) if device is not None else _default_device()
        self.head_dim = head_dim
        self.block_dim = block_dim
        self.n_blocks = head_dim // block_dim
        self.n_centroids = n_centroids
        self.c = c
        self.mode = "rotated" if use_rotation else mode
        self.n_refine_dsq = n_refine_dsq
        self.use_rotation = self.mode == "rotated"
        self.n_heavy = n_heavy
        dev = self.device
        self.centroids = torch.zeros((self.n_blocks, n_centroids, block_dim), dtype=torch.float32,
                                     device=dev)
        self.permutation = torch.arange(head_dim, dtype=torch.int32, device=dev)
        self.inv_permutation = torch.arange(head_dim, dtype=torch.int32, device=dev)
        self.mixed_high_precision_blocks = torch.zeros(self.n_blocks, dtype=torch.bool, device=dev)
        self.mixed_block_mass = torch.zeros(self.n_blocks, dtype=torch.float32, device=dev)
        self.last_score_backend = "none"
        if self.use_rotation:
            self.rotation = generate_rotation_matrix(head_dim, seed=rotation_seed, device=dev)
        else:
            self.rotation = torch.eye(head_dim, dtype=torch.float32, device=dev)
        self._heavy_u8 = None

    # ------------------------------------------------------------ state
    def state_dict(self) -> dict:
        """Codec state for save/load (the reference keeps it as attributes only)."""
        return {
            "mode": self.mode, "head_dim": self.head_dim, "block_dim": self.block_dim,
            "n_centroids": self.n_centroids,
            "centroids": self.centroids.detach().cpu(),
            "permutation": self.permutation.detach().cpu(),
            "inv_permutation": self.inv_permutation.detach().cpu(),
            "heavy": self.mixed_high_precision_blocks.detach().cpu(),
            "rotation": self.rotation.detach().cpu(),
        }

    def load_state_dict(self, st: dict) -> "SunShapeBlockCodec":
        dev = self.device
        if "mode" in st:
            self.mode = str(st["mode"])
            self.use_rotation = self.mode == "rotated"
        self.centroids = K.cuda_tensor(st["centroids"], torch.float32, dev).clone()
        if self.centroids.shape != (self.n_blocks, self.n_centroids, self.block_dim):
            raise ValueError(f"centroids shape {tuple(self.centroids.shape)} does not match codec")
        perm = st.get("permutation")
        if perm is not None:
            self.permutation = K.cuda_tensor(perm, torch.int32, dev)
            inv = st.get("inv_permutation")
            self.inv_permutation = (K.cuda_tensor(inv, torch.int32, dev) if inv is not None
                                    else invert_permutation(self.permutation).to(dev))
        heavy = st.get("heavy")
        if heavy is not None:
            self.mixed_high_precision_blocks = K.cuda_tensor(heavy, torch.bool, dev)
        rot = st.get("rotation")
        if rot is not None:
            self.rotation = K.cuda_tensor(rot, torch.float32, dev)
        self._heavy_u8 = None
        return self

    # ------------------------------------------------------------ transforms
    def _is_perm(self) -> bool:
        return self.mode in PERM_MODES

    def _forward_transform(self, x: torch.Tensor) -> torch.Tensor:
        """codec.py:273-282."""
        if self._is_perm():
            return apply_permutation(x, self.permutation)
        if self.use_rotation:
            return K.rotate_rows(x, self.rotation.T)
        return x

    def _inverse_transform(self, x: torch.Tensor) -> torch.Tensor:
        """codec.py:284-293."""
        if self._is_perm():
            return apply_permutation(x, self.inv_permutation)
        if self.use_rotation:
            return K.rotate_rows(x, self.rotation)
        return x

    @property
    def has_heavy(self) -> bool:
        return self.mode == "profileperm_mixed_precision" and bool(self.mixed_high_precision_blocks.any())

    @property
    def heavy_u8(self) -> torch.Tensor | None:
        if not self.has_heavy:
            return None
        if self._heavy_u8 is None:
            self._heavy_u8 = self.mixed_high_precision_blocks.to(torch.uint8).contiguous()
        return self._heavy_u8

    @property
    def n_heavy_blocks(self) -> int:
        return int(self.mixed_high_precision_blocks.sum()) if self.has_heavy else 0

    # ------------------------------------------------------------ fit
    def fit(self, q_cal, k_cal, kmeans_iters: int = 25, seed: int = 0) -> "SunShapeBlockCodec":
        """codec.py:299-418. Returns self."""
        dev = self.device
        q = K.cuda_tensor(q_cal, torch.float32, dev)
        k = K.cuda_tensor(k_cal, torch.float32, dev)
        nb, bd, kc = self.n_blocks, self.block_dim, self.n_centroids
        heavy = torch.zeros(nb, dtype=torch.bool, device=dev)
        if self.mode == "rotated":
            q = _matmul_f32(q, self.rotation.T)
            k = _matmul_f32(k, self.rotation.T)
            self.permutation = torch.arange(self.head_dim, dtype=torch.int32, device=dev)
        elif self.mode in ("profileperm_baseline", "profileperm_mixed_precision"):
            perm = covariance_block_permutation(q, bd).to(dev)
            self.permutation = perm
            self.inv_permutation = invert_permutation(perm).to(dev)
            q = apply_permutation(q, perm)
            k = apply_permutation(k, perm)
            if self.mode == "profileperm_mixed_precision":
                heavy, mass = mixed_precision_block_mask(q, bd, 0.5, n_heavy=self.n_heavy)
                heavy = heavy.to(dev)
                self.mixed_block_mass = mass.to(dev)
        else:
            raise ValueError(f"fit is not implemented for mode {self.mode} in this build")
        self.mixed_high_precision_blocks = heavy
        if self.mode != "profileperm_mixed_precision":
            self.mixed_block_mass = torch.zeros(nb, dtype=torch.float32, device=dev)
        self._heavy_u8 = None

        k = k.contiguous()
        n = k.shape[0]
        if n <= kc:
            cents = torch.zeros((nb, kc, bd), dtype=torch.float32, device=dev)
            cents[:, :n, :] = k.reshape(n, nb, bd).permute(1, 0, 2)
        else:
            init = np.stack([_kmeans_init(n, kc, seed + b) for b in range(nb)])  # (nb, K)
            idx = torch.as_tensor(init, device=dev, dtype=torch.long)
            kb = k.reshape(n, nb, bd)
            cents = kb[idx, torch.arange(nb, device=dev)[:, None], :]  # (nb, K, bd)
            cents = _kmeans_blocks(k, cents.contiguous(), kmeans_iters)
        cents[heavy] = 0.0
        if self.mode == "profileperm_mixed_precision" and self.n_refine_dsq > 0:
            cents = self._refine_centroids(q, k, cents, self.n_refine_dsq)
        self.centroids = cents.contiguous()
        return self

    def _refine_centroids(self, q, k, cents, n_steps: int, step_size: float = 0.1):
        """Attention-aware centroid refinement (codec.py:111-189), run by fit in
        mixed-precision mode with identity metric and all blocks active."""
        nb, kc, bd = cents.shape
        d = self.head_dim
        sc = math.sqrt(d)
        qs = q[: min(128, q.shape[0])].contiguous()
        ks = k[: min(1024, k.shape[0])].contiguous()
        ref = cents.clone()
        assign = K.vq_assign(ks, ref)  # (n, nb) exact nearest
        ar = torch.arange(nb, device=ks.device)
        k_hat = ref[ar[None, :], assign.long(), :].reshape(ks.shape[0], d)
        for _ in range(n_steps):
            p_o = torch.softmax(_matmul_f32(qs, ks.T) / sc, dim=-1)
            p_h = torch.softmax(_matmul_f32(qs, k_hat.T) / sc, dim=-1)
            err = p_h - p_o
            sens = p_h * (1.0 - p_h)
            g_att = _matmul_f32((err * sens).T, qs) / sc
            g_tot = (k_hat - ks) + 0.5 * g_att
            assign = K.vq_assign(ks, ref).long()  # per-block assignment with current centroids
            gb = g_tot.reshape(-1, nb, bd)
            flat = (ar[None, :] * kc + assign).reshape(-1)
            sums = torch.zeros((nb * kc, bd), dtype=torch.float32, device=ks.device)
            sums.index_add_(0, flat, gb.reshape(-1, bd))
            cnt = torch.zeros(nb * kc, dtype=torch.float32, device=ks.device)
            cnt.index_add_(0, flat, torch.ones_like(flat, dtype=torch.float32))
            upd = torch.where(cnt[:, None] > 0, sums / cnt.clamp(min=1)[:, None], torch.zeros_like(sums))
            ref = ref - step_size * upd.reshape(nb, kc, bd)
            k_hat = ref[ar[None, :], assign, :].reshape(ks.shape[0], d)
        return ref

    # ------------------------------------------------------------ quantize
    def quantize(self, keys) -> SunShapeQuantized:
        """codec.py:424-514: nearest centroid per block on the GPU."""
        x = K.cuda_tensor(keys, device=self.device)
        if x.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            x = x.float()
        perm = None
        if self._is_perm():
            perm = self.permutation
        elif self.use_rotation:
            x = K.rotate_rows(x, self.rotation.T)
        n = x.shape[0]
        pt = None
        if self.has_heavy:
            pt = torch.zeros((n, self.n_blocks, self.block_dim), dtype=torch.float32,
                             device=self.device)
        idx = K.vq_assign(x, self.centroids, perm=perm, heavy=self.heavy_u8, out_pt=pt)
        return SunShapeQuantized(
            indices=idx, head_dim=self.head_dim, block_dim=self.block_dim, n_blocks=self.n_blocks,
            passthrough_blocks=(self.mixed_high_precision_blocks
                                if self.mode == "profileperm_mixed_precision" else None),
            passthrough_values=pt)

    def dequantize(self, quantized: SunShapeQuantized) -> torch.Tensor:
        """codec.py:516-543: concatenated centroids in codec space, heavy blocks
        restored from the float32 passthrough, then the inverse transform."""
        idx = K.cuda_tensor(quantized.indices, torch.uint8, self.device)
        out = K.vq_dequant(idx, self.centroids)  # codec space, (N, head_dim) f32
        pb = quantized.passthrough_blocks
        if pb is not None and bool(torch.as_tensor(pb).any()):
            if quantized.passthrough_values is None:
                raise ValueError("Mixed-precision missing passthrough values.")
            hm = K.cuda_tensor(pb, torch.bool, self.device).repeat_interleave(self.block_dim)
            ptv = K.cuda_tensor(quantized.passthrough_values, torch.float32, self.device)
            out[:, hm] = ptv.reshape(ptv.shape[0], -1)[:, hm]
        return self._inverse_transform(out)

    def __call__(self, keys) -> torch.Tensor:
        """Quantize then dequantize (codec.py:545-547)."""
        return self.dequantize(self.quantize(keys))

    # ------------------------------------------------------------ scores
    def precompute_query_centroid_dots(self, query) -> torch.Tensor:
        """qdots[q, b, c] = <q_b, C[b, c]> (codec.py:553-573); query (n_qh,
        head_dim) already in codec space. One launch of ss_query_centroid_dots."""
        q = K.cuda_tensor(query, torch.float32, self.device).reshape(-1, self.head_dim).contiguous()
        out = torch.empty((q.shape[0], self.n_blocks, self.n_centroids), dtype=torch.float32,
                          device=self.device)
        K.L.call("ss_query_centroid_dots", K.L.ptr(q), q.shape[0], self.head_dim,
                 K.L.ptr(self.centroids), self.block_dim, self.n_centroids, K.L.ptr(out),
                 K.L.stream_ptr(self.device))
        return out

    def attention_scores(self, query, quantized: SunShapeQuantized, *,
                         prefer_metal: bool = True) -> torch.Tensor:
        """scores[q, t] = sum_b qdots[q, b, idx[t, b]] (codec.py:575-637), with
        the query x centroid table built in shared memory by the kernel.
        Passthrough blocks contribute through their centroids, as in the
        reference."""
        q = K.cuda_tensor(query, torch.float32, self.device)
        q = self._forward_transform(q).contiguous()
        idx = K.cuda_tensor(quantized.indices, torch.uint8, self.device)
        self.last_score_backend = "cuda"
        return K.vq_scores(q, self.centroids, idx)

    def heldout_logit_mse(self, q_test, k_test) -> float:
        """E[(q . (k - k_hat))^2] (codec.py:639-650)."""
        q = K.cuda_tensor(q_test, torch.float32, self.device)
        k = K.cuda_tensor(k_test, torch.float32, self.device)
        delta = k - self(k)
        return float(((q * delta).sum(dim=1) ** 2).mean())
