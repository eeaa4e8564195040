"""Host-side fit helpers: ProfilePerm, rotations, block masks (rotation.py of
the reference). These are small O(d^2)-O(d^3) calibration computations that
the reference also runs on the host; the statistics are computed with torch
(on the tensors' device) and the greedy/sorting control flow runs on the host.
"""

from __future__ import annotations

import math

import numpy as np
import torch


def _as_f32(x, device=None) -> torch.Tensor:
    if isinstance(x, torch.Tensor):
        t = x
    else:
        t = torch.as_tensor(np.asarray(x))
    if device is not None:
        t = t.to(device)
    return t.to(torch.float32)


def _matmul_f32(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Full-precision fp32 matmul (no TF32 on CUDA)."""
    if a.is_cuda:
        prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        try:
            return a @ b
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev
    return a @ b


def generate_rotation_matrix(d: int, seed: int = 0, device=None) -> torch.Tensor:
    """Haar-random rotation by QR of a seeded Gaussian with the sign fix of
    rotation.py:29-50 (R <- Q * sign(diag(R_qr))).

    The reference draws the Gaussian with MLX's RNG; this draws it with
    numpy.random.default_rng(seed), so matrices are reproducible but differ
    from MLX's for the same seed.
    """
    g = np.random.default_rng(seed).standard_normal((d, d)).astype(np.float32)
    q, r = np.linalg.qr(g.astype(np.float64))
    q = q * np.sign(np.diag(r))[None, :]
    return torch.as_tensor(q.astype(np.float32), device=device)


def generate_wht_signs(d: int, seed: int = 0) -> np.ndarray:
    """Random +-1 signs for the randomized Walsh-Hadamard transform
    (rotation.py:66-84)."""
    if d <= 0 or d & (d - 1):
        raise ValueError(f"WHT requires d to be a power of 2, got {d}")
    rng = np.random.RandomState(seed)
    return rng.choice([-1.0, 1.0], size=d).astype(np.float32)


def apply_wht(x, signs, inverse: bool = False) -> torch.Tensor:
    """R x with R = H_d diag(signs) / sqrt(d) (or its inverse), rotation.py:87-134."""
    x = _as_f32(x)
    d = x.shape[-1]
    if d <= 0 or d & (d - 1):
        raise ValueError(f"WHT requires last dim to be a power of 2, got {d}")
    s = _as_f32(signs, x.device)
    y = x if inverse else x * s
    shape = y.shape
    y = y.reshape(-1, d).clone()
    h = 1
    while h < d:
        y = y.reshape(-1, d // (2 * h), 2, h)
        a, b = y[:, :, 0, :].clone(), y[:, :, 1, :].clone()
        y[:, :, 0, :], y[:, :, 1, :] = a + b, a - b
        y = y.reshape(-1, d)
        h *= 2
    y = y.reshape(shape) / math.sqrt(d)
    return y * s if inverse else y


def _covariance(x: torch.Tensor) -> torch.Tensor:
    c = x - x.mean(dim=0, keepdim=True)
    return _matmul_f32(c.T, c) / max(1, x.shape[0] - 1)


def covariance_block_permutation(q_cal, block_dim: int) -> torch.Tensor:
    """ProfilePerm (rotation.py:186-248): repeatedly seed a block with the
    remaining dimension of largest total |cov| affinity and grow it with the
    candidate of largest affinity to the block's members."""
    q = _as_f32(q_cal)
    aff = _covariance(q).abs().cpu().numpy()
    np.fill_diagonal(aff, 0.0)
    d = aff.shape[0]
    left = list(range(d))
    order: list[int] = []
    while left:
        if len(left) <= block_dim:
            order.extend(left)
            break
        seed = left[int(aff[left].sum(axis=1).argmax())]
        blk = [seed]
        left.remove(seed)
        while len(blk) < block_dim and left:
            gain = aff[np.array(left)][:, np.array(blk)].sum(axis=1)
            pick = left[int(gain.argmax())]
            blk.append(pick)
            left.remove(pick)
        order.extend(blk)
    return torch.tensor(order, dtype=torch.int32)


def invert_permutation(perm) -> torch.Tensor:
    """rotation.py:251-259."""
    p = torch.as_tensor(perm).long()
    inv = torch.empty_like(p)
    inv[p] = torch.arange(p.numel(), device=p.device)
    return inv.to(torch.int32)


def apply_permutation(x, perm):
    """rotation.py:262-266: gather along the last dimension."""
    if perm is None or torch.as_tensor(perm).numel() == 0:
        return x
    x = torch.as_tensor(x)
    return x[..., torch.as_tensor(perm, device=x.device).long()]


def positive_excess_kurtosis(q) -> torch.Tensor:
    """rotation.py:361-369."""
    q = _as_f32(q)
    c = q - q.mean(dim=0, keepdim=True)
    var = torch.clamp((c * c).mean(dim=0), min=1e-12)
    ex = (c ** 4).mean(dim=0) / (var * var) - 3.0
    return torch.clamp(ex, min=0.0)


def mixed_precision_block_mask(q_cal, block_dim: int, mass_threshold: float = 0.5,
                               n_heavy: int | None = None):
    """Heavy-tailed block mask (rotation.py:372-404): the smallest set of
    highest-kurtosis-mass blocks whose normalised mass reaches the threshold,
    or, with ``n_heavy``, exactly that many of the highest-mass blocks."""
    k = positive_excess_kurtosis(q_cal)
    nb = k.shape[0] // block_dim
    mass = k.reshape(nb, block_dim).sum(dim=1)
    normed = (mass / torch.clamp(mass.sum(), min=1e-12)).cpu().numpy()
    ranked = np.argsort(normed)[::-1]
    if n_heavy is None:
        cum = np.cumsum(normed[ranked])
        cut = max(1, min(int((cum < mass_threshold).sum()) + 1, nb))
    else:
        cut = int(n_heavy)
    heavy = np.zeros(nb, dtype=bool)
    heavy[ranked[:cut]] = True
    return torch.as_tensor(heavy), mass


def block_local_cov_metric(q_cal, perm, block_dim: int) -> torch.Tensor:
    """Block-diagonal covariance metric of the permuted queries (rotation.py:274-303)."""
    c = _covariance(apply_permutation(_as_f32(q_cal), perm))
    out = torch.zeros_like(c)
    for b in range(c.shape[0] // block_dim):
        sl = slice(b * block_dim, (b + 1) * block_dim)
        out[sl, sl] = c[sl, sl]
    return out


def block_affinity_gate(q_cal, block_dim: int):
    """Per-block variance share and the >=50 % mass active set (rotation.py:311-353)."""
    q = _as_f32(q_cal)
    c = q - q.mean(dim=0, keepdim=True)
    var = (c * c).mean(dim=0)
    nb = var.shape[0] // block_dim
    mass = var.reshape(nb, block_dim).sum(dim=1)
    aff = mass / torch.clamp(mass.sum(), min=1e-12)
    a = aff.cpu().numpy()
    ranked = np.argsort(a)[::-1]
    cut = max(1, min(int((np.cumsum(a[ranked]) < 0.5).sum()) + 1, nb))
    act = np.zeros(nb, dtype=bool)
    act[ranked[:cut]] = True
    active = torch.as_tensor(act, device=aff.device)
    w = aff * active.float()
    return w / torch.clamp(w.max(), min=1e-12), active


def safe_normalize(x, axis: int = -1, eps: float = 1e-8):
    """Unit-normalise, leaving zero vectors unchanged (rotation.py:412-420)."""
    x = _as_f32(x)
    n = torch.linalg.norm(x, dim=axis, keepdim=True)
    safe = torch.where(n < eps, torch.ones_like(n), n)
    return x / safe, n
