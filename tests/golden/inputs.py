"""Deterministic seeded inputs shared by the fixture generator and the tests.

Every generator uses ``numpy.random.default_rng`` (or, where a reference
test used it, the legacy ``numpy.random.seed``), so the same arrays are
rebuilt on any machine; fixtures store only reference outputs.
"""

from __future__ import annotations

import numpy as np


def gaussian_qk(seed: int, n_q: int, n_k: int, d: int):
    """q then k, i.i.d. N(0,1) float32 from one generator (config 1 recipe)."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((n_q, d)).astype(np.float32)
    k = rng.standard_normal((n_k, d)).astype(np.float32)
    return q, k


def small_codec_inputs():
    """head_dim 64 calibration set, like the reference test fixtures
    (tests_mlx/test_sunshape_mlx.py:43-69: keys (512,64), queries (256,64))."""
    k = np.random.default_rng(42).standard_normal((512, 64)).astype(np.float32)
    q = np.random.default_rng(137).standard_normal((256, 64)).astype(np.float32)
    return q, k


def channel_sigma(d: int, seed: int = 1) -> np.ndarray:
    """Per-channel std, log-normal(0, 0.5) (configs 2/3/5 key recipe)."""
    return np.exp(np.random.default_rng(seed).normal(0.0, 0.5, size=d)).astype(np.float32)


def anisotropic(n: int, d: int, seed: int, sigma: np.ndarray, dtype=np.float16):
    x = np.random.default_rng(seed).standard_normal((n, d)).astype(np.float32) * sigma[None, :]
    return x.astype(dtype)


def heavy_tailed_queries(n: int, d: int, seed: int = 5):
    """Gaussian queries with a few Student-t(3) channels so the kurtosis mask
    of the mixed-precision mode has structure."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((n, d)).astype(np.float32)
    ch = rng.choice(d, size=d // 6, replace=False)
    q[:, ch] = rng.standard_t(3.0, size=(n, ch.size)).astype(np.float32)
    return q


def assign_known_answer():
    """test_kernels.py:404-423 inputs: legacy seed 333, keys (32,128),
    centroids (16,256,8)."""
    np.random.seed(333)
    keys = np.random.randn(32, 128).astype(np.float32)
    cents = np.random.randn(16, 256, 8).astype(np.float32)
    return keys, cents


def kv_stream(seed: int, b: int, h: int, t: int, d: int, sigma=None):
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((b, h, t, d)).astype(np.float32)
    if sigma is not None:
        k = k * sigma
    v = rng.standard_normal((b, h, t, d)).astype(np.float32)
    return k.astype(np.float16), v.astype(np.float16)


def decode_queries(seed: int, b: int, hq: int, tq: int, d: int):
    return np.random.default_rng(seed).standard_normal((b, hq, tq, d)).astype(np.float16)
