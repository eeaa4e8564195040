"""NumPy restatement of the reference's CPU semantics for the SunShape path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the product package
never imports this file.

Every function cites the reference file:line it restates (paths relative to
the reference project root, gauravsaini/sunshape-mlx). All arithmetic is
float32 where the reference computes in float32, with the same reduction
orders where those are observable:

* block distances are ``np.sum((k - c) ** 2, axis=-1)`` (codec.py:497-499),
  which NumPy evaluates as a fixed pairwise tree for 8-wide blocks and a
  left-to-right sum for blocks narrower than 8;
* the k-means update is ``np.add.at`` (sequential float32 adds in point
  order) followed by a float64 division cast back to float32
  (codec.py:94-100).
"""

from __future__ import annotations

import math

import numpy as np

__all__ = [
    "kmeans", "kmeans_assign_blas", "kmeans_update",
    "covariance", "covariance_block_permutation", "invert_permutation",
    "apply_permutation", "positive_excess_kurtosis", "mixed_precision_block_mask",
    "heaviest_blocks_mask", "refine_centroids", "rotation_matrix_np", "fit", "forward_transform",
    "inverse_transform", "quantize", "block_distances", "dequantize",
    "query_centroid_dots", "attention_scores", "scale_queries", "sdpa",
    "pack_indices", "unpack_indices", "packed_dim", "quantize_values",
    "dequantize_values", "TQ_CODEBOOKS", "tq_tables", "tq_quantize",
    "tq_dequantize", "tq_group_quantize", "tq_group_dequantize",
    "scalar_quantize", "decode_attention_fp", "lse_merge",
]

PERM_MODES = ("profileperm_baseline", "profileperm_localmetric_dsq",
              "profileperm_mixed_precision")


# --------------------------------------------------------------------------
# k-means (codec.py:53-103)
# --------------------------------------------------------------------------

def kmeans_assign_blas(data: np.ndarray, cents: np.ndarray) -> np.ndarray:
    """Assignment step of codec.py:88-91: ||x||^2 + ||c||^2 - 2 x.c, argmin."""
    x_sq = np.sum(data ** 2, axis=1, keepdims=True)
    c_sq = np.sum(cents ** 2, axis=1, keepdims=True).T
    d = x_sq + c_sq - 2.0 * data @ cents.T
    return np.argmin(d, axis=1)


def kmeans_update(data: np.ndarray, assign: np.ndarray, cents: np.ndarray) -> np.ndarray:
    """Update step of codec.py:94-100 (np.add.at means, empty keeps old)."""
    k = cents.shape[0]
    acc = np.zeros_like(cents)
    cnt = np.zeros(k, dtype=np.float64)
    np.add.at(acc, assign, data)
    np.add.at(cnt, assign, 1.0)
    used = cnt > 0
    acc[used] /= cnt[used, None]
    acc[~used] = cents[~used]
    return acc


def kmeans(data, n_centroids: int, n_iters: int = 25, seed: int = 0) -> np.ndarray:
    """Lloyd k-means, codec.py:53-103 (RandomState(seed) permutation init)."""
    data = np.asarray(data, dtype=np.float32)
    n, d = data.shape
    if n <= n_centroids:  # codec.py:73-76
        out = np.zeros((n_centroids, d), dtype=np.float32)
        out[:n] = data
        return out
    pick = np.random.RandomState(seed).permutation(n)[:n_centroids]
    cents = data[pick].copy()
    for _ in range(n_iters):
        cents = kmeans_update(data, kmeans_assign_blas(data, cents), cents)
    return cents.astype(np.float32)


# --------------------------------------------------------------------------
# ProfilePerm and block masks (rotation.py)
# --------------------------------------------------------------------------

def covariance(x: np.ndarray) -> np.ndarray:
    """rotation.py:179-183."""
    x = np.asarray(x, dtype=np.float32)
    c = x - np.mean(x, axis=0, keepdims=True)
    return (c.T @ c) / np.float32(max(1, x.shape[0] - 1))


def covariance_block_permutation(q_cal, block_dim: int) -> np.ndarray:
    """Greedy seed-and-grow block packing, rotation.py:186-248."""
    aff = np.abs(covariance(q_cal))
    np.fill_diagonal(aff, 0.0)
    d = aff.shape[0]
    left = set(range(d))
    order: list[int] = []
    while left:
        rows = sorted(left)
        if len(rows) <= block_dim:
            order.extend(rows)
            break
        seed = rows[int(aff[rows].sum(axis=1).argmax())]
        blk = [seed]
        left.remove(seed)
        while len(blk) < block_dim and left:
            cand = sorted(left)
            gain = aff[np.array(cand)][:, np.array(blk)].sum(axis=1)
            pick = cand[int(gain.argmax())]
            blk.append(pick)
            left.remove(pick)
        order.extend(blk)
    return np.array(order, dtype=np.int32)


def invert_permutation(perm) -> np.ndarray:
    """rotation.py:251-259."""
    perm = np.asarray(perm)
    inv = np.empty_like(perm)
    inv[perm] = np.arange(perm.shape[0], dtype=perm.dtype)
    return inv


def apply_permutation(x, perm):
    """rotation.py:262-266."""
    if perm is None or np.size(perm) == 0:
        return x
    return np.asarray(x)[..., np.asarray(perm)]


def positive_excess_kurtosis(q) -> np.ndarray:
    """rotation.py:361-369."""
    q = np.asarray(q, dtype=np.float32)
    c = q - np.mean(q, axis=0, keepdims=True)
    var = np.maximum(np.mean(np.square(c), axis=0), np.float32(1e-12))
    ex = np.mean(c ** 4, axis=0) / np.square(var) - np.float32(3.0)
    return np.maximum(ex, 0.0).astype(np.float32)


def mixed_precision_block_mask(q_cal, block_dim: int, mass_threshold: float = 0.5):
    """rotation.py:372-404: smallest top-kurtosis block set reaching the mass."""
    k = positive_excess_kurtosis(q_cal)
    nb = k.shape[0] // block_dim
    mass = k.reshape(nb, block_dim).sum(axis=1)
    normed = mass / np.maximum(mass.sum(), np.float32(1e-12))
    ranked = np.argsort(normed)[::-1]
    cum = np.cumsum(normed[ranked])
    cut = max(1, min(int((cum < mass_threshold).sum()) + 1, nb))
    heavy = np.zeros(nb, dtype=bool)
    heavy[ranked[:cut]] = True
    return heavy, mass


def heaviest_blocks_mask(q_cal, block_dim: int, n_heavy: int) -> np.ndarray:
    """Fixed-count variant (the n_heavy option): the n_heavy highest-mass blocks
    under the kurtosis ranking of rotation.py:386-398."""
    k = positive_excess_kurtosis(q_cal)
    nb = k.shape[0] // block_dim
    mass = k.reshape(nb, block_dim).sum(axis=1)
    normed = mass / np.maximum(mass.sum(), np.float32(1e-12))
    ranked = np.argsort(normed)[::-1]
    heavy = np.zeros(nb, dtype=bool)
    heavy[ranked[:n_heavy]] = True
    return heavy


def _softmax_np(x: np.ndarray) -> np.ndarray:
    """codec.py:192-195 (float32)."""
    e = np.exp(x - x.max(axis=-1, keepdims=True))
    return e / e.sum(axis=-1, keepdims=True)


def refine_centroids(q_cal, k_cal, cents, e_metric, block_dim: int, n_steps: int = 3,
                     step_size: float = 0.1, block_affinity=None, active_blocks=None):
    """Attention-aware centroid refinement, codec.py:111-189 (run by fit for
    every mode except profileperm_baseline and rotated, codec.py:400-410)."""
    d = k_cal.shape[-1]
    nb = d // block_dim
    sc = math.sqrt(d)
    qs = np.asarray(q_cal[:min(128, q_cal.shape[0])], dtype=np.float32)
    ks = np.asarray(k_cal[:min(1024, k_cal.shape[0])], dtype=np.float32)
    e = np.asarray(e_metric, dtype=np.float32)
    ref = np.array(cents, dtype=np.float32).copy()
    ba = np.ones(nb, np.float32) if block_affinity is None else np.asarray(block_affinity, np.float32)
    ab = np.ones(nb, bool) if active_blocks is None else np.asarray(active_blocks, bool)

    def assign(b):
        sl = slice(b * block_dim, (b + 1) * block_dim)
        eb = e[sl, sl]
        return sl, np.argmin(block_distances(ks[:, sl] @ eb.T, ref[b] @ eb.T), axis=1)

    k_hat = np.zeros_like(ks)
    for b in range(nb):
        sl, a = assign(b)
        k_hat[:, sl] = ref[b][a]
    for _ in range(n_steps):
        p_o = _softmax_np((qs @ ks.T) / sc)
        p_h = _softmax_np((qs @ k_hat.T) / sc)
        err = p_h - p_o
        sens = p_h * (1.0 - p_h)
        g_att = ((err * sens).T @ qs) / sc
        g_tot = (k_hat - ks) + 0.5 * g_att
        for b in range(nb):
            if not ab[b]:
                continue
            sl, a = assign(b)
            new = ref[b].copy()
            step = step_size * float(ba[b])
            for ci in range(ref.shape[1]):
                sel = a == ci
                if sel.any():
                    new[ci] -= step * g_tot[sel, sl].mean(axis=0)
            ref[b] = new
            k_hat[:, sl] = new[a]
    return ref


def rotation_matrix_np(d: int, seed: int) -> np.ndarray:
    """Haar rotation by QR with the det(+1)-style sign fix of rotation.py:29-50.

    The reference draws G with the MLX RNG, which cannot be reproduced
    without MLX; this draws G with NumPy's default_rng(seed). Both sides of
    every parity test receive the same matrix explicitly.
    """
    g = np.random.default_rng(seed).standard_normal((d, d)).astype(np.float32)
    q, r = np.linalg.qr(g.astype(np.float64))
    q = q * np.sign(np.diag(r))[None, :]
    return q.astype(np.float32)


# --------------------------------------------------------------------------
# Codec: fit / quantize / dequantize / scores (codec.py)
# --------------------------------------------------------------------------

def fit(q_cal, k_cal, *, head_dim: int, block_dim: int = 8, n_centroids: int = 256,
        mode: str = "profileperm_baseline", kmeans_iters: int = 25, seed: int = 0,
        rotation: np.ndarray | None = None, n_heavy: int | None = None,
        n_refine_dsq: int = 3) -> dict:
    """codec.py:299-418 for the profileperm_baseline / _mixed_precision /
    rotated modes (E is the identity in all three)."""
    nb = head_dim // block_dim
    q = np.asarray(q_cal, dtype=np.float32)
    k = np.asarray(k_cal, dtype=np.float32)
    perm = np.arange(head_dim, dtype=np.int32)
    heavy = np.zeros(nb, dtype=bool)
    if mode == "rotated":
        q = q @ rotation.T
        k = k @ rotation.T
    elif mode in ("profileperm_baseline", "profileperm_mixed_precision"):
        perm = covariance_block_permutation(q, block_dim)
        q = apply_permutation(q, perm)
        k = apply_permutation(k, perm)
        if mode == "profileperm_mixed_precision":
            if n_heavy is None:
                heavy, _ = mixed_precision_block_mask(q, block_dim, 0.5)
            else:
                heavy = heaviest_blocks_mask(q, block_dim, n_heavy)
    else:
        raise ValueError(f"oracle fit: unsupported mode {mode}")
    cents = np.zeros((nb, n_centroids, block_dim), dtype=np.float32)
    for b in range(nb):
        if heavy[b]:
            continue
        sl = slice(b * block_dim, (b + 1) * block_dim)
        cents[b] = kmeans(k[:, sl], n_centroids, kmeans_iters, seed + b)
    if mode == "profileperm_mixed_precision" and n_refine_dsq > 0:
        cents = refine_centroids(q, k, cents, np.eye(head_dim, dtype=np.float32),
                                 block_dim, n_steps=n_refine_dsq)
    return {
        "mode": mode, "head_dim": head_dim, "block_dim": block_dim,
        "n_blocks": nb, "n_centroids": n_centroids, "centroids": cents,
        "permutation": perm, "inv_permutation": invert_permutation(perm),
        "heavy": heavy,
        "rotation": (rotation if mode == "rotated" else np.eye(head_dim, dtype=np.float32)),
    }


def forward_transform(state: dict, x):
    """codec.py:273-282."""
    x = np.asarray(x, dtype=np.float32)
    if state["mode"] in PERM_MODES:
        return apply_permutation(x, state["permutation"])
    if state["mode"] == "rotated":
        return x @ state["rotation"].T
    return x


def inverse_transform(state: dict, x):
    """codec.py:284-293."""
    if state["mode"] in PERM_MODES:
        return apply_permutation(x, state["inv_permutation"])
    if state["mode"] == "rotated":
        return x @ state["rotation"]
    return x


def block_distances(kb: np.ndarray, cb: np.ndarray) -> np.ndarray:
    """(N, K) squared distances exactly as codec.py:497-498 evaluates them."""
    diff = kb[:, None, :] - cb[None, :, :]
    return np.sum(diff ** 2, axis=-1)


def quantize(state: dict, keys):
    """NumPy quantize path, codec.py:424-514. Returns (indices u8, passthrough
    f32 (N, nb, bd) or None)."""
    x = forward_transform(state, keys)
    n = x.shape[0]
    nb, bd = state["n_blocks"], state["block_dim"]
    mixed = state["mode"] == "profileperm_mixed_precision" and state["heavy"].any()
    idx = np.zeros((n, nb), dtype=np.int32)
    ptv = np.zeros((n, nb, bd), dtype=np.float32) if mixed else None
    for b in range(nb):
        sl = slice(b * bd, (b + 1) * bd)
        if mixed and state["heavy"][b]:
            ptv[:, b, :] = x[:, sl]
            continue
        idx[:, b] = np.argmin(block_distances(x[:, sl], state["centroids"][b]), axis=1)
    dt = np.uint8 if state["n_centroids"] <= 256 else np.uint16
    return idx.astype(dt), ptv


def dequantize(state: dict, idx, passthrough=None) -> np.ndarray:
    """codec.py:516-543."""
    idx = np.asarray(idx).astype(np.int64)
    nb, bd = state["n_blocks"], state["block_dim"]
    out = np.zeros((idx.shape[0], state["head_dim"]), dtype=np.float32)
    for b in range(nb):
        sl = slice(b * bd, (b + 1) * bd)
        if state["mode"] == "profileperm_mixed_precision" and state["heavy"][b]:
            out[:, sl] = passthrough[:, b, :]
        else:
            out[:, sl] = state["centroids"][b][idx[:, b]]
    return inverse_transform(state, out)


def query_centroid_dots(state: dict, q_transformed) -> np.ndarray:
    """codec.py:553-573: qdots[q,b,c] = <q_b, C[b,c]> (float32)."""
    q = np.asarray(q_transformed, dtype=np.float32)
    qb = q.reshape(q.shape[0], state["n_blocks"], state["block_dim"])
    return np.einsum("qbd,bcd->qbc", qb, state["centroids"]).astype(np.float32)


def attention_scores(state: dict, query, idx) -> np.ndarray:
    """codec.py:575-637 gather path: sum_b qdots[q, b, idx[t, b]] (no scale;
    passthrough blocks contribute their zero centroids, as in the reference)."""
    lut = query_centroid_dots(state, forward_transform(state, query))
    idx = np.asarray(idx).astype(np.int64)
    nb = state["n_blocks"]
    g = lut[:, np.arange(nb)[None, :], idx]  # (nq, T, nb)
    return g.sum(axis=2, dtype=np.float32)


# --------------------------------------------------------------------------
# SDPA over the cache (attention.py:166-352, 2-pass fallback semantics)
# --------------------------------------------------------------------------

def scale_queries(queries: np.ndarray, scale: float) -> np.ndarray:
    """attention.py:208: queries * scale in the queries' own dtype (a Python
    scalar takes the array's dtype), then used in float32."""
    if queries.dtype == np.float16:
        return (queries * np.float16(scale)).astype(np.float16)
    return (queries.astype(np.float32) * np.float32(scale)).astype(np.float32)


def _softmax_precise(s: np.ndarray) -> np.ndarray:
    m = s.max(axis=-1, keepdims=True)
    e = np.exp((s - m).astype(np.float64))
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)


def sdpa(queries, state: dict, idx, values, scale: float, mask=None,
         buffer_keys=None, buffer_values=None) -> np.ndarray:
    """attention.py:166-352 (2-pass path).

    queries (B, Hq, Tq, D); idx (B, Hkv, Tc, nb) compressed key indices;
    values (B, Hkv, Tc, D) the compressed-token values as the cache returns
    them; buffer_keys / buffer_values (B, Hkv, Tb, D) the full-precision tail
    (hybrid cache). Output (B, Hq, Tq, D) float32.
    """
    queries = np.asarray(queries)
    b_, hq, tq, d = queries.shape
    hkv = idx.shape[1]
    rep = hq // hkv
    tc = idx.shape[2]
    tb = 0 if buffer_keys is None else buffer_keys.shape[2]
    tkv = tc + tb
    out = np.zeros((b_, hq, tq, d), dtype=np.float32)
    if tkv == 0:
        return out
    qs = scale_queries(queries, scale).astype(np.float32)
    for b in range(b_):
        for h in range(hkv):
            v_all = []
            if tc:
                v_all.append(np.asarray(values[b, h], dtype=np.float32))
            if tb:
                v_all.append(np.asarray(buffer_values[b, h], dtype=np.float32))
            v_all = np.concatenate(v_all, axis=0)
            for r in range(rep):
                qh = h * rep + r
                q = qs[b, qh]  # (Tq, D) original basis
                parts = []
                if tc:
                    parts.append(attention_scores(state, q, idx[b, h]))
                if tb:
                    parts.append(q @ np.asarray(buffer_keys[b, h], dtype=np.float32).T)
                s = np.concatenate(parts, axis=1).astype(np.float32)
                if isinstance(mask, str) and mask == "causal":
                    off = tkv - tq
                    ok = (off + np.arange(tq))[:, None] >= np.arange(tkv)[None, :]
                    s = np.where(ok, s, np.finfo(np.float32).min)
                elif mask is not None and not isinstance(mask, str):
                    m = np.asarray(mask)
                    if m.dtype == bool:
                        s = np.where(m, s, np.finfo(np.float32).min)
                    else:
                        s = s + m.astype(np.float32)
                out[b, qh] = _softmax_precise(s) @ v_all
    return out


def decode_attention_fp(q_scaled_t: np.ndarray, state: dict, idx: np.ndarray,
                        values: np.ndarray) -> tuple:
    """Unnormalised online-softmax triple (m, l, o) for one (b, kv-head) and
    its query rows, as produced per split by a split-KV decode; used to check
    the log-sum-exp merge. q_scaled_t is already in codec space."""
    lut = query_centroid_dots(state, q_scaled_t)
    nb = state["n_blocks"]
    s = lut[:, np.arange(nb)[None, :], idx.astype(np.int64)].sum(axis=2)
    m = s.max(axis=1)
    p = np.exp((s - m[:, None]).astype(np.float64))
    l_ = p.sum(axis=1)
    o = p @ values.astype(np.float64)
    return m.astype(np.float32), l_.astype(np.float32), o.astype(np.float32)


def lse_merge(ms, ls, os_):
    """Merge per-shard (m, l, o) triples: o = sum_g o_g e^{m_g-m*} / sum_g l_g e^{m_g-m*}."""
    ms = np.asarray(ms, np.float64)
    mstar = ms.max(axis=0)
    w = np.exp(ms - mstar[None])
    l_ = (np.asarray(ls, np.float64) * w).sum(axis=0)
    o = (np.asarray(os_, np.float64) * w[..., None]).sum(axis=0)
    return (o / l_[..., None]).astype(np.float32)


# --------------------------------------------------------------------------
# Bit packing and grouped value quantization (kernels.py:1102-1269)
# --------------------------------------------------------------------------

def packed_dim(d: int, bits: int) -> int:
    """value_codecs.py:90-101."""
    if bits == 2:
        return d // 16
    if bits == 3:
        return (d + 9) // 10
    if bits == 4:
        return d // 8
    raise ValueError(bits)


def pack_indices(idx, bits: int) -> np.ndarray:
    """kernels.py:1102-1137: element i of each word-group sits at bits [i*bits, ...)."""
    idx = np.asarray(idx).astype(np.uint32)
    d = idx.shape[-1]
    per = {2: 16, 3: 10, 4: 8}[bits]
    if bits == 3 and d % 10:
        pad = [(0, 0)] * (idx.ndim - 1) + [(0, 10 - d % 10)]
        idx = np.pad(idx, pad)
        d = idx.shape[-1]
    g = idx.reshape(*idx.shape[:-1], d // per, per) & np.uint32((1 << bits) - 1)
    sh = (np.arange(per, dtype=np.uint32) * bits)
    return np.bitwise_or.reduce(g << sh, axis=-1).astype(np.uint32)


def unpack_indices(packed, d: int, bits: int) -> np.ndarray:
    """kernels.py:1140-1163."""
    packed = np.asarray(packed, dtype=np.uint32)
    per = {2: 16, 3: 10, 4: 8}[bits]
    sh = (np.arange(per, dtype=np.uint32) * bits)
    e = (packed[..., None] >> sh) & np.uint32((1 << bits) - 1)
    e = e.reshape(*packed.shape[:-1], packed.shape[-1] * per)
    return e[..., :d]


def quantize_values(values, bits: int = 4, group_size: int = 64):
    """kernels.py:1173-1228: asymmetric min-max per group."""
    v = np.asarray(values, dtype=np.float32)
    lead = v.shape[:-1]
    d = v.shape[-1]
    g = d // group_size
    vg = v.reshape(*lead, g, group_size)
    lo = vg.min(axis=-1, keepdims=True)
    hi = vg.max(axis=-1, keepdims=True)
    sc = (hi - lo) / np.float32(2 ** bits - 1)
    sc = np.where(sc < np.float32(1e-8), np.float32(1e-8), sc).astype(np.float32)
    q = np.round((vg - lo) / sc).astype(np.int32)
    q = np.clip(q, 0, 2 ** bits - 1).astype(np.uint8)
    return (pack_indices(q.reshape(*lead, d), bits), sc[..., 0], lo[..., 0], g)


def dequantize_values(packed, scales, zeros, d: int, bits: int = 4, group_size: int = 64):
    """kernels.py:1231-1269: q * scale + zero."""
    q = unpack_indices(packed, d, bits).astype(np.float32)
    g = d // group_size
    qg = q.reshape(*q.shape[:-1], g, group_size)
    v = qg * np.asarray(scales, np.float32)[..., None] + np.asarray(zeros, np.float32)[..., None]
    return v.reshape(*q.shape[:-1], d).astype(np.float32)


# --------------------------------------------------------------------------
# TurboQuant values (value_codecs.py:20-177, kernels.py:453-507)
# --------------------------------------------------------------------------

# Lloyd-Max levels / decision boundaries of N(0, 1) for 1-4 bits, the
# published optimal scalar quantizer tables (value_codecs.py:20-87).
TQ_CODEBOOKS = {
    1: ([-0.7978845608028654, 0.7978845608028654], [0.0]),
    2: ([-1.510417608611893, -0.4527800346911237, 0.4527800346911237, 1.510417608611893],
        [-0.9815988216515084, 0.0, 0.9815988216515084]),
    3: ([-2.151945705166112, -1.3439092791423422, -0.7560052816730181, -0.2450941791152904,
         0.2450941791152904, 0.7560052816730181, 1.3439092791423422, 2.151945705166112],
        [-1.7479274921542272, -1.0499572804076802, -0.5005497303941542, 0.0,
         0.5005497303941542, 1.0499572804076802, 1.7479274921542272]),
    4: ([-2.732896755154294, -2.069364258154187, -1.618400443227723, -1.2565648452462146,
         -0.9426291036999694, -0.6569817464411519, -0.38818871416000605, -0.12844300124876415,
         0.12844300124876415, 0.38818871416000605, 0.6569817464411519, 0.9426291036999694,
         1.2565648452462146, 1.618400443227723, 2.069364258154187, 2.732896755154294],
        [-2.4011305066542405, -1.8438823506909552, -1.4374826442369688, -1.099596974473092,
         -0.7998054250705606, -0.522585230300579, -0.2583158577043851, 0.0,
         0.2583158577043851, 0.522585230300579, 0.7998054250705606, 1.099596974473092,
         1.4374826442369688, 1.8438823506909552, 2.4011305066542405]),
}


def tq_tables(head_dim: int, bits: int):
    """value_codecs.py:148-151: levels and boundaries scaled by 1/sqrt(D)."""
    lv, bd = TQ_CODEBOOKS[bits]
    s = 1.0 / math.sqrt(head_dim)
    return (np.array([c * s for c in lv], dtype=np.float32),
            np.array([b * s for b in bd], dtype=np.float32))


def scalar_quantize(values, boundaries) -> np.ndarray:
    """kernels.py:453-507: idx = #{j : v > boundary_j} (uint8)."""
    v = np.asarray(values, dtype=np.float32)
    out = np.zeros(v.shape, dtype=np.uint8)
    for b in np.asarray(boundaries, dtype=np.float32):
        out += (v > b).astype(np.uint8)
    return out


def tq_quantize(values, rotation, bits: int):
    """value_codecs.py:159-171: per-token norm, unit @ R^T, boundary count, pack."""
    v = np.asarray(values, dtype=np.float32)
    d = v.shape[-1]
    _, bnd = tq_tables(d, bits)
    n = np.sqrt(np.sum(v * v, axis=-1, keepdims=True)).astype(np.float32)
    unit = v / np.maximum(n, np.float32(1e-8))
    r = unit @ np.asarray(rotation, np.float32).T
    return pack_indices(scalar_quantize(r, bnd), bits), n[..., 0]


def tq_dequantize(packed, norms, rotation, bits: int, d: int):
    """value_codecs.py:173-177: levels[idx] @ R * norm."""
    lv, _ = tq_tables(d, bits)
    idx = unpack_indices(packed, d, bits).astype(np.int64)
    return (lv[idx] @ np.asarray(rotation, np.float32)) * np.asarray(norms, np.float32)[..., None]


def tq_group_quantize(values, rotation, bits: int, group_size: int):
    """Per-group-scaled TurboQuant (fp16 scale per group of channels, the value
    format of the 32768-token decode workload; an extension of
    value_codecs.py:159-171): r = v @ R^T; per group of ``group_size``
    channels s = fp16(||r_g|| / sqrt(group_size)); idx = #{j : r > B_j * s}
    with the unscaled N(0,1) boundaries B; 2-bit packed as kernels.py:1102."""
    v = np.asarray(values, dtype=np.float32)
    d = v.shape[-1]
    lv, bd = TQ_CODEBOOKS[bits]
    bd = np.array(bd, dtype=np.float32)
    r = v @ np.asarray(rotation, np.float32).T
    lead = r.shape[:-1]
    g = d // group_size
    rg = r.reshape(*lead, g, group_size)
    s = np.sqrt(np.sum(rg * rg, axis=-1) / np.float32(group_size)).astype(np.float32)
    s16 = s.astype(np.float16)
    thr = bd[None, :] * s16.astype(np.float32)[..., None]  # (..., g, nbnd)
    idx = np.zeros(rg.shape, dtype=np.uint8)
    for j in range(bd.shape[0]):
        idx += (rg > thr[..., j:j + 1]).astype(np.uint8)
    return pack_indices(idx.reshape(*lead, d), bits), s16


def tq_group_dequantize(packed, scales16, rotation, bits: int, d: int, group_size: int):
    """Inverse of tq_group_quantize: (L[idx] * s_g) @ R."""
    lv = np.array(TQ_CODEBOOKS[bits][0], dtype=np.float32)
    idx = unpack_indices(packed, d, bits).astype(np.int64)
    g = d // group_size
    r = lv[idx].reshape(*idx.shape[:-1], g, group_size)
    r = r * np.asarray(scales16).astype(np.float32)[..., None]
    return r.reshape(*idx.shape[:-1], d) @ np.asarray(rotation, np.float32)
