"""The CPU oracle against golden vectors produced by the reference's own code
(tests/golden/make_golden.py) and against the explicit NumPy known answers of
the reference's test_kernels.py."""

import math

import numpy as np
import pytest

import inputs as I
import oracle as O
from conftest import golden


@pytest.fixture(scope="module")
def cfg1_state():
    q, k = I.gaussian_qk(42, 1024, 2048, 128)
    return O.fit(q, k, head_dim=128, kmeans_iters=15, seed=42), q, k


def test_fit_d64_matches_reference():
    q, k = I.small_codec_inputs()
    g = golden("codec_d64")
    st = O.fit(q, k, head_dim=64, kmeans_iters=10, seed=42)
    np.testing.assert_array_equal(st["permutation"], g["permutation"])
    np.testing.assert_array_equal(st["inv_permutation"], g["inv_permutation"])
    np.testing.assert_array_equal(st["centroids"], g["centroids"])
    idx, _ = O.quantize(st, k)
    np.testing.assert_array_equal(idx, g["indices"])
    np.testing.assert_array_equal(O.dequantize(st, idx), g["k_hat"])
    np.testing.assert_allclose(O.attention_scores(st, q[:8], idx), g["scores"], atol=1e-5)


def test_cfg1_fit_quantize_scores(cfg1_state):
    st, q, k = cfg1_state
    g = golden("cfg1")
    np.testing.assert_array_equal(st["permutation"], g["permutation"])
    np.testing.assert_array_equal(st["centroids"], g["centroids"])
    idx, _ = O.quantize(st, k[:128])
    np.testing.assert_array_equal(idx, g["indices"])
    full, _ = O.quantize(st, k)
    np.testing.assert_array_equal(O.dequantize(st, full), g["k_hat"])
    np.testing.assert_allclose(O.attention_scores(st, q[:8], idx), g["scores"], atol=1e-5)


def test_assign_known_answer_seed333():
    keys, cents = I.assign_known_answer()
    st = {"mode": "profileperm_baseline", "head_dim": 128, "block_dim": 8, "n_blocks": 16,
          "n_centroids": 256, "centroids": cents, "permutation": np.arange(128),
          "heavy": np.zeros(16, bool)}
    idx, _ = O.quantize(st, keys)
    np.testing.assert_array_equal(idx, golden("assign333")["indices"])


def test_mixed_precision_fit_with_refinement():
    g = golden("mixed")
    qm = I.heavy_tailed_queries(512, 64, seed=5)
    km = np.random.default_rng(6).standard_normal((512, 64)).astype(np.float32)
    st = O.fit(qm, km, head_dim=64, mode="profileperm_mixed_precision", kmeans_iters=5, seed=3)
    np.testing.assert_array_equal(st["heavy"], g["heavy"])
    np.testing.assert_array_equal(st["permutation"], g["permutation"])
    np.testing.assert_array_equal(st["centroids"], g["centroids"])
    idx, pt = O.quantize(st, km[:64])
    np.testing.assert_array_equal(idx, g["indices"])
    np.testing.assert_array_equal(pt, g["passthrough"])
    np.testing.assert_array_equal(O.dequantize(st, idx, pt), g["k_hat"])
    np.testing.assert_allclose(O.attention_scores(st, qm[:4], idx), g["scores"], atol=1e-5)


def test_rotated_mode():
    g = golden("rotated")
    q, k = I.small_codec_inputs()
    st = O.fit(q, k, head_dim=64, mode="rotated", kmeans_iters=5, seed=1, rotation=g["rotation"])
    np.testing.assert_array_equal(st["centroids"], g["centroids"])
    idx, _ = O.quantize(st, k[:64])
    np.testing.assert_array_equal(idx, g["indices"])
    np.testing.assert_allclose(O.dequantize(st, idx), g["k_hat"], atol=1e-6)


def _cache_idx(st, K):
    return np.stack([np.stack([O.quantize(st, K[b, h])[0] for h in range(K.shape[1])])
                     for b in range(K.shape[0])])


def test_sdpa_simple_cache(cfg1_state):
    st = cfg1_state[0]
    g = golden("sdpa_simple")
    kk, vv = I.kv_stream(11, 2, 2, 100, 128)
    k3, v3 = I.kv_stream(13, 2, 2, 3, 128)
    K = np.concatenate([kk, k3], 2)
    V = np.concatenate([vv, v3], 2)
    idx = _cache_idx(st, K)
    np.testing.assert_array_equal(idx, g["key_indices"])
    sc = 1 / math.sqrt(128)
    qd = I.decode_queries(12, 2, 8, 1, 128)
    tol = dict(atol=2e-3, rtol=2e-3)  # golden outputs are fp16
    np.testing.assert_allclose(O.sdpa(qd, st, idx[:, :, :100], vv, sc), g["out_decode"], **tol)
    q3 = I.decode_queries(14, 2, 8, 3, 128)
    np.testing.assert_allclose(O.sdpa(q3, st, idx, V, sc, mask="causal"), g["out_causal"], **tol)
    np.testing.assert_allclose(O.sdpa(q3, st, idx, V, sc, mask=g["bool_mask"]), g["out_bool_mask"], **tol)
    np.testing.assert_allclose(O.sdpa(q3, st, idx, V, sc, mask=g["add_mask"]), g["out_add_mask"], **tol)


@pytest.mark.parametrize("name", ["hyb_fp16_b32", "hyb_grouped4_b32", "hyb_grouped2_b0",
                                  "hyb_tq2_b32", "hyb_tq2_b0", "hyb_tq4_b0", "hyb_vq_b32"])
def test_sdpa_hybrid(cfg1_state, name):
    st = cfg1_state[0]
    g = golden(name)
    bsz = g["key_indices"].shape[0]
    kk, vv = I.kv_stream(21, bsz, 2, 100, 128)
    c = int(g["compressed_offset"])
    b = int(g["buffer_offset"])
    assert c + b == 100
    np.testing.assert_array_equal(_cache_idx(st, kk[:, :, :c]), g["key_indices"])
    np.testing.assert_array_equal(g["buffer_keys"][:, :, :b], kk[:, :, c:])
    qd = I.decode_queries(12, 2, 8, 1, 128)[:bsz]
    o = O.sdpa(qd, st, g["key_indices"], g["values"][:, :, :c], 1 / math.sqrt(128),
               buffer_keys=g["buffer_keys"] if b else None,
               buffer_values=g["buffer_values"] if b else None)
    np.testing.assert_allclose(o, g["out"], atol=2e-3, rtol=2e-3)
    if "values_packed" in g and "value_scales" in g:  # grouped
        bits = 4 if "grouped4" in name else 2
        p, s, z, _ = O.quantize_values(vv[:, :, :c].astype(np.float32), bits, 64)
        np.testing.assert_array_equal(p, g["values_packed"])
        np.testing.assert_array_equal(s, g["value_scales"])
        np.testing.assert_array_equal(z, g["value_zeros"])
    if "value_norms" in g:
        bits = 4 if "tq4" in name else 2
        p, n = O.tq_quantize(vv[:, :, :c].astype(np.float32), g["rotation"], bits)
        np.testing.assert_array_equal(p, g["values_packed"])
        np.testing.assert_array_equal(n, g["value_norms"])


def test_hybrid_flush_bookkeeping():
    g = golden("hyb_flush_seq")
    # offsets after appends [16, 24, 1, 1, 40] with buffer 32, then trim(5), trim(40)
    want = [(16, 0, 16), (40, 8, 32), (41, 9, 32), (42, 10, 32), (82, 50, 32), (77, 50, 27),
            (37, 37, 0)]
    assert [tuple(int(x) for x in r) for r in g["offsets"]] == want


def test_packing_known_answers():
    g = golden("packing")
    for bits in (2, 3, 4):
        d = g[f"idx{bits}"].shape[1]
        np.testing.assert_array_equal(O.pack_indices(g[f"idx{bits}"], bits), g[f"packed{bits}"])
        np.testing.assert_array_equal(O.unpack_indices(g[f"packed{bits}"], d, bits), g[f"idx{bits}"])
    np.testing.assert_array_equal(O.pack_indices(g["idx3_d27"], 3), g["packed3_d27"])
    # boundary values and stray bits (test_kernels.py:86-103, 265-284)
    full = np.full((1, 30), 7, np.uint8)
    p = O.pack_indices(full, 3)
    assert int(p[0, 0]) >> 30 == 0
    np.testing.assert_array_equal(O.unpack_indices(p, 30, 3), full)


def test_grouped_values_known_answers():
    g = golden("grouped_values")
    for bits in (2, 4):
        p, s, z, n = O.quantize_values(g["values"], bits, 64)
        np.testing.assert_array_equal(p, g[f"packed{bits}"])
        np.testing.assert_array_equal(s, g[f"scales{bits}"])
        np.testing.assert_array_equal(z, g[f"zeros{bits}"])
        deq = O.dequantize_values(p, s, z, 128, bits, 64)
        np.testing.assert_array_equal(deq, g[f"deq{bits}"])
        rel = np.sqrt(np.mean((deq - g["values"]) ** 2)) / np.std(g["values"])
        assert rel < (0.15 if bits == 4 else 0.55)  # test_kernels.py:129


def test_turboquant_values_known_answers():
    g = golden("turboquant_values")
    for bits in (2, 3, 4):
        p, n = O.tq_quantize(g["values"], g[f"rotation{bits}"], bits)
        np.testing.assert_array_equal(p, g[f"packed{bits}"])
        np.testing.assert_array_equal(n, g[f"norms{bits}"])
        np.testing.assert_allclose(O.tq_dequantize(p, n, g[f"rotation{bits}"], bits, 128),
                                   g[f"deq{bits}"], atol=1e-5)
    d = O.tq_dequantize(*O.tq_quantize(g["values"], g["rotation2"], 2), g["rotation2"], 2, 128)
    assert np.mean((d - g["values"]) ** 2) < 1.5  # tests_mlx:495-504


def test_scalar_quantize_known_answer():
    g = golden("scalar_quantize")
    np.testing.assert_array_equal(O.scalar_quantize(g["values"], g["boundaries"]), g["indices"])


def test_fused_block_vq_helper():
    g = golden("fused_block_vq")
    st = {"n_blocks": 16, "block_dim": 8, "centroids": g["centroids"]}
    qd = O.query_centroid_dots(st, g["queries"])
    s = qd[:, np.arange(16)[None, :], g["indices"].astype(np.int64)].sum(axis=2)
    tq, tkv = 4, 32
    ok = (np.arange(tkv - tq, tkv))[:, None] >= np.arange(tkv)[None, :]
    s = np.where(ok, s, np.finfo(np.float32).min)
    w = np.exp(s - s.max(1, keepdims=True))
    w /= w.sum(1, keepdims=True)
    np.testing.assert_allclose(w @ g["values"], g["out"], atol=5e-3)


def test_lse_merge_is_exact_split():
    rng = np.random.default_rng(0)
    st = {"n_blocks": 16, "block_dim": 8, "centroids": rng.standard_normal((16, 256, 8)).astype(np.float32)}
    idx = rng.integers(0, 256, (500, 16)).astype(np.uint8)
    v = rng.standard_normal((500, 128)).astype(np.float32)
    q = (rng.standard_normal((4, 128)) * 0.1).astype(np.float32)
    m, l_, o = O.decode_attention_fp(q, st, idx, v)
    full = o / l_[:, None]
    parts = [O.decode_attention_fp(q, st, idx[a:b], v[a:b]) for a, b in ((0, 123), (123, 400), (400, 500))]
    got = O.lse_merge([p[0] for p in parts], [p[1] for p in parts], [p[2] for p in parts])
    np.testing.assert_allclose(got, full, rtol=1e-5, atol=1e-6)
