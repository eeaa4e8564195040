"""GPU parity of the codec kernels against the oracle and the reference's
golden vectors. Index outputs must be bit-exact; near-tie exceptions are
counted and must be genuine ties (relative distance gap < 1e-6)."""

import numpy as np
import pytest
import torch

import inputs as I
import oracle as O
from conftest import golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ss(cuda_ok):
    import sunshape_mlx_b200 as ss

    return ss


def _codec_from(ss, st_like, head_dim, mode="profileperm_baseline", **kw):
    c = ss.SunShapeBlockCodec(head_dim=head_dim, mode=mode, **kw)
    c.load_state_dict(st_like)
    return c


def test_assign_known_answer_seed333(ss):
    keys, cents = I.assign_known_answer()
    got = ss.block_vq_quantize_metal(keys, cents, 16, 256, 8, 128).cpu().numpy()
    np.testing.assert_array_equal(got, golden("assign333")["indices"])


@pytest.mark.parametrize("bd,k,n,dt", [(8, 256, 3001, np.float32), (8, 256, 4096, np.float16),
                                      (4, 256, 777, np.float32), (8, 64, 130, np.float32),
                                      (16, 256, 65, np.float32), (2, 16, 33, np.float32)])
def test_assign_bit_exact_vs_numpy(ss, bd, k, n, dt):
    rng = np.random.default_rng(bd * 1000 + k + n)
    d = 128
    keys = (rng.standard_normal((n, d)) * rng.uniform(0.2, 3.0, d)).astype(dt)
    cents = rng.standard_normal((d // bd, k, bd)).astype(np.float32)
    got = ss.block_vq_quantize_metal(keys, cents, d // bd, k, bd, d).cpu().numpy()
    st = {"mode": "profileperm_baseline", "head_dim": d, "block_dim": bd, "n_blocks": d // bd,
          "n_centroids": k, "centroids": cents, "permutation": np.arange(d), "heavy": np.zeros(d // bd, bool)}
    want, _ = O.quantize(st, keys.astype(np.float32))
    np.testing.assert_array_equal(got, want)


def test_assign_with_permutation_and_strided_rows(ss):
    from sunshape_mlx_b200 import kernels as K

    rng = np.random.default_rng(5)
    B, H, T, D, cap = 2, 3, 77, 128, 256
    keys = torch.tensor(rng.standard_normal((B, H, T, D)), dtype=torch.float16, device="cuda")
    cents = torch.tensor(rng.standard_normal((16, 256, 8)), dtype=torch.float32, device="cuda")
    perm = torch.tensor(rng.permutation(D), dtype=torch.int32, device="cuda")
    store = torch.full((B, H, cap, 16), 255, dtype=torch.uint8, device="cuda")
    K.vq_assign(keys.reshape(B * H, T, D), cents, perm=perm,
                out_idx=store[:, :, 10:10 + T].reshape(B * H, T, 16))
    st = {"mode": "profileperm_baseline", "head_dim": D, "block_dim": 8, "n_blocks": 16,
          "n_centroids": 256, "centroids": cents.cpu().numpy(), "permutation": perm.cpu().numpy(),
          "heavy": np.zeros(16, bool)}
    kn = keys.float().cpu().numpy()
    for b in range(B):
        for h in range(H):
            want, _ = O.quantize(st, kn[b, h])
            np.testing.assert_array_equal(store[b, h, 10:10 + T].cpu().numpy(), want)
    assert int((store[:, :, :10] != 255).sum()) == 0 and int((store[:, :, 10 + T:] != 255).sum()) == 0


def test_cfg1_quantize_dequant_scores_with_reference_state(ss):
    g = golden("cfg1")
    q, k = I.gaussian_qk(42, 1024, 2048, 128)
    c = _codec_from(ss, {"centroids": g["centroids"], "permutation": g["permutation"]}, 128)
    qz = c.quantize(k[:128])
    np.testing.assert_array_equal(qz.indices.cpu().numpy(), g["indices"])
    np.testing.assert_array_equal(c(k).cpu().numpy(), g["k_hat"])
    np.testing.assert_allclose(c.attention_scores(q[:8], qz).cpu().numpy(), g["scores"], atol=1e-4)
    assert c.last_score_backend == "cuda"


def test_cfg1_fit_on_gpu(ss):
    g = golden("cfg1")
    q, k = I.gaussian_qk(42, 1024, 2048, 128)
    c = ss.SunShapeBlockCodec(head_dim=128).fit(q, k, kmeans_iters=15, seed=42)
    np.testing.assert_array_equal(c.permutation.cpu().numpy(), g["permutation"])
    cg = c.centroids.cpu().numpy()
    n_diff = int((cg != g["centroids"]).any(axis=-1).sum())
    # centroid-by-centroid parity; the reference's assignment uses BLAS dot
    # products whose rounding order is not specified, so near-tie reassignments
    # may move a few centroids.
    assert n_diff <= 0.02 * cg.shape[0] * cg.shape[1], n_diff
    st = O.fit(q, k, head_dim=128, kmeans_iters=15, seed=42)
    x = O.apply_permutation(k, st["permutation"])
    def distortion(cents):
        tot = 0.0
        for b in range(16):
            d = O.block_distances(x[:, b * 8:(b + 1) * 8], cents[b])
            tot += float(d.min(axis=1).mean())
        return tot
    assert abs(distortion(cg) / distortion(g["centroids"]) - 1) < 1e-3


def test_kmeans_update_bit_exact(ss):
    from sunshape_mlx_b200 import _lib as L

    rng = np.random.default_rng(3)
    n, nb, bd, k = 4096, 16, 8, 256
    x = rng.standard_normal((n, nb * bd)).astype(np.float32)
    cin = rng.standard_normal((nb, k, bd)).astype(np.float32)
    assign = rng.integers(0, k - 3, (n, nb)).astype(np.uint8)  # leave empty clusters
    xt, at, ct = (torch.tensor(a, device="cuda") for a in (x, assign, cin))
    out = torch.empty_like(ct)
    L.call("ss_kmeans_update", L.ptr(xt), n, nb, bd, L.ptr(at), L.ptr(ct), L.ptr(out), k,
           L.stream_ptr())
    for b in range(nb):
        want = O.kmeans_update(x[:, b * bd:(b + 1) * bd], assign[:, b].astype(np.int64), cin[b])
        np.testing.assert_array_equal(out[b].cpu().numpy(), want)


@pytest.mark.parametrize("n,bd,k", [(30000, 4, 256), (777, 16, 64), (50000, 8, 256)])
def test_kmeans_update_bit_exact_sizes(ss, n, bd, k):
    """Sorted (n <= 49152) and scanning (larger n) update kernels, np.add.at order."""
    from sunshape_mlx_b200 import _lib as L

    rng = np.random.default_rng(n + bd)
    nb = 128 // bd
    x = rng.standard_normal((n, nb * bd)).astype(np.float32)
    cin = rng.standard_normal((nb, k, bd)).astype(np.float32)
    assign = rng.integers(0, k - 5, (n, nb)).astype(np.uint8)
    assign[: n // 3, 0] = 7  # one heavily used cluster
    xt, at, ct = (torch.tensor(a, device="cuda") for a in (x, assign, cin))
    out = torch.empty_like(ct)
    L.call("ss_kmeans_update", L.ptr(xt), n, nb, bd, L.ptr(at), L.ptr(ct), L.ptr(out), k,
           L.stream_ptr())
    got = out.cpu().numpy()
    for b in range(nb):
        want = O.kmeans_update(x[:, b * bd:(b + 1) * bd], assign[:, b].astype(np.int64), cin[b])
        np.testing.assert_array_equal(got[b], want)


def test_kmeans_expanded_assignment_matches_blas_form(ss):
    from sunshape_mlx_b200 import kernels as K

    rng = np.random.default_rng(9)
    x = rng.standard_normal((4096, 8)).astype(np.float32)
    c = x[rng.permutation(4096)[:256]].copy()
    got = K.vq_assign(torch.tensor(x, device="cuda"), torch.tensor(c[None], device="cuda"),
                      dist_mode=1).cpu().numpy()[:, 0]
    want = O.kmeans_assign_blas(x, c)
    bad = np.nonzero(got != want)[0]
    for i in bad:  # only genuine near-ties may differ
        d = O.block_distances(x[i:i + 1], c)[0]
        assert abs(d[got[i]] - d[want[i]]) <= 1e-5 * max(1.0, abs(d[want[i]]))
    assert bad.size <= 4


def test_mixed_precision_with_reference_state(ss):
    g = golden("mixed")
    km = np.random.default_rng(6).standard_normal((512, 64)).astype(np.float32)
    c = _codec_from(ss, {"centroids": g["centroids"], "permutation": g["permutation"],
                         "heavy": g["heavy"]}, 64, mode="profileperm_mixed_precision")
    qz = c.quantize(km[:64])
    np.testing.assert_array_equal(qz.indices.cpu().numpy(), g["indices"])
    np.testing.assert_array_equal(qz.passthrough_values.cpu().numpy(), g["passthrough"])
    np.testing.assert_array_equal(c.dequantize(qz).cpu().numpy(), g["k_hat"])
    qm = I.heavy_tailed_queries(512, 64, seed=5)
    np.testing.assert_allclose(c.attention_scores(qm[:4], qz).cpu().numpy(), g["scores"], atol=1e-4)


def test_mixed_fit_on_gpu_matches_reference_mask(ss):
    g = golden("mixed")
    qm = I.heavy_tailed_queries(512, 64, seed=5)
    km = np.random.default_rng(6).standard_normal((512, 64)).astype(np.float32)
    c = ss.SunShapeBlockCodec(head_dim=64, mode="profileperm_mixed_precision").fit(qm, km, 5, 3)
    np.testing.assert_array_equal(c.mixed_high_precision_blocks.cpu().numpy(), g["heavy"])
    np.testing.assert_array_equal(c.permutation.cpu().numpy(), g["permutation"])
    np.testing.assert_allclose(c.centroids.cpu().numpy(), g["centroids"], atol=2e-3)


def test_rotated_mode_with_reference_state(ss):
    g = golden("rotated")
    q, k = I.small_codec_inputs()
    c = _codec_from(ss, {"centroids": g["centroids"], "rotation": g["rotation"], "mode": "rotated"},
                    64, mode="rotated", use_rotation=True)
    qz = c.quantize(k[:64])
    got = qz.indices.cpu().numpy()
    assert (got != g["indices"]).mean() < 0.005  # GPU vs BLAS rotation rounding: near-ties only
    st = {"mode": "rotated", "head_dim": 64, "block_dim": 8, "n_blocks": 8, "n_centroids": 256,
          "centroids": g["centroids"], "rotation": g["rotation"], "heavy": np.zeros(8, bool)}
    np.testing.assert_allclose(c.dequantize(qz).cpu().numpy(), O.dequantize(st, got), atol=1e-5)


def test_block_vq_score_from_table(ss):
    rng = np.random.default_rng(55)  # test_kernels.py:163-194
    qd = rng.standard_normal((4, 16, 256)).astype(np.float32)
    idx = rng.integers(0, 256, (32, 16)).astype(np.uint8)
    got = ss.block_vq_score_metal(qd, idx, 4, 32, 16, 256).cpu().numpy()
    want = qd[:, np.arange(16)[None, :], idx.astype(np.int64)].sum(axis=2)
    assert np.abs(got - want).max() < 1e-3
    got2 = ss.block_vq_score_metal(qd[:2, :8, :64], idx[:16, :8] % 64, 2, 16, 8, 64)
    assert tuple(got2.shape) == (2, 16)


@pytest.mark.parametrize("B,T,heavy,kdt", [(2, 3, False, torch.float16), (1, 40, True, torch.float32),
                                           (3, 2500, True, torch.float16), (2, 2049, False, torch.bfloat16),
                                           (4, 2100, False, torch.float16)])
def test_cache_append_matches_assign_and_values(ss, B, T, heavy, kdt):
    """ss_cache_append (one launch for decode-sized appends, the assignment
    dispatch plus a row copy above 4096 rows): indices equal ss_vq_assign's,
    heavy blocks land in the fp16 stream, values are stored as fp16, and rows
    outside the write position are untouched."""
    from sunshape_mlx_b200 import kernels as K

    rng = np.random.default_rng(70 + T)
    qc = I.heavy_tailed_queries(1024, 128, seed=3)
    kc = rng.standard_normal((2048, 128)).astype(np.float32)
    mode = "profileperm_mixed_precision" if heavy else "profileperm_baseline"
    codec = ss.SunShapeBlockCodec(head_dim=128, mode=mode, **({"n_heavy": 4} if heavy else {}))
    codec.fit(qc, kc, kmeans_iters=2, seed=0)
    cache = ss.create_kv_cache(codec, n_kv_heads=2)
    cache.defer_append = False  # this test is about ss_cache_append itself
    k0 = torch.tensor(rng.standard_normal((B, 2, 37, 128)), device="cuda").half()
    cache.append(k0, k0 * 2)
    k = torch.tensor(rng.standard_normal((B, 2, T, 128)), device="cuda").to(kdt)
    v = torch.tensor(rng.standard_normal((B, 2, T, 128)), device="cuda").to(kdt)
    cache.append(k, v)
    assert cache.offset == 37 + T
    want = K.vq_assign(k.reshape(B * 2, T, 128), codec.centroids,
                       perm=codec.permutation, heavy=codec.heavy_u8).reshape(B, 2, T, -1)
    assert torch.equal(cache._key_indices[:, :, 37:37 + T], want)
    assert torch.equal(cache._values[:, :, 37:37 + T], v.half())
    assert torch.equal(cache._values[:, :, :37], (k0 * 2).half())
    if heavy:
        hp = torch.nonzero(codec.heavy_u8).flatten().tolist()
        kp = k.float()[..., codec.permutation.long()].reshape(B, 2, T, -1, 8)
        assert torch.equal(cache._key_heavy[:, :, 37:37 + T],
                           kp[:, :, :, hp].reshape(B, 2, T, -1).half())
