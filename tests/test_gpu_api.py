"""GPU checks of the API edges around the hot path: the hybrid cache's
flush/trim bookkeeping against the reference's own record, update_and_fetch's
deferred keys, make_mask, nbytes / compression_ratio, the kernel dispatch
counters and backend breadcrumbs, and the query x centroid table."""

import math

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


@pytest.fixture(scope="module")
def cfg1_codec(ss):
    g = golden("cfg1")
    c = ss.SunShapeBlockCodec(head_dim=128)
    c.load_state_dict({"centroids": g["centroids"], "permutation": g["permutation"]})
    return c


def test_hybrid_flush_trim_sequence_matches_reference(ss, cfg1_codec):
    """The reference's hybrid cache (cache.py:656-710 append/flush,
    954-963 trim) recorded (offset, compressed, buffered) after appends of
    16, 24, 1, 1, 40 tokens with buffer_size 32, then trim(5) and trim(40),
    and the surviving key indices."""
    g = golden("hyb_flush_seq")
    hc = ss.create_kv_cache(cfg1_codec, n_kv_heads=2, buffer_size=32, value_backend="fp16")
    assert isinstance(hc, ss.HybridSunShapeKVCache)
    offs = []
    for i, t in enumerate([16, 24, 1, 1, 40]):
        kk, vv = I.kv_stream(30 + i, 1, 2, t, 128)
        hc.update_and_fetch(kk, vv)
        offs.append((hc.offset, hc.compressed_offset, hc.buffer_offset))
    hc.trim(5)
    offs.append((hc.offset, hc.compressed_offset, hc.buffer_offset))
    hc.trim(40)
    offs.append((hc.offset, hc.compressed_offset, hc.buffer_offset))
    assert offs == [tuple(int(x) for x in r) for r in g["offsets"]]
    np.testing.assert_array_equal(hc.key_indices.cpu().numpy(), g["key_indices"])


def test_update_and_fetch_defers_keys(ss, cfg1_codec):
    """mlx-lm call order: update_and_fetch then the patched SDPA. The fused
    kernel reads the index stream itself, so the returned keys are never
    dequantized on that path; reading them gives the dequantized keys."""
    from sunshape_mlx_b200 import patch
    from sunshape_mlx_b200.cache import DeferredTensor

    cache = ss.create_kv_cache(cfg1_codec, n_kv_heads=2)
    kk, vv = I.kv_stream(41, 2, 2, 300, 128)
    k_out, v_out = cache.update_and_fetch(kk, vv)
    assert isinstance(k_out, DeferredTensor) and tuple(k_out.shape) == (2, 2, 300, 128)
    assert k_out.dtype == torch.float32
    q = torch.tensor(I.decode_queries(42, 2, 8, 1, 128), device="cuda").half()
    patch.apply()
    try:
        out = patch.current_sdpa()(q, k_out, v_out, cache=cache, scale=1 / math.sqrt(128), mask=None)
    finally:
        patch.revert()
    assert not k_out.is_materialized
    torch.testing.assert_close(out, ss.sunshape_sdpa(q, cache, 1 / math.sqrt(128)), rtol=0, atol=0)
    torch.testing.assert_close(k_out.materialize(), cache.keys, rtol=0, atol=0)
    cache.eager_fetch = True
    k2, _ = cache.update_and_fetch(*I.kv_stream(43, 2, 2, 1, 128))
    assert isinstance(k2, torch.Tensor) and k2.shape[2] == 301
    hy = ss.create_kv_cache(cfg1_codec, n_kv_heads=2, value_backend="grouped", value_bits=4)
    hk, hv = hy.update_and_fetch(kk, vv)
    assert isinstance(hk, DeferredTensor) and isinstance(hv, DeferredTensor)
    torch.testing.assert_close(hk.materialize(), hy.keys)
    torch.testing.assert_close(hv.materialize(), hy.values)


def test_make_mask_nbytes_and_compression(ss, cfg1_codec):
    """make_mask (cache.py:310-329): "none" for an empty step, "causal", or
    an fp16 array with 0 where key <= query position and fp16 min elsewhere;
    nbytes counts the real batch (the reference assumes batch 1, cache.py:268-294)."""
    cache = ss.create_kv_cache(cfg1_codec, n_kv_heads=2)
    assert cache.make_mask(0) == "none"
    kk, vv = I.kv_stream(44, 3, 2, 10, 128)
    cache.append(kk, vv)
    assert cache.make_mask(4) == "causal"
    m = cache.make_mask(4, return_array=True).cpu()
    assert m.dtype == torch.float16
    qp = np.arange(10, 14)[:, None]
    kp = np.arange(14)[None, :]
    want = np.where(qp >= kp, 0.0, np.finfo(np.float16).min).astype(np.float16)
    np.testing.assert_array_equal(m.numpy().astype(np.float16), want)
    assert cache.nbytes == 3 * 2 * 10 * (16 + 256)
    assert cache.nbytes_equivalent_fp16 == 2 * 3 * 2 * 10 * 128 * 2
    assert abs(cache.compression_ratio - (2 * 128 * 2) / (16 + 256)) < 1e-9


def test_kernel_stats_and_backend_breadcrumbs(ss, cfg1_codec):
    ss.reset_kernel_stats()
    cache = ss.create_kv_cache(cfg1_codec, n_kv_heads=2)
    kk, vv = I.kv_stream(45, 1, 2, 50, 128)
    cache.append(kk, vv)
    q = I.decode_queries(46, 1, 8, 1, 128)
    ss.sunshape_sdpa(q, cache, 0.088)
    st = ss.get_kernel_stats()
    assert st.get("ss_decode_attn", 0) >= 1
    # the append is deferred into the decode launch (or, when that does not
    # apply, a separate ss_cache_append / ss_vq_assign)
    assert (st.get("ss_cache_append", 0) + st.get("ss_vq_assign", 0)
            + st.get("ss_cache_append (fused into ss_decode_attn)", 0)) >= 1
    assert cfg1_codec.last_score_backend == "cuda_fused"
    qz = cfg1_codec.quantize(torch.tensor(kk[0, 0], device="cuda"))
    cfg1_codec.attention_scores(torch.randn(4, 128, device="cuda"), qz)
    assert cfg1_codec.last_score_backend == "cuda"
    ss.reset_kernel_stats()
    assert ss.get_kernel_stats() == {}


def test_query_centroid_dots_kernel(ss, cfg1_codec):
    """precompute_query_centroid_dots (codec.py:553-573) on its own kernel,
    against the oracle's einsum (pinned by the reference's cfg1 scores)."""
    g = golden("cfg1")
    q_cal, _ = I.gaussian_qk(42, 1024, 2048, 128)
    st = {"mode": "profileperm_baseline", "head_dim": 128, "block_dim": 8, "n_blocks": 16,
          "n_centroids": 256, "centroids": g["centroids"], "permutation": g["permutation"],
          "heavy": np.zeros(16, bool)}
    qt = O.forward_transform(st, q_cal[:8])
    want = O.query_centroid_dots(st, qt)
    ss.reset_kernel_stats()
    got = cfg1_codec.precompute_query_centroid_dots(torch.tensor(qt, device="cuda"))
    assert ss.get_kernel_stats().get("ss_query_centroid_dots") == 1
    assert tuple(got.shape) == (8, 16, 256)
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-5, atol=1e-5)
    # the gather over these tables reproduces the reference's cfg1 scores
    scores = want[:, np.arange(16)[None, :], g["indices"].astype(np.int64)].sum(-1)
    np.testing.assert_allclose(scores, g["scores"], atol=1e-4)


@pytest.mark.parametrize("d,rows,odt", [(128, 1000, torch.float32), (64, 77, torch.float32),
                                        (128, 129, torch.float16)])
def test_rotate_rows_kernel(ss, d, rows, odt):
    """The data-path rotations (rotated-mode keys, codec.py:273-293; the
    TurboQuant value basis of the fp16 tail) on the library's own kernel,
    against a float64 product."""
    from sunshape_mlx_b200 import kernels as K

    g = torch.Generator(device="cuda").manual_seed(d + rows)
    x = torch.randn((rows, d), generator=g, device="cuda")
    m = ss.generate_rotation_matrix(d, seed=3, device="cuda")
    ss.reset_kernel_stats()
    got = K.rotate_rows(x, m.T, odt)
    assert ss.get_kernel_stats().get("ss_rotate_rows") == 1
    want = x.double() @ m.T.double()
    if odt == torch.float32:
        assert float((got.double() - want).abs().max()) < 1e-5
    else:
        torch.testing.assert_close(got, want.half(), rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("kind,T,dt", [("perm", 1, torch.float16), ("perm", 3, torch.bfloat16),
                                       ("mixed", 1, torch.float32), ("bd4", 1, torch.float16)])
def test_deferred_append_fused_into_decode(ss, kind, T, dt):
    """A decode step's append (update_and_fetch) handed to the next
    sunshape_sdpa, whose table launch quantizes and stores the new tokens:
    the cache streams and the output equal those of a separate append
    (ss_cache_append) bit for bit, over several steps; any other reader
    (keys, trim, a second append) writes a pending append first."""
    rng = np.random.default_rng(7)
    kc = rng.standard_normal((2048, 128)).astype(np.float32)
    qc = I.heavy_tailed_queries(1024, 128, seed=3)
    if kind == "mixed":
        codec = ss.SunShapeBlockCodec(head_dim=128, mode="profileperm_mixed_precision", n_heavy=4)
    else:
        codec = ss.SunShapeBlockCodec(head_dim=128, block_dim=4 if kind == "bd4" else 8)
    codec.fit(qc, kc, kmeans_iters=2, seed=0)
    caches = [ss.create_kv_cache(codec, n_kv_heads=4) for _ in range(2)]
    caches[1].defer_append = False
    g = torch.Generator(device="cuda").manual_seed(11)
    pre_k = torch.randn((2, 4, 300, 128), generator=g, device="cuda").to(dt)
    pre_v = torch.randn((2, 4, 300, 128), generator=g, device="cuda").to(dt)
    for c in caches:
        c.append(pre_k, pre_v)
    for step in range(4):
        k = torch.randn((2, 4, T, 128), generator=g, device="cuda").to(dt)
        v = torch.randn((2, 4, T, 128), generator=g, device="cuda").to(dt)
        q = torch.randn((2, 16, 1, 128), generator=g, device="cuda").half()
        outs = []
        for c in caches:
            c.update_and_fetch(k, v)
            outs.append(ss.sunshape_sdpa(q, c, 1 / math.sqrt(128)))
        assert caches[0]._pending is None
        torch.testing.assert_close(outs[0], outs[1], rtol=0, atol=0)
        assert torch.equal(caches[0].key_indices, caches[1].key_indices)
        assert torch.equal(caches[0].values, caches[1].values)
        if kind == "mixed":
            assert torch.equal(caches[0]._key_heavy[:, :, :caches[0].offset],
                               caches[1]._key_heavy[:, :, :caches[1].offset])
    # readers other than the fused decode write the pending tokens first
    k = torch.randn((2, 4, T, 128), generator=g, device="cuda").to(dt)
    for c in caches:
        c.append(k, k)
    assert caches[0]._pending is not None
    torch.testing.assert_close(caches[0].keys, caches[1].keys, rtol=0, atol=0)
    assert caches[0]._pending is None
    for c in caches:
        c.append(k, k)
        c.trim(1)
    assert torch.equal(caches[0].key_indices, caches[1].key_indices)


def test_pinned_host_append_and_output(ss, cfg1_codec):
    """Page-locked host tensors for a decode step: the new K/V token is read
    by the append kernel from host memory in place, and the attention output
    is written straight into a host tensor; results equal the device path."""
    caches = [ss.create_kv_cache(cfg1_codec, n_kv_heads=2) for _ in range(2)]
    kk, vv = I.kv_stream(51, 2, 2, 500, 128)
    for c in caches:
        c.append(kk, vv)
    g = torch.Generator().manual_seed(5)
    for step in range(3):
        k = torch.randn((2, 2, 1, 128), generator=g).half().pin_memory()
        v = torch.randn((2, 2, 1, 128), generator=g).half().pin_memory()
        q = torch.randn((2, 8, 1, 128), generator=g).half()
        qd = q.cuda()
        host_out = torch.empty((2, 8, 1, 128), dtype=torch.float16).pin_memory()
        caches[0].append(k, v)                      # stays on the host until the launch
        assert not caches[0]._pending[0].is_cuda
        r0 = ss.sunshape_sdpa(qd, caches[0], 0.088, out=host_out)
        caches[1].append(k.cuda(), v.cuda())
        r1 = ss.sunshape_sdpa(qd, caches[1], 0.088)
        torch.cuda.synchronize()
        assert r0 is host_out
        torch.testing.assert_close(host_out, r1.cpu(), rtol=0, atol=0)
        assert torch.equal(caches[0].key_indices, caches[1].key_indices)
        assert torch.equal(caches[0].values, caches[1].values)
    # a pending host append written by another reader (flush through ss_cache_append)
    k = torch.randn((2, 2, 1, 128), generator=g).half().pin_memory()
    caches[0].append(k, k)
    caches[1].append(k.cuda(), k.cuda())
    assert torch.equal(caches[0].key_indices, caches[1].key_indices)
