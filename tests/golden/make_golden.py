"""Generate golden vectors by running the REFERENCE package's own code.

Run where the reference tree is available, naming its root directory:

    SUNSHAPE_REF=<path to the reference tree> python tests/golden/make_golden.py

The reference imports ``mlx.core``; MLX is not installable here, so
``mlx_numpy_shim.py`` is put in its place. Every Metal wrapper then takes its
own ``return None`` fallback, i.e. the reference runs the CPU code paths it
runs on any non-Apple machine (NumPy quantize loop, 2-pass SDPA, MLX-op
packing/value codecs). Inputs come from ``inputs.py``; only outputs (and the
few parameters drawn inside the reference, like the rotation matrix) are
stored, as compressed ``.npz`` files next to this script.
"""

from __future__ import annotations

import math
import os
import sys
import tempfile
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import inputs as I  # noqa: E402
import mlx_numpy_shim  # noqa: E402


def _import_reference(ref_root: str):
    tmp = tempfile.mkdtemp(prefix="sunshape_ref_")
    os.symlink(ref_root, os.path.join(tmp, "sunshape_mlx"))
    sys.path.insert(0, tmp)
    mlx_pkg = types.ModuleType("mlx")
    mlx_pkg.core = mlx_numpy_shim
    sys.modules["mlx"] = mlx_pkg
    sys.modules["mlx.core"] = mlx_numpy_shim
    import sunshape_mlx  # noqa: F401
    return sys.modules["sunshape_mlx"]


def _save(name: str, **arrays):
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **{k: np.asarray(v) for k, v in arrays.items()})
    print(f"wrote {path}: {sorted(arrays)}")


def main():
    ref_root = os.environ.get("SUNSHAPE_REF")
    if not ref_root:
        raise SystemExit("set SUNSHAPE_REF to the root of the reference tree")
    ss = _import_reference(ref_root)
    from sunshape_mlx.codec import SunShapeBlockCodec
    from sunshape_mlx import kernels as K
    from sunshape_mlx.cache import create_kv_cache, HybridSunShapeKVCache
    from sunshape_mlx.attention import sunshape_sdpa
    from sunshape_mlx.value_codecs import TurboQuantValueCodec

    # A. head_dim 64 baseline codec (test fixture analogue)
    q, k = I.small_codec_inputs()
    c = SunShapeBlockCodec(head_dim=64, block_dim=8, n_centroids=256, mode="profileperm_baseline")
    c.fit(q, k, kmeans_iters=10, seed=42)
    qz = c.quantize(k)
    _save("codec_d64", permutation=c.permutation, inv_permutation=c.inv_permutation,
          centroids=c.centroids, indices=qz.indices, k_hat=c.dequantize(qz),
          scores=c.attention_scores(q[:8], qz), backend=np.array(c.last_score_backend))

    # B. config 1: D=128, fit on q (1024) / k (2048), 15 iters, seed 42
    q, k = I.gaussian_qk(42, 1024, 2048, 128)
    c1 = SunShapeBlockCodec(head_dim=128, block_dim=8, n_centroids=256, mode="profileperm_baseline")
    c1.fit(q, k, kmeans_iters=15, seed=42)
    qz = c1.quantize(k[:128])
    _save("cfg1", permutation=c1.permutation, centroids=c1.centroids, indices=qz.indices,
          k_hat=c1(k), scores=c1.attention_scores(q[:8], qz))

    # C. assignment known answer (test_kernels.py:404-439)
    keys, cents = I.assign_known_answer()
    ca = SunShapeBlockCodec(head_dim=128, block_dim=8, n_centroids=256, mode="profileperm_baseline")
    ca.centroids = cents
    got = ca.quantize(keys).indices
    ref = np.zeros((32, 16), dtype=np.int32)
    for b in range(16):
        d = keys[:, b * 8:(b + 1) * 8][:, None, :] - cents[b][None]
        ref[:, b] = np.argmin(np.sum(d ** 2, axis=-1), axis=1)
    assert np.array_equal(got.astype(np.int32), ref)
    _save("assign333", indices=got)

    # D. mixed precision (heavy-tailed queries)
    qm = I.heavy_tailed_queries(512, 64, seed=5)
    km = np.random.default_rng(6).standard_normal((512, 64)).astype(np.float32)
    cm = SunShapeBlockCodec(head_dim=64, block_dim=8, n_centroids=256, mode="profileperm_mixed_precision")
    cm.fit(qm, km, kmeans_iters=5, seed=3)
    qz = cm.quantize(km[:64])
    _save("mixed", permutation=cm.permutation, centroids=cm.centroids,
          heavy=cm.mixed_high_precision_blocks, indices=qz.indices,
          passthrough=qz.passthrough_values, k_hat=cm.dequantize(qz),
          scores=cm.attention_scores(qm[:4], qz))

    # E. rotated mode
    q, k = I.small_codec_inputs()
    cr = SunShapeBlockCodec(head_dim=64, block_dim=8, n_centroids=256, mode="rotated",
                            use_rotation=True, rotation_seed=7)
    cr.fit(q, k, kmeans_iters=5, seed=1)
    qz = cr.quantize(k[:64])
    _save("rotated", rotation=cr.rotation, centroids=cr.centroids, indices=qz.indices,
          k_hat=cr.dequantize(qz), scores=cr.attention_scores(q[:4], qz))

    scale = 1.0 / math.sqrt(128)

    # F. simple cache (fp16 values) + SDPA, decode and causal prefill
    kk, vv = I.kv_stream(11, 2, 2, 100, 128)
    cache = create_kv_cache(c1, n_kv_heads=2)
    cache.update_and_fetch(kk, vv)
    qd = I.decode_queries(12, 2, 8, 1, 128)
    out_decode = sunshape_sdpa(qd, cache, scale, mask=None)
    k3, v3 = I.kv_stream(13, 2, 2, 3, 128)
    cache.update_and_fetch(k3, v3)
    q3 = I.decode_queries(14, 2, 8, 3, 128)
    out_causal = sunshape_sdpa(q3, cache, scale, mask="causal")
    bmask = np.random.default_rng(15).random((3, 103)) > 0.3
    bmask[:, 0] = True
    out_bmask = sunshape_sdpa(q3, cache, scale, mask=bmask)
    amask = (np.random.default_rng(16).standard_normal((3, 103)) * 2.0).astype(np.float32)
    out_amask = sunshape_sdpa(q3, cache, scale, mask=amask)
    _save("sdpa_simple", key_indices=cache.key_indices, out_decode=out_decode,
          out_causal=out_causal, bool_mask=bmask, out_bool_mask=out_bmask,
          add_mask=amask, out_add_mask=out_amask, offset=np.array(cache.offset),
          backend=np.array(c1.last_score_backend))

    # G/H/I. hybrid caches
    for name, kw in [
        ("hyb_fp16_b32", dict(buffer_size=32)),
        ("hyb_grouped4_b32", dict(value_backend="grouped", value_bits=4, buffer_size=32)),
        ("hyb_grouped2_b0", dict(value_backend="grouped", value_bits=2, buffer_size=0)),
        ("hyb_tq2_b32", dict(value_backend="turboquant", value_bits=2, buffer_size=32)),
        ("hyb_tq2_b0", dict(value_backend="turboquant", value_bits=2, buffer_size=0)),
        ("hyb_tq4_b0", dict(value_backend="turboquant", value_bits=4, buffer_size=0)),
        ("hyb_vq_b32", dict(value_backend="sunshape", value_bits=1, buffer_size=32)),
    ]:
        # The reference's empty-buffer accessor returns batch size 1
        # (cache.py:830-835), so buffer_size=0 with B>1 raises IndexError in
        # attention.py:272; those cases use B=1.
        bsz = 1 if kw["buffer_size"] == 0 else 2
        kk, vv = I.kv_stream(21, bsz, 2, 100, 128)
        hc = create_kv_cache(c1, n_kv_heads=2, **kw)
        assert isinstance(hc, HybridSunShapeKVCache)
        hc.update_and_fetch(kk, vv)
        out = sunshape_sdpa(qd[:bsz], hc, scale, mask=None)
        extra = {}
        if hc.value_backend == "grouped":
            extra = dict(values_packed=hc._values_packed[:, :, :hc.compressed_offset],
                         value_scales=hc._value_scales[:, :, :hc.compressed_offset],
                         value_zeros=hc._value_zeros[:, :, :hc.compressed_offset])
        elif hc.value_backend == "turboquant":
            extra = dict(values_packed=hc._values_packed[:, :, :hc.compressed_offset],
                         value_norms=hc._value_norms[:, :, :hc.compressed_offset],
                         rotation=hc._value_codec_impl.rotation)
        elif hc.value_backend == "sunshape":
            extra = dict(value_indices=hc._value_indices[:, :, :hc.compressed_offset])
        _save(name, key_indices=hc.key_indices, buffer_keys=hc.buffer_keys,
              buffer_values=hc.buffer_values, values=hc.values, out=out,
              compressed_offset=np.array(hc.compressed_offset),
              buffer_offset=np.array(hc.buffer_offset), **extra)

    # J. hybrid flush bookkeeping over a sequence of appends
    hc = create_kv_cache(c1, n_kv_heads=2, buffer_size=32, value_backend="fp16")
    offs = []
    for i, t in enumerate([16, 24, 1, 1, 40]):
        kk, vv = I.kv_stream(30 + i, 1, 2, t, 128)
        hc.update_and_fetch(kk, vv)
        offs.append((hc.offset, hc.compressed_offset, hc.buffer_offset))
    hc.trim(5)
    offs.append((hc.offset, hc.compressed_offset, hc.buffer_offset))
    hc.trim(40)
    offs.append((hc.offset, hc.compressed_offset, hc.buffer_offset))
    _save("hyb_flush_seq", offsets=np.array(offs), key_indices=hc.key_indices)

    # K. packing (test_kernels.py:49-103)
    np.random.seed(42)
    packs = {}
    for bits, mx_, d in [(2, 3, 128), (3, 7, 100), (4, 15, 128)]:
        idx = np.random.randint(0, mx_ + 1, size=(32, d), dtype=np.uint8)
        packs[f"idx{bits}"] = idx
        packs[f"packed{bits}"] = K.pack_indices(idx, bits=bits)
    np.random.seed(99)
    idx27 = np.random.randint(0, 8, size=(5, 27), dtype=np.uint8)
    packs["idx3_d27"] = idx27
    packs["packed3_d27"] = K.pack_indices(idx27, bits=3)
    _save("packing", **packs)

    # L. grouped value quantization (test_kernels.py:105-131)
    np.random.seed(123)
    vals = np.random.randn(64, 128).astype(np.float32)
    gq = {"values": vals}
    for bits in (2, 4):
        p, s, z, g = K.quantize_values(vals, bits=bits, group_size=64)
        gq[f"packed{bits}"], gq[f"scales{bits}"], gq[f"zeros{bits}"] = p, s, z
        gq[f"deq{bits}"] = K.dequantize_values(p, s, z, D=128, bits=bits, group_size=64)
    _save("grouped_values", **gq)

    # M. TurboQuant value codec
    vals = np.random.default_rng(21).standard_normal((64, 128)).astype(np.float32)
    tq = {"values": vals}
    for bits in (2, 3, 4):
        codec = TurboQuantValueCodec(head_dim=128, bits=bits, seed=43)
        p, n = codec.quantize(vals)
        tq[f"rotation{bits}"] = codec.rotation
        tq[f"packed{bits}"], tq[f"norms{bits}"] = p, n
        tq[f"deq{bits}"] = codec.dequantize(p, n)
    _save("turboquant_values", **tq)

    # N. scalar quantize (test_kernels.py:134-160)
    np.random.seed(77)
    bnd = np.array([-1.0, -0.5, 0.0, 0.5, 1.0], dtype=np.float32)
    vals = np.random.randn(100, 64).astype(np.float32)
    sq, backend = K.quantize_scalar_to_indices(vals, bnd, prefer_metal=False)
    _save("scalar_quantize", values=vals, boundaries=bnd, indices=sq)

    # O. pure-op fused attention (test_kernels.py:197-247 inputs)
    np.random.seed(42)
    cents = np.random.randn(16, 256, 8).astype(np.float32)
    idx = np.random.randint(0, 256, size=(32, 16), dtype=np.int32)
    vals = np.random.randn(32, 128).astype(np.float32)
    qq = np.random.randn(4, 128).astype(np.float32)
    qdots = np.einsum("qbd,bcd->qbc", qq.reshape(4, 16, 8), cents)
    fo = K.fused_block_vq_attention(qdots, idx, vals, T_q=4, T_kv=32, n_blocks=16,
                                    n_centroids=256, head_dim=128)
    _save("fused_block_vq", centroids=cents, indices=idx, values=vals, queries=qq, out=fo)
    print("reference version", ss.__version__)


if __name__ == "__main__":
    main()
