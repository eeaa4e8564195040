"""GPU parity of the fused decode / prefill attention over the compressed
cache (ss_decode_attn) against the reference's golden outputs, the oracle,
and a plain-torch fp64 reference. Tolerance: 1e-3 relative (max-abs error /
max-abs reference) for float32 semantics; fp16 outputs are additionally
compared with the reference's fp16 outputs at 2e-3 absolute."""

import math

import numpy as np
import pytest
import torch

import gpu_ref as G
import inputs as I
import oracle as O
from conftest import golden

pytestmark = pytest.mark.gpu
REL = 1e-3


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


def _check(out, want16=None, want32=None, rel=REL):
    o = out.float()
    if want16 is not None:
        w = torch.as_tensor(np.asarray(want16, np.float32), device=o.device)
        assert float((o - w).abs().max()) < 2e-3
    if want32 is not None:
        w = torch.as_tensor(np.asarray(want32, np.float32), device=o.device) if not torch.is_tensor(want32) else want32
        assert G.rel_err(o, w) < rel, G.rel_err(o, w)


def test_sdpa_simple_cache_golden(ss, cfg1_codec):
    g = golden("sdpa_simple")
    sc = 1 / math.sqrt(128)
    stt = {"mode": "profileperm_baseline", "head_dim": 128, "block_dim": 8, "n_blocks": 16,
           "n_centroids": 256, "centroids": golden("cfg1")["centroids"],
           "permutation": golden("cfg1")["permutation"], "heavy": np.zeros(16, bool),
           "inv_permutation": O.invert_permutation(golden("cfg1")["permutation"])}
    cache = ss.create_kv_cache(cfg1_codec, n_kv_heads=2)
    assert isinstance(cache, ss.SunShapeKVCache)
    kk, vv = I.kv_stream(11, 2, 2, 100, 128)
    k_out, v_out = cache.update_and_fetch(kk, vv)
    assert cache.offset == 100 and tuple(v_out.shape) == (2, 2, 100, 128)
    qd = I.decode_queries(12, 2, 8, 1, 128)
    out = ss.sunshape_sdpa(qd, cache, sc)
    assert out.dtype == torch.float16
    idx = cache.key_indices.cpu().numpy()
    _check(out, g["out_decode"], O.sdpa(qd, stt, idx, vv, sc))
    k3, v3 = I.kv_stream(13, 2, 2, 3, 128)
    cache.update_and_fetch(k3, v3)
    np.testing.assert_array_equal(cache.key_indices.cpu().numpy(), g["key_indices"])
    V = np.concatenate([vv, v3], 2)
    q3 = I.decode_queries(14, 2, 8, 3, 128)
    idx = cache.key_indices.cpu().numpy()
    _check(ss.sunshape_sdpa(q3, cache, sc, mask="causal"), g["out_causal"],
           O.sdpa(q3, stt, idx, V, sc, mask="causal"))
    _check(ss.sunshape_sdpa(q3, cache, sc, mask=g["bool_mask"]), g["out_bool_mask"],
           O.sdpa(q3, stt, idx, V, sc, mask=g["bool_mask"]))
    _check(ss.sunshape_sdpa(q3, cache, sc, mask=g["add_mask"]), g["out_add_mask"],
           O.sdpa(q3, stt, idx, V, sc, mask=g["add_mask"]))
    # round-trip keys property == oracle dequantize
    np.testing.assert_array_equal(cache.keys.cpu().numpy()[1, 0],
                                  O.dequantize(stt, idx[1, 0]))


@pytest.mark.parametrize("name,kw", [
    ("hyb_fp16_b32", dict(buffer_size=32)),
    ("hyb_grouped4_b32", dict(value_backend="grouped", value_bits=4, buffer_size=32)),
    ("hyb_grouped2_b0", dict(value_backend="grouped", value_bits=2, buffer_size=0)),
    ("hyb_tq2_b32", dict(value_backend="turboquant", value_bits=2, buffer_size=32)),
    ("hyb_tq2_b0", dict(value_backend="turboquant", value_bits=2, buffer_size=0)),
    ("hyb_tq4_b0", dict(value_backend="turboquant", value_bits=4, buffer_size=0)),
    ("hyb_vq_b32", dict(value_backend="sunshape", value_bits=1, buffer_size=32)),
])
def test_sdpa_hybrid_golden(ss, cfg1_codec, name, kw):
    g = golden(name)
    bsz = g["key_indices"].shape[0]
    if "value_norms" in g:
        kw = dict(kw, value_rotation=g["rotation"])
    cache = ss.create_kv_cache(cfg1_codec, n_kv_heads=2, **kw)
    kk, vv = I.kv_stream(21, bsz, 2, 100, 128)
    cache.update_and_fetch(kk, vv)
    assert cache.compressed_offset == int(g["compressed_offset"])
    assert cache.buffer_offset == int(g["buffer_offset"])
    np.testing.assert_array_equal(cache.key_indices.cpu().numpy(), g["key_indices"])
    qd = I.decode_queries(12, 2, 8, 1, 128)[:bsz]
    out = ss.sunshape_sdpa(qd, cache, 1 / math.sqrt(128))
    # oracle on the values the cache decodes (fp16 like the reference's cache.values)
    vals = cache.values.float().cpu().numpy()
    c = cache.compressed_offset
    stt = {"mode": "profileperm_baseline", "head_dim": 128, "block_dim": 8, "n_blocks": 16,
           "n_centroids": 256, "centroids": golden("cfg1")["centroids"],
           "permutation": golden("cfg1")["permutation"], "heavy": np.zeros(16, bool)}
    b = cache.buffer_offset
    want = O.sdpa(qd, stt, g["key_indices"], vals[:, :, :c], 1 / math.sqrt(128),
                  buffer_keys=kk[:, :, c:] if b else None, buffer_values=vv[:, :, c:] if b else None)
    _check(out, g["out"], want, rel=2e-3)
    if cache.value_backend == "grouped":
        np.testing.assert_array_equal(cache.values_packed_raw.cpu().numpy().view(np.uint32),
                                      g["values_packed"])
        np.testing.assert_array_equal(cache.value_scales_raw.cpu().numpy(), g["value_scales"])


def _random_cache_setup(B, Hkv, T, D=128, bd=8, k=256, seed=0, vfmt="fp16"):
    rng = np.random.default_rng(seed)
    nb = D // bd
    cents = torch.tensor(rng.standard_normal((nb, k, bd)) * 0.7, dtype=torch.float32, device="cuda")
    perm = torch.tensor(rng.permutation(D), dtype=torch.int32, device="cuda")
    cap = -(-T // 256) * 256
    idx = torch.zeros((B, Hkv, cap, nb), dtype=torch.uint8, device="cuda")
    idx[:, :, :T] = torch.randint(0, k, (B, Hkv, T, nb), device="cuda", dtype=torch.uint8)
    v = torch.zeros((B, Hkv, cap, D), dtype=torch.float16, device="cuda")
    v[:, :, :T] = torch.randn((B, Hkv, T, D), device="cuda").half()
    return cents, perm, idx, v, cap


def _ref_from(cents, perm, idx, v, q, scale, T, causal=False):
    inv = torch.argsort(perm.long())
    kc = G.dequant_codec_space(idx[:, :, :T], cents)
    k = kc[..., inv]
    qs = G.scaled_queries(q, scale)
    return G.attention(qs, k, v[:, :, :T].float(), causal=causal)


@pytest.mark.parametrize("B,Hkv,Hq,Tq,T,D,causal,max_ctas", [
    (2, 8, 32, 1, 8192, 128, False, 0),     # cfg2 shape, 2 sequences
    (1, 2, 8, 1, 1, 128, False, 0),         # single token
    (1, 2, 8, 1, 129, 128, False, 0),       # ragged tail tile
    (3, 2, 2, 1, 1000, 128, False, 0),      # no GQA (R = 1)
    (1, 1, 8, 1, 5000, 128, False, 3),      # R = 8, 3 CTAs -> cross-CTA merges
    (2, 4, 16, 2, 3001, 128, True, 0),      # Tq = 2 causal, R = 8
    (1, 2, 8, 5, 700, 128, True, 7),        # 20 rows -> 3 row groups
    (2, 2, 4, 1, 2048, 64, False, 0),       # head_dim 64
    (1, 1, 4, 1, 40000, 128, False, 148),   # one pair spread over many CTAs
])
def test_decode_random_vs_torch(ss, B, Hkv, Hq, Tq, T, D, causal, max_ctas):
    from sunshape_mlx_b200.attention import _run_decode

    cents, perm, idx, v, cap = _random_cache_setup(B, Hkv, T, D, seed=T + Hq)
    q = torch.randn((B, Hq, Tq, D), device="cuda").half()
    out = torch.empty_like(q)
    spec = dict(tc=T, cap=cap, idx=idx, v=v, max_ctas=max_ctas)
    _run_decode(q, centroids=cents, perm=perm, scale=1 / math.sqrt(D), spec=spec, causal=causal,
                out=out)
    want = _ref_from(cents, perm, idx, v, q, 1 / math.sqrt(D), T, causal)
    assert G.rel_err(out, want) < REL, G.rel_err(out, want)


def test_decode_invariant_to_cta_split(ss):
    from sunshape_mlx_b200.attention import _run_decode

    cents, perm, idx, v, cap = _random_cache_setup(2, 4, 6000, seed=11)
    q = torch.randn((2, 16, 1, 128), device="cuda").half()
    outs = []
    for mc in (1, 5, 37, 148):
        o = torch.empty((2, 16, 1, 128), dtype=torch.float32, device="cuda")
        _run_decode(q, centroids=cents, perm=perm, scale=0.088, spec=dict(tc=6000, cap=cap, idx=idx, v=v, max_ctas=mc),
                    causal=False, out=o)
        outs.append(o)
    # different split points change each warp's running max and so the fp16
    # rounding of P; results agree to the parity tolerance
    for o in outs[1:]:
        assert G.rel_err(o, outs[0]) < REL
    from sunshape_mlx_b200 import _lib as L
    from sunshape_mlx_b200.attention import _WS
    for ws in _WS.values():
        L.call("ss_decode_check", L.ptr(ws), L.stream_ptr())
        # the 8 units' arrival counters (bytes 256..288) are back at zero
        assert int(ws[256:256 + 4 * 8].view(torch.int32).abs().sum()) == 0


def test_quantized_values_decode_vs_torch(ss):
    from sunshape_mlx_b200.attention import _run_decode

    B, H, T, D = 2, 4, 3000, 128
    cents, perm, idx, v, cap = _random_cache_setup(B, H, T, seed=2)
    vals = torch.randn((B, H, cap, D), device="cuda")
    for kind in ("grouped2", "grouped4", "tq_ref", "tq_group"):
        if kind.startswith("grouped"):
            bits = int(kind[-1])
            codec = ss.GroupedValueCodec(head_dim=D, bits=bits, group_size=64)
            p, s, z = codec.quantize(vals)
            spec = dict(tc=T, cap=cap, idx=idx, vq=p, vs=s, vz=z, bits=bits, group=64,
                        levels=codec.levels(None))
            deq = codec.dequantize(p, s, z)
        else:
            codec = ss.TurboQuantValueCodec(head_dim=D, bits=2, group_size=None if kind == "tq_ref" else 32)
            p, s = codec.quantize(vals)
            vs = s if s.dim() == 4 else s.unsqueeze(-1)
            spec = dict(tc=T, cap=cap, idx=idx, vq=p, vs=vs, vz=None, bits=2,
                        group=codec.group_size or D, levels=codec.levels(None), v_rot=codec.rotation)
            deq = codec.dequantize(p, s)
        q = torch.randn((B, 4 * H, 1, D), device="cuda").half()
        out = torch.empty_like(q)
        _run_decode(q, centroids=cents, perm=perm, scale=0.088, spec=spec, causal=False, out=out)
        want = _ref_from(cents, perm, idx, deq.half(), q, 0.088, T)
        assert G.rel_err(out, want) < 2e-3, (kind, G.rel_err(out, want))


@pytest.mark.parametrize("T", [77, 129, 3000])
def test_tq_group32_fragment_decode_ragged(ss, T):
    """2-bit values with fp16 scales per 32 channels, 4 query rows per kv-head:
    the kernel decodes the codes straight into the P.V MMA fragments. Ragged
    lengths leave a partial last tile, and the rows past the end hold NaN
    scales: those tokens must contribute exactly nothing. Checked per element
    against float64 attention over the values as the kernel rounds them
    (fp16(level * scale) in the rotated basis), rotated back."""
    from sunshape_mlx_b200.attention import _run_decode

    B, H, D = 2, 4, 128
    cents, perm, idx, _, cap = _random_cache_setup(B, H, T, seed=70 + T)
    vals = torch.randn((B, H, cap, D), device="cuda")
    codec = ss.TurboQuantValueCodec(head_dim=D, bits=2, group_size=32)
    p, s = codec.quantize(vals)
    assert s.dtype == torch.float16 and s.shape[-1] == D // 32
    s = s.clone()
    s[:, :, T:] = float("nan")
    spec = dict(tc=T, cap=cap, idx=idx, vq=p, vs=s, vz=None, bits=2, group=32,
                levels=codec.levels(None), v_rot=codec.rotation)
    q = torch.randn((B, 4 * H, 1, D), device="cuda")
    out = torch.empty_like(q)
    _run_decode(q, centroids=cents, perm=perm, scale=0.088, spec=spec, causal=False, out=out)
    # values in the rotated basis, rounded as the kernel rounds them
    words = p[:, :, :T].to(torch.int64) & 0xFFFFFFFF
    sh = torch.arange(16, device="cuda", dtype=torch.int64) * 2
    codes = ((words.unsqueeze(-1) >> sh) & 3).reshape(B, H, T, D)
    lv = torch.tensor(codec.levels(None)[:4], dtype=torch.float32, device="cuda")
    r = (lv[codes] * s[:, :, :T].float().repeat_interleave(32, dim=-1)).half()
    want = _ref_from(cents, perm, idx, r, q, 0.088, T).double() @ codec.rotation.double()
    err = (out.double() - want).abs()
    mref = want.abs().max()
    assert torch.isfinite(out).all()
    assert float(err.max() / mref) < 1e-3
    assert float((err / (2e-3 * want.abs() + 1e-4 * mref)).max()) <= 1.0


@pytest.mark.parametrize("hq", [8, 16])  # 16: 8 rows per kv-head, tables split into 2 row groups
def test_mixed_precision_heavy_blocks_exact_scoring(ss, hq):
    rng = np.random.default_rng(4)
    qc = I.heavy_tailed_queries(2048, 128, seed=7)
    kc = rng.standard_normal((2048, 128)).astype(np.float32)
    codec = ss.SunShapeBlockCodec(head_dim=128, mode="profileperm_mixed_precision", n_heavy=4)
    codec.fit(qc, kc, kmeans_iters=4, seed=0)
    assert codec.n_heavy_blocks == 4
    cache = ss.create_kv_cache(codec, n_kv_heads=2)
    kk, vv = I.kv_stream(8, 1, 2, 700, 128)
    cache.update_and_fetch(kk, vv)
    q = I.decode_queries(9, 1, hq, 1, 128)
    out = ss.sunshape_sdpa(q, cache, 1 / math.sqrt(128))
    # reference semantics with heavy blocks restored: q . dequantize(quantize(k))
    khat = torch.stack([torch.stack([codec(torch.tensor(kk[0, h], device="cuda")) for h in range(2)])])
    want = G.attention(G.scaled_queries(torch.tensor(q, device="cuda"), 1 / math.sqrt(128)), khat,
                       torch.tensor(vv, device="cuda").float())
    assert G.rel_err(out, want) < REL


@pytest.mark.parametrize("n_heavy,hq,qdt,vals", [
    (2, 8, torch.float16, "fp16"), (4, 16, torch.float32, "fp16"), (8, 8, torch.float32, "fp16"),
    (8, 16, torch.float16, "grouped2"), (3, 8, torch.float32, "fp16"), (6, 16, torch.float16, "fp16"),
    (12, 8, torch.float16, "grouped2"), (4, 8, torch.bfloat16, "grouped2")])
def test_heavy_block_scoring_shapes(ss, n_heavy, hq, qdt, vals):
    """Heavy-block dot products over every heavy width: 16/32/64 heavy dims
    take the warp-MMA path (fp16 keys x hi+lo split queries), 24/48/96 the
    per-lane path; fp32 and bf16 queries exercise the lo half of the split."""
    rng = np.random.default_rng(40 + n_heavy)
    qc = I.heavy_tailed_queries(2048, 128, seed=8)
    kc = rng.standard_normal((2048, 128)).astype(np.float32)
    codec = ss.SunShapeBlockCodec(head_dim=128, mode="profileperm_mixed_precision", n_heavy=n_heavy)
    codec.fit(qc, kc, kmeans_iters=3, seed=0)
    assert codec.n_heavy_blocks == n_heavy
    kw = {} if vals == "fp16" else dict(value_backend="grouped", value_bits=2, buffer_size=0)
    cache = ss.create_kv_cache(codec, n_kv_heads=2, **kw)
    kk, vv = I.kv_stream(11, 1, 2, 1000, 128)
    vv = vv * 2.0
    cache.update_and_fetch(kk, vv)
    q = torch.tensor(I.decode_queries(12, 1, hq, 1, 128), device="cuda").to(qdt) * 3
    out = ss.sunshape_sdpa(q, cache, 1 / math.sqrt(128))
    khat = torch.stack([torch.stack([codec(torch.tensor(kk[0, h], device="cuda")) for h in range(2)])])
    vt = torch.tensor(vv, device="cuda")
    if vals != "fp16":
        vc = ss.GroupedValueCodec(head_dim=128, bits=2, group_size=64)
        p_, s_, z_ = vc.quantize(vt.half())
        vt = vc.dequantize(p_, s_, z_)
    want = G.attention(G.scaled_queries(q, 1 / math.sqrt(128)), khat, vt.float())
    tol = 4e-3 if qdt == torch.bfloat16 else 2e-3  # bf16 output: half an ulp is 2^-9 relative
    assert G.rel_err(out, want) < tol, G.rel_err(out, want)


@pytest.mark.parametrize("vbd,vmode,buf,tq", [
    (4, "profileperm_baseline", 0, 1), (8, "profileperm_baseline", 32, 1),
    (16, "profileperm_baseline", 0, 1), (4, "rotated", 16, 1),
    (8, "rotated", 0, 1), (4, "profileperm_baseline", 16, 5)])
def test_vq_values_fused_decode(ss, vbd, vmode, buf, tq):
    """value_backend="sunshape" (cache.py:785-812): block-VQ value indices
    decoded inside the fused kernel from an fp16 centroid table, accumulated
    in the value codec's basis and transformed back once; compared with the
    reference semantics softmax(q k_hat^T) v_hat, v_hat = fp16(dequantize(v))."""
    rng = np.random.default_rng(60 + vbd + 3 * buf + tq + len(vmode))
    kc = rng.standard_normal((2048, 128)).astype(np.float32)
    qc = rng.standard_normal((1024, 128)).astype(np.float32)
    kcodec = ss.SunShapeBlockCodec(head_dim=128, block_dim=4)
    kcodec.fit(qc, kc, kmeans_iters=3, seed=0)
    vcal = rng.standard_normal((2048, 128)).astype(np.float32)
    vcodec = ss.SunShapeBlockCodec(head_dim=128, block_dim=vbd, mode=vmode)
    vcodec.fit(qc, vcal, kmeans_iters=3, seed=1)
    cache = ss.create_kv_cache(kcodec, n_kv_heads=2, value_backend="sunshape", value_bits=8,
                               value_codec=vcodec, buffer_size=buf)
    kk, vv = I.kv_stream(21, 2, 2, 777, 128)
    cache.update_and_fetch(kk, vv)
    q = torch.tensor(I.decode_queries(22, 2, 8, tq, 128), device="cuda")
    out = ss.sunshape_sdpa(q, cache, 1 / math.sqrt(128), mask="causal" if tq > 1 else None)
    kt = torch.tensor(kk, device="cuda")
    vt = torch.tensor(vv, device="cuda")
    c = 777 - buf
    khat = torch.cat([torch.stack([torch.stack([kcodec(kt[b, h, :c]) for h in range(2)]) for b in range(2)]),
                      kt[:, :, c:].half().float()], 2)
    vhat = torch.cat([torch.stack([torch.stack([vcodec(vt[b, h, :c]) for h in range(2)]) for b in range(2)]).half(),
                      vt[:, :, c:].half()], 2)
    want = G.attention(G.scaled_queries(q, 1 / math.sqrt(128)), khat, vhat.float(), causal=tq > 1)
    assert G.rel_err(out, want) < 2e-3, G.rel_err(out, want)
    # the cache's decoded values agree with the codec (the unfused view)
    torch.testing.assert_close(cache.values[:, :, :c].float(), vhat[:, :, :c].float())


def test_empty_cache_returns_zeros(ss, cfg1_codec):
    cache = ss.create_kv_cache(cfg1_codec, n_kv_heads=2)
    q = torch.randn((1, 4, 1, 128), device="cuda").half()
    assert float(ss.sunshape_sdpa(q, cache, 0.1).abs().max()) == 0.0


def test_reference_fused_wrappers_known_answers(ss):
    """test_kernels.py [11] [12] [14] [15] [16] [17]: fused kernels vs the
    explicit NumPy softmax references."""
    def khat(c, idx):
        return np.concatenate([c[b][idx[:, b]] for b in range(16)], axis=1)

    def ref(q, k, v, causal=False):
        s = q @ k.T
        if causal:
            tq, tkv = s.shape
            ok = np.arange(tkv - tq, tkv)[:, None] >= np.arange(tkv)[None, :]
            s = np.where(ok, s, -1e30)
        w = np.exp(s - s.max(-1, keepdims=True))
        return (w / w.sum(-1, keepdims=True)) @ v

    for seed, tq, tkv, causal, scale, tol in [(111, 1, 64, False, 1.0, 5e-3), (222, 4, 32, True, 1.0, 5e-3),
                                              (444, 1, 512, False, 0.1, 1e-2)]:
        np.random.seed(seed)
        c = np.random.randn(16, 256, 8).astype(np.float32)
        idx = np.random.randint(0, 256, size=(tkv, 16), dtype=np.uint8)
        v = (np.random.randn(tkv, 128) * scale).astype(np.float32)
        q = (np.random.randn(tq, 128) * scale).astype(np.float32)
        if causal:
            got = ss.fused_attention_causal_metal(q, c, idx, v, tq, tkv, 16, 256, 128, q_offset=tkv - tq)
        else:
            got = ss.fused_attention_metal(q, c, idx, v, tq, tkv, 16, 256, 128)
        assert np.abs(got.cpu().numpy() - ref(q, khat(c, idx), v, causal)).max() < tol
    for seed, tq, tkv, causal, bits in [(555, 1, 64, False, 4), (666, 4, 32, True, 4), (777, 1, 64, False, 2)]:
        np.random.seed(seed)
        c = np.random.randn(16, 256, 8).astype(np.float32)
        idx = np.random.randint(0, 256, size=(tkv, 16), dtype=np.uint8)
        q = np.random.randn(tq, 128).astype(np.float32)
        v = np.random.randn(tkv, 128).astype(np.float32)
        p, s, z, _ = O.quantize_values(v, bits, 64)
        deq = O.dequantize_values(p, s, z, 128, bits, 64)
        fn = ss.fused_attention_dequant_causal_metal if causal else ss.fused_attention_dequant_metal
        kw = dict(q_offset=tkv - tq) if causal else {}
        got = fn(q, c, idx, p.view(np.int32), s, z, tq, tkv, 16, 256, 128, bits, 64, **kw)
        assert np.abs(got.cpu().numpy() - ref(q, khat(c, idx), deq, causal)).max() < 5e-3


def test_splitkv_partials_merge_single_gpu(ss, cfg1_codec):
    from sunshape_mlx_b200 import splitkv
    from sunshape_mlx_b200.attention import decode_partials

    kk, vv = I.kv_stream(31, 1, 2, 3000, 128)
    full = ss.create_kv_cache(cfg1_codec, n_kv_heads=2)
    full.append(kk, vv)
    shards = []
    for r in range(3):
        lo, hi = splitkv.shard_range(3000, r, 3)
        c = ss.create_kv_cache(cfg1_codec, n_kv_heads=2)
        c.append(kk[:, :, lo:hi], vv[:, :, lo:hi])
        shards.append(c)
    q = torch.tensor(I.decode_queries(32, 1, 8, 1, 128), device="cuda")
    parts = torch.stack([decode_partials(q, c, 0.088) for c in shards])
    got = splitkv.merge_partials(parts, q.shape, q.dtype)
    want = ss.sunshape_sdpa(q, full, 0.088)
    assert float((got.float() - want.float()).abs().max()) < 2e-3
