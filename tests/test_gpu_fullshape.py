"""Decode parity at the full sizes of the two long benchmark workloads.

* the 2-bit TurboQuant-value workload: B=64, 32q/8kv, T_kv=32768, rotated
  values with fp16 scales per 32 channels, buffer_size 0;
* the long single sequence: B=1, 64q/8kv, T_kv=524288, mixed-precision keys
  (4 of 16 blocks stored fp16), fp16 values, plus the split-KV path
  (per-shard (o, m, l) partials merged by ss_lse_merge).

The caches are built exactly as ``bench.py --config 3|5`` builds them. The
fused kernel writes fp32 outputs here, so the comparison measures the
kernel's arithmetic (fp16 softmax weights into the P.V MMA, fp32
accumulation) rather than the fp16 output rounding. The reference for a
(batch, kv-head) pair is computed in float64 by plain torch from the cache's
own stored codes: keys = centroid rows (plus the stored fp16 heavy blocks)
in the original basis, values = the stored 2-bit codes times their scales,
rotated back, rounded to fp16 as the reference's ``cache.values`` is
(cache.py:774-784), softmax in float64 (attention.py:307-350 semantics).

Tolerances (written here, checked per pair):
  * max |err| / max |ref| < 1e-3                      (fp32 semantics bound)
  * per element |err| <= 2e-3 * |ref| + 1e-4 * max|ref|  (every element)
  * ||err||_2 / ||ref||_2 < 1e-3
The per-element bound needs the softmax weights at better than fp16
precision (2^-11 relative rounding of each weight shifts every output
element by ~3e-4 of its own size): the kernel feeds P to the MMA as fp16
hi + lo pairs. For the TurboQuant values the per-element bound applies to the
kernel's own value rounding (fp16 in the rotated basis); the comparison with
the reference's rounding (fp16 after the inverse rotation) uses the
norm-wise bounds, as the two roundings differ per element.
"""

import math
import os
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

REL_MAX = 1e-3
REL_ELEM = 2e-3
ATOL_FRAC = 1e-4
REL_L2 = 1e-3


@pytest.fixture(scope="module")
def ss(cuda_ok):
    import sunshape_mlx_b200 as ss

    return ss


def _keys_pair(codec, spec, b, h, T):
    """(T, D) f32 keys of pair (b, h) in the original basis, from the stored
    indices and (mixed precision) the stored fp16 heavy blocks."""
    cents = codec.centroids  # (nb, K, bd)
    nb, _, bd = cents.shape
    idx = spec["idx"][b, h, :T].long()
    kc = cents[torch.arange(nb, device=idx.device), idx]  # (T, nb, bd)
    kh = spec.get("kheavy")
    if kh is not None:
        heavy = torch.nonzero(codec.mixed_high_precision_blocks).flatten().tolist()
        hv = kh[b, h, :T].float().reshape(T, len(heavy), bd)
        for j, blk in enumerate(heavy):
            kc[:, blk] = hv[:, j]
    kc = kc.reshape(T, nb * bd)
    inv = torch.argsort(codec.permutation.long())
    return kc[:, inv]


def _tq_values_pair(spec, b, h, T, basis="original"):
    """(T, D) values of pair (b, h) decoded from the 2-bit codes: level x
    fp16 group scale in the rotated basis. basis="original": rotated back and
    rounded to fp16, as the reference's cache.values; basis="rotated": rounded
    to fp16 in the rotated basis (the kernel accumulates there and rotates the
    output once, which is the same sum up to where the fp16 rounding falls)."""
    words = spec["vq"][b, h, :T]            # (T, D/16) int32, 16 codes per word
    D = words.shape[1] * 16
    sh = torch.arange(16, device=words.device, dtype=torch.int32) * 2
    codes = ((words.unsqueeze(-1) >> sh) & 3).reshape(T, D).long()
    lv = torch.tensor(spec["levels"][:4], dtype=torch.float32, device=words.device)
    g = int(spec["group"])
    sc = spec["vs"][b, h, :T].float()       # (T, D/g)
    r = lv[codes] * sc.repeat_interleave(g, dim=1)
    if basis == "rotated":
        return r.half()
    v = r.double() @ spec["v_rot"].double()
    return v.half()


def _ref_pair(qs, k, v):
    """qs (R, D) f32 scaled queries; k (T, D); v (T, D) -> (R, D) f64 softmax."""
    s = qs.double() @ k.double().T
    w = torch.softmax(s, dim=-1)
    return w @ v.double()


def _check(got, want, tag, per_element=True):
    err = (got.double() - want).abs()
    mref = want.abs().max()
    rel_max = float(err.max() / mref)
    rel_l2 = float(err.norm() / want.norm())
    bound = REL_ELEM * want.abs() + ATOL_FRAC * mref
    worst = float((err / bound).max())
    print(f"{tag}: max-rel {rel_max:.2e} l2-rel {rel_l2:.2e} elem/bound {worst:.3f}")
    assert rel_max < REL_MAX, (tag, rel_max)
    assert rel_l2 < REL_L2, (tag, rel_l2)
    if per_element:
        assert worst <= 1.0, (tag, worst)


def _scaled(q, scale):
    return (q.float() * float(np.float16(scale))).half().float()


def _decode_f32(q, cache, scale, spec=None, part_out=None):
    from sunshape_mlx_b200.attention import _run_decode

    codec = cache.codec
    spec = spec or cache.attention_spec()
    out = None if part_out is not None else torch.empty(q.shape, dtype=torch.float32, device=q.device)
    n_heavy = codec.n_heavy_blocks if spec.get("kheavy") is not None else 0
    _run_decode(q, centroids=codec.centroids, perm=codec.permutation, scale=scale, spec=spec,
                causal=False, out=out, heavy=codec.heavy_u8, n_heavy=n_heavy, part_out=part_out)
    return out


def test_cfg3_full_shape_parity(ss):
    import bench

    dev = torch.device("cuda", 0)
    codec, cache, q = bench._build_cfg3(dev)
    c = bench.CFG3
    assert cache.offset == c["T"] and tuple(q.shape) == (c["B"], c["HQ"], 1, 128)
    scale = 1 / math.sqrt(128)
    out32 = _decode_f32(q, cache, scale)
    out16 = ss.sunshape_sdpa(q, cache, scale)       # the product path, fp16 out
    spec = cache.attention_spec()
    rep = c["HQ"] // c["HKV"]
    qs = _scaled(q, scale)
    for b, h in [(0, 0), (17, 3), (40, 5), (c["B"] - 1, c["HKV"] - 1)]:
        k = _keys_pair(codec, spec, b, h, c["T"])
        got = out32[b, h * rep:(h + 1) * rep, 0]
        qp = qs[b, h * rep:(h + 1) * rep, 0]
        # the kernel's arithmetic, element by element: same fp16 values (in
        # the rotated basis), float64 softmax, output rotated back
        vr = _tq_values_pair(spec, b, h, c["T"], basis="rotated")
        want_r = _ref_pair(qp, k, vr) @ spec["v_rot"].double()
        _check(got, want_r, f"cfg3 pair ({b},{h}) f32, rotated-basis values")
        # against the reference's own rounding of the values (fp16 after the
        # inverse rotation): the two roundings differ by half an fp16 ulp per
        # value, so this comparison is held to the norm-wise bounds
        v = _tq_values_pair(spec, b, h, c["T"])
        want = _ref_pair(qp, k, v)
        _check(got, want, f"cfg3 pair ({b},{h}) f32, reference rounding", per_element=False)
        e16 = float((out16[b, h * rep:(h + 1) * rep, 0].double() - want).abs().max())
        assert e16 < 2e-3 * float(want.abs().max()) + 1e-3, e16
    assert torch.isfinite(out16).all()


@pytest.fixture(scope="module")
def cfg5(ss):
    import bench

    dev = torch.device("cuda", 0)
    codec, cache, q = bench._build_cfg5(dev, 0, 1)
    assert cache.offset == bench.CFG5["T"] and codec.n_heavy_blocks == 4
    yield codec, cache, q
    del cache
    torch.cuda.empty_cache()


def test_cfg5_full_shape_parity(ss, cfg5):
    import bench

    codec, cache, q = cfg5
    c = bench.CFG5
    scale = 1 / math.sqrt(128)
    out32 = _decode_f32(q, cache, scale)
    spec = cache.attention_spec()
    rep = c["HQ"] // c["HKV"]
    qs = _scaled(q, scale)
    for h in range(c["HKV"]):
        k = _keys_pair(codec, spec, 0, h, c["T"])
        v = spec["v"][0, h, :c["T"]]
        want = _ref_pair(qs[0, h * rep:(h + 1) * rep, 0], k, v)
        _check(out32[0, h * rep:(h + 1) * rep, 0], want, f"cfg5 kv-head {h} f32")


@pytest.mark.parametrize("n_shards", [2, 4, 8])
def test_cfg5_split_partials_merge(ss, cfg5, n_shards):
    """The split-KV step of the multi-GPU long-context decode on one GPU:
    each shard's (o, m, l) rows from ss_decode_attn_partial over its token
    range (views into the one cache), merged by ss_lse_merge, equal the
    unsplit decode."""
    from sunshape_mlx_b200 import splitkv

    codec, cache, q = cfg5
    T = cache.offset
    scale = 1 / math.sqrt(128)
    base = cache.attention_spec()
    parts = []
    for r in range(n_shards):
        lo, hi = splitkv.shard_range(T, r, n_shards)
        assert lo % 128 == 0
        spec = dict(base)
        spec["tc"] = hi - lo
        for key in ("idx", "v", "kheavy"):
            spec[key] = base[key][:, :, lo:]
        part = torch.empty((q.shape[1], 130), dtype=torch.float32, device=q.device)
        _decode_f32(q, cache, scale, spec=spec, part_out=part)
        parts.append(part)
    merged = splitkv.merge_partials(torch.stack(parts), q.shape, torch.float32)
    full = _decode_f32(q, cache, scale)
    err = float((merged - full).abs().max() / full.abs().max())
    print(f"cfg5 split x{n_shards}: max-rel vs unsplit {err:.2e}")
    assert err < REL_MAX
