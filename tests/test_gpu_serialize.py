"""Cache save/load (prompt-cache serialization): a restored cache decodes
bit-identically and keeps appending like the original (the reference only
exposes the raw arrays, cache.py:256-262, 988-998)."""

import math

import numpy as np
import pytest
import torch

import inputs as I

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ss(cuda_ok):
    import sunshape_mlx_b200 as ss

    return ss


@pytest.fixture(scope="module")
def codec(ss):
    q, k = I.small_codec_inputs()
    q = np.concatenate([q, q], 1)[:, :128]
    k = np.concatenate([k, k[::-1]], 1)[:, :128]
    return ss.SunShapeBlockCodec(head_dim=128).fit(q, k, kmeans_iters=3, seed=0)


@pytest.mark.parametrize("kw", [
    dict(), dict(buffer_size=32), dict(value_backend="grouped", value_bits=4, buffer_size=16),
    dict(value_backend="turboquant", value_bits=2, buffer_size=0),
    dict(value_backend="turboquant", value_bits=2, tq_group_size=32, buffer_size=8),
    dict(value_backend="sunshape", value_bits=1, buffer_size=32)])
def test_save_load_roundtrip(ss, codec, tmp_path, kw):
    cache = ss.create_kv_cache(codec, n_kv_heads=2, **kw)
    kk, vv = I.kv_stream(3, 2, 2, 300, 128)
    cache.append(torch.tensor(kk, device="cuda"), torch.tensor(vv, device="cuda"))
    path = tmp_path / "cache.pt"
    ss.save_cache(cache, path)
    back = ss.load_cache(path)
    assert type(back) is type(cache) and back.offset == cache.offset
    q = torch.tensor(I.decode_queries(4, 2, 8, 1, 128), device="cuda")
    a = ss.sunshape_sdpa(q, cache, 1 / math.sqrt(128))
    b = ss.sunshape_sdpa(q, back, 1 / math.sqrt(128))
    assert torch.equal(a, b)
    # both keep decoding the same way after more tokens
    k2, v2 = I.kv_stream(5, 2, 2, 40, 128)
    for c in (cache, back):
        c.append(torch.tensor(k2, device="cuda"), torch.tensor(v2, device="cuda"))
    assert torch.equal(ss.sunshape_sdpa(q, cache, 1 / math.sqrt(128)),
                       ss.sunshape_sdpa(q, back, 1 / math.sqrt(128)))
