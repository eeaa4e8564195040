"""Device-side give-ups are reported, and the library keeps working after one.

Every wait of the decode kernel (ss_decode_attn) and of the tensor-core
assignment kernel is bounded; a wait that runs out makes the launch give up
and report through the workspace error word and the process error sink. The
reference has no such path: its wrappers return None on any exception and
the caller falls back (kernels.py:99-116). Here the failure is produced
without any GPU fault: the wait bound is set to 1 ms and a test hook makes
the producer (decode) or the loader (assignment) skip one tile's copies, so
the consumers' waits on that tile run out. Then:
  * the product API raises SunShapeCudaError with SS_ERR_TIMEOUT,
  * the next normal call succeeds and matches the reference.
"""

import math

import numpy as np
import pytest
import torch

import gpu_ref as G

pytestmark = pytest.mark.gpu
WAIT_NS = 1_000_000  # 1 ms


@pytest.fixture(scope="module")
def ss(cuda_ok):
    import sunshape_mlx_b200 as ss

    return ss


def _cache(ss, seed=3, T=3000):
    rng = np.random.default_rng(seed)
    kc = rng.standard_normal((2048, 128)).astype(np.float32)
    qc = rng.standard_normal((1024, 128)).astype(np.float32)
    codec = ss.SunShapeBlockCodec(head_dim=128)
    codec.fit(qc, kc, kmeans_iters=2, seed=0)
    cache = ss.create_kv_cache(codec, n_kv_heads=4)
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = torch.randn((2, 4, T, 128), generator=g, device="cuda").half()
    v = torch.randn((2, 4, T, 128), generator=g, device="cuda").half()
    cache.append(k, v)
    q = torch.randn((2, 16, 1, 128), generator=g, device="cuda").half()
    return codec, cache, q, k, v


def _want(codec, cache, q, v):
    k = cache.keys  # dequantised keys (ss_vq_dequant, pinned bit-exact elsewhere)
    return G.attention(G.scaled_queries(q, 1 / math.sqrt(128)), k, v.float())


def test_decode_wait_timeout_is_reported_then_recovers(ss):
    from sunshape_mlx_b200 import _lib as L
    from sunshape_mlx_b200.attention import PreparedDecode

    L.check_device_errors()  # nothing pending from earlier tests
    codec, cache, q, _, v = _cache(ss)
    scale = 1 / math.sqrt(128)
    bad = PreparedDecode(q, cache, scale, wait_limit_ns=WAIT_NS, _test_skip_tile=0)
    with pytest.raises(L.SunShapeCudaError) as ei:
        bad.run(check=True)
    assert ei.value.code == L.SS_ERR_TIMEOUT
    # the workspace word carries the same report (and is cleared by reading it)
    rc = L.load().ss_decode_check(L.ptr(bad.ws), L.stream_ptr())
    assert rc == L.SS_ERR_TIMEOUT
    assert L.load().ss_decode_check(L.ptr(bad.ws), L.stream_ptr()) == L.SS_OK
    # a following normal call through the public API succeeds and is correct
    out = ss.sunshape_sdpa(q, cache, scale, check=True)
    want = _want(codec, cache, q, v)
    assert G.rel_err(out, want) < 2e-3
    good = PreparedDecode(q, cache, scale, wait_limit_ns=WAIT_NS)
    assert G.rel_err(good.run(check=True), want) < 2e-3


def test_decode_give_up_raises_on_the_next_call(ss):
    """Without check=True the launch returns at once; the give-up is seen by
    the next call of the product API (no synchronization needed for that)."""
    from sunshape_mlx_b200 import _lib as L
    from sunshape_mlx_b200.attention import PreparedDecode

    codec, cache, q, _, v = _cache(ss, seed=4, T=1500)
    scale = 1 / math.sqrt(128)
    PreparedDecode(q, cache, scale, wait_limit_ns=WAIT_NS, _test_skip_tile=2).run()
    torch.cuda.synchronize()
    with pytest.raises(L.SunShapeCudaError) as ei:
        ss.sunshape_sdpa(q, cache, scale)
    assert ei.value.code == L.SS_ERR_TIMEOUT and "decode" in str(ei.value)
    for ws in __import__("sunshape_mlx_b200.attention", fromlist=["_WS"])._WS.values():
        L.load().ss_decode_check(L.ptr(ws), L.stream_ptr())
    out = ss.sunshape_sdpa(q, cache, scale, check=True)
    assert G.rel_err(out, _want(codec, cache, q, v)) < 2e-3


def test_assign_wait_timeout_is_reported_then_recovers(ss):
    from sunshape_mlx_b200 import _lib as L
    from sunshape_mlx_b200 import kernels as K

    rng = np.random.default_rng(9)
    cents = torch.tensor(rng.standard_normal((16, 256, 8)), dtype=torch.float32, device="cuda")
    keys = torch.randn((32768, 128), device="cuda").half()
    lib = L.load()
    K.set_assign_path("tensor")
    try:
        lib.ss_set_assign_wait(WAIT_NS, 1)  # the loader never stages tile 0
        try:
            K.vq_assign(keys, cents)
            with pytest.raises(L.SunShapeCudaError) as ei:
                L.check_device_errors()
            assert ei.value.code == L.SS_ERR_TIMEOUT and "assignment" in str(ei.value)
            with pytest.raises(L.SunShapeCudaError):
                K.assign_check()  # the kernel's own sticky status says the same
        finally:
            lib.ss_set_assign_wait(0, 0)
        got = K.vq_assign(keys, cents)
        K.assign_check()
        L.check_device_errors()
    finally:
        K.set_assign_path("simt")
    want = K.vq_assign(keys, cents)
    K.set_assign_path("auto")
    assert torch.equal(got, want)
