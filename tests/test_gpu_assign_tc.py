"""GPU parity of the tensor-core (tcgen05) nearest-centroid assignment.

The tensor-core kernel screens distances as a GEMM and re-scores near ties
exactly, so its indices must equal, bit for bit, both the CUDA-core kernel
and the oracle (the reference's NumPy quantize, codec.py:472-514), including
on inputs built to be full of exact ties, keys too large for fp16, NaN keys,
heavy (pass-through) blocks and strided cache layouts."""

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K(cuda_ok):
    from sunshape_mlx_b200 import kernels as K

    yield K
    K.set_assign_path("auto")


def _run(K, path, keys, cents, **kw):
    K.set_assign_path(path)
    try:
        out = K.vq_assign(keys, cents, **kw)
        K.assign_check(keys.device)
        return out
    finally:
        K.set_assign_path("auto")


def _state(cents, perm=None, heavy=None):
    nb, k, bd = cents.shape
    d = nb * bd
    return {"mode": "profileperm_mixed_precision" if heavy is not None else "profileperm_baseline",
            "head_dim": d, "block_dim": bd, "n_blocks": nb, "n_centroids": k, "centroids": cents,
            "permutation": np.arange(d) if perm is None else perm,
            "heavy": np.zeros(nb, bool) if heavy is None else heavy}


@pytest.mark.parametrize("bd,k,n,dt", [
    (8, 256, 4096, torch.float16), (8, 256, 1000, torch.float32), (8, 256, 777, torch.bfloat16),
    (4, 256, 1300, torch.float16), (16, 256, 600, torch.float32), (8, 64, 640, torch.float16),
    (8, 128, 513, torch.float32), (4, 64, 900, torch.float16), (8, 192, 300, torch.float32)])
def test_tensor_path_bit_exact(K, bd, k, n, dt):
    rng = np.random.default_rng(bd * 7919 + k * 31 + n)
    d = 128
    sig = np.exp(rng.normal(0, 0.5, d)).astype(np.float32)
    keys = (rng.standard_normal((n, d)) * sig).astype(np.float32)
    kt = torch.tensor(keys, device="cuda").to(dt)
    cents = (rng.standard_normal((d // bd, k, bd)) * 0.8).astype(np.float32)
    ct = torch.tensor(cents, device="cuda")
    got = _run(K, "tensor", kt, ct).cpu().numpy()
    ref = _run(K, "simt", kt, ct).cpu().numpy()
    np.testing.assert_array_equal(got, ref)
    want, _ = O.quantize(_state(cents), kt.float().cpu().numpy())
    np.testing.assert_array_equal(got, want)


def test_exact_ties_and_duplicates(K):
    """Duplicate centroids and keys equal to centroids give exact distance
    ties; the lowest index must win, as np.argmin does."""
    rng = np.random.default_rng(11)
    nb, k, bd, n = 16, 256, 8, 2048
    cents = rng.standard_normal((nb, k, bd)).astype(np.float16).astype(np.float32)
    cents[:, 200:] = cents[:, 100:156]           # exact duplicates, higher index
    cents[:, 7] = cents[:, 3]
    pick = rng.integers(0, k, (n, nb))
    keys = np.stack([cents[b, pick[:, b]] for b in range(nb)], 1).reshape(n, nb * bd)
    keys[::3] += (rng.standard_normal((len(keys[::3]), nb * bd)) * 1e-3).astype(np.float32)
    kt = torch.tensor(keys, device="cuda", dtype=torch.float16)
    ct = torch.tensor(cents, device="cuda")
    got = _run(K, "tensor", kt, ct).cpu().numpy()
    want, _ = O.quantize(_state(cents), kt.float().cpu().numpy())
    np.testing.assert_array_equal(got, want)
    assert (got < 200).all()  # duplicates resolve to the first copy


def test_scale_extremes_overflow_and_nan(K):
    """Centroids far from 1 (per-block power-of-two scaling), keys beyond the
    fp16 range after scaling, and NaN keys all take the exact path."""
    rng = np.random.default_rng(12)
    nb, k, bd, n = 16, 256, 8, 1024
    cents = rng.standard_normal((nb, k, bd)).astype(np.float32)
    cents[0] *= 1e-6
    cents[1] *= 3e4
    cents[2] *= 1e-30
    keys = rng.standard_normal((n, nb * bd)).astype(np.float32)
    keys[:, 0:8] *= 1e-6
    keys[:, 8:16] *= 3e4
    keys[:, 16:24] *= 1e-30
    keys[5, 40:48] = 1e9                        # does not fit fp16 after scaling
    keys[6, 50] = np.nan
    keys[7, 60] = np.inf
    kt = torch.tensor(keys, device="cuda")
    ct = torch.tensor(cents, device="cuda")
    got = _run(K, "tensor", kt, ct).cpu().numpy()
    ref = _run(K, "simt", kt, ct).cpu().numpy()
    np.testing.assert_array_equal(got, ref)
    ok = np.ones(n, bool)
    ok[[6, 7]] = False                           # NaN/inf rows: compare with the CUDA-core kernel only
    want, _ = O.quantize(_state(cents), keys[ok])
    np.testing.assert_array_equal(got[ok], want)


def test_expanded_mode_matches_cuda_core_kernel(K):
    """dist_mode 1 (k-means assignment, codec.py:88-91): same exact formula in
    both kernels, so indices agree bit for bit."""
    rng = np.random.default_rng(13)
    for bd, dt in ((8, torch.float32), (4, torch.float32), (16, torch.float16)):
        x = rng.standard_normal((4096, 128)).astype(np.float32)
        c = np.stack([x[rng.permutation(4096)[:256], b * bd:(b + 1) * bd] for b in range(128 // bd)])
        xt = torch.tensor(x, device="cuda").to(dt)
        ct = torch.tensor(c, device="cuda")
        got = _run(K, "tensor", xt, ct, dist_mode=1).cpu().numpy()
        ref = _run(K, "simt", xt, ct, dist_mode=1).cpu().numpy()
        np.testing.assert_array_equal(got, ref)


def test_permutation_heavy_blocks_and_strided_cache(K):
    rng = np.random.default_rng(14)
    B, H, T, D, cap = 2, 4, 300, 128, 512
    keys = torch.tensor(rng.standard_normal((B, H, T, D)) * 2, dtype=torch.float16, device="cuda")
    cents = torch.tensor(rng.standard_normal((16, 256, 8)), dtype=torch.float32, device="cuda")
    perm = torch.tensor(rng.permutation(D), dtype=torch.int32, device="cuda")
    heavy = np.zeros(16, bool)
    heavy[[1, 6, 11, 15]] = True
    ht = torch.tensor(heavy.astype(np.uint8), device="cuda")
    outs = {}
    for path in ("tensor", "simt"):
        store = torch.full((B, H, cap, 16), 255, dtype=torch.uint8, device="cuda")
        hv = torch.zeros((B, H, cap, 32), dtype=torch.float16, device="cuda")
        pt = torch.zeros((B * H * T, 16, 8), dtype=torch.float32, device="cuda")
        K.set_assign_path(path)
        try:
            K.vq_assign(keys.reshape(B * H, T, D), cents, perm=perm, heavy=ht,
                        out_idx=store[:, :, 7:7 + T].reshape(B * H, T, 16),
                        out_heavy=hv[:, :, 7:7 + T].reshape(B * H, T, 32), out_pt=pt)
            K.assign_check()
        finally:
            K.set_assign_path("auto")
        outs[path] = (store.cpu().numpy(), hv.cpu().numpy(), pt.cpu().numpy())
    for a, b in zip(outs["tensor"], outs["simt"]):
        np.testing.assert_array_equal(a, b)
    store = outs["tensor"][0]
    assert (store[:, :, :7] == 255).all() and (store[:, :, 7 + T:] == 255).all()
    st = _state(cents.cpu().numpy(), perm.cpu().numpy(), heavy)
    kn = keys.float().cpu().numpy()
    for b in range(B):
        for h in range(H):
            want, ptv = O.quantize(st, kn[b, h])
            np.testing.assert_array_equal(store[b, h, 7:7 + T], want)


def test_cache_fill_scale_agrees_with_cuda_core_kernel(K):
    """Config-2 shape cache fill (16 x 8 x 8192 fp16 keys): tensor == CUDA-core."""
    g = torch.Generator(device="cuda").manual_seed(21)
    sig = torch.exp(torch.randn(128, device="cuda", generator=g) * 0.5)
    keys = (torch.randn(16 * 8, 8192, 128, device="cuda", generator=g) * sig).half()
    cents = torch.randn(16, 256, 8, device="cuda", generator=g) * 0.9
    perm = torch.randperm(128, device="cuda", generator=g).int()
    a = _run(K, "tensor", keys, cents, perm=perm)
    b = _run(K, "simt", keys, cents, perm=perm)
    assert torch.equal(a, b)


def test_auto_path_small_and_unsupported_shapes(K):
    """Auto uses the CUDA-core kernel for tiny or unsupported shapes; forcing
    the tensor path on an unsupported shape raises."""
    rng = np.random.default_rng(15)
    cents = torch.tensor(rng.standard_normal((64, 16, 2)), dtype=torch.float32, device="cuda")
    keys = torch.tensor(rng.standard_normal((700, 128)), dtype=torch.float32, device="cuda")
    a = K.vq_assign(keys, cents)
    want, _ = O.quantize(_state(cents.cpu().numpy()), keys.cpu().numpy())
    np.testing.assert_array_equal(a.cpu().numpy(), want)
    K.set_assign_path("tensor")
    try:
        with pytest.raises(RuntimeError):
            K.vq_assign(keys, cents)
    finally:
        K.set_assign_path("auto")
