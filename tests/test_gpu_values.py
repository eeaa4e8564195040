"""GPU parity of the value codecs and bit packing."""

import numpy as np
import pytest
import torch

import oracle as O
from conftest import golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ss(cuda_ok):
    import sunshape_mlx_b200 as ss

    return ss


def _u32(t):
    return t.cpu().numpy().view(np.uint32)


def test_pack_unpack_golden(ss):
    g = golden("packing")
    for bits in (2, 3, 4):
        idx = g[f"idx{bits}"]
        p = ss.pack_indices(idx, bits)
        np.testing.assert_array_equal(_u32(p), g[f"packed{bits}"])
        np.testing.assert_array_equal(ss.unpack_indices(p, idx.shape[1], bits).cpu().numpy(), idx)
    p = ss.pack_indices(g["idx3_d27"], 3)
    np.testing.assert_array_equal(_u32(p), g["packed3_d27"])
    full = np.full((1, 30), 7, np.uint8)
    p = ss.pack_indices(full, 3)
    assert int(_u32(p)[0, 0]) >> 30 == 0
    with pytest.raises(ValueError):
        ss.pack_indices(np.zeros((1, 30), np.uint8), 2)


def test_grouped_values_golden(ss):
    g = golden("grouped_values")
    for bits in (2, 4):
        p, s, z, n = ss.quantize_values(g["values"], bits=bits, group_size=64)
        np.testing.assert_array_equal(_u32(p), g[f"packed{bits}"])
        np.testing.assert_array_equal(s.cpu().numpy(), g[f"scales{bits}"])
        np.testing.assert_array_equal(z.cpu().numpy(), g[f"zeros{bits}"])
        d = ss.dequantize_values(p, s, z, D=128, bits=bits, group_size=64)
        np.testing.assert_array_equal(d.cpu().numpy(), g[f"deq{bits}"])


@pytest.mark.parametrize("bits,gs", [(2, 16), (3, 32), (4, 128)])
def test_grouped_values_vs_oracle(ss, bits, gs):
    rng = np.random.default_rng(bits)
    v = (rng.standard_normal((257, 128)) * 3).astype(np.float16)
    v[5, :gs] = 1.5  # constant group -> scale floor 1e-8
    p, s, z, _ = ss.quantize_values(torch.tensor(v, device="cuda"), bits=bits, group_size=gs)
    po, so, zo, _ = O.quantize_values(v.astype(np.float32), bits, gs)
    np.testing.assert_array_equal(_u32(p), po)
    np.testing.assert_array_equal(s.cpu().numpy(), so)
    np.testing.assert_array_equal(z.cpu().numpy(), zo)


def _near_boundary_only(r, bnd, got, want, tol=1e-5):
    bad = np.argwhere(got != want)
    for i, j in bad:
        assert np.min(np.abs(r[i, j] - bnd)) < tol, (i, j, r[i, j])
    return len(bad)


def test_turboquant_values_golden(ss):
    g = golden("turboquant_values")
    for bits in (2, 3, 4):
        codec = ss.TurboQuantValueCodec(head_dim=128, bits=bits, rotation=g[f"rotation{bits}"])
        p, n = codec.quantize(g["values"])
        np.testing.assert_allclose(n.cpu().numpy(), g[f"norms{bits}"], rtol=1e-6)
        got = O.unpack_indices(_u32(p), 128, bits)
        want = O.unpack_indices(g[f"packed{bits}"], 128, bits)
        v = g["values"]
        unit = v / np.maximum(np.linalg.norm(v, axis=1, keepdims=True), 1e-8)
        r = unit @ g[f"rotation{bits}"].T
        _, bnd = O.tq_tables(128, bits)
        assert _near_boundary_only(r, bnd, got, want) <= 3
        d = codec.dequantize(p, n).cpu().numpy()
        np.testing.assert_allclose(d, O.tq_dequantize(_u32(p), n.cpu().numpy(), g[f"rotation{bits}"], bits, 128),
                                   atol=1e-5)


def test_turboquant_group_extension_vs_oracle(ss):
    rng = np.random.default_rng(43)
    rot = O.rotation_matrix_np(128, 43)
    v = rng.standard_normal((300, 128)).astype(np.float16)
    codec = ss.TurboQuantValueCodec(head_dim=128, bits=2, rotation=rot, group_size=32)
    p, s = codec.quantize(torch.tensor(v, device="cuda"))
    po, so = O.tq_group_quantize(v.astype(np.float32), rot, 2, 32)
    np.testing.assert_allclose(s.cpu().numpy().astype(np.float32), so.astype(np.float32), rtol=1e-3)
    got = O.unpack_indices(_u32(p), 128, 2)
    want = O.unpack_indices(po, 128, 2)
    assert (got != want).mean() < 1e-3
    d = codec.dequantize(p, s).cpu().numpy()
    ref = O.tq_group_dequantize(_u32(p), s.cpu().numpy(), rot, 2, 128, 32)
    np.testing.assert_allclose(d, ref, atol=1e-4)


def test_scalar_quantize_golden(ss):
    g = golden("scalar_quantize")
    out, backend = ss.kernels.quantize_scalar_to_indices(g["values"], g["boundaries"])
    np.testing.assert_array_equal(out.cpu().numpy(), g["indices"])
    assert backend == "cuda"
