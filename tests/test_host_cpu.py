"""Host-side logic of the package checked on CPU against the oracle:
ProfilePerm, kurtosis masks, permutation helpers, WHT; plus the split-KV
merge orchestration over a 2-rank gloo group."""

import os

import numpy as np
import pytest
import torch

import inputs as I
import oracle as O
from sunshape_mlx_b200 import rotation as R


def test_profileperm_matches_oracle():
    q, _ = I.gaussian_qk(42, 1024, 2048, 128)
    np.testing.assert_array_equal(R.covariance_block_permutation(torch.tensor(q), 8).numpy(),
                                  O.covariance_block_permutation(q, 8))
    q64, _ = I.small_codec_inputs()
    np.testing.assert_array_equal(R.covariance_block_permutation(q64, 8).numpy(),
                                  O.covariance_block_permutation(q64, 8))


def test_permutation_helpers():
    q, _ = I.small_codec_inputs()
    p = R.covariance_block_permutation(q, 8)
    inv = R.invert_permutation(p)
    np.testing.assert_array_equal(p.numpy()[inv.numpy()], np.arange(64))
    x = torch.tensor(q)
    np.testing.assert_array_equal(R.apply_permutation(R.apply_permutation(x, p), inv).numpy(), q)


def test_mixed_mask_matches_oracle():
    qm = I.heavy_tailed_queries(512, 64, seed=5)
    h, mass = R.mixed_precision_block_mask(torch.tensor(qm), 8)
    ho, mo = O.mixed_precision_block_mask(qm, 8)
    np.testing.assert_array_equal(h.numpy(), ho)
    np.testing.assert_allclose(mass.numpy(), mo, rtol=1e-5)
    h4, _ = R.mixed_precision_block_mask(torch.tensor(qm), 8, n_heavy=4)
    np.testing.assert_array_equal(h4.numpy(), O.heaviest_blocks_mask(qm, 8, 4))
    assert int(h4.sum()) == 4


def test_rotation_is_orthogonal_and_matches_oracle():
    r = R.generate_rotation_matrix(64, seed=0)
    np.testing.assert_allclose((r @ r.T).numpy(), np.eye(64), atol=1e-5)
    np.testing.assert_array_equal(r.numpy(), O.rotation_matrix_np(64, 0))


def test_wht_roundtrip_and_norm():
    s = R.generate_wht_signs(64, seed=42)
    assert set(np.unique(s)) <= {-1.0, 1.0}
    x = torch.randn(16, 64)
    y = R.apply_wht(x, s)
    np.testing.assert_allclose(R.apply_wht(y, s, inverse=True).numpy(), x.numpy(), atol=1e-4)
    np.testing.assert_allclose(y.norm(dim=1).numpy(), x.norm(dim=1).numpy(), atol=1e-4)
    with pytest.raises(ValueError, match="power of 2"):
        R.generate_wht_signs(48)


def test_safe_normalize():
    xn, n = R.safe_normalize([[3.0, 4.0], [0.0, 0.0]])
    assert abs(float(xn[0].norm()) - 1) < 1e-6 and not torch.isnan(xn).any()


def _gloo_worker(rank, world, port, q):
    import torch.distributed as dist
    from sunshape_mlx_b200 import splitkv

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(0)
    st = {"n_blocks": 16, "block_dim": 8,
          "centroids": rng.standard_normal((16, 256, 8)).astype(np.float32)}
    idx = rng.integers(0, 256, (1000, 16)).astype(np.uint8)
    v = rng.standard_normal((1000, 128)).astype(np.float32)
    qq = (rng.standard_normal((4, 128)) * 0.1).astype(np.float32)
    lo, hi = splitkv.shard_range(1000, rank, world)
    m, l_, o = O.decode_attention_fp(qq, st, idx[lo:hi], v[lo:hi])
    part = torch.tensor(np.concatenate([o, m[:, None], l_[:, None]], axis=1))
    gathered = splitkv.all_gather_partials(part)
    got = O.lse_merge(gathered[:, :, 128].numpy(), gathered[:, :, 129].numpy(),
                      gathered[:, :, :128].numpy())
    m0, l0, o0 = O.decode_attention_fp(qq, st, idx, v)
    q.put((rank, float(np.abs(got - o0 / l0[:, None]).max())))
    dist.destroy_process_group()


def test_splitkv_gather_two_ranks_gloo():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=60) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, err in res:
        assert err < 1e-5


def test_shard_range_covers_everything():
    from sunshape_mlx_b200 import splitkv

    for n, w in [(1000, 3), (524288, 8), (7, 8), (0, 2)]:
        spans = [splitkv.shard_range(n, r, w) for r in range(w)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


def test_decode_schedule_partition():
    """The decode kernel's static schedule (csrc/decode_attn.cu: make_sched,
    range_start, cta_of): ranges tile the (unit, tile) sequence in order,
    every tile maps to the CTA whose range holds it, and no empty range sits
    inside a unit (the cross-CTA merge counts every CTA of a unit)."""
    import random
    def make(total, tpu, w, grid): return (total, tpu, w, total + w * (total // tpu - 1), grid)
    def start(s, k):
        total, tpu, w, cost, grid = s
        if k >= grid: return total
        y = k * cost; pg = (tpu + w) * grid; j = y // pg; x = (y - j * pg + grid - 1) // grid
        t = j * tpu + x if x < tpu else (j + 1) * tpu
        return min(t, total)
    def cta_of(s, t):
        total, tpu, w, cost, grid = s
        return (t + w * (t // tpu)) * grid // cost

    rng = random.Random(1)
    for _ in range(1500):
        tpu = rng.choice([1, 2, 3, 7, 64, 65, 256, 4096])
        nu = rng.randint(1, 200)
        total = tpu * nu
        grid = rng.randint(1, min(148, total))
        w = 0 if nu == 1 else rng.choice([0, 1, 8, 20])
        s = make(total, tpu, w, grid)
        st = [start(s, k) for k in range(grid + 1)]
        assert st[0] == 0 and st[-1] == total and all(a <= b for a, b in zip(st, st[1:]))
        for t in range(0, total, max(1, total // 200)):
            k = cta_of(s, t)
            assert st[k] <= t < st[k + 1]
        for u in range(nu):
            f, l = cta_of(s, u * tpu), cta_of(s, (u + 1) * tpu - 1)
            assert all(st[k + 1] > st[k] for k in range(f, l + 1))


def test_deferred_tensor_computes_once_on_first_use():
    """update_and_fetch's deferred keys: shape/dtype without computing; any
    use computes once; torch functions and operators see the real tensor."""
    import torch

    from sunshape_mlx_b200.cache import DeferredTensor

    calls = []

    def fn():
        calls.append(1)
        return torch.arange(6, dtype=torch.float32).reshape(1, 1, 2, 3)

    d = DeferredTensor(fn, (1, 1, 2, 3), torch.float32, torch.device("cpu"))
    assert d.shape == (1, 1, 2, 3) and d.dtype == torch.float32 and d.ndim == 4
    assert d.size(2) == 2 and not d.is_materialized and not calls
    assert float((d * 2).sum()) == 30.0
    assert torch.equal(torch.cat([d, d], 2)[0, 0, 2], torch.tensor([0.0, 1.0, 2.0]))
    assert float(d[0, 0, 1, 2]) == 5.0 and d.float().shape == (1, 1, 2, 3)
    assert d.is_materialized and len(calls) == 1
