"""ss_decode_attn_noalloc: decode attention for callers that cannot allocate
device memory (allocator-less runtimes, code confined to another framework's
memory pool). It keeps its scratch in a fixed device array inside the library
instead of a caller workspace. Checked through the C ABI against the regular
ss_decode_attn on the same inputs, on two calls in a row (the second call
reuses the array the first one left behind). Collected last on purpose."""

import ctypes as C
import math

import pytest
import torch

pytestmark = pytest.mark.gpu
REL = 1e-3


def _rel(a, b):
    return float((a.float() - b.float()).abs().max() / b.float().abs().max())


def test_noalloc_matches_workspace_entry_point(cuda_ok):
    from sunshape_mlx_b200 import _lib as L
    from sunshape_mlx_b200.attention import _fill_args, workspace_for

    g = torch.Generator(device="cuda").manual_seed(5)
    B, HKV, HQ, T, D, NB, K = 2, 4, 16, 3000, 128, 16, 256
    cap = 3072
    cents = torch.randn((NB, K, 8), generator=g, device="cuda") * 0.7
    perm = torch.randperm(D, generator=g, device="cuda").to(torch.int32)
    idx = torch.randint(0, K, (B, HKV, cap, NB), generator=g, device="cuda", dtype=torch.uint8)
    v = torch.randn((B, HKV, cap, D), generator=g, device="cuda").half()
    lib = L.load()
    st = L.stream_ptr()
    L.reset_kernel_stats()
    for step in range(2):
        q = torch.randn((B, HQ, 1, D), generator=g, device="cuda").half()
        spec = dict(tc=T - step * 700, cap=cap, idx=idx, v=v)
        ref = torch.empty_like(q)
        a, keep = _fill_args(q, cents, perm, 1 / math.sqrt(D), spec, False, ref)
        ws = workspace_for(q.device, lib.ss_decode_workspace_size(C.byref(a)))
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        L.check("ss_decode_attn", lib.ss_decode_attn(C.byref(a), st))
        out = torch.full_like(q, float("nan"))
        b, keep2 = _fill_args(q, cents, perm, 1 / math.sqrt(D), spec, False, out)
        L.check("ss_decode_attn_noalloc", lib.ss_decode_attn_noalloc(C.byref(b), st))
        torch.cuda.synchronize()
        assert not torch.isnan(out.float()).any()
        assert _rel(out, ref) < REL, (step, _rel(out, ref))
    # no device-side wait gave up in either call (the error word of the fixed
    # array is sticky; this reads and clears it), and the calls are counted
    # under their own name
    assert lib.ss_decode_noalloc_check(st) == L.SS_OK
    stats = L.kernel_stats()
    assert stats.get("ss_decode_attn_noalloc") == 2 and stats.get("ss_decode_attn") == 2


def test_noalloc_rejects_oversized_problem(cuda_ok):
    from sunshape_mlx_b200 import _lib as L

    a = L.DecodeArgs()
    a.b, a.hq, a.hkv, a.tq, a.d, a.bd, a.k, a.tc = 4096, 32, 8, 1, 128, 8, 256, 1 << 20
    rc = L.load().ss_decode_attn_noalloc(C.byref(a), L.stream_ptr())
    assert rc == 5 and "fixed" in L.last_error()
