"""C-ABI checks that need no GPU: the library builds/loads, exports every
entry point the header declares, the ctypes struct mirrors the C layout, and
argument validation rejects bad calls before touching a device."""

import ctypes as C
import os
import re
import subprocess
import tempfile

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "sunshape_b200.h")


def _declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|void|const char\*)\s+(ss_\w+)\(", src, re.M)))


@pytest.fixture(scope="module")
def lib():
    from sunshape_mlx_b200 import build, _lib as L

    build.build()
    return L.load()


def test_library_exports_every_declared_symbol(lib):
    from sunshape_mlx_b200 import _lib as L

    names = _declared()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(L.EXPORTED), set(names) ^ set(L.EXPORTED)
    nm = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True, text=True).stdout
    for n in names:
        assert re.search(rf"\bT {n}\b", nm), n


def test_abi_version(lib):
    assert lib.ss_abi_version() == 101


def test_decode_args_layout_matches_header():
    from sunshape_mlx_b200 import _lib as L

    fields = ["q", "scale", "centroids", "n_heavy", "tc", "vfmt", "v_levels", "v_rot", "ttail",
              "causal", "mask_mode", "out", "workspace", "max_ctas", "wait_limit_ns",
              "test_skip_tile", "app_keys", "app_dtype", "app_value_row_stride", "app_rows"]
    prog = "#include <cstdio>\n#include <cstddef>\n#include \"%s\"\nint main(){printf(\"%%zu\", sizeof(ss_decode_args));%s}\n" % (
        HEADER, "".join(f'printf(" %zu", offsetof(ss_decode_args, {f}));' for f in fields))
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "l.cpp"), os.path.join(d, "l")
        open(src, "w").write(prog)
        subprocess.run(["g++", src, "-o", exe], check=True)
        got = [int(x) for x in subprocess.run([exe], capture_output=True, text=True).stdout.split()]
    want = [C.sizeof(L.DecodeArgs)] + [getattr(L.DecodeArgs, f).offset for f in fields]
    assert got == want


def test_bad_arguments_are_rejected_without_a_device(lib):
    from sunshape_mlx_b200 import _lib as L

    rc = lib.ss_vq_assign(None, 0, 1, 1, 0, 0, 128, None, None, 8, 256, None, None, 0, 0, None, 0,
                          0, None, 0, None)
    assert rc == 1
    assert "null" in L.last_error()
    rc = lib.ss_kmeans_update(None, 10, 16, 8, None, None, None, 256, None)
    assert rc == 1
    rc = lib.ss_pack_indices(C.c_void_p(16), 1, 30, 5, C.c_void_p(16), None)
    assert rc == 1 and "bits" in L.last_error()
    a = L.DecodeArgs()
    a.d = 96  # unsupported head_dim
    a.hq = a.hkv = 1
    assert lib.ss_decode_attn(C.byref(a), None) == 1
    assert "head_dim" in L.last_error()
    assert lib.ss_lse_merge(None, 2, 4, 128, None, None, 0, 128, None) == 1


def test_workspace_size_is_positive(lib):
    from sunshape_mlx_b200 import _lib as L

    a = L.DecodeArgs()
    a.b, a.hq, a.hkv, a.tq, a.d, a.bd, a.k, a.tc = 16, 32, 8, 1, 128, 8, 256, 8192
    n = lib.ss_decode_workspace_size(C.byref(a))
    assert n > 0


def test_kernel_stats_roundtrip(lib):
    from sunshape_mlx_b200 import _lib as L

    L.reset_kernel_stats()
    assert L.kernel_stats() == {}
