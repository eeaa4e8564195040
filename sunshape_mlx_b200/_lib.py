"""ctypes binding of libsunshape_b200.so (the C ABI in include/sunshape_b200.h).

The library is loaded on first use. If it is missing or cannot be loaded the
import fails loudly: there is no CPU fallback anywhere in this package.
Every wrapper here takes torch CUDA tensors, checks them, and forwards raw
pointers plus the current CUDA stream.
"""

from __future__ import annotations

import ctypes as C
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsunshape_b200.so")

SS_OK = 0
SS_ERR_TIMEOUT = 4
STATUS_NAMES = {1: "bad argument", 2: "unsupported", 3: "CUDA error", 4: "timeout",
                5: "workspace"}
SS_F32, SS_F16, SS_BF16 = 0, 1, 2
SS_V_F16, SS_V_QUANT, SS_V_VQ = 0, 1, 2

_DTYPE_CODE = {torch.float32: SS_F32, torch.float16: SS_F16, torch.bfloat16: SS_BF16}


class SunShapeCudaError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed ({STATUS_NAMES.get(code, code)}): {msg}")
        self.code = code


vp = C.c_void_p
i32 = C.c_int
i64 = C.c_int64
f32 = C.c_float


class DecodeArgs(C.Structure):
    """Mirror of ss_decode_args (field order and types must match the header)."""

    _fields_ = [
        ("q", vp), ("q_dtype", i32), ("q_sb", i64), ("q_sh", i64), ("q_st", i64),
        ("b", i32), ("hq", i32), ("hkv", i32), ("tq", i32), ("d", i32),
        ("scale", f32),
        ("perm", vp), ("rot_k", vp), ("centroids", vp),
        ("bd", i32), ("k", i32),
        ("heavy", vp), ("n_heavy", i32),
        ("tc", i64),
        ("idx", vp), ("idx_pair_stride", i64),
        ("kheavy", vp), ("kheavy_pair_stride", i64),
        ("vfmt", i32),
        ("v", vp), ("v_pair_stride", i64),
        ("vq", vp), ("vq_pair_stride", i64),
        ("v_bits", i32), ("v_group", i32),
        ("v_scales", vp), ("v_scale_dtype", i32), ("vs_pair_stride", i64),
        ("v_zeros", vp), ("vz_pair_stride", i64),
        ("v_levels", f32 * 16),
        ("v_rot", vp),
        ("v_idx", vp), ("vi_pair_stride", i64), ("v_cents", vp), ("v_bd", i32), ("v_k", i32),
        ("ttail", i64),
        ("k_tail", vp), ("v_tail", vp), ("tail_pair_stride", i64),
        ("causal", i32),
        ("mask", vp), ("mask_stride", i64),
        ("mask_mode", i32),
        ("out", vp), ("out_dtype", i32), ("o_sb", i64), ("o_sh", i64), ("o_st", i64),
        ("workspace", vp), ("workspace_bytes", C.c_size_t),
        ("max_ctas", i32),
        ("wait_limit_ns", i64), ("test_skip_tile", i64),
        ("app_keys", vp), ("app_values", vp), ("app_dtype", i32),
        ("app_key_pair_stride", i64), ("app_key_row_stride", i64),
        ("app_value_pair_stride", i64), ("app_value_row_stride", i64),
        ("app_rows", i64),
    ]


class AppendArgs(C.Structure):
    """Mirror of ss_append_args."""

    _fields_ = [
        ("keys", vp), ("key_dtype", i32), ("key_group_stride", i64), ("key_row_stride", i64),
        ("values", vp), ("value_dtype", i32), ("value_group_stride", i64),
        ("value_row_stride", i64),
        ("n_groups", i64), ("rows", i64),
        ("d", i32),
        ("perm", vp), ("centroids", vp), ("bd", i32), ("k", i32), ("heavy", vp),
        ("idx", vp), ("idx_group_stride", i64), ("idx_row_stride", i64),
        ("kheavy", vp), ("kheavy_group_stride", i64), ("kheavy_row_stride", i64),
        ("v", vp), ("v_group_stride", i64), ("v_row_stride", i64),
    ]


_SIGS = {
    "ss_abi_version": ([], i32),
    "ss_last_error": ([], C.c_char_p),
    "ss_device_sm_count": ([], i32),
    "ss_kernel_stats": ([C.c_char_p, C.c_size_t], i32),
    "ss_reset_kernel_stats": ([], None),
    "ss_vq_assign": ([vp, i32, i64, i64, i64, i64, i32, vp, vp, i32, i32, vp, vp, i64, i64,
                      vp, i64, i64, vp, i32, vp], i32),
    "ss_kmeans_update": ([vp, i64, i32, i32, vp, vp, vp, i32, vp], i32),
    "ss_vq_scores": ([vp, i32, i32, vp, i32, i32, vp, i64, i64, vp, i64, vp], i32),
    "ss_vq_scores_lut": ([vp, i32, i32, i32, vp, i64, i64, vp, i64, vp], i32),
    "ss_vq_dequant": ([vp, i64, i64, i64, i64, vp, i32, i32, i32, vp, vp, vp, i64, i64, vp,
                       i32, i64, i64, vp], i32),
    "ss_value_encode_grouped": ([vp, i32, i64, i64, i64, i64, i32, i32, i32, vp, i64, i64, vp,
                                 vp, i64, i64, vp], i32),
    "ss_value_encode_tq": ([vp, i32, i64, i64, i64, i64, i32, i32, i32, i32, vp, vp, vp, i64,
                            i64, vp, i64, i64, vp], i32),
    "ss_scalar_quantize": ([vp, i64, vp, i32, vp, vp], i32),
    "ss_pack_indices": ([vp, i64, i32, i32, vp, vp], i32),
    "ss_unpack_indices": ([vp, i64, i32, i32, vp, vp], i32),
    "ss_value_decode": ([vp, i64, i64, i64, i64, i32, i32, i32, vp, vp, i32, vp, i64, i64, vp,
                         vp, i32, i64, i64, vp], i32),
    "ss_decode_workspace_size": ([C.POINTER(DecodeArgs)], C.c_size_t),
    "ss_decode_attn": ([C.POINTER(DecodeArgs), vp], i32),
    "ss_cache_append": ([C.POINTER(AppendArgs), vp], i32),
    "ss_decode_attn_partial": ([C.POINTER(DecodeArgs), vp, vp], i32),
    "ss_decode_check": ([vp, vp], i32),
    "ss_set_assign_path": ([i32], i32),
    "ss_vq_assign_check": ([vp], i32),
    "ss_decode_attn_noalloc": ([C.POINTER(DecodeArgs), vp], i32),
    "ss_lse_merge": ([vp, i32, i64, i32, vp, vp, i32, i64, vp], i32),
    "ss_decode_noalloc_check": ([vp], i32),
    "ss_set_error_sink": ([vp], i32),
    "ss_set_assign_wait": ([i64, i64], i32),
    "ss_query_centroid_dots": ([vp, i64, i32, vp, i32, i32, vp, vp], i32),
    "ss_rotate_rows": ([vp, i64, i32, i64, vp, vp, i32, i64, vp], i32),
}

EXPORTED = tuple(_SIGS)

_lib = None
_lock = threading.Lock()


def load(path: str | None = None) -> C.CDLL:
    """Loads (once) and returns the shared library; raises if it is missing."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise ImportError(
                f"SunShape CUDA library not found at {p}; build it with "
                "`python -m sunshape_mlx_b200.build` (there is no CPU fallback)")
        lib = C.CDLL(p)
        for name, (argt, rest) in _SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes = argt
            fn.restype = rest
        _lib = lib
        _attach_error_sink(lib)
        return lib


# ------------------------------------------------------------------ device-side give-ups
# A page-locked host word that the decode and tensor-core assignment kernels
# OR a code into when one of their bounded waits gives up (ss_set_error_sink).
# Reading it costs no synchronization, so every product entry point checks it
# before launching and raises for a launch that failed earlier.
_SINK = None
_SINK_WORD = None


def _attach_error_sink(lib) -> None:
    global _SINK, _SINK_WORD
    if not torch.cuda.is_available():
        return
    t = torch.zeros(1, dtype=torch.int32).pin_memory()
    if lib.ss_set_error_sink(C.c_void_p(t.data_ptr())) != SS_OK:
        raise SunShapeCudaError("ss_set_error_sink", 1, lib.ss_last_error().decode())
    _SINK = t
    _SINK_WORD = C.c_int.from_address(t.data_ptr())


WAIT_CODES = {1: "decode producer stage wait", 2: "decode copy drain", 4: "decode tile wait",
              8: "decode table wait", 16: "tensor-core assignment pipeline wait"}


def poll_device_errors() -> None:
    """Raises SunShapeCudaError (SS_ERR_TIMEOUT) if a kernel launched since
    the last poll gave up on a bounded device-side wait; its output was then
    invalid. Clears the word. Does not synchronize: a launch still running is
    seen by a later poll (``check_device_errors`` synchronizes first)."""
    w = _SINK_WORD
    if w is None or w.value == 0:
        return
    code = w.value
    w.value = 0
    what = ", ".join(n for b, n in WAIT_CODES.items() if code & b) or str(code)
    raise SunShapeCudaError("device wait", SS_ERR_TIMEOUT,
                            f"a device-side wait gave up ({what}); the output of that launch is invalid")


def check_device_errors(device=None) -> None:
    """Synchronizes the current stream of `device`, then ``poll_device_errors``."""
    torch.cuda.current_stream(device).synchronize()
    poll_device_errors()


def last_error() -> str:
    return load().ss_last_error().decode()


def check(fn: str, code: int) -> None:
    if code != SS_OK:
        raise SunShapeCudaError(fn, code, last_error())


def call(fn: str, *args) -> None:
    """Calls C entry point `fn`, raising SunShapeCudaError on failure."""
    check(fn, getattr(load(), fn)(*args))


# ------------------------------------------------------------------ helpers

def ptr(t: torch.Tensor | None):
    if t is None:
        return None
    return C.c_void_p(t.data_ptr())


def stream_ptr(device: torch.device | None = None):
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}") from None


def require_cuda(*tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError(
                "SunShape B200 kernels need CUDA tensors (there is no CPU fallback); "
                f"got a tensor on {t.device}")


def kernel_stats() -> dict[str, int]:
    lib = load()
    n = lib.ss_kernel_stats(None, 0)
    buf = C.create_string_buffer(n + 1)
    lib.ss_kernel_stats(buf, n + 1)
    out = {}
    for line in buf.value.decode().splitlines():
        k, v = line.split("=")
        out[k] = int(v)
    return out


def reset_kernel_stats() -> None:
    load().ss_reset_kernel_stats()
