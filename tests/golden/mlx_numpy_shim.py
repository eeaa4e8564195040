"""A NumPy-backed stand-in for the small part of ``mlx.core`` that the
reference package touches, so the reference's own Python code can run in a
container without MLX and produce golden vectors.

Used only by ``tests/golden/make_golden.py`` (fixture generation, run in a
container that has the reference tree). ``mx.fast.metal_kernel`` returns a
kernel object whose call raises, so every reference wrapper takes its own
documented fallback (``return None`` -> NumPy/MLX-op path), which is exactly
what the reference executes on a non-Apple CPU.

``mx.random`` is backed by ``numpy.random.default_rng(seed)``; the reference
draws its rotation matrix from MLX's RNG, which cannot be reproduced here, so
fixtures record the matrix that was used.
"""

from __future__ import annotations

import types

import numpy as np

float16 = np.float16
float32 = np.float32
float64 = np.float64
int32 = np.int32
int64 = np.int64
uint8 = np.uint8
uint16 = np.uint16
uint32 = np.uint32
bool_ = np.bool_
Dtype = type
cpu = "cpu"
gpu = "gpu"


class _ArrayMeta(type):
    def __instancecheck__(cls, obj):
        return isinstance(obj, np.ndarray)


class array(metaclass=_ArrayMeta):
    """``mx.array(x, dtype)``: Python floats default to float32, ints to int32."""

    def __new__(cls, x, dtype=None):
        if dtype is None:
            if isinstance(x, np.ndarray):
                return x.copy()
            a = np.asarray(x)
            if a.dtype == np.float64:
                a = a.astype(np.float32)
            elif a.dtype == np.int64:
                a = a.astype(np.int32)
            return a
        return np.array(x, dtype=dtype)


def eval(*args, **kwargs):  # noqa: A001 - mirrors mlx.core.eval
    return None


def zeros(shape, dtype=np.float32):
    return np.zeros(shape, dtype=dtype)


def ones(shape, dtype=np.float32):
    return np.ones(shape, dtype=dtype)


def full(shape, val, dtype=np.float32):
    return np.full(shape, val, dtype=dtype)


def zeros_like(x):
    return np.zeros_like(x)


def ones_like(x):
    return np.ones_like(x)


def eye(n, dtype=np.float32):
    return np.eye(n, dtype=dtype)


def arange(*args, dtype=None):
    a = np.arange(*args)
    if dtype is not None:
        return a.astype(dtype)
    return a.astype(np.int32) if a.dtype.kind == "i" else a.astype(np.float32)


def _axis_kw(kw):
    return {k: v for k, v in kw.items() if k in ("axis", "keepdims")}


def sum(x, axis=None, keepdims=False):  # noqa: A001
    x = np.asarray(x)
    r = np.sum(x, axis=axis, keepdims=keepdims)
    return r.astype(x.dtype) if x.dtype.kind == "f" else r


def mean(x, axis=None, keepdims=False):
    x = np.asarray(x)
    return np.mean(x, axis=axis, keepdims=keepdims).astype(x.dtype if x.dtype.kind == "f" else np.float32)


def max(x, axis=None, keepdims=False):  # noqa: A001
    return np.max(x, axis=axis, keepdims=keepdims)


def min(x, axis=None, keepdims=False):  # noqa: A001
    return np.min(x, axis=axis, keepdims=keepdims)


maximum = np.maximum
minimum = np.minimum
where = np.where
abs = np.abs  # noqa: A001
square = np.square
sign = np.sign
diag = np.diag
einsum = np.einsum
take_along_axis = np.take_along_axis
concatenate = np.concatenate
stack = np.stack
clip = np.clip
left_shift = np.left_shift
right_shift = np.right_shift
bitwise_and = np.bitwise_and
finfo = np.finfo


def round(x, decimals=0):  # noqa: A001
    return np.round(x, decimals)


def pad(x, pad_width, constant_values=0):
    return np.pad(x, pad_width, constant_values=constant_values)


def softmax(x, axis=-1, precise=False):
    x = np.asarray(x)
    m = np.max(x, axis=axis, keepdims=True)
    e = np.exp((x - m).astype(np.float64 if precise else x.dtype))
    return (e / np.sum(e, axis=axis, keepdims=True)).astype(x.dtype)


class _Linalg:
    @staticmethod
    def norm(x, axis=None, keepdims=False):
        x = np.asarray(x)
        return np.sqrt(np.sum(x * x, axis=axis, keepdims=keepdims)).astype(x.dtype)

    @staticmethod
    def qr(a, stream=None):
        return np.linalg.qr(np.asarray(a))

    @staticmethod
    def pinv(a, stream=None):
        return np.linalg.pinv(np.asarray(a)).astype(np.asarray(a).dtype)


linalg = _Linalg()


class _Random:
    _rng = np.random.default_rng(0)

    def seed(self, s):
        _Random._rng = np.random.default_rng(s)

    def normal(self, shape, dtype=np.float32):
        return _Random._rng.standard_normal(shape).astype(dtype)


random = _Random()


class _MetalKernel:
    def __init__(self, **kw):
        self.name = kw.get("name")

    def __call__(self, *a, **kw):
        raise RuntimeError("Metal is not available (NumPy stand-in for mlx.core)")


fast = types.SimpleNamespace(metal_kernel=lambda **kw: _MetalKernel(**kw))
