"""SunShape KV caches resident in GPU memory (cache.py of the reference).

Layouts (all contiguous, per (batch, kv-head) pair a fixed-capacity stream):
  key indices   (B, H, cap, n_blocks) uint8
  heavy keys    (B, H, cap, n_heavy * block_dim) fp16   (mixed-precision codec)
  fp16 values   (B, H, cap, D) fp16
  grouped       packed (B, H, cap, words) + scales/zeros (B, H, cap, G) f32
  turboquant    packed (B, H, cap, words) + norms (B, H, cap) f32
                (or per-group fp16 scales (B, H, cap, G) in the grouped variant)
  hybrid tail   fp16 keys/values (B, H, bufcap, D) in the original basis
Capacities grow in 256-token steps (cache.py:33) and tails in 128-token
multiples, so every stream holds whole tiles of the fused attention kernel.
Appends quantize keys and encode values directly into the cache slices.
"""

from __future__ import annotations

import torch

from . import _lib as L
from . import kernels as K
from .codec import SunShapeBlockCodec
from .value_codecs import GroupedValueCodec, TurboQuantValueCodec, build_value_codec

__all__ = ["SunShapeKVCache", "HybridSunShapeKVCache", "create_kv_cache", "save_cache",
           "load_cache", "DeferredTensor"]

_STEP = 256
_DEFAULT_BUFFER_SIZE = 128
_TAIL_STEP = 128


def _round_up(x: int, m: int) -> int:
    return ((x + m - 1) // m) * m


def _grow(old: torch.Tensor | None, shape: tuple, used: int, dtype, device, fill_zero=True):
    """New buffer of `shape`; copies old[:, :, :used] over."""
    new = (torch.zeros if fill_zero else torch.empty)(shape, dtype=dtype, device=device)
    if old is not None and used > 0:
        new[:, :, :used] = old[:, :, :used]
    return new


def _causal_mask(offset: int, n: int, return_array: bool):
    """mlx-lm style mask for n new queries at positions [offset, offset+n)."""
    if offset == 0 and n == 0:
        return "none"
    if not return_array:
        return "causal"
    qpos = torch.arange(offset, offset + n)
    kpos = torch.arange(offset + n)
    ok = qpos[:, None] >= kpos[None, :]
    return torch.where(ok, torch.tensor(0.0), torch.tensor(torch.finfo(torch.float16).min)).to(
        torch.float16)


class DeferredTensor:
    """A tensor computed on first use: what ``update_and_fetch`` returns for
    the dequantized keys (and decoded values), which mlx-lm-style callers
    pass straight to the patched SDPA. The fused kernel reads the cache's
    streams in place and never looks at them, so materializing them on every
    step (a full O(T) dequantization per layer, cache.py:205, 211-240 of the
    reference) is skipped unless something actually reads them.

    ``shape``/``dtype``/``device``/``ndim`` are known without computing; any
    other use (indexing, arithmetic, torch functions, attribute access)
    materializes it once, from the cache's storage at that moment with the
    token count of the call that made it. A caller that keeps it across a
    later append, flush or trim calls ``materialize()`` first."""

    __slots__ = ("_fn", "_shape", "_dtype", "_device", "_t")

    def __init__(self, fn, shape, dtype, device):
        self._fn, self._shape, self._dtype, self._device, self._t = fn, torch.Size(shape), dtype, device, None

    shape = property(lambda self: self._shape)
    dtype = property(lambda self: self._dtype)
    device = property(lambda self: self._device)
    ndim = property(lambda self: len(self._shape))
    is_materialized = property(lambda self: self._t is not None)

    def size(self, dim=None):
        return self._shape if dim is None else self._shape[dim]

    def dim(self) -> int:
        return len(self._shape)

    def materialize(self) -> torch.Tensor:
        if self._t is None:
            self._t = self._fn()
            self._fn = None
        return self._t

    def __getattr__(self, name):
        return getattr(self.materialize(), name)

    @classmethod
    def __torch_function__(cls, func, types, args=(), kwargs=None):
        def conv(x):
            if isinstance(x, DeferredTensor):
                return x.materialize()
            if isinstance(x, (list, tuple)):
                return type(x)(conv(y) for y in x)
            if isinstance(x, dict):
                return {k: conv(v) for k, v in x.items()}
            return x
        return func(*conv(args), **conv(kwargs or {}))

    def __getitem__(self, i):
        return self.materialize()[i]

    def __len__(self) -> int:
        return self._shape[0]

    def __iter__(self):
        return iter(self.materialize())

    def __array__(self, dtype=None):
        a = self.materialize().cpu().numpy()
        return a if dtype is None else a.astype(dtype)

    def __repr__(self) -> str:
        state = "materialized" if self._t is not None else "deferred"
        return f"DeferredTensor(shape={tuple(self._shape)}, dtype={self._dtype}, {state})"


def _binop(name):
    def f(self, *a):
        return getattr(self.materialize(), name)(*[x.materialize() if isinstance(x, DeferredTensor) else x for x in a])
    f.__name__ = name
    return f


for _n in ("__add__", "__radd__", "__sub__", "__rsub__", "__mul__", "__rmul__", "__truediv__",
           "__rtruediv__", "__matmul__", "__rmatmul__", "__neg__", "__pow__", "__eq__", "__ne__",
           "__lt__", "__le__", "__gt__", "__ge__", "__abs__"):
    setattr(DeferredTensor, _n, _binop(_n))
DeferredTensor.__hash__ = object.__hash__


class SunShapeKVCache:
    """Keys as block-VQ indices + fp16 values (cache.py:59-336)."""

    def __init__(self, codec: SunShapeBlockCodec, *, n_kv_heads: int = 1,
                 head_dim: int | None = None, dtype=torch.float16):
        self.codec = codec
        self.device = codec.device
        self.n_kv_heads = n_kv_heads
        self.head_dim = head_dim or codec.head_dim
        self.block_dim = codec.block_dim
        self.n_blocks = codec.n_blocks
        self.n_centroids = codec.n_centroids
        self.dtype = dtype
        self.offset = 0
        self._key_indices = None
        self._key_heavy = None
        self._values = None
        self._capacity = 0
        self._batch = 0
        self._epoch = 0          # bumped whenever the storage is reallocated
        self._assign_memo = None
        self._sdpa_memo = None
        self.eager_fetch = False  # True: update_and_fetch materializes keys (reference behaviour)
        # A decode step's append is handed to the next sunshape_sdpa call, which
        # quantizes and stores the tokens in its own table launch
        # (ss_decode_args.app_*); any other reader writes them first.
        self.defer_append = True
        self._pending = None      # (keys, values, offset, tokens) not yet written

    # ------------------------------------------------------------ storage
    def _ensure_capacity(self, B: int, new_tokens: int) -> None:
        """cache.py:102-150: grow to a multiple of 256 tokens."""
        need = self.offset + new_tokens
        if self._key_indices is not None and B != self._batch:
            raise ValueError(f"batch size changed from {self._batch} to {B}")
        if need <= self._capacity:
            return
        self._epoch += 1
        cap = _round_up(need, _STEP)
        H, dev = self.n_kv_heads, self.device
        self._key_indices = _grow(self._key_indices, (B, H, cap, self.n_blocks), self.offset,
                                  torch.uint8, dev)
        self._values = _grow(self._values, (B, H, cap, self.head_dim), self.offset,
                             torch.float16, dev)
        nh = self.codec.n_heavy_blocks
        if nh:
            self._key_heavy = _grow(self._key_heavy, (B, H, cap, nh * self.block_dim),
                                    self.offset, torch.float16, dev)
        self._capacity = cap
        self._batch = B

    def append(self, keys, values) -> None:
        """Quantize and store new tokens without materialising anything
        (the write half of update_and_fetch). Page-locked host tensors
        (``pin_memory()``) of a deferred decode-step append are not copied:
        the kernel that writes them reads them from host memory directly."""
        L.poll_device_errors()
        if _pinned(keys) and _pinned(values) and self.defer_append:
            k, v = keys, values
        else:
            k = K.cuda_tensor(keys, device=self.device)
            v = K.cuda_tensor(values, device=self.device)
        B, H, T, D = k.shape
        if H != self.n_kv_heads:
            raise AssertionError(f"Expected {self.n_kv_heads} kv heads, got {H}")
        if D != self.head_dim:
            raise AssertionError(f"Expected head_dim {self.head_dim}, got {D}")
        if T == 0:
            return
        self._flush_pending()
        self._ensure_capacity(B, T)
        o = self.offset
        codec = self.codec
        if (self.defer_append and B * H * T <= 4096 and not codec.use_rotation
                and codec.block_dim in (4, 8) and k.stride(3) == 1 and v.shape == k.shape
                and v.stride(3) == 1 and k.stride(0) == H * k.stride(1)
                and v.stride(0) == H * v.stride(1)):
            self._pending = (k, v, o, T)
            self.offset += T
            return
        if not k.is_cuda:
            k, v = K.cuda_tensor(k, device=self.device), K.cuda_tensor(v, device=self.device)
        if not self._append_fast(k, v, o):
            _quantize_keys_into(self.codec, k, self._key_indices[:, :, o:o + T],
                                None if self._key_heavy is None else self._key_heavy[:, :, o:o + T])
            self._values.narrow(2, o, T).copy_(v)
        self.offset += T

    def _append_fast(self, k: torch.Tensor, v: torch.Tensor, o: int) -> bool:
        """ss_cache_append: keys quantized into the index stream and values
        stored at token o in one launch, with an argument block kept from the
        last call (rebuilt on reallocation or a layout change), so a decode
        step's append is one short C call."""
        codec = self.codec
        B, H, T, D = k.shape
        if (codec.use_rotation or k.stride(3) != 1 or k.stride(0) != H * k.stride(1)
                or v.shape != k.shape or v.stride(3) != 1 or v.stride(0) != H * v.stride(1)):
            return False
        key = (self._epoch, k.dtype, k.stride(1), k.stride(2), v.dtype, v.stride(1), v.stride(2),
               codec.centroids.data_ptr(), codec.permutation.data_ptr(), codec._is_perm(),
               codec.n_heavy_blocks)
        memo = self._assign_memo
        if memo is None or memo[0] != key:
            L = K.L
            a = L.AppendArgs()
            a.key_dtype, a.key_group_stride, a.key_row_stride = L.dtype_code(k.dtype), k.stride(1), k.stride(2)
            a.value_dtype, a.value_group_stride, a.value_row_stride = L.dtype_code(v.dtype), v.stride(1), v.stride(2)
            a.n_groups, a.d = B * H, D
            perm = codec.permutation if codec._is_perm() else None
            a.perm = L.ptr(perm)
            a.centroids = L.ptr(codec.centroids)
            a.bd, a.k = codec.block_dim, codec.n_centroids
            a.heavy = L.ptr(codec.heavy_u8)
            ki, kh, vv = self._key_indices, self._key_heavy, self._values
            a.idx_group_stride, a.idx_row_stride = ki.stride(1), ki.stride(2)
            if kh is not None:
                a.kheavy_group_stride, a.kheavy_row_stride = kh.stride(1), kh.stride(2)
            a.v_group_stride, a.v_row_stride = vv.stride(1), vv.stride(2)
            bases = (ki.data_ptr(), None if kh is None else kh.data_ptr(), vv.data_ptr())
            memo = (key, a, L.C.byref(a), L.load().ss_cache_append, bases,
                    (ki.stride(2), 0 if kh is None else 2 * kh.stride(2), 2 * vv.stride(2)),
                    [codec, perm])
            self._assign_memo = memo
        _, a, ref, fn, (ki_p, kh_p, v_p), (irs, hrs2, vrs2), _ = memo
        a.keys = k.data_ptr()
        a.values = v.data_ptr()
        a.rows = T
        a.idx = ki_p + o * irs
        if kh_p is not None:
            a.kheavy = kh_p + o * hrs2
        a.v = v_p + o * vrs2
        rc = fn(ref, K.L.stream_ptr(self.device))
        if rc:
            K.L.check("ss_cache_append", rc)
        return True

    def _flush_pending(self) -> None:
        """Writes a deferred append now (one ss_cache_append launch)."""
        pend = self._pending
        if pend is None:
            return
        self._pending = None
        k, v, o, T = pend
        if not self._append_fast(k, v, o):
            if not k.is_cuda:
                k, v = K.cuda_tensor(k, device=self.device), K.cuda_tensor(v, device=self.device)
            _quantize_keys_into(self.codec, k, self._key_indices[:, :, o:o + T],
                                None if self._key_heavy is None else self._key_heavy[:, :, o:o + T])
            self._values.narrow(2, o, T).copy_(v)

    def update_and_fetch(self, keys, values):
        """cache.py:156-205: append, then return (keys, values) as stored.
        The keys are a DeferredTensor (dequantized on first use only: the
        fused SDPA reads the index stream itself); ``eager_fetch = True``
        returns the dequantized tensor at once, as the reference does."""
        self.append(keys, values)
        return self._fetch_keys(), self.values

    def _fetch_keys(self):
        if self.eager_fetch or self._key_indices is None or self.offset == 0:
            return self.keys
        idx, kh, t = self._key_indices, self._key_heavy, self.offset
        codec = self.codec

        def fetch():
            self._flush_pending()
            return _dequantize_keys(codec, idx[:, :, :t], None if kh is None else kh[:, :, :t])
        return DeferredTensor(
            fetch,
            (self._batch, self.n_kv_heads, t, self.head_dim), torch.float32, self.device)

    # ------------------------------------------------------------ views
    @property
    def keys(self) -> torch.Tensor:
        """Dequantized keys (B, H, T, D) float32 (cache.py:211-240)."""
        self._flush_pending()
        if self._key_indices is None or self.offset == 0:
            return torch.zeros((1, self.n_kv_heads, 0, self.head_dim), dtype=torch.float32,
                               device=self.device)
        return _dequantize_keys(self.codec, self._key_indices[:, :, :self.offset],
                                None if self._key_heavy is None else self._key_heavy[:, :, :self.offset])

    @property
    def values(self) -> torch.Tensor:
        self._flush_pending()
        if self._values is None or self.offset == 0:
            return torch.zeros((1, self.n_kv_heads, 0, self.head_dim), dtype=self.dtype,
                               device=self.device)
        return self._values[:, :, :self.offset]

    @property
    def key_indices(self) -> torch.Tensor:
        self._flush_pending()
        if self._key_indices is None or self.offset == 0:
            return torch.zeros((1, self.n_kv_heads, 0, self.n_blocks), dtype=torch.uint8,
                               device=self.device)
        return self._key_indices[:, :, :self.offset]

    @property
    def state(self):
        return (self.key_indices, self.values)

    # ------------------------------------------------------------ fused-attention view
    def attention_spec(self, flush: bool = True) -> dict:
        """Streams and token count for the fused kernel. flush=False leaves a
        deferred append pending (the caller's launch writes it)."""
        if flush:
            self._flush_pending()
        cap = self._capacity
        spec = dict(tc=self.offset, cap=cap, idx=self._key_indices, v=self._values)
        if self._key_heavy is not None:
            spec["kheavy"] = self._key_heavy
        return spec

    # ------------------------------------------------------------ accounting
    @property
    def nbytes(self) -> int:
        if self._key_indices is None:
            return 0
        B, T = self._batch, self.offset
        nh = self.codec.n_heavy_blocks
        return (B * self.n_kv_heads * T * self.n_blocks + B * self.n_kv_heads * T * self.head_dim * 2
                + B * self.n_kv_heads * T * nh * self.block_dim * 2)

    @property
    def nbytes_equivalent_fp16(self) -> int:
        if self.offset == 0:
            return 0
        B = self._batch or 1
        return 2 * B * self.n_kv_heads * self.offset * self.head_dim * 2

    @property
    def compression_ratio(self) -> float:
        fp16 = self.nbytes_equivalent_fp16
        return 1.0 if fp16 == 0 else fp16 / max(1, self.nbytes)

    def is_trimmable(self) -> bool:
        return True

    def trim(self, n: int) -> None:
        self._flush_pending()
        self.offset = max(0, self.offset - n)

    def empty(self) -> bool:
        return self.offset == 0

    def make_mask(self, N: int, return_array: bool = False, window_size=None, **kwargs):
        return _causal_mask(self.offset, N, return_array)

    def __repr__(self) -> str:
        return (f"SunShapeKVCache(offset={self.offset}, head_dim={self.head_dim}, "
                f"n_blocks={self.n_blocks}, n_centroids={self.n_centroids}, "
                f"compression={self.compression_ratio:.1f}x)")


def _pinned(x) -> bool:
    """A page-locked host tensor (readable by the GPU in place)."""
    return isinstance(x, torch.Tensor) and not x.is_cuda and x.is_pinned()


def _quantize_keys_into(codec: SunShapeBlockCodec, keys: torch.Tensor, idx_out: torch.Tensor,
                        heavy_out: torch.Tensor | None) -> None:
    """Assigns (B, H, T, D) keys straight into a strided cache slice."""
    if codec.use_rotation:
        keys = K.rotate_rows(keys, codec.rotation.T)
        perm = None
    else:
        perm = codec.permutation if codec._is_perm() else None
    B, H, T, D = keys.shape
    K.vq_assign(keys.reshape(B * H, T, D), codec.centroids, perm=perm, heavy=codec.heavy_u8,
                out_idx=idx_out.reshape(B * H, T, -1) if _viewable(idx_out) else idx_out,
                out_heavy=None if heavy_out is None else heavy_out.reshape(B * H, T, -1))


def _viewable(t: torch.Tensor) -> bool:
    return t.stride(0) == t.stride(1) * t.shape[1]


def _dequantize_keys(codec: SunShapeBlockCodec, idx: torch.Tensor,
                     heavy_vals: torch.Tensor | None) -> torch.Tensor:
    inv = codec.inv_permutation if codec._is_perm() else None
    out = K.vq_dequant(idx, codec.centroids, inv_perm=inv,
                       heavy=codec.heavy_u8 if heavy_vals is not None else None,
                       heavy_vals=heavy_vals)
    if codec.use_rotation:
        out = K.rotate_rows(out, codec.rotation)
    return out


class HybridSunShapeKVCache:
    """fp16 recent-token buffer + compressed tail (cache.py:348-998)."""

    def __init__(self, codec: SunShapeBlockCodec, *, n_kv_heads: int = 1,
                 head_dim: int | None = None, dtype=torch.float16,
                 buffer_size: int = _DEFAULT_BUFFER_SIZE, value_backend: str | None = None,
                 value_bits: int | None = None, value_group_size: int = 64, value_seed: int = 43,
                 value_codec: SunShapeBlockCodec | None = None, prefer_metal_kernels: bool = True,
                 tq_group_size: int | None = None, value_rotation=None):
        self.codec = codec
        self.device = codec.device
        self.n_kv_heads = n_kv_heads
        self.head_dim = head_dim or codec.head_dim
        self.block_dim = codec.block_dim
        self.n_blocks = codec.n_blocks
        self.n_centroids = codec.n_centroids
        self.dtype = dtype
        self.buffer_size = buffer_size
        self.value_backend = value_backend or ("fp16" if value_bits is None else "grouped")
        self.value_bits = value_bits
        self.value_group_size = value_group_size
        self.value_seed = value_seed
        self.prefer_metal_kernels = prefer_metal_kernels
        self.value_codec = value_codec
        self.last_value_quant_backend = "none"
        if self.value_backend not in {"fp16", "grouped", "turboquant", "sunshape"}:
            raise ValueError(f"Unsupported value backend: {self.value_backend}")
        if self.value_backend != "fp16" and self.value_bits is None:
            raise ValueError(f"value_bits is required for value backend {self.value_backend}")
        if self.value_backend == "grouped" and self.head_dim % self.value_group_size != 0:
            raise ValueError(
                f"head_dim ({self.head_dim}) must be divisible by "
                f"value_group_size ({self.value_group_size}) for value quantization")
        if self.value_backend == "sunshape":
            self.value_codec = self.value_codec or codec
            if self.value_codec.head_dim != self.head_dim:
                raise ValueError("SunShape value codec head_dim must match cache head_dim")
            self.value_n_blocks = self.value_codec.n_blocks
            self.value_n_centroids = self.value_codec.n_centroids
        else:
            self.value_n_blocks = 0
            self.value_n_centroids = 0
        self._value_codec_impl = None
        if self.value_backend in ("grouped", "turboquant"):
            self._value_codec_impl = build_value_codec(
                self.value_backend, head_dim=self.head_dim, value_bits=self.value_bits or 0,
                value_group_size=self.value_group_size, value_seed=self.value_seed,
                prefer_metal=prefer_metal_kernels, tq_group_size=tq_group_size,
                device=self.device)
            if value_rotation is not None and self.value_backend == "turboquant":
                c = self._value_codec_impl
                c.rotation = K.cuda_tensor(value_rotation, torch.float32, self.device)
                c.rotation_t = c.rotation.T.contiguous()
        self._compressed_offset = 0
        self._buffer_offset = 0
        self._batch = 0
        self._key_buffer = None
        self._value_buffer = None
        # TurboQuant values are attended in the rotated basis; the fp16 tail is
        # kept there too (v R^T) so one accumulator covers all tokens.
        self._value_buffer_rot = None
        self._vq_tables = None   # (key, fp16 value centroids, inverse-transform matrix)
        self._key_indices = None
        self._key_heavy = None
        self._values_packed = None
        self._value_scales = None
        self._value_zeros = None
        self._value_norms = None
        self._value_indices = None
        self._values_fp16 = None
        self._compressed_capacity = 0
        self._epoch = 0          # bumped whenever compressed storage is reallocated
        self._assign_memo = None
        self._sdpa_memo = None
        self.eager_fetch = False  # True: update_and_fetch materializes (reference behaviour)

    @property
    def offset(self) -> int:
        return self._compressed_offset + self._buffer_offset

    # ------------------------------------------------------------ append / flush
    def _ensure_compressed(self, B: int, n: int) -> None:
        need = self._compressed_offset + n
        if need <= self._compressed_capacity:
            return
        cap = _round_up(need, _STEP)
        self._epoch += 1
        H, dev, u = self.n_kv_heads, self.device, self._compressed_offset
        self._key_indices = _grow(self._key_indices, (B, H, cap, self.n_blocks), u, torch.uint8, dev)
        nh = self.codec.n_heavy_blocks
        if nh:
            self._key_heavy = _grow(self._key_heavy, (B, H, cap, nh * self.block_dim), u,
                                    torch.float16, dev)
        vc = self._value_codec_impl
        if self.value_backend == "grouped":
            self._values_packed = _grow(self._values_packed, (B, H, cap, vc.packed_dim), u, torch.int32, dev)
            self._value_scales = _grow(self._value_scales, (B, H, cap, vc.n_groups), u, torch.float32, dev)
            self._value_zeros = _grow(self._value_zeros, (B, H, cap, vc.n_groups), u, torch.float32, dev)
        elif self.value_backend == "turboquant":
            self._values_packed = _grow(self._values_packed, (B, H, cap, vc.packed_dim), u, torch.int32, dev)
            if vc.group_size is None:
                self._value_norms = _grow(self._value_norms, (B, H, cap), u, torch.float32, dev)
            else:
                self._value_norms = _grow(self._value_norms, (B, H, cap, vc.n_scale_groups), u,
                                          torch.float16, dev)
        elif self.value_backend == "sunshape":
            self._value_indices = _grow(self._value_indices, (B, H, cap, self.value_n_blocks), u,
                                        torch.uint8, dev)
        else:
            self._values_fp16 = _grow(self._values_fp16, (B, H, cap, self.head_dim), u,
                                      torch.float16, dev)
        self._compressed_capacity = cap

    def _flush_buffer(self, B: int, n: int) -> None:
        """Moves the oldest n buffered tokens to compressed storage (cache.py:463-650)."""
        n = min(n, self._buffer_offset)
        if n <= 0:
            return
        self._ensure_compressed(B, n)
        c0 = self._compressed_offset
        kf = self._key_buffer[:, :, :n]
        vf = self._value_buffer[:, :, :n]
        _quantize_keys_into(self.codec, kf, self._key_indices[:, :, c0:c0 + n],
                            None if self._key_heavy is None else self._key_heavy[:, :, c0:c0 + n])
        vc = self._value_codec_impl
        if self.value_backend == "grouped":
            vc.quantize_into(vf, self._values_packed[:, :, c0:c0 + n],
                             self._value_scales[:, :, c0:c0 + n], self._value_zeros[:, :, c0:c0 + n])
            self.last_value_quant_backend = vc.last_quantize_backend
        elif self.value_backend == "turboquant":
            vc.quantize_into(vf, self._values_packed[:, :, c0:c0 + n], self._value_norms[:, :, c0:c0 + n])
            self.last_value_quant_backend = vc.last_quantize_backend
        elif self.value_backend == "sunshape":
            _quantize_keys_into(self.value_codec, vf, self._value_indices[:, :, c0:c0 + n], None)
            self.last_value_quant_backend = "sunshape"
        else:
            self._values_fp16[:, :, c0:c0 + n] = vf
            self.last_value_quant_backend = "fp16"
        rem = self._buffer_offset - n
        if rem > 0:
            self._key_buffer[:, :, :rem] = self._key_buffer[:, :, n:n + rem].clone()
            self._value_buffer[:, :, :rem] = self._value_buffer[:, :, n:n + rem].clone()
            if self._value_buffer_rot is not None:
                self._value_buffer_rot[:, :, :rem] = self._value_buffer_rot[:, :, n:n + rem].clone()
        self._compressed_offset += n
        self._buffer_offset = rem

    def append(self, keys, values) -> None:
        """Append to the fp16 buffer and flush overflow (cache.py:656-710)."""
        L.poll_device_errors()
        k = K.cuda_tensor(keys, device=self.device)
        v = K.cuda_tensor(values, device=self.device)
        B, H, T, D = k.shape
        if H != self.n_kv_heads or D != self.head_dim:
            raise AssertionError("kv heads / head_dim mismatch")
        if self._batch and B != self._batch:
            raise ValueError(f"batch size changed from {self._batch} to {B}")
        self._batch = B
        if self.buffer_size == 0 and self._buffer_offset == 0 and self._append_vq_fast(k, v):
            return
        need = self._buffer_offset + T
        cur = 0 if self._key_buffer is None else self._key_buffer.shape[2]
        if need > cur:
            size = _round_up(max(self.buffer_size, need, 2 * cur if cur else 0, 1), _TAIL_STEP)
            self._key_buffer = _grow(self._key_buffer, (B, H, size, D), self._buffer_offset,
                                     torch.float16, self.device)
            self._value_buffer = _grow(self._value_buffer, (B, H, size, D), self._buffer_offset,
                                       torch.float16, self.device)
            if self.value_backend == "turboquant" or self._vq_transformed():
                self._value_buffer_rot = _grow(self._value_buffer_rot, (B, H, size, D),
                                               self._buffer_offset, torch.float16, self.device)
        b0 = self._buffer_offset
        self._key_buffer[:, :, b0:b0 + T] = k
        self._value_buffer[:, :, b0:b0 + T] = v
        if self._value_buffer_rot is not None:
            if self.value_backend == "turboquant":
                rt = self._value_codec_impl.rotation_t
                self._value_buffer_rot[:, :, b0:b0 + T] = K.rotate_rows(v, rt, torch.float16)
            else:  # block-VQ values: the value codec's own basis
                self._value_buffer_rot[:, :, b0:b0 + T] = \
                    self.value_codec._forward_transform(v.float()).half()
        self._buffer_offset += T
        if self._buffer_offset > self.buffer_size:
            self._flush_buffer(B, self._buffer_offset - self.buffer_size)

    def update_and_fetch(self, keys, values):
        """cache.py:656-710. Keys and values come back as DeferredTensors
        (computed on first use; the fused SDPA reads the streams itself);
        ``eager_fetch = True`` materializes them at once, as the reference."""
        self.append(keys, values)
        if self.eager_fetch or self.offset == 0:
            return self.keys, self.values
        shape = (max(self._batch, 1), self.n_kv_heads, self.offset, self.head_dim)
        snap = self._snapshot()
        return (DeferredTensor(lambda: snap.keys, shape, torch.float32, self.device),
                DeferredTensor(lambda: snap.values, shape, self.dtype, self.device))

    def _snapshot(self):
        """A shallow copy holding the current streams and offsets (the token
        counts of this call for views computed later)."""
        import copy

        return copy.copy(self)

    # ------------------------------------------------------------ views
    @property
    def keys(self) -> torch.Tensor:
        parts = []
        if self._compressed_offset > 0:
            c = self._compressed_offset
            parts.append(_dequantize_keys(self.codec, self._key_indices[:, :, :c],
                                          None if self._key_heavy is None else self._key_heavy[:, :, :c]))
        if self._buffer_offset > 0:
            parts.append(self._key_buffer[:, :, :self._buffer_offset].float())
        if not parts:
            return torch.zeros((max(self._batch, 1), self.n_kv_heads, 0, self.head_dim),
                               dtype=torch.float32, device=self.device)
        return torch.cat(parts, dim=2)

    def _compressed_values(self, out_dtype=torch.float16) -> torch.Tensor | None:
        c = self._compressed_offset
        if c == 0:
            return None
        vc = self._value_codec_impl
        if self.value_backend == "grouped":
            return vc.dequantize(self._values_packed[:, :, :c], self._value_scales[:, :, :c],
                                 self._value_zeros[:, :, :c], out_dtype=out_dtype)
        if self.value_backend == "turboquant":
            return vc.dequantize(self._values_packed[:, :, :c], self._value_norms[:, :, :c],
                                 out_dtype=out_dtype)
        if self.value_backend == "sunshape":
            return _dequantize_keys(self.value_codec, self._value_indices[:, :, :c], None).to(out_dtype)
        return self._values_fp16[:, :, :c]

    @property
    def values(self) -> torch.Tensor:
        """Compressed values decoded (in the cache dtype) followed by the buffer."""
        parts = []
        cv = self._compressed_values(torch.float16)
        if cv is not None:
            parts.append(cv)
        if self._buffer_offset > 0:
            parts.append(self._value_buffer[:, :, :self._buffer_offset])
        if not parts:
            return torch.zeros((max(self._batch, 1), self.n_kv_heads, 0, self.head_dim),
                               dtype=self.dtype, device=self.device)
        return torch.cat(parts, dim=2)

    @property
    def key_indices(self) -> torch.Tensor:
        if self._key_indices is None or self._compressed_offset == 0:
            return torch.zeros((max(self._batch, 1), self.n_kv_heads, 0, self.n_blocks),
                               dtype=torch.uint8, device=self.device)
        return self._key_indices[:, :, :self._compressed_offset]

    @property
    def buffer_keys(self) -> torch.Tensor:
        if self._key_buffer is None or self._buffer_offset == 0:
            return torch.zeros((max(self._batch, 1), self.n_kv_heads, 0, self.head_dim),
                               dtype=torch.float16, device=self.device)
        return self._key_buffer[:, :, :self._buffer_offset]

    @property
    def buffer_values(self) -> torch.Tensor:
        if self._value_buffer is None or self._buffer_offset == 0:
            return torch.zeros((max(self._batch, 1), self.n_kv_heads, 0, self.head_dim),
                               dtype=torch.float16, device=self.device)
        return self._value_buffer[:, :, :self._buffer_offset]

    @property
    def compressed_offset(self) -> int:
        return self._compressed_offset

    @property
    def buffer_offset(self) -> int:
        return self._buffer_offset

    @property
    def values_packed_raw(self):
        if self.value_backend != "grouped" or self._compressed_offset == 0:
            return None
        return self._values_packed[:, :, :self._compressed_offset]

    @property
    def value_scales_raw(self):
        if self.value_backend != "grouped" or self._compressed_offset == 0:
            return None
        return self._value_scales[:, :, :self._compressed_offset]

    @property
    def value_zeros_raw(self):
        if self.value_backend != "grouped" or self._compressed_offset == 0:
            return None
        return self._value_zeros[:, :, :self._compressed_offset]

    @property
    def can_fuse_value_dequant(self) -> bool:
        return self.value_backend == "grouped" and self._compressed_offset > 0

    def _append_vq_fast(self, k: torch.Tensor, v: torch.Tensor) -> bool:
        """No fp16 tail and block-VQ values: new keys and values go straight
        into the index streams, one ss_vq_assign each, from argument tuples
        kept until the storage is reallocated (a decode step's append is
        otherwise dominated by host work). Same indices as the buffered path,
        which quantizes the same fp16-stored tokens."""
        kc, vc = self.codec, self.value_codec
        if (self.value_backend != "sunshape" or kc.use_rotation or vc.use_rotation
                or kc.n_heavy_blocks or vc.n_heavy_blocks):
            return False
        B, H, T, D = k.shape
        # the buffered path stores tokens in fp16 before quantizing them
        k16 = k if k.dtype == torch.float16 else k.half()
        v16 = v if v.dtype == torch.float16 else v.half()
        for t in (k16, v16):
            if t.stride(3) != 1 or t.stride(0) != H * t.stride(1):
                return False
        self._ensure_compressed(B, T)
        key = (self._epoch, k16.stride(1), k16.stride(2), v16.stride(1), v16.stride(2),
               kc.centroids.data_ptr(), vc.centroids.data_ptr(), kc.permutation.data_ptr(),
               vc.permutation.data_ptr())
        memo = self._assign_memo
        if memo is None or memo[0] != key:
            L = K.L
            fn = L.load().ss_vq_assign
            calls = []
            for cd, src, dst in ((kc, k16, self._key_indices), (vc, v16, self._value_indices)):
                perm = cd.permutation if cd._is_perm() else None
                calls.append((src is k16, L.ptr(perm), L.ptr(cd.centroids), cd.block_dim,
                              cd.n_centroids, dst.data_ptr(), dst.stride(1), dst.stride(2),
                              src.stride(1), src.stride(2), [perm, cd]))
            memo = (key, fn, calls)
            self._assign_memo = memo
        _, fn, calls = memo
        o = self._compressed_offset
        st = K.L.stream_ptr(self.device)
        C = K.L.C
        for is_key, perm_p, cents_p, bd, kn, dst_p, dgs, drs, sgs, srs, _ in calls:
            src = k16 if is_key else v16
            rc = fn(C.c_void_p(src.data_ptr()), K.L.SS_F16, B * H, T, sgs, srs, D, perm_p, cents_p,
                    bd, kn, None, C.c_void_p(dst_p + o * drs), dgs, drs, None, 0, 0, None, 0, st)
            if rc:
                K.L.check("ss_vq_assign", rc)
        self._compressed_offset += T
        self.last_value_quant_backend = "sunshape"
        return True

    def _vq_transformed(self) -> bool:
        vc = self.value_codec
        return self.value_backend == "sunshape" and (vc._is_perm() or vc.use_rotation)

    def _vq_value_tables(self):
        """Block-VQ values for the fused decode: the value centroids in fp16
        (the dtype the reference's cache returns dequantised values in,
        cache.py:785-812) and the codec's inverse transform as a (D, D) matrix
        M with x = y @ M (a permutation matrix, the rotation, or None)."""
        vc = self.value_codec
        key = (vc.centroids.data_ptr(), vc.centroids._version, vc.use_rotation,
               vc.permutation.data_ptr(), vc.permutation._version)
        if self._vq_tables is None or self._vq_tables[0] != key:
            cents = vc.centroids.to(torch.float16).contiguous()
            vrot = None
            if vc._is_perm() or vc.use_rotation:
                eye = torch.eye(self.head_dim, dtype=torch.float32, device=self.device)
                vrot = vc._inverse_transform(eye).contiguous()
            self._vq_tables = (key, cents, vrot)
        return self._vq_tables[1], self._vq_tables[2]

    # ------------------------------------------------------------ fused-attention view
    def attention_spec(self) -> dict:
        spec = dict(tc=self._compressed_offset, cap=self._compressed_capacity)
        if self._compressed_offset > 0:
            spec["idx"] = self._key_indices
            if self._key_heavy is not None:
                spec["kheavy"] = self._key_heavy
            vc = self._value_codec_impl
            if self.value_backend == "fp16":
                spec["v"] = self._values_fp16
            elif self.value_backend == "sunshape":
                cents, vrot = self._vq_value_tables()
                spec.update(vi=self._value_indices, v_cents=cents)
                if vrot is not None:
                    spec["v_rot"] = vrot
            elif self.value_backend == "grouped":
                spec.update(vq=self._values_packed, vs=self._value_scales, vz=self._value_zeros,
                            bits=vc.bits, group=vc.group_size, levels=vc.levels(self.device))
            else:
                norms = self._value_norms
                spec.update(vq=self._values_packed,
                            vs=norms if norms.dim() == 4 else norms.unsqueeze(-1), vz=None,
                            bits=vc.bits, group=vc.group_size or self.head_dim,
                            levels=vc.levels(self.device), v_rot=vc.rotation)
        if self._buffer_offset > 0:
            vt = self._value_buffer_rot if self._value_buffer_rot is not None else self._value_buffer
            spec.update(k_tail=self._key_buffer, v_tail=vt, ttail=self._buffer_offset)
            if self._value_buffer_rot is not None and "v_rot" not in spec:
                spec["v_rot"] = (self._value_codec_impl.rotation if self.value_backend == "turboquant"
                                 else self._vq_value_tables()[1])
        return spec

    # ------------------------------------------------------------ accounting
    @property
    def nbytes(self) -> int:
        """Storage bytes of compressed + buffered tokens for the real batch size
        (the reference's version assumes batch 1, cache.py:907)."""
        B = max(self._batch, 1)
        H, c, b = self.n_kv_heads, self._compressed_offset, self._buffer_offset
        idx = B * H * c * self.n_blocks
        idx += B * H * c * self.codec.n_heavy_blocks * self.block_dim * 2
        vc = self._value_codec_impl
        if self.value_backend == "grouped" and c:
            val = B * H * c * (vc.packed_dim * 4 + vc.n_groups * 8)
        elif self.value_backend == "turboquant" and c:
            sc = 4 if vc.group_size is None else 2 * vc.n_scale_groups
            val = B * H * c * (vc.packed_dim * 4 + sc)
        elif self.value_backend == "sunshape" and c:
            val = B * H * c * self.value_n_blocks
        else:
            val = B * H * c * self.head_dim * 2
        return idx + val + B * H * b * self.head_dim * 4

    @property
    def nbytes_equivalent_fp16(self) -> int:
        if self.offset == 0:
            return 0
        return 2 * max(self._batch, 1) * self.n_kv_heads * self.offset * self.head_dim * 2

    @property
    def compression_ratio(self) -> float:
        fp16 = self.nbytes_equivalent_fp16
        return 1.0 if fp16 == 0 else fp16 / max(1, self.nbytes)

    def is_trimmable(self) -> bool:
        return True

    def trim(self, n: int) -> None:
        """Drops n tokens from the end: buffer first, then compressed (cache.py:954-963)."""
        if n <= 0:
            return
        bt = min(n, self._buffer_offset)
        self._buffer_offset -= bt
        rest = n - bt
        if rest > 0:
            self._compressed_offset = max(0, self._compressed_offset - rest)

    def empty(self) -> bool:
        return self.offset == 0

    def make_mask(self, N: int, return_array: bool = False, window_size=None, **kwargs):
        return _causal_mask(self.offset, N, return_array)

    @property
    def state(self):
        parts = []
        if self._compressed_offset > 0:
            parts.append(self.key_indices)
        if self._buffer_offset > 0:
            parts.append(self.buffer_keys)
        if not parts:
            parts.append(torch.zeros((1,), device=self.device))
        return tuple(parts)

    def __repr__(self) -> str:
        return (f"HybridSunShapeKVCache(offset={self.offset}, compressed={self._compressed_offset}, "
                f"buffer={self._buffer_offset}, value_backend={self.value_backend}, "
                f"compression={self.compression_ratio:.1f}x)")


def create_kv_cache(codec: SunShapeBlockCodec, *, n_kv_heads: int = 1, head_dim: int | None = None,
                    dtype=torch.float16, value_backend: str = "fp16", value_bits: int | None = None,
                    value_group_size: int = 64, value_seed: int = 43,
                    value_codec: SunShapeBlockCodec | None = None,
                    buffer_size: int = _DEFAULT_BUFFER_SIZE, prefer_metal_kernels: bool = True,
                    tq_group_size: int | None = None, value_rotation=None):
    """cache.py:1006-1107: fp16 values with the default buffer -> simple cache;
    anything else -> hybrid cache."""
    if value_backend == "fp16" and buffer_size == _DEFAULT_BUFFER_SIZE:
        return SunShapeKVCache(codec, n_kv_heads=n_kv_heads, head_dim=head_dim, dtype=dtype)
    return HybridSunShapeKVCache(
        codec, n_kv_heads=n_kv_heads, head_dim=head_dim, dtype=dtype, buffer_size=buffer_size,
        value_backend=value_backend, value_bits=value_bits, value_group_size=value_group_size,
        value_seed=value_seed, value_codec=value_codec, prefer_metal_kernels=prefer_metal_kernels,
        tq_group_size=tq_group_size, value_rotation=value_rotation)


# ---------------------------------------------------------------- serialization
# The reference only exposes the raw arrays (`state`, cache.py:256-262,
# 988-998); these save and restore a cache completely (codec, value codec,
# every stream and the offsets), so a prompt cache can be stored and decoding
# resumed from it with identical results.
_DTYPES = {str(d): d for d in (torch.float16, torch.bfloat16, torch.float32)}


def _codec_from_state(st: dict, device) -> SunShapeBlockCodec:
    c = SunShapeBlockCodec(head_dim=int(st["head_dim"]), block_dim=int(st["block_dim"]),
                           n_centroids=int(st["n_centroids"]), mode=str(st["mode"]),
                           device=device)
    return c.load_state_dict(st)


def _cache_state(cache) -> dict:
    if hasattr(cache, "_flush_pending"):
        cache._flush_pending()
    fields = {}
    for name, val in vars(cache).items():
        if name.endswith("_memo") or name in ("codec", "value_codec", "_value_codec_impl", "device"):
            continue
        if isinstance(val, torch.Tensor):
            fields[name] = val.detach().cpu()
        elif isinstance(val, torch.dtype):
            fields[name] = str(val)
        elif val is None or isinstance(val, (bool, int, float, str)):
            fields[name] = val
    st = {"kind": type(cache).__name__, "codec": cache.codec.state_dict(), "fields": fields}
    vc = getattr(cache, "value_codec", None)
    if vc is not None and vc is not cache.codec:
        st["value_codec"] = vc.state_dict()
    impl = getattr(cache, "_value_codec_impl", None)
    if impl is not None and getattr(impl, "rotation", None) is not None:
        st["value_rotation"] = impl.rotation.detach().cpu()
        st["tq_group_size"] = getattr(impl, "group_size", None)
    return st


def _restore_fields(cache, fields: dict) -> None:
    for name, val in fields.items():
        if isinstance(val, torch.Tensor):
            val = val.to(cache.device)
        elif name == "dtype" or (isinstance(val, str) and val in _DTYPES and name.endswith("dtype")):
            val = _DTYPES.get(val, val)
        setattr(cache, name, val)
    if hasattr(cache, "_epoch"):
        cache._epoch += 1  # cached launch arguments refer to the old storage


def cache_state_dict(cache) -> dict:
    """CPU-tensor state of a SunShape cache (simple or hybrid), codec included."""
    return _cache_state(cache)


def cache_from_state_dict(st: dict, device=None, codec: SunShapeBlockCodec | None = None):
    """Rebuilds a cache saved by :func:`cache_state_dict` on `device`."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    codec = codec or _codec_from_state(st["codec"], dev)
    f = st["fields"]
    dtype = _DTYPES.get(f.get("dtype"), torch.float16)
    if st["kind"] == "SunShapeKVCache":
        cache = SunShapeKVCache(codec, n_kv_heads=int(f["n_kv_heads"]),
                                head_dim=int(f["head_dim"]), dtype=dtype)
    elif st["kind"] == "HybridSunShapeKVCache":
        vcodec = _codec_from_state(st["value_codec"], dev) if "value_codec" in st else None
        cache = HybridSunShapeKVCache(
            codec, n_kv_heads=int(f["n_kv_heads"]), head_dim=int(f["head_dim"]), dtype=dtype,
            buffer_size=int(f["buffer_size"]), value_backend=f["value_backend"],
            value_bits=f["value_bits"], value_group_size=int(f["value_group_size"]),
            value_seed=int(f["value_seed"]), value_codec=vcodec,
            tq_group_size=st.get("tq_group_size"), value_rotation=st.get("value_rotation"))
    else:
        raise ValueError(f"unknown cache kind {st['kind']!r}")
    _restore_fields(cache, f)
    return cache


def save_cache(cache, path) -> None:
    """Writes a cache (and its codecs) to `path` (torch.save of CPU tensors)."""
    torch.save(cache_state_dict(cache), path)


def load_cache(path, device=None, codec: SunShapeBlockCodec | None = None):
    """Loads a cache written by :func:`save_cache`; decoding continues from it."""
    return cache_from_state_dict(torch.load(path, map_location="cpu", weights_only=False),
                                 device=device, codec=codec)

