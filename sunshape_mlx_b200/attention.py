"""SunShape scaled-dot-product attention over the compressed cache
(attention.py of the reference).

``sunshape_sdpa`` launches one fused kernel for the whole (B, Hq, Tq) output
(ss_decode_attn): query x centroid tables in shared memory, the uint8 index
and value streams read once per kv-head for all of its GQA query heads,
online softmax, P.V on the tensor cores, fp16 tail of the hybrid cache and
causal / array masks handled in the same pass. There is no 2-pass or CPU
path: unsupported configurations raise.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L
from . import kernels as K
from .cache import HybridSunShapeKVCache, SunShapeKVCache

__all__ = ["sunshape_sdpa", "decode_partials", "workspace_for", "PreparedDecode"]

_WS: dict[tuple, torch.Tensor] = {}


def workspace_for(device: torch.device, nbytes: int) -> torch.Tensor:
    """Zero-initialised decode workspace, one per (device, stream), grown on
    demand. The kernel leaves its arrival counters at zero on exit, so the
    buffer is reused without clearing; calls sharing it are stream-ordered."""
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    ws = _WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        _WS[key] = ws
    return ws


def _fill_args(q: torch.Tensor, centroids: torch.Tensor, perm, scale: float, spec: dict,
               causal: bool, out: torch.Tensor | None, mask=None, rot_k=None, heavy=None,
               n_heavy: int = 0) -> tuple[L.DecodeArgs, list]:
    keep = []  # tensors that must outlive the call
    a = L.DecodeArgs()
    B, Hq, Tq, D = q.shape
    a.q = q.data_ptr()
    a.q_dtype = L.dtype_code(q.dtype)
    a.q_sb, a.q_sh, a.q_st = q.stride(0), q.stride(1), q.stride(2)
    if q.stride(3) != 1:
        raise ValueError("queries must be contiguous in head_dim")
    idx = spec.get("idx")
    v = spec.get("v")
    vq = spec.get("vq")
    k_tail = spec.get("k_tail")
    ref = idx if idx is not None else k_tail
    if ref is None:
        raise ValueError("empty cache spec")
    a.b = B
    a.hkv = ref.shape[1]
    a.hq, a.tq, a.d = Hq, Tq, D
    a.scale = float(scale)
    a.perm = perm.data_ptr() if perm is not None else None
    a.rot_k = rot_k.data_ptr() if rot_k is not None else None
    nb, k, bd = centroids.shape
    a.centroids = centroids.data_ptr()
    a.bd, a.k = bd, k
    a.heavy = heavy.data_ptr() if heavy is not None else None
    a.n_heavy = n_heavy
    tc = int(spec.get("tc", 0))
    a.tc = tc
    if tc > 0:
        a.idx = idx.data_ptr()
        a.idx_pair_stride = idx.stride(1)
        kh = spec.get("kheavy")
        if n_heavy:
            a.kheavy = kh.data_ptr()
            a.kheavy_pair_stride = kh.stride(1)
        vi = spec.get("vi")
        if v is not None:
            a.vfmt = L.SS_V_F16
            a.v = v.data_ptr()
            a.v_pair_stride = v.stride(1)
        elif vi is not None:
            a.vfmt = L.SS_V_VQ
            a.v_idx = vi.data_ptr()
            a.vi_pair_stride = vi.stride(1)
            vc = spec["v_cents"]
            a.v_cents = vc.data_ptr()
            a.v_k, a.v_bd = vc.shape[1], vc.shape[2]
        else:
            a.vfmt = L.SS_V_QUANT
            a.vq = vq.data_ptr()
            a.vq_pair_stride = vq.stride(1)
            a.v_bits = int(spec["bits"])
            a.v_group = int(spec["group"])
            vs = spec["vs"]
            a.v_scales = vs.data_ptr()
            a.v_scale_dtype = L.SS_F32 if vs.dtype == torch.float32 else L.SS_F16
            a.vs_pair_stride = vs.stride(1)
            vz = spec.get("vz")
            if vz is not None:
                a.v_zeros = vz.data_ptr()
                a.vz_pair_stride = vz.stride(1)
            lv = list(spec["levels"]) + [0.0] * (16 - len(spec["levels"]))
            a.v_levels = (C.c_float * 16)(*lv)
    else:
        a.vfmt = L.SS_V_F16 if v is not None or vq is None else L.SS_V_QUANT  # tail only
    vr = spec.get("v_rot")
    if vr is not None:
        vr = vr.contiguous()
        keep.append(vr)
        a.v_rot = vr.data_ptr()
    tt = int(spec.get("ttail", 0))
    a.ttail = tt
    if tt > 0:
        a.k_tail = k_tail.data_ptr()
        a.v_tail = spec["v_tail"].data_ptr()
        a.tail_pair_stride = k_tail.stride(1)
        if spec["v_tail"].stride(1) != k_tail.stride(1):
            raise ValueError("tail keys and values must share the layout")
    a.causal = 1 if causal else 0
    if mask is not None:
        m = mask
        keep.append(m)
        a.mask = m.data_ptr()
        a.mask_stride = m.stride(0)
        a.mask_mode = spec.get("mask_mode", 0)
    if out is not None:
        a.out = out.data_ptr()
        a.out_dtype = L.dtype_code(out.dtype)
        a.o_sb, a.o_sh, a.o_st = out.stride(0), out.stride(1), out.stride(2)
    a.max_ctas = int(spec.get("max_ctas", 0))
    return a, keep


def _run_decode(q: torch.Tensor, *, centroids: torch.Tensor, perm, scale: float, spec: dict,
                causal: bool, out: torch.Tensor | None, mask=None, rot_k=None, heavy=None,
                n_heavy: int = 0, part_out: torch.Tensor | None = None) -> None:
    a, keep = _fill_args(q, centroids, perm, scale, spec, causal, out, mask, rot_k, heavy, n_heavy)
    lib = L.load()
    nbytes = lib.ss_decode_workspace_size(C.byref(a))
    if nbytes == 0:
        raise L.SunShapeCudaError("ss_decode_workspace_size", 1, L.last_error())
    ws = workspace_for(q.device, nbytes)
    a.workspace = ws.data_ptr()
    a.workspace_bytes = ws.numel()
    st = L.stream_ptr(q.device)
    if part_out is None:
        L.check("ss_decode_attn", lib.ss_decode_attn(C.byref(a), st))
    else:
        L.check("ss_decode_attn_partial",
                lib.ss_decode_attn_partial(C.byref(a), C.c_void_p(part_out.data_ptr()), st))
    del keep


def _prepare_mask(mask, tq: int, tkv: int, device) -> tuple[torch.Tensor | None, int, bool]:
    """(float mask, mask_mode, causal) from None / "causal" / array masks."""
    if mask is None or (isinstance(mask, str) and mask == "none"):
        return None, 0, False
    if isinstance(mask, str):
        if mask == "causal":
            return None, 0, True
        raise ValueError(f"unsupported mask {mask!r}")
    m = K.cuda_tensor(mask, device=device)
    while m.dim() > 2 and m.shape[0] == 1:
        m = m[0]
    if m.dim() != 2:
        raise ValueError("array masks must be 2-D (T_q, T_kv)")
    m = m.expand(tq, tkv)
    if m.dtype == torch.bool:
        return m.to(torch.float32).contiguous(), 1, False
    return m.to(torch.float32).contiguous(), 0, False


def sunshape_sdpa(queries, cache, scale: float, mask=None, *, check: bool = False,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """Scaled dot-product attention over a SunShape cache (attention.py:166-352).

    queries (B, n_q_heads, T_q, D) in the model basis; the cache's key indices,
    value payload and (hybrid) fp16 tail are read in place. Output has the
    queries' dtype.

    Every call first raises SunShapeCudaError (timeout) if an earlier launch
    gave up on a bounded device-side wait (its output was invalid); with
    ``check=True`` the call also synchronizes and checks its own launch.

    ``out`` (optional, queries' shape and dtype) receives the result: a CUDA
    tensor, or a page-locked host tensor that the kernel writes in place
    (the result then needs no separate device-to-host copy; it is complete
    once the stream reaches this point).
    """
    L.poll_device_errors()
    res = _sdpa(queries, cache, scale, mask, out)
    if check:
        L.check_device_errors(cache.device)
    return res


def _sdpa(queries, cache, scale: float, mask=None, out_user=None) -> torch.Tensor:
    q = K.cuda_tensor(queries, device=cache.device)
    if out_user is not None:
        if tuple(out_user.shape) != tuple(q.shape) or out_user.dtype != q.dtype:
            raise ValueError("out must have the queries' shape and dtype")
        if not (out_user.is_cuda or out_user.is_pinned()) or out_user.stride(-1) != 1:
            raise ValueError("out must be a CUDA or page-locked host tensor, contiguous in head_dim")
        if not out_user.is_cuda and not q.is_contiguous():
            raise ValueError("a host out needs contiguous queries")
    B, Hq, Tq, D = q.shape
    if Hq % cache.n_kv_heads:
        raise ValueError("n_q_heads must be a multiple of n_kv_heads")
    tkv = cache.offset
    if tkv == 0:
        if out_user is not None:
            out_user.zero_()
            return out_user
        return torch.zeros_like(q)
    if mask is None and (isinstance(cache, SunShapeKVCache) or
                         (isinstance(cache, HybridSunShapeKVCache) and cache._buffer_offset == 0)):
        return _sdpa_simple_fast(q, cache, scale, out_user)
    codec = cache.codec
    spec = cache.attention_spec()
    m, mode, causal = _prepare_mask(mask, Tq, tkv, q.device)
    spec["mask_mode"] = mode
    out = out_user if out_user is not None else torch.empty_like(q)
    perm = codec.permutation if codec._is_perm() else None
    rot_k = codec.rotation.contiguous() if codec.use_rotation else None
    n_heavy = codec.n_heavy_blocks if spec.get("kheavy") is not None else 0
    _run_decode(q, centroids=codec.centroids, perm=perm, scale=scale, spec=spec, causal=causal,
                out=out, mask=m, rot_k=rot_k, heavy=codec.heavy_u8, n_heavy=n_heavy)
    codec.last_score_backend = "cuda_fused"
    return out


def _sdpa_simple_fast(q: torch.Tensor, cache, scale: float, out_user=None) -> torch.Tensor:
    """sunshape_sdpa without a mask for the simple cache, or a hybrid cache
    whose fp16 tail is empty (then every token is compressed): the argument block
    is kept on the cache and rebuilt only when the storage is reallocated or
    the query layout, dtype or scale changes; per call only the query and
    output pointers and the token count are updated."""
    codec = cache.codec
    vcod = getattr(cache, "value_codec", None)
    key = (cache._epoch, tuple(q.shape), tuple(q.stride()), q.dtype, float(scale),
           codec.centroids.data_ptr(), codec.permutation.data_ptr(), codec.use_rotation,
           None if vcod is None else (vcod.centroids.data_ptr(), vcod.centroids._version))
    memo = cache._sdpa_memo
    pend = getattr(cache, "_pending", None)
    if memo is None or memo[0] != key:
        spec = cache.attention_spec(flush=False) if pend is not None else cache.attention_spec()
        perm = codec.permutation if codec._is_perm() else None
        rot_k = codec.rotation.contiguous() if codec.use_rotation else None
        n_heavy = codec.n_heavy_blocks if spec.get("kheavy") is not None else 0
        out = torch.empty_like(q)
        a, keep = _fill_args(q, codec.centroids, perm, scale, spec, False, out, None, rot_k,
                             codec.heavy_u8, n_heavy)
        keep += [spec, rot_k]
        lib = L.load()
        memo = (key, a, keep, lib, C.byref(a), {})
        cache._sdpa_memo = memo
    _, a, _, lib, ref, ws_by_tiles = memo
    if out_user is not None and out_user.stride() != q.stride():
        raise ValueError("out must have the queries' strides")
    out = out_user if out_user is not None else torch.empty_like(q)
    a.q = q.data_ptr()
    a.out = out.data_ptr()
    a.tc = cache.offset
    # the workspace size depends on the token count only through its tiles;
    # workspaces belong to a stream
    sp = torch.cuda.current_stream(q.device).cuda_stream
    tiles = ((cache.offset + 127) >> 7, sp)
    ws = ws_by_tiles.get(tiles)
    if ws is None:
        nbytes = lib.ss_decode_workspace_size(ref)
        if nbytes == 0:
            raise L.SunShapeCudaError("ss_decode_workspace_size", 1, L.last_error())
        ws = workspace_for(q.device, nbytes)
        if len(ws_by_tiles) > 64:
            ws_by_tiles.clear()
        ws_by_tiles[tiles] = ws
    a.workspace = ws.data_ptr()
    a.workspace_bytes = ws.numel()
    if pend is not None:
        # the deferred append of this step is written by this launch's table
        # kernel (ss_decode_args.app_*); fall back to a separate append when
        # the fused form does not apply
        k, v, o, T = pend
        a.app_keys, a.app_values, a.app_dtype = k.data_ptr(), v.data_ptr(), L.dtype_code(k.dtype)
        a.app_key_pair_stride, a.app_key_row_stride = k.stride(1), k.stride(2)
        a.app_value_pair_stride, a.app_value_row_stride = v.stride(1), v.stride(2)
        a.app_rows = T if o + T == cache.offset and k.dtype == v.dtype else 0
        if a.app_rows == 0:
            a.app_keys = None
            cache._flush_pending()
        rc = lib.ss_decode_attn(ref, C.c_void_p(sp))
        a.app_keys, a.app_values, a.app_rows = None, None, 0
        if rc == 2 and cache._pending is not None:  # unsupported fused form
            cache._flush_pending()
            rc = lib.ss_decode_attn(ref, C.c_void_p(sp))
        cache._pending = None
    else:
        rc = lib.ss_decode_attn(ref, C.c_void_p(sp))
    if rc:
        L.check("ss_decode_attn", rc)
    codec.last_score_backend = "cuda_fused"
    return out


def decode_partials(queries, cache, scale: float) -> torch.Tensor:
    """This shard's unnormalised (o, m, l) per query row, f32
    (B * Hq * Tq, D + 2): the input of the cross-GPU log-sum-exp merge."""
    L.poll_device_errors()
    q = K.cuda_tensor(queries, device=cache.device)
    B, Hq, Tq, D = q.shape
    part = torch.empty((B * Hq * Tq, D + 2), dtype=torch.float32, device=q.device)
    if cache.offset == 0:
        part[:, :D] = 0
        part[:, D] = float("-inf")
        part[:, D + 1] = 0
        return part
    codec = cache.codec
    spec = cache.attention_spec()
    perm = codec.permutation if codec._is_perm() else None
    rot_k = codec.rotation.contiguous() if codec.use_rotation else None
    n_heavy = codec.n_heavy_blocks if spec.get("kheavy") is not None else 0
    _run_decode(q, centroids=codec.centroids, perm=perm, scale=scale, spec=spec, causal=False,
                out=None, rot_k=rot_k, heavy=codec.heavy_u8, n_heavy=n_heavy, part_out=part)
    return part


class PreparedDecode:
    """A decode launch with its argument block built once: ``run()`` is a
    single C call (no tensor allocation), suitable for tight decode loops and
    CUDA-graph capture. The cache must not be reallocated (grown) between
    ``run()`` calls; queries are read from ``q`` and the result written to
    ``out`` in place."""

    def __init__(self, q: torch.Tensor, cache, scale: float, out: torch.Tensor | None = None,
                 max_ctas: int = 0, wait_limit_ns: int = 0, _test_skip_tile: int = -1,
                 part_out: torch.Tensor | None = None):
        codec = cache.codec
        self.q = q
        # part_out (B*Hq*Tq, D+2) f32: write this shard's (o, m, l) rows instead
        # of the output (the split-KV step, ss_decode_attn_partial)
        self.part_out = part_out
        self.out = None if part_out is not None else (out if out is not None else torch.empty_like(q))
        spec = cache.attention_spec()
        spec["max_ctas"] = max_ctas
        perm = codec.permutation if codec._is_perm() else None
        rot_k = codec.rotation.contiguous() if codec.use_rotation else None
        n_heavy = codec.n_heavy_blocks if spec.get("kheavy") is not None else 0
        self._a, self._keep = _fill_args(q, codec.centroids, perm, scale, spec, False, self.out,
                                         None, rot_k, codec.heavy_u8, n_heavy)
        self._keep += [spec, rot_k]
        lib = L.load()
        nbytes = lib.ss_decode_workspace_size(C.byref(self._a))
        if nbytes == 0:
            raise L.SunShapeCudaError("ss_decode_workspace_size", 1, L.last_error())
        self.ws = workspace_for(q.device, nbytes)
        self._a.workspace = self.ws.data_ptr()
        self._a.workspace_bytes = self.ws.numel()
        # bound of the kernel's device-side waits (0: 2 s); the skip hook makes
        # the waits on one tile run out (tests of the timeout path)
        self._a.wait_limit_ns = int(wait_limit_ns)
        self._a.test_skip_tile = int(_test_skip_tile) + 1 if _test_skip_tile >= 0 else 0
        self._lib = lib
        self._ref = C.byref(self._a)
        self._part_ptr = C.c_void_p(part_out.data_ptr()) if part_out is not None else None
        self.device = q.device

    def run(self, stream=None, check: bool = False) -> torch.Tensor:
        """One launch. Raises first if an earlier launch gave up on a bounded
        device-side wait; ``check=True`` also synchronizes the stream and
        checks this launch."""
        w = L._SINK_WORD
        if w is not None and w.value:
            L.poll_device_errors()
        st = C.c_void_p(stream if stream is not None else torch.cuda.current_stream(self.device).cuda_stream)
        if self.part_out is None:
            rc = self._lib.ss_decode_attn(self._ref, st)
        else:
            rc = self._lib.ss_decode_attn_partial(self._ref, self._part_ptr, st)
        if rc:
            L.check("ss_decode_attn", rc)
        if check:
            if stream is not None:
                torch.cuda.synchronize(self.device)
            L.check_device_errors(self.device)
        return self.out if self.part_out is None else self.part_out
