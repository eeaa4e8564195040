"""Value codecs for hybrid SunShape caches (value_codecs.py of the reference).

Both encoders run as sm_100a kernels. ``TurboQuantValueCodec`` keeps the
reference's format (per-token float32 norm, Haar rotation, Lloyd-Max levels
scaled by 1/sqrt(D)) by default; ``group_size`` selects the per-group scaled
variant (fp16 RMS scale per group of channels in the rotated basis) used by
the long-context benchmark configurations.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from . import _lib as L
from . import kernels as K
from .rotation import generate_rotation_matrix

__all__ = ["GroupedValueCodec", "TurboQuantValueCodec", "build_value_codec",
           "TURBOQUANT_CODEBOOKS"]

# Lloyd-Max optimal scalar quantizers of N(0, 1) (levels, decision
# boundaries) for 1-4 bits -- the published tables the reference embeds at
# value_codecs.py:20-87.
TURBOQUANT_CODEBOOKS: dict[int, tuple[list[float], list[float]]] = {
    1: ([-0.7978845608028654, 0.7978845608028654], [0.0]),
    2: ([-1.510417608611893, -0.4527800346911237, 0.4527800346911237, 1.510417608611893],
        [-0.9815988216515084, 0.0, 0.9815988216515084]),
    3: ([-2.151945705166112, -1.3439092791423422, -0.7560052816730181, -0.2450941791152904,
         0.2450941791152904, 0.7560052816730181, 1.3439092791423422, 2.151945705166112],
        [-1.7479274921542272, -1.0499572804076802, -0.5005497303941542, 0.0,
         0.5005497303941542, 1.0499572804076802, 1.7479274921542272]),
    4: ([-2.732896755154294, -2.069364258154187, -1.618400443227723, -1.2565648452462146,
         -0.9426291036999694, -0.6569817464411519, -0.38818871416000605, -0.12844300124876415,
         0.12844300124876415, 0.38818871416000605, 0.6569817464411519, 0.9426291036999694,
         1.2565648452462146, 1.618400443227723, 2.069364258154187, 2.732896755154294],
        [-2.4011305066542405, -1.8438823506909552, -1.4374826442369688, -1.099596974473092,
         -0.7998054250705606, -0.522585230300579, -0.2583158577043851, 0.0,
         0.2583158577043851, 0.522585230300579, 0.7998054250705606, 1.099596974473092,
         1.4374826442369688, 1.8438823506909552, 2.4011305066542405]),
}


def _rows(x: torch.Tensor):
    """(x as (G, T, D) strided view, G, T)."""
    if x.dim() == 1:
        x = x[None]
    x3 = x.reshape(-1, *x.shape[-2:]) if x.dim() > 2 else x[None]
    return x3, x3.shape[0], x3.shape[1]


@dataclass
class GroupedValueCodec:
    """Asymmetric per-group min-max values (value_codecs.py:104-133)."""
    head_dim: int
    bits: int
    group_size: int = 64
    name: str = "grouped"
    last_quantize_backend: str = "cuda"

    @property
    def packed_dim(self) -> int:
        return K.packed_dim(self.head_dim, self.bits)

    @property
    def n_groups(self) -> int:
        return self.head_dim // self.group_size

    def levels(self, device) -> list[float]:
        return [float(i) for i in range(2 ** self.bits)]

    def quantize(self, values):
        p, s, z, _ = K.quantize_values(values, bits=self.bits, group_size=self.group_size)
        self.last_quantize_backend = "cuda"
        return p, s, z

    def quantize_into(self, values: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor,
                      zeros: torch.Tensor) -> None:
        """Encodes (G, T, D) rows straight into strided cache slices."""
        v3, g, t = _rows(values)
        p3, _, _ = _rows(packed)
        s3, _, _ = _rows(scales)
        z3, _, _ = _rows(zeros)
        if s3.stride() != z3.stride():
            raise ValueError("scales and zeros must share strides")
        L.call("ss_value_encode_grouped", L.ptr(v3), L.dtype_code(v3.dtype), g, t, v3.stride(0),
               v3.stride(1), self.head_dim, self.bits, self.group_size, L.ptr(p3), p3.stride(0),
               p3.stride(1), L.ptr(s3), L.ptr(z3), s3.stride(0), s3.stride(1),
               L.stream_ptr(v3.device))
        self.last_quantize_backend = "cuda"

    def dequantize(self, packed, scales, zeros, out_dtype=torch.float32) -> torch.Tensor:
        return K.dequantize_values(packed, scales, zeros, D=self.head_dim, bits=self.bits,
                                   group_size=self.group_size, out_dtype=out_dtype)


@dataclass
class TurboQuantValueCodec:
    """Rotated scalar-quantized values (value_codecs.py:136-177).

    group_size=None: the reference format (per-token f32 norm, levels/sqrt(D)).
    group_size=g: per-group fp16 scale s = ||r_g||/sqrt(g) in the rotated basis,
    levels unscaled (an extension used by the long-context configuration).
    """
    head_dim: int
    bits: int
    seed: int = 43
    prefer_metal: bool = True
    group_size: int | None = None
    device: object = None
    rotation: torch.Tensor | None = None
    name: str = "turboquant"
    last_quantize_backend: str = "none"
    centroids: torch.Tensor = field(init=False)
    boundaries: torch.Tensor = field(init=False)

    def __post_init__(self) -> None:
        if self.bits not in (2, 3, 4):
            raise ValueError(f"TurboQuant values support 2, 3, or 4 bits, got {self.bits}")
        if self.group_size is not None and self.head_dim % self.group_size:
            raise ValueError("head_dim must be a multiple of group_size")
        dev = torch.device(self.device) if self.device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.device = dev
        lv, bd = TURBOQUANT_CODEBOOKS[self.bits]
        sc = 1.0 / math.sqrt(self.head_dim) if self.group_size is None else 1.0
        self.centroids = torch.tensor([c * sc for c in lv], dtype=torch.float32, device=dev)
        self.boundaries = torch.tensor([b * sc for b in bd], dtype=torch.float32, device=dev)
        if self.rotation is None:
            self.rotation = generate_rotation_matrix(self.head_dim, seed=self.seed, device=dev)
        else:
            self.rotation = K.cuda_tensor(self.rotation, torch.float32, dev)
        self.rotation_t = self.rotation.T.contiguous()

    @property
    def packed_dim(self) -> int:
        return K.packed_dim(self.head_dim, self.bits)

    @property
    def mode(self) -> int:
        return 0 if self.group_size is None else 1

    @property
    def n_scale_groups(self) -> int:
        return 1 if self.group_size is None else self.head_dim // self.group_size

    @property
    def scale_dtype(self) -> torch.dtype:
        return torch.float32 if self.group_size is None else torch.float16

    def levels(self, device=None) -> list[float]:
        return [float(x) for x in self.centroids.cpu()]

    def quantize_into(self, values: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor) -> None:
        v3, g, t = _rows(values)
        p3, _, _ = _rows(packed)
        if scales.dim() == values.dim() - 1:  # per-token norms (..., T)
            s3 = scales.reshape(-1, scales.shape[-1]) if scales.dim() > 1 else scales[None]
            ss0, ss1 = s3.stride(0), s3.stride(1)
        else:
            s3, _, _ = _rows(scales)
            ss0, ss1 = s3.stride(0), s3.stride(1)
        L.call("ss_value_encode_tq", L.ptr(v3), L.dtype_code(v3.dtype), g, t, v3.stride(0),
               v3.stride(1), self.head_dim, self.bits, self.mode, self.group_size or self.head_dim,
               L.ptr(self.rotation), L.ptr(self.boundaries), L.ptr(p3), p3.stride(0),
               p3.stride(1), L.ptr(s3), ss0, ss1, L.stream_ptr(v3.device))
        self.last_quantize_backend = "cuda"

    def quantize(self, values):
        """Returns (packed words, norms (..,) f32) or (packed, scales (.., G) f16)."""
        v = K.cuda_tensor(values, device=self.device)
        if v.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            v = v.float()
        lead = v.shape[:-1]
        packed = torch.empty((*lead, self.packed_dim), dtype=torch.int32, device=v.device)
        if self.group_size is None:
            sc = torch.empty(lead, dtype=torch.float32, device=v.device)
        else:
            sc = torch.empty((*lead, self.n_scale_groups), dtype=torch.float16, device=v.device)
        self.quantize_into(v, packed, sc)
        return packed, sc

    def dequantize(self, packed, norms, out_dtype=torch.float32) -> torch.Tensor:
        p = K.cuda_tensor(packed, device=self.device)
        if p.dtype != torch.int32:
            p = p.view(torch.int32) if p.element_size() == 4 else p.to(torch.int32)
        s = K.cuda_tensor(norms, device=self.device)
        d = self.head_dim
        g = self.n_scale_groups
        rows = p.numel() // p.shape[-1]
        out = torch.empty((*p.shape[:-1], d), dtype=out_dtype, device=p.device)
        sdt = L.SS_F32 if s.dtype == torch.float32 else L.SS_F16
        L.call("ss_value_decode", L.ptr(p), 1, rows, 0, p.shape[-1], d, self.bits,
               self.group_size or d, L.ptr(self.centroids), L.ptr(s), sdt, None, 0, g,
               L.ptr(self.rotation), L.ptr(out), L.dtype_code(out_dtype), 0, d,
               L.stream_ptr(p.device))
        return out


def build_value_codec(value_backend: str, *, head_dim: int, value_bits: int,
                      value_group_size: int = 64, value_seed: int = 43, prefer_metal: bool = True,
                      tq_group_size: int | None = None, device=None):
    """value_codecs.py:180-201."""
    if value_backend == "fp16":
        return None
    if value_backend == "grouped":
        return GroupedValueCodec(head_dim=head_dim, bits=value_bits, group_size=value_group_size)
    if value_backend == "turboquant":
        return TurboQuantValueCodec(head_dim=head_dim, bits=value_bits, seed=value_seed,
                                    prefer_metal=prefer_metal, group_size=tq_group_size,
                                    device=device)
    raise ValueError(f"Unsupported value backend: {value_backend}")
