"""SunShape block-VQ KV-cache compression on NVIDIA B200 (sm_100a).

Drop-in for the hot path of gauravsaini/sunshape-mlx: the codec
(fit / quantize / dequantize / attention_scores), the KV caches and the
SDPA entry, with every on-device step a hand-written CUDA kernel behind the
C ABI in include/sunshape_b200.h. Tensors are torch CUDA tensors.
"""

from .rotation import (
    apply_permutation,
    apply_wht,
    block_affinity_gate,
    block_local_cov_metric,
    covariance_block_permutation,
    generate_rotation_matrix,
    generate_wht_signs,
    invert_permutation,
    mixed_precision_block_mask,
    positive_excess_kurtosis,
    safe_normalize,
)
from .codec import SunShapeBlockCodec, SunShapeQuantized
from .cache import (HybridSunShapeKVCache, SunShapeKVCache, create_kv_cache, load_cache,
                    save_cache)
from .attention import sunshape_sdpa
from .kernels import (
    block_vq_quantize_metal,
    block_vq_score_metal,
    dequantize_values,
    fused_attention_causal_metal,
    fused_attention_dequant_causal_metal,
    fused_attention_dequant_metal,
    fused_attention_metal,
    fused_block_vq_attention,
    get_kernel_stats,
    pack_indices,
    quantize_values,
    reset_kernel_stats,
    unpack_indices,
)
from .value_codecs import GroupedValueCodec, TurboQuantValueCodec

__version__ = "0.3.0+b200"

__all__ = [
    "SunShapeBlockCodec", "SunShapeQuantized", "SunShapeKVCache", "HybridSunShapeKVCache",
    "sunshape_sdpa", "generate_rotation_matrix", "generate_wht_signs", "apply_wht",
    "covariance_block_permutation", "invert_permutation", "apply_permutation",
    "block_local_cov_metric", "block_affinity_gate", "mixed_precision_block_mask",
    "positive_excess_kurtosis", "safe_normalize", "pack_indices", "unpack_indices",
    "quantize_values", "dequantize_values", "fused_block_vq_attention", "fused_attention_metal",
    "fused_attention_causal_metal", "fused_attention_dequant_metal",
    "fused_attention_dequant_causal_metal", "block_vq_quantize_metal", "GroupedValueCodec",
    "TurboQuantValueCodec", "create_kv_cache", "get_kernel_stats", "reset_kernel_stats",
    "save_cache", "load_cache",
]
