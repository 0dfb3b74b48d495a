"""aethelstream_b200 -- B200 (sm_100a) per-layer optimizer step of AethelStream.

NF4 weight dequantisation, GaLore projection (tcgen05 tensor cores), INT8
low-rank Adam, back-projection with a fused NF4 weight write, and a LOMO fused
full-rank update, behind the C ABI in include/aeth_galore.h.  Importing this
package loads libaeth_galore.so and raises ImportError if it is missing: there
is no CPU fallback.
"""
from . import _lib
from ._lib import AethError, load

load()  # fail loudly at import time when the native library is absent

from .galore import (  # noqa: E402
    AdamWConfig,
    apply_galore_bf16_update,
    decode_int4_to_fp16,
    decode_int8_to_fp16,
    ClipResult,
    GaLoreConfig,
    GaLoreOptimizer,
    LayerRankConfig,
    LomoState,
    NF4Tensor,
    ProjectorKind,
    deferred_apply_with_clip,
    lomo_sqnorm,
    lomo_update,
    nf4_dequantize,
    nf4_quantize,
    randomized_svd,
    randomized_svd_fast,
    randomized_svd_sketch,
)

__all__ = [
    "AdamWConfig", "apply_galore_bf16_update", "decode_int4_to_fp16", "decode_int8_to_fp16", "AethError", "ClipResult", "GaLoreConfig", "GaLoreOptimizer", "LayerRankConfig", "LomoState", "NF4Tensor",
    "ProjectorKind", "deferred_apply_with_clip", "load", "lomo_sqnorm", "lomo_update", "nf4_dequantize", "nf4_quantize", "randomized_svd", "randomized_svd_fast", "randomized_svd_sketch",
    "_lib",
]
