"""torque_mlx_b200 — B200-native (sm_100a) packed-KV decode path of torque-mlx.

Rotation-native KV cache: keys/values rotated by Pi = D1 H D2 / sqrt(d),
quantized to a global 2/3/4-bit Lloyd-Max codebook and bit-packed into uint32
words; decode attention runs straight on the packed codes.  The public names
mirror the reference package ``torque_mlx``; all compute runs in the CUDA
library ``libtorque_b200.so`` (C ABI in include/torque_b200.h).
"""

from .config import RotationMode, TorqueConfig
from .layout import CacheMetadata, PackedKVLayout, build_variant_id
from .quantization import (
    SUPPORTED_BIT_WIDTHS,
    WORD_BITS,
    Codebook,
    build_gaussian_codebook,
    codebook_boundaries,
    dequantize,
    kv_bytes_per_token,
    load_codebook,
    pack_indices,
    pack_indices_batched,
    packed_words_for_head_dim,
    quantize,
    save_codebook,
    unpack_indices,
)
from .rotation import RotationSpec, apply_structured_rotation, validate_head_dim
from .cache import TorqueKVCache, TorqueKVCacheB200, TorqueKVCacheMLX
from .ops import (
    cuda_available,
    decode_packed_attention,
    decode_packed_attention_split,
    decode_packed_attention_split_batched,
    decode_packed_attention_split_batched_with_current,
    dequantize_packed,
    lse_merge,
    quantize_and_pack_rows,
    quantize_and_pack_rows_dual,
    quantize_and_pack_rows_dual_metal,
    quantize_and_pack_rows_metal,
)

__all__ = [
    "CacheMetadata", "Codebook", "PackedKVLayout", "RotationMode", "RotationSpec", "SUPPORTED_BIT_WIDTHS",
    "TorqueConfig", "TorqueKVCache", "TorqueKVCacheB200", "TorqueKVCacheMLX", "WORD_BITS",
    "apply_structured_rotation", "build_gaussian_codebook", "build_variant_id", "codebook_boundaries",
    "cuda_available", "decode_packed_attention", "decode_packed_attention_split",
    "decode_packed_attention_split_batched", "decode_packed_attention_split_batched_with_current", "dequantize",
    "dequantize_packed", "kv_bytes_per_token", "load_codebook", "lse_merge", "pack_indices", "pack_indices_batched",
    "packed_words_for_head_dim", "quantize", "quantize_and_pack_rows", "quantize_and_pack_rows_dual",
    "quantize_and_pack_rows_dual_metal", "quantize_and_pack_rows_metal",
    "save_codebook", "unpack_indices", "validate_head_dim",
]
from .artifact import (  # noqa: E402
    TorqueArtifact,
    TorqueArtifactManifest,
    build_torque_artifact,
    convert_npz_checkpoint,
    load_torque_artifact,
)
from .conversion import FusedAttentionWeights, fuse_attention_weights  # noqa: E402

__all__ += ["FusedAttentionWeights", "TorqueArtifact", "TorqueArtifactManifest", "build_torque_artifact",
            "convert_npz_checkpoint", "fuse_attention_weights", "load_torque_artifact"]
