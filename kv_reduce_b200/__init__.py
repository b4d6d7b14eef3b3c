"""kv_reduce_b200: B200-native (sm_100a) packed draft-KV cache and decode attention.

Drop-in for the packed draft-KV path of KV_Reduce:
  * ``kv_reduce_b200.packed_kv_cache``     <- kv_reduce.packed_kv_cache
  * ``kv_reduce_b200.packed_kv_attention`` <- kv_reduce.triton_packed_kv_attention
  * ``kv_reduce_b200.streaming``           <- PackedLayer / PackedCache of
    kv_reduce/experiments/packed_review.py, on a preallocated cache
All compute runs in libkvr.so (CUDA C++ for sm_100a, C ABI in include/kvr.h).
"""
from .packed_kv_cache import (  # noqa: F401
    FULL_PRECISION_BITS,
    PackedKVComponent,
    key_scale_pairs,
    pack_kivi_kv,
    pack_per_channel_grouped_affine,
    pack_per_token_affine,
    pack_unsigned,
    packed_num_bytes,
    tensor_bytes,
    unpack_unsigned,
)
from .packed_kv_attention import (  # noqa: F401
    DecodeLaunch,
    PackedDecoder,
    SimtDecodeLaunch,
    check_finite_outputs,
    lse_merge,
    packed_kv_decode_attention,
    packed_kv_decode_attention_layers,
    packed_kv_decode_attention_simt,
    theoretical_attention_flops,
)
from .streaming import PackedCache, PackedKVCache, PackedKVCacheLayer, PackedLayer  # noqa: F401

__version__ = "0.1.0"
