"""``torch.ops.kvr.*``: the packed draft-KV path as PyTorch custom operators.

Each operator wraps one library launcher over plain tensors (the fields of
the packed components) and has a fake (meta) implementation giving output
shapes and dtypes without running anything, so code that calls the path can
be traced by ``torch.compile`` / ``torch.export`` and captured in CUDA
graphs with the library kernels as opaque nodes.

    kvr::pack_per_token(values, bits) -> (payload, scale, offset)
        packed_kv_cache.py:159-192
    kvr::pack_grouped(keys, bits, group_size, residual_length)
        -> (payload, scale, offset, residual)          packed_kv_cache.py:195-253
    kvr::decode_attention(query, key_payload, key_scale, key_offset,
        key_residual, value_payload, value_scale, value_offset, seq_len,
        key_bits, value_bits, group_size, prefix_len, split_tokens) -> out
        triton_packed_kv_attention.py:284-389
    kvr::lse_merge(part_ml, part_o) -> out           (cross-GPU partial merge)

Import this module to register them.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .packed_kv_attention import lse_merge as _lse_merge
from .packed_kv_attention import packed_kv_decode_attention
from .packed_kv_cache import (
    PackedKVComponent,
    _quantized_prefix_length,
    pack_per_channel_grouped_affine,
    pack_per_token_affine,
    packed_num_bytes,
)

Tensor = torch.Tensor


@torch.library.custom_op("kvr::pack_per_token", mutates_args=())
def pack_per_token(values: Tensor, bits: int) -> Tuple[Tensor, Tensor, Tensor]:
    if not 2 <= bits <= 8:
        raise ValueError("kvr::pack_per_token packs 2- to 8-bit codes.")
    c = pack_per_token_affine(values, bits)
    return c.payload, c.scale, c.offset


@pack_per_token.register_fake
def _(values: Tensor, bits: int) -> Tuple[Tensor, Tensor, Tensor]:
    payload = values.new_empty(packed_num_bytes(values.numel(), bits), dtype=torch.uint8)
    meta = (*values.shape[:-1], 1)
    return payload, values.new_empty(meta, dtype=torch.bfloat16), values.new_empty(meta, dtype=torch.bfloat16)


@torch.library.custom_op("kvr::pack_grouped", mutates_args=())
def pack_grouped(keys: Tensor, bits: int, group_size: int, residual_length: int
                 ) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    if not 2 <= bits <= 8:
        raise ValueError("kvr::pack_grouped packs 2- to 8-bit codes.")
    c = pack_per_channel_grouped_affine(keys, bits, group_size=group_size, residual_length=residual_length)
    # the residual can be a view of the input (one b*h slab): an operator output must own its storage
    return c.payload, c.scale, c.offset, c.residual.clone()


@pack_grouped.register_fake
def _(keys: Tensor, bits: int, group_size: int, residual_length: int) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    seq_len, head_dim = int(keys.shape[-2]), int(keys.shape[-1])
    prefix = _quantized_prefix_length(seq_len, group_size, residual_length)
    residual = keys.new_empty((*keys.shape[:-2], seq_len - prefix, head_dim))
    if prefix == 0:
        empty_meta = keys.new_empty(0, dtype=torch.bfloat16)
        return keys.new_empty(0, dtype=torch.uint8), empty_meta, keys.new_empty(0, dtype=torch.bfloat16), residual
    bh = keys.numel() // (seq_len * head_dim)
    meta = (*keys.shape[:-2], prefix // group_size, 1, head_dim)
    return (keys.new_empty(packed_num_bytes(bh * prefix * head_dim, bits), dtype=torch.uint8),
            keys.new_empty(meta, dtype=torch.bfloat16), keys.new_empty(meta, dtype=torch.bfloat16), residual)


@torch.library.custom_op("kvr::decode_attention", mutates_args=())
def decode_attention(query: Tensor, key_payload: Tensor, key_scale: Tensor, key_offset: Tensor,
                     key_residual: Optional[Tensor], value_payload: Tensor, value_scale: Tensor,
                     value_offset: Tensor, seq_len: int, key_bits: int, value_bits: int, group_size: int,
                     prefix_len: int, split_tokens: int) -> Tensor:
    batch, head_dim = int(query.shape[0]), int(query.shape[-1])
    kv_heads = int(value_scale.shape[1]) if value_scale.dim() >= 3 else 1
    shape = (batch, kv_heads, int(seq_len), head_dim)
    k = PackedKVComponent(key_payload, key_scale, key_offset, key_residual, shape, int(key_bits),
                          "per_channel_grouped_affine", query.dtype, int(group_size), int(prefix_len))
    v = PackedKVComponent(value_payload, value_scale, value_offset, None, shape, int(value_bits),
                          "per_token_affine", query.dtype)
    return packed_kv_decode_attention(query, k, v, split_tokens=split_tokens)


@decode_attention.register_fake
def _(query, key_payload, key_scale, key_offset, key_residual, value_payload, value_scale, value_offset,
      seq_len, key_bits, value_bits, group_size, prefix_len, split_tokens):
    return torch.empty_like(query)


@torch.library.custom_op("kvr::lse_merge", mutates_args=())
def lse_merge(part_ml: Tensor, part_o: Tensor) -> Tensor:
    return _lse_merge(part_ml, part_o)


@lse_merge.register_fake
def _(part_ml: Tensor, part_o: Tensor) -> Tensor:
    return part_o.new_empty((int(part_o.shape[1]), int(part_o.shape[2])), dtype=torch.bfloat16)


def decode_attention_from(query: Tensor, packed_keys: PackedKVComponent, packed_values: PackedKVComponent, *,
                          split_tokens: int = 0) -> Tensor:
    """``torch.ops.kvr.decode_attention`` over packed components."""
    return torch.ops.kvr.decode_attention(
        query, packed_keys.payload, packed_keys.scale, packed_keys.offset, packed_keys.residual,
        packed_values.payload, packed_values.scale, packed_values.offset, int(packed_keys.shape[-2]),
        int(packed_keys.bits), int(packed_values.bits), int(packed_keys.group_size),
        int(packed_keys.prefix_length), int(split_tokens))
