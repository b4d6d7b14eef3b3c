"""``torch.ops.kvr.*``: the packed draft-KV path as PyTorch operators.

The decode operators are C++ (libkvr_torch.so, ``TORCH_LIBRARY(kvr, m)`` over
libkvr.so's C ABI): their checks, stride and pointer work and launch run
without Python.  The packing operators are Python custom operators over the
packing kernels.  Every operator has a fake (meta) implementation giving
output shapes and dtypes without running anything, so code that calls the
path can be traced by ``torch.compile`` / ``torch.export`` and captured in
CUDA graphs with the library kernels as opaque nodes.

    kvr::pack_per_token(values, bits) -> (payload, scale, offset)
        packed_kv_cache.py:159-192
    kvr::pack_grouped(keys, bits, group_size, residual_length)
        -> (payload, scale, offset, residual)          packed_kv_cache.py:195-253
    kvr::decode_attention(query, key_payload, key_scale, key_offset,
        key_residual, value_payload, value_scale, value_offset, seq_len,
        key_bits, value_bits, group_size, prefix_len, split_tokens=0,
        block_tokens=32, out_fp32=False, shapes=None, layouts=3,
        key_scale_pairs=None) -> out                   triton_packed_kv_attention.py:284-389
    kvr::decode_step(query, k_new, v_new, <streaming layer buffers>, lengths,
        geom, key_scale_pairs=None) -> out
                              packed_review.py:23-31 + :78 on a streaming layer
    kvr::lse_merge(part_ml, part_o) -> out           (cross-GPU partial merge)

Import this module to register them.
"""
from __future__ import annotations

from typing import Tuple

import torch

from . import _lib
from .packed_kv_attention import scale_pairs_of
from .packed_kv_cache import (
    PackedKVComponent,
    _quantized_prefix_length,
    pack_per_channel_grouped_affine,
    pack_per_token_affine,
    packed_num_bytes,
)

Tensor = torch.Tensor

_lib.load_torch_ops()


@torch.library.register_fake("kvr::decode_attention")
def _(query, key_payload, key_scale, key_offset, key_residual, value_payload, value_scale, value_offset,
      seq_len, key_bits, value_bits, group_size, prefix_len, split_tokens=0, block_tokens=32, out_fp32=False,
      shapes=None, layouts=3, key_scale_pairs=None):
    return query.new_empty(query.shape, dtype=torch.float32 if out_fp32 else query.dtype)


@torch.library.register_fake("kvr::decode_step")
def _(query, k_new, v_new, key_payload, key_scale, key_offset, key_residual, value_payload, value_scale,
      value_offset, lengths, geom, key_scale_pairs=None):
    return query.new_empty(query.shape)


@torch.library.register_fake("kvr::lse_merge")
def _(part_ml, part_o):
    return part_o.new_empty((int(part_o.shape[1]), int(part_o.shape[2])), dtype=torch.bfloat16)


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


def decode_attention_from(query: Tensor, packed_keys: PackedKVComponent, packed_values: PackedKVComponent, *,
                          split_tokens: int = 0) -> Tensor:
    """``torch.ops.kvr.decode_attention`` over packed components."""
    return torch.ops.kvr.decode_attention(
        query, packed_keys.payload, packed_keys.scale, packed_keys.offset, packed_keys.residual,
        packed_values.payload, packed_values.scale, packed_values.offset, int(packed_keys.shape[-2]),
        int(packed_keys.bits), int(packed_values.bits), int(packed_keys.group_size),
        int(packed_keys.prefix_length), int(split_tokens), key_scale_pairs=scale_pairs_of(packed_keys))
