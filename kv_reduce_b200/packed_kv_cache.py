"""Bit-packed KV tensors: the API of kv_reduce/packed_kv_cache.py on sm_100a.

Same names, argument meaning, layouts and ``ValueError`` preconditions as the
reference module (kv_reduce/packed_kv_cache.py:15-275); every byte of
payload and every bf16 metadata bit is produced by CUDA kernels in libkvr.so
and is bit-identical to the reference's output for the same bf16 input.

Differences, all raised as errors rather than silently handled:
  * tensors must live on a CUDA device (the reference also runs on CPU);
  * inputs must be bf16 and ``metadata_dtype`` bf16 (the reference accepts
    other float dtypes; bf16 is what its draft-cache path uses).
"""
from __future__ import annotations

from dataclasses import dataclass
from math import ceil
from typing import Tuple

import torch

from . import _lib

FULL_PRECISION_BITS = 16


def _quantized_prefix_length(seq_len: int, group_size: int, residual_length: int) -> int:
    """P = floor(max(0, S - R) / G) * G  (packed_kv_cache.py:15-19)."""
    if group_size <= 0 or residual_length < 0:
        raise ValueError("group_size must be positive and residual_length non-negative.")
    eligible = max(0, int(seq_len) - int(residual_length))
    return (eligible // int(group_size)) * int(group_size)


def packed_num_bytes(num_values: int, bits: int) -> int:
    """ceil(n * bits / 8)  (packed_kv_cache.py:22-25)."""
    if bits < 1 or bits > 8:
        raise ValueError("Packed values require between 1 and 8 bits.")
    return ceil(int(num_values) * int(bits) / 8)


def tensor_bytes(tensor: torch.Tensor | None) -> int:
    """Logical bytes of a tensor (packed_kv_cache.py:97-98)."""
    return 0 if tensor is None else tensor.numel() * tensor.element_size()


def pack_unsigned(values: torch.Tensor, bits: int) -> torch.Tensor:
    """Pack unsigned codes into a flat LSB-first uint8 stream (packed_kv_cache.py:28-63)."""
    if bits < 1 or bits > 8:
        raise ValueError("bits must be in [1, 8].")
    flat = values.reshape(-1).to(torch.uint8).contiguous()
    if flat.numel() == 0:
        return torch.empty(0, dtype=torch.uint8, device=values.device)
    dev = _lib.require_cuda(flat)
    maximum = int(flat.max().item())
    if maximum >= (1 << bits):
        raise ValueError(f"Value {maximum} cannot be represented with {bits} bits.")
    out = torch.empty(packed_num_bytes(flat.numel(), bits), dtype=torch.uint8, device=dev)
    _lib.call("kvr_pack_unsigned", flat.data_ptr(), flat.numel(), bits, out.data_ptr(), _lib.stream_ptr(dev))
    return out


def unpack_unsigned(payload: torch.Tensor, bits: int, num_values: int) -> torch.Tensor:
    """Inverse of pack_unsigned (packed_kv_cache.py:66-94)."""
    if bits < 1 or bits > 8:
        raise ValueError("bits must be in [1, 8].")
    if payload.dtype != torch.uint8:
        raise ValueError("payload must have dtype torch.uint8.")
    expected = packed_num_bytes(num_values, bits)
    if payload.numel() != expected:
        raise ValueError(f"Expected {expected} packed bytes, received {payload.numel()}.")
    if num_values == 0:
        return torch.empty(0, dtype=torch.uint8, device=payload.device)
    dev = _lib.require_cuda(payload)
    src = payload.reshape(-1).contiguous()
    out = torch.empty(num_values, dtype=torch.uint8, device=dev)
    _lib.call("kvr_unpack_unsigned", src.data_ptr(), num_values, bits, out.data_ptr(), _lib.stream_ptr(dev))
    return out


def _numel(shape: Tuple[int, ...]) -> int:
    result = 1
    for dimension in shape:
        result *= int(dimension)
    return result


def _bh_stride(t: torch.Tensor, compact: int, what: str) -> int:
    """Stride between consecutive (b, h) slabs of a packed tensor.

    A flat / fully contiguous tensor (the reference's layout) has slabs of
    `compact` elements back to back.  A view [B, H, ...] into a larger
    capacity buffer (kv_reduce_b200.streaming) carries its slab stride in
    dimension 1; the trailing dimensions must be contiguous.
    """
    if t.dim() <= 1 or t.is_contiguous():
        return compact
    if t.dim() < 3 or t.stride(0) != t.shape[1] * t.stride(1):
        raise ValueError(f"{what}: unsupported strides {tuple(t.stride())}.")
    inner = t[0, 0]
    if not inner.is_contiguous():
        raise ValueError(f"{what}: inner dimensions must be contiguous.")
    return t.stride(1)


_OUT_DTYPES = {torch.bfloat16: 0, torch.float32: 1, torch.float16: 2}


@dataclass
class PackedKVComponent:
    """Packed storage record, fields as packed_kv_cache.py:101-112."""

    payload: torch.Tensor
    scale: torch.Tensor | None
    offset: torch.Tensor | None
    residual: torch.Tensor | None
    shape: Tuple[int, ...]
    bits: int
    layout: str
    output_dtype: torch.dtype
    group_size: int = 0
    prefix_length: int = 0
    # Keys only, optional: the scales as fp16 pairs in the decode kernel's
    # register order (key_scale_pairs), a lookup table derived from `scale`
    # when the group is packed.  Not part of the reference's record and not
    # counted in its byte properties; the decode reads it in place of `scale`.
    scale_pairs: torch.Tensor | None = None

    @property
    def payload_bytes(self) -> int:
        return tensor_bytes(self.payload) + tensor_bytes(self.residual)

    @property
    def metadata_bytes(self) -> int:
        return tensor_bytes(self.scale) + tensor_bytes(self.offset)

    @property
    def storage_bytes(self) -> int:
        return self.payload_bytes + self.metadata_bytes

    def unpack(self) -> torch.Tensor:
        """Dequantize to ``output_dtype`` on the GPU (packed_kv_cache.py:126-149).

        ``code * scale + offset`` in fp32 with two roundings, then a cast,
        bit-identical to the reference.
        """
        if self.layout == "native":
            return self.payload.reshape(self.shape)
        if self.layout not in ("per_token_affine", "per_channel_grouped_affine"):
            raise ValueError(f"Unsupported packed layout: {self.layout}")
        if self.output_dtype not in _OUT_DTYPES:
            raise ValueError(f"Unsupported output dtype {self.output_dtype}.")
        shape = tuple(int(s) for s in self.shape)
        seq_len, head_dim = shape[-2], shape[-1]
        bh = _numel(shape[:-2])
        src = self.payload if self.payload.numel() or self.residual is None else self.residual
        dev = _lib.require_cuda(src)
        out = torch.empty(shape, dtype=self.output_dtype, device=dev)
        if out.numel() == 0:
            return out
        a = _lib.DequantArgs()
        a.out = out.data_ptr()
        a.out_dtype = _OUT_DTYPES[self.output_dtype]
        a.bh, a.seq_len, a.head_dim, a.bits = bh, seq_len, head_dim, int(self.bits)
        row_bytes_num = head_dim * int(self.bits)
        if self.layout == "per_token_affine":
            rows = seq_len
            a.group_size = 0
            a.prefix_len = seq_len
        else:
            rows = int(self.prefix_length)
            a.group_size = int(self.group_size)
            a.prefix_len = rows
        if rows > 0:
            if row_bytes_num % 8 == 0:
                a.payload_bh_stride = _bh_stride(self.payload, rows * row_bytes_num // 8, "payload")
            a.payload = self.payload.data_ptr()
            meta_compact = rows if self.layout == "per_token_affine" else (rows // self.group_size) * head_dim
            _check_meta(self.scale, "scale")
            _check_meta(self.offset, "offset")
            a.meta_bh_stride = _bh_stride(self.scale, meta_compact, "scale")
            a.scale = self.scale.data_ptr()
            a.offset = self.offset.data_ptr()
        if self.layout == "per_channel_grouped_affine" and rows < seq_len:
            res = self.residual
            if res is None or res.dtype != torch.bfloat16:
                raise ValueError("key residual must be a bf16 tensor.")
            a.residual_bh_stride = _bh_stride(res, (seq_len - rows) * head_dim, "residual")
            a.residual = res.data_ptr()
        _lib.call("kvr_dequantize", a, _lib.stream_ptr(dev))
        return out


def _check_meta(t: torch.Tensor | None, what: str) -> None:
    if t is None or t.dtype != torch.bfloat16:
        raise ValueError(f"{what} must be a bf16 tensor (metadata_dtype=torch.bfloat16).")


def _check_input(x: torch.Tensor, metadata_dtype: torch.dtype) -> torch.device:
    if x.dtype != torch.bfloat16:
        raise ValueError("kv_reduce_b200 packs bf16 tensors only.")
    if metadata_dtype != torch.bfloat16:
        raise ValueError("kv_reduce_b200 stores bf16 metadata only (metadata_dtype=torch.bfloat16).")
    if x.dim() < 2:
        raise ValueError("KV tensors need at least [tokens, head_dim] dimensions.")
    return _lib.require_cuda(x)


def pack_per_token_affine(
    values: torch.Tensor,
    bits: int,
    *,
    metadata_dtype: torch.dtype = torch.bfloat16,
) -> PackedKVComponent:
    """Per-token affine values (packed_kv_cache.py:159-192), fused on the GPU."""
    if bits >= FULL_PRECISION_BITS:
        return PackedKVComponent(
            payload=values.contiguous(), scale=None, offset=None, residual=None,
            shape=tuple(values.shape), bits=FULL_PRECISION_BITS, layout="native",
            output_dtype=values.dtype,
        )
    if bits < 2 or bits > 8:
        raise ValueError("Affine KV quantization supports 2 through 8 bits.")
    dev = _check_input(values, metadata_dtype)
    x = values.contiguous()
    head_dim = int(x.shape[-1])
    rows = x.numel() // head_dim if head_dim else 0
    payload = torch.empty(packed_num_bytes(x.numel(), bits), dtype=torch.uint8, device=dev)
    meta_shape = (*x.shape[:-1], 1)
    scale = torch.empty(meta_shape, dtype=metadata_dtype, device=dev)
    offset = torch.empty(meta_shape, dtype=metadata_dtype, device=dev)
    if rows > 0:
        a = _lib.TokenQuantArgs()
        a.x, a.x_bh_stride, a.x_row_stride = x.data_ptr(), rows * head_dim, head_dim
        a.payload, a.payload_bh_stride = payload.data_ptr(), packed_num_bytes(rows * head_dim, bits)
        a.scale, a.offset, a.meta_bh_stride = scale.data_ptr(), offset.data_ptr(), rows
        a.bh, a.rows, a.row0, a.head_dim, a.bits = 1, rows, 0, head_dim, bits
        scratch = None
        if (head_dim * bits) % 8:
            scratch = torch.empty(rows * head_dim, dtype=torch.uint8, device=dev)
            a.codes_scratch = scratch.data_ptr()
        _lib.call("kvr_quantize_per_token", a, _lib.stream_ptr(dev))
    return PackedKVComponent(
        payload=payload, scale=scale, offset=offset, residual=None, shape=tuple(values.shape),
        bits=bits, layout="per_token_affine", output_dtype=values.dtype,
    )


def key_scale_pairs(scale: torch.Tensor, bits: int, *, out: torch.Tensor | None = None, group0: int = 0,
                    groups: int | None = None) -> torch.Tensor | None:
    """fp16 pairs of the key scales in the decode kernel's register order
    (kvr_key_scale_pairs): a tensor with ``scale``'s layout ([..., groups, 1,
    D] 16-bit words), or ``out`` with groups [group0, group0 + groups)
    filled.  None when the decode kernel does not cover the geometry
    (head_dim outside {64, 128} or bits outside {2, 4, 8})."""
    D = int(scale.shape[-1]) if scale.dim() else 0
    if D not in (64, 128) or bits not in (2, 4, 8) or scale.dim() < 3 or scale.numel() == 0:
        return None
    if out is None:
        out = torch.empty(scale.shape, dtype=torch.int16, device=scale.device)
    n_groups = int(scale.shape[-3])
    bh = scale.numel() // (n_groups * D)
    sb = n_groups * D if scale.is_contiguous() else int(scale.stride(-4))
    ob = int(out.shape[-3]) * D if out.is_contiguous() else int(out.stride(-4))
    a = _lib.ScalePairsArgs()
    a.scale, a.scale_bh_stride = scale.data_ptr(), sb
    a.pairs, a.pairs_bh_stride = out.data_ptr(), ob
    a.bh, a.groups, a.group0 = bh, n_groups - group0 if groups is None else int(groups), int(group0)
    a.head_dim, a.key_bits = D, int(bits)
    _lib.call("kvr_key_scale_pairs", a, _lib.stream_ptr(scale.device))
    return out


def pack_per_channel_grouped_affine(
    keys: torch.Tensor,
    bits: int,
    *,
    group_size: int = 32,
    residual_length: int = 128,
    metadata_dtype: torch.dtype = torch.bfloat16,
) -> PackedKVComponent:
    """Per-channel keys grouped along tokens + BF16 residual (packed_kv_cache.py:195-253)."""
    if bits >= FULL_PRECISION_BITS:
        return PackedKVComponent(
            payload=keys.contiguous(), scale=None, offset=None, residual=None,
            shape=tuple(keys.shape), bits=FULL_PRECISION_BITS, layout="native",
            output_dtype=keys.dtype,
        )
    if bits < 2 or bits > 8:
        raise ValueError("Affine KV quantization supports 2 through 8 bits.")
    prefix_length = _quantized_prefix_length(keys.shape[-2], group_size, residual_length)
    dev = _check_input(keys, metadata_dtype)
    x = keys.contiguous()
    residual = x[..., prefix_length:, :].contiguous()
    if prefix_length == 0:
        return PackedKVComponent(
            payload=torch.empty(0, dtype=torch.uint8, device=dev),
            scale=torch.empty(0, dtype=metadata_dtype, device=dev),
            offset=torch.empty(0, dtype=metadata_dtype, device=dev),
            residual=residual, shape=tuple(keys.shape), bits=bits,
            layout="per_channel_grouped_affine", output_dtype=keys.dtype,
            group_size=group_size, prefix_length=0,
        )
    seq_len, head_dim = int(x.shape[-2]), int(x.shape[-1])
    bh = x.numel() // (seq_len * head_dim)
    groups = prefix_length // group_size
    payload = torch.empty(packed_num_bytes(bh * prefix_length * head_dim, bits), dtype=torch.uint8, device=dev)
    meta_shape = (*x.shape[:-2], groups, 1, head_dim)
    scale = torch.empty(meta_shape, dtype=metadata_dtype, device=dev)
    offset = torch.empty(meta_shape, dtype=metadata_dtype, device=dev)
    a = _lib.GroupQuantArgs()
    a.x, a.x_bh_stride, a.x_row_stride = x.data_ptr(), seq_len * head_dim, head_dim
    a.payload = payload.data_ptr()
    a.payload_bh_stride = (prefix_length * head_dim * bits) // 8
    a.scale, a.offset, a.meta_bh_stride = scale.data_ptr(), offset.data_ptr(), groups * head_dim
    a.bh, a.groups, a.group0, a.group_size, a.head_dim, a.bits = bh, groups, 0, group_size, head_dim, bits
    scratch = None
    if (head_dim * bits) % 8:
        scratch = torch.empty(bh * prefix_length * head_dim, dtype=torch.uint8, device=dev)
        a.codes_scratch = scratch.data_ptr()
    _lib.call("kvr_quantize_grouped", a, _lib.stream_ptr(dev))
    return PackedKVComponent(
        payload=payload, scale=scale, offset=offset, residual=residual, shape=tuple(keys.shape),
        bits=bits, layout="per_channel_grouped_affine", output_dtype=keys.dtype,
        group_size=group_size, prefix_length=prefix_length, scale_pairs=key_scale_pairs(scale, bits),
    )


def pack_kivi_kv(
    keys: torch.Tensor,
    values: torch.Tensor,
    *,
    k_bits: int,
    v_bits: int,
    group_size: int = 32,
    residual_length: int = 128,
    metadata_dtype: torch.dtype = torch.bfloat16,
) -> Tuple[PackedKVComponent, PackedKVComponent]:
    """(grouped keys, per-token values)  (packed_kv_cache.py:256-275)."""
    return (
        pack_per_channel_grouped_affine(
            keys, k_bits, group_size=group_size, residual_length=residual_length,
            metadata_dtype=metadata_dtype,
        ),
        pack_per_token_affine(values, v_bits, metadata_dtype=metadata_dtype),
    )
