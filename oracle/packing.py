"""numpy restatement of kv_reduce/packed_kv_cache.py -- test infrastructure only.

All arithmetic is float32 with the reference's operation order, so codes and
bf16 metadata are bit-identical to the reference (pinned against golden
vectors made from the reference itself).  bf16 tensors are carried as their
uint16 bit patterns.
"""
from __future__ import annotations

from math import ceil
from typing import Dict, Tuple

import numpy as np

F32 = np.float32


# ------------------------------------------------------------------ bf16 bits
def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns -> float32 (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even (Tensor.to(bfloat16))."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


# --------------------------------------------------------------- primitives
def quantized_prefix_length(seq_len: int, group_size: int, residual_length: int) -> int:
    """P = floor(max(0, S-R)/G)*G  (packed_kv_cache.py:15-19)."""
    if group_size <= 0 or residual_length < 0:
        raise ValueError("group_size must be positive and residual_length non-negative.")
    return (max(0, int(seq_len) - int(residual_length)) // int(group_size)) * int(group_size)


def packed_num_bytes(n: int, bits: int) -> int:
    """packed_kv_cache.py:22-25."""
    return ceil(int(n) * int(bits) / 8)


def pack_unsigned(codes: np.ndarray, bits: int) -> np.ndarray:
    """LSB-first bit stream, value i at bit i*bits (packed_kv_cache.py:28-63)."""
    flat = np.asarray(codes, dtype=np.uint8).reshape(-1).astype(np.uint32)
    n = flat.size
    out = np.zeros(packed_num_bytes(n, bits), dtype=np.uint32)
    if n == 0:
        return out.astype(np.uint8)
    pos = np.arange(n, dtype=np.int64) * bits
    byte, off = pos >> 3, (pos & 7).astype(np.uint32)
    np.add.at(out, byte, (flat << off) & 0xFF)
    cross = off + bits > 8
    if cross.any():
        np.add.at(out, byte[cross] + 1, flat[cross] >> (8 - off[cross]))
    return out.astype(np.uint8)


def unpack_unsigned(payload: np.ndarray, bits: int, n: int) -> np.ndarray:
    """Inverse of pack_unsigned (packed_kv_cache.py:66-94)."""
    p = np.asarray(payload, dtype=np.uint8).reshape(-1).astype(np.uint32)
    if n == 0:
        return np.zeros(0, dtype=np.uint8)
    pos = np.arange(n, dtype=np.int64) * bits
    byte, off = pos >> 3, (pos & 7).astype(np.uint32)
    nxt = np.where(byte + 1 < p.size, p[np.minimum(byte + 1, p.size - 1)], 0)
    raw = (p[byte] | (nxt << 8)) >> off
    return (raw & ((1 << bits) - 1)).astype(np.uint8)


# ----------------------------------------------------------------- quantizer
def _affine(x: np.ndarray, mn: np.ndarray, mx: np.ndarray, bits: int) -> Tuple[np.ndarray, np.ndarray]:
    """scale = max(max-min, 1e-8)/(2^b-1); code = clamp(rint((x-min)/scale)).

    packed_kv_cache.py:181-182 and :240-241 (IEEE float32 division,
    round half to even)."""
    scale = np.maximum((mx - mn).astype(F32), F32(1e-8)) / F32((1 << bits) - 1)
    scale = scale.astype(F32)
    q = np.rint(((x - mn).astype(F32) / scale).astype(F32))
    q = np.clip(q, 0, (1 << bits) - 1).astype(np.uint8)
    return q, scale


def quantize_per_token(x_bits: np.ndarray, bits: int) -> Dict[str, np.ndarray]:
    """pack_per_token_affine (packed_kv_cache.py:159-192) on bf16 bits [..., D]."""
    x = bf16_to_f32(x_bits)
    mn = x.min(axis=-1, keepdims=True)
    mx = x.max(axis=-1, keepdims=True)
    codes, scale = _affine(x, mn, mx, bits)
    return {
        "codes": codes,
        "payload": pack_unsigned(codes, bits),
        "scale": f32_to_bf16(scale),
        "offset": f32_to_bf16(mn),
    }


def quantize_grouped(x_bits: np.ndarray, bits: int, group_size: int, residual_length: int) -> Dict[str, np.ndarray]:
    """pack_per_channel_grouped_affine (packed_kv_cache.py:195-253) on bf16 bits [..., S, D]."""
    S, D = x_bits.shape[-2], x_bits.shape[-1]
    P = quantized_prefix_length(S, group_size, residual_length)
    residual = np.ascontiguousarray(x_bits[..., P:, :])
    lead = x_bits.shape[:-2]
    if P == 0:
        return {"P": P, "codes": np.zeros((*lead, 0, D), np.uint8), "payload": np.zeros(0, np.uint8),
                "scale": np.zeros(0, np.uint16), "offset": np.zeros(0, np.uint16), "residual": residual}
    x = bf16_to_f32(x_bits[..., :P, :]).reshape(*lead, P // group_size, group_size, D)
    mn = x.min(axis=-2, keepdims=True)
    mx = x.max(axis=-2, keepdims=True)
    codes, scale = _affine(x, mn, mx, bits)
    return {
        "P": P,
        "codes": codes.reshape(*lead, P, D),
        "payload": pack_unsigned(codes, bits),
        "scale": f32_to_bf16(scale),
        "offset": f32_to_bf16(mn),
        "residual": residual,
    }


def dequant_per_token(payload: np.ndarray, scale_bits: np.ndarray, offset_bits: np.ndarray, bits: int,
                      shape: Tuple[int, ...]) -> np.ndarray:
    """fp32 unpack of per-token values: code*scale + offset, two roundings (:130-131)."""
    n = int(np.prod(shape))
    q = unpack_unsigned(payload, bits, n).reshape(shape).astype(F32)
    return ((q * bf16_to_f32(scale_bits)).astype(F32) + bf16_to_f32(offset_bits)).astype(F32)


def dequant_grouped(payload: np.ndarray, scale_bits: np.ndarray, offset_bits: np.ndarray,
                    residual_bits: np.ndarray, bits: int, shape: Tuple[int, ...], P: int,
                    group_size: int) -> np.ndarray:
    """fp32 unpack of grouped keys + BF16 residual (:132-148)."""
    lead, D = tuple(shape[:-2]), shape[-1]
    parts = []
    if P > 0:
        q = unpack_unsigned(payload, bits, int(np.prod(lead)) * P * D)
        q = q.reshape(*lead, P // group_size, group_size, D).astype(F32)
        pre = ((q * bf16_to_f32(scale_bits)).astype(F32) + bf16_to_f32(offset_bits)).astype(F32)
        parts.append(pre.reshape(*lead, P, D))
    if shape[-2] > P:
        parts.append(bf16_to_f32(residual_bits))
    return np.concatenate(parts, axis=-2)
