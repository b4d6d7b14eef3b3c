"""The reference's unfused CPU decode path, restated -- CPU baseline only.

kv_reduce/experiments/benchmark_packed_kv_attention.py:236-240 times
``gqa_attention(query, packed_keys.unpack(), packed_values.unpack())``:
unpack_unsigned (packed_kv_cache.py:66-94), dequantize q*scale+offset in
fp32 and cast to bf16 (:126-149), then scaled_dot_product_attention with
enable_gqa (:58-76).  The reference package cannot travel to the GPU host,
so this module restates that operator sequence with the same torch CPU ops
and is timed there as the reference arm.  Used only by bench.py's
CPU-baseline leg and by tests; tests/test_oracle_golden.py pins its output
to the reference's own.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Tuple

import numpy as np
import torch
import torch.nn.functional as F

from . import packing


@dataclass
class CpuPacked:
    payload: torch.Tensor          # uint8 flat
    scale: torch.Tensor            # bf16
    offset: torch.Tensor           # bf16
    residual: torch.Tensor | None  # bf16 [B, H, S-P, D]
    shape: Tuple[int, ...]
    bits: int
    prefix_length: int = 0
    group_size: int = 0

    @property
    def storage_bytes(self) -> int:
        n = self.payload.numel() + 2 * (self.scale.numel() + self.offset.numel())
        return n + (0 if self.residual is None else 2 * self.residual.numel())


def _bits_tensor(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits, dtype=np.uint16).view(np.int16)).view(torch.bfloat16)


def pack_cpu(keys_bits: np.ndarray, values_bits: np.ndarray, k_bits: int, v_bits: int, group_size: int,
             residual_length: int) -> Tuple[CpuPacked, CpuPacked]:
    """Pack with the numpy oracle and wrap as CPU torch tensors."""
    kq = packing.quantize_grouped(keys_bits, k_bits, group_size, residual_length)
    vq = packing.quantize_per_token(values_bits, v_bits)
    shape = tuple(keys_bits.shape)
    P = kq["P"]
    kmeta = (*shape[:-2], P // group_size, 1, shape[-1])
    k = CpuPacked(torch.from_numpy(kq["payload"]), _bits_tensor(kq["scale"]).reshape(kmeta),
                  _bits_tensor(kq["offset"]).reshape(kmeta), _bits_tensor(kq["residual"]), shape, k_bits, P,
                  group_size)
    v = CpuPacked(torch.from_numpy(vq["payload"]), _bits_tensor(vq["scale"]), _bits_tensor(vq["offset"]), None,
                  shape, v_bits)
    return k, v


def _unpack_unsigned(payload: torch.Tensor, bits: int, n: int) -> torch.Tensor:
    if bits == 8:
        return payload[:n]
    if bits in (2, 4):
        per = 8 // bits
        shifts = torch.arange(per, dtype=torch.int32) * bits
        return ((payload.to(torch.int32).unsqueeze(-1) >> shifts) & ((1 << bits) - 1)).reshape(-1)[:n].to(torch.uint8)
    idx = torch.arange(n, dtype=torch.int64) * bits
    byte, off = torch.div(idx, 8, rounding_mode="floor"), torch.remainder(idx, 8).to(torch.int32)
    p32 = payload.to(torch.int32)
    raw = p32[byte] >> off
    cross = off + bits > 8
    if bool(cross.any()):
        raw[cross] |= p32[byte[cross] + 1] << (8 - off[cross])
    return (raw & ((1 << bits) - 1)).to(torch.uint8)


def unpack_values(v: CpuPacked, dtype=torch.bfloat16) -> torch.Tensor:
    q = _unpack_unsigned(v.payload, v.bits, int(np.prod(v.shape))).reshape(v.shape)
    return (q.float() * v.scale.float() + v.offset.float()).to(dtype)


def unpack_keys(k: CpuPacked, dtype=torch.bfloat16) -> torch.Tensor:
    lead, D, P, G = k.shape[:-2], k.shape[-1], k.prefix_length, k.group_size
    n = int(np.prod(lead)) * P * D
    q = _unpack_unsigned(k.payload, k.bits, n).reshape(*lead, P // G, G, D)
    prefix = (q.float() * k.scale.float() + k.offset.float()).reshape(*lead, P, D)
    if k.residual is not None and k.residual.shape[-2] > 0:
        prefix = torch.cat((prefix.to(dtype), k.residual.to(dtype)), dim=-2)
    return prefix.to(dtype)


def unfused_decode(query: torch.Tensor, k: CpuPacked, v: CpuPacked) -> torch.Tensor:
    """unpack keys, unpack values, SDPA with GQA: the reference's unfused step."""
    keys, values = unpack_keys(k), unpack_values(v)
    return F.scaled_dot_product_attention(query, keys, values, is_causal=False, enable_gqa=True)
