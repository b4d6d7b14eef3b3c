"""Seeded synthetic packed-KV workloads with the shapes of the benchmark configs.

No dataset is involved: the reference benchmarks draw K/V/Q from normal
distributions (kv_reduce/experiments/benchmark_fused_packed_kv_attention.py:
124-149).  These configs add the outlier key channels KIVI is designed for:
a fixed, seeded set of channels scaled up in every token and head.
"""
from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Dict, List, Tuple

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    batch: int
    q_heads: int
    kv_heads: int
    head_dim: int
    seq_len: int
    k_bits: int
    v_bits: int
    group_size: int
    residual_length: int
    layers: int
    outliers: int = 4
    outlier_scale: float = 10.0
    value_std: float = 1.0
    seed: int = 0
    draft_steps: int = 0

    @property
    def prefix_len(self) -> int:
        eligible = max(0, self.seq_len - self.residual_length)
        return (eligible // self.group_size) * self.group_size

    def scaled(self, **kw) -> "Workload":
        return replace(self, **kw)


CONFIGS: Dict[str, Workload] = {
    # single layer, CPU-runnable: 1K tokens, residual 0
    "1": Workload("qwen2.5-1.5b-1k-k4v4-r0", 1, 12, 2, 128, 1024, 4, 4, 32, 0, 1),
    # full Qwen2.5-1.5B-geometry draft cache, 32K tokens, 28 layers
    "2": Workload("qwen2.5-1.5b-32k-k4v4", 1, 12, 2, 128, 32768, 4, 4, 32, 128, 28),
    # Llama-3.2-1B geometry, batch 32, 8K tokens, mixed precision
    "3a": Workload("llama3.2-1b-b32-8k-k8v4", 32, 32, 8, 64, 8192, 8, 4, 32, 128, 16, outliers=8,
                   outlier_scale=8.0, value_std=0.5),
    "3b": Workload("llama3.2-1b-b32-8k-k4v8", 32, 32, 8, 64, 8192, 4, 8, 32, 128, 16, outliers=8,
                   outlier_scale=8.0, value_std=0.5),
    # KIVI-2 stress: batch 64, 16K tokens, K2V2
    "4": Workload("qwen2.5-1.5b-b64-16k-k2v2", 64, 12, 2, 128, 16384, 2, 2, 32, 128, 28),
    # speculative draft loop: 4 x (append one token + decode), batch 128, 4K
    "5": Workload("qwen2.5-1.5b-b128-4k-k4v4-draft4", 128, 12, 2, 128, 4096, 4, 4, 32, 128, 28, draft_steps=4),
}


def outlier_channels(wl: Workload) -> List[int]:
    g = torch.Generator().manual_seed(wl.seed)
    return sorted(torch.randperm(wl.head_dim, generator=g)[: wl.outliers].tolist())


def _gen(device: torch.device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def make_layer_kv(wl: Workload, layer: int, device: torch.device | str = "cuda",
                  seq_len: int | None = None, batch: int | None = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """K, V bf16 [B, HKV, S, D] for one layer (seed = wl.seed + layer)."""
    device = torch.device(device)
    S = wl.seq_len if seq_len is None else seq_len
    B = wl.batch if batch is None else batch
    shape = (B, wl.kv_heads, S, wl.head_dim)
    g = _gen(device, wl.seed * 1000 + layer)
    k = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    chans = outlier_channels(wl)
    if chans:
        k[..., chans] *= wl.outlier_scale
    v = torch.randn(shape, generator=g, device=device, dtype=torch.float32) * wl.value_std
    return k.to(torch.bfloat16), v.to(torch.bfloat16)


def make_query(wl: Workload, layer: int, device: torch.device | str = "cuda", step: int = 0,
               batch: int | None = None) -> torch.Tensor:
    device = torch.device(device)
    B = wl.batch if batch is None else batch
    g = _gen(device, 7_000_000 + wl.seed * 1000 + layer * 16 + step)
    return torch.randn((B, wl.q_heads, 1, wl.head_dim), generator=g, device=device,
                       dtype=torch.float32).to(torch.bfloat16)


def layer_bytes(wl: Workload, seq_len: int | None = None, batch: int | None = None) -> Dict[str, int]:
    """Algorithmic bytes one decode step reads/writes for one layer.

    packed key payload + key scale/offset + BF16 key residual + value payload
    + value scale/offset + query + output.  Split partials and L2 re-reads
    are not counted.
    """
    S = wl.seq_len if seq_len is None else seq_len
    B = wl.batch if batch is None else batch
    D, H = wl.head_dim, wl.kv_heads
    P = (max(0, S - wl.residual_length) // wl.group_size) * wl.group_size
    bh = B * H
    out = {
        "key_payload": bh * P * D * wl.k_bits // 8,
        "key_meta": bh * (P // wl.group_size) * D * 2 * 2,
        "key_residual": bh * (S - P) * D * 2,
        "value_payload": bh * S * D * wl.v_bits // 8,
        "value_meta": bh * S * 2 * 2,
        "query": B * wl.q_heads * D * 2,
        "output": B * wl.q_heads * D * 2,
    }
    out["total"] = sum(out.values())
    out["cache"] = out["total"] - out["query"] - out["output"]
    return out
