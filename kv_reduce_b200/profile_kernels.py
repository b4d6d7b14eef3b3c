"""Run every library kernel once at one layer of the 32K Qwen2.5-1.5B geometry
(B=1, 2 KV heads, 12 query heads, D=128, K4V4, group 32, residual 128), for a
profiler's launch list (``ncu ... python -m kv_reduce_b200.profile_kernels``).

Each kernel runs ``--repeat`` times after one warm-up round, on inputs larger
than the 126 MB L2 where the kernel's own traffic allows (the bf16 keys and
values of one 32K layer are 16.8 MB each, so the packing kernels are measured
on 8 layers' worth of rows at once).
"""
from __future__ import annotations

import argparse

import torch

import kv_reduce_b200 as kvr
from kv_reduce_b200 import workloads


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--repeat", type=int, default=2)
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    wl = workloads.CONFIGS["2"]
    B8 = 8   # batch the packing inputs to 8 sequences: 134 MB of bf16 keys + values per kernel

    k8, v8 = workloads.make_layer_kv(wl, 0, device=dev, batch=B8)
    k1, v1 = k8[:1].contiguous(), v8[:1].contiguous()
    q = workloads.make_query(wl, 0, device=dev)
    for _ in range(1 + args.repeat):
        # kvr::quant_group_kernel, kvr::quant_token_kernel (pack_kivi_kv)
        pk8, pv8 = kvr.pack_kivi_kv(k8, v8, k_bits=4, v_bits=4, group_size=32, residual_length=128)
        # kvr::dequant_kernel (PackedKVComponent.unpack)
        pk8.unpack()
        pv8.unpack()
        # decode_kernel (one layer)
        pk, pv = kvr.pack_kivi_kv(k1, v1, k_bits=4, v_bits=4, group_size=32, residual_length=128)
        kvr.packed_kv_decode_attention(q, pk, pv)
        # append_kernel + residual flush (streaming cache, 32 appended tokens then commit)
        layer = kvr.PackedKVCacheLayer(1, wl.kv_heads, wl.head_dim, capacity=wl.seq_len + 256, device=dev)
        layer.prefill(k1, v1)
        for t in range(32):
            layer.append(k1[:, :, t:t + 1], v1[:, :, t:t + 1])
        layer.commit()
        # lse_merge_kernel (cross-GPU partial merge of 4 shards)
        rows = wl.layers * wl.q_heads
        ml = torch.zeros(4, rows, 2, device=dev)
        o = torch.randn(4, rows, wl.head_dim, device=dev)
        kvr.lse_merge(ml, o)
        # pack_unsigned / unpack_unsigned (codes <-> bit stream)
        codes = torch.randint(0, 16, (k8.numel(),), dtype=torch.uint8, device=dev)
        payload = kvr.pack_unsigned(codes, 4)
        kvr.unpack_unsigned(payload, 4, codes.numel())
        torch.cuda.synchronize()
        del pk8, pv8, pk, pv, layer


if __name__ == "__main__":
    main()
