"""Tensor cores vs CUDA cores for the packed decode attention: the measured A/B.

The decode kernel runs its GQA-group x token tiles on the tensor cores
(``kvr_decode_attention``: mma.sync m16n8k16, codes as fp16 operands).  The
alternative is the same computation on the CUDA cores
(``kvr_decode_attention_simt``: fp32 FMA, same packed layout, same split-K
and LSE merge, every packed byte shared by the group's query heads).  The
tensor-core kernel is the one the library uses because it measures faster;
this module is that measurement:

    python -m kv_reduce_b200.engine_ab [--configs 2,4] [--steps 20]

prints one JSON line per workload and engine (all layers of a decode step,
one launch per 32 layers, replayed as a CUDA graph, CUDA events; every
workload's packed cache is larger than the 126 MB L2, so no flush), with the
step time, the achieved algorithmic HBM bandwidth, its fraction of the
measured copy peak and the largest difference between the engines' outputs.
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

from . import _lib, workloads
from .packed_kv_attention import DecodeLaunch, _effective_split, _geometry, _layer_ptrs, _validate
from .packed_kv_cache import PackedKVComponent, pack_kivi_kv

ENGINES = ("tensor", "simt")


class SimtDecodeLaunch(DecodeLaunch):
    """A prepared decode launch on the CUDA-core engine."""

    def __init__(self, geom, layers, device, split_tokens: int = 0, stream: int | None = None,
                 out_fp32: bool = False) -> None:
        super().__init__(geom, layers, device, split_tokens=split_tokens, stream=stream, out_fp32=out_fp32)
        n = int(_lib.load().kvr_decode_simt_workspace(self.args))
        if n == 0:
            raise ValueError("this geometry is not supported by the CUDA-core engine")
        self.simt_workspace = torch.empty(n, dtype=torch.uint8, device=device)
        self.args.workspace, self.args.workspace_bytes = self.simt_workspace.data_ptr(), n

    def __call__(self) -> None:
        _lib.check("kvr_decode_attention_simt", _lib.load().kvr_decode_attention_simt(self.args, self.stream))


def simt_decode(query: torch.Tensor, packed_keys: PackedKVComponent, packed_values: PackedKVComponent, *,
                split_tokens: int = 0, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """packed_kv_decode_attention computed by the CUDA-core engine."""
    _validate(query, packed_keys, packed_values, 32)
    query = query.contiguous()
    geom = _geometry(query, packed_keys, packed_values)
    out_fp32 = out_dtype == torch.float32
    out = torch.empty_like(query, dtype=torch.float32) if out_fp32 else torch.empty_like(query)
    launch = SimtDecodeLaunch(geom, [_layer_ptrs(query, out, packed_keys, packed_values)], query.device,
                              split_tokens=_effective_split(split_tokens, 32), out_fp32=out_fp32)
    launch()
    return out


def _hbm_peak() -> float:
    path = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0


def measure(key: str, steps: int, warmup: int) -> list[dict]:
    wl = workloads.CONFIGS[key]
    device = torch.device("cuda", 0)
    ks, vs, qs = [], [], []
    for layer in range(wl.layers):
        k, v = workloads.make_layer_kv(wl, layer, device=device)
        pk, pv = pack_kivi_kv(k, v, k_bits=wl.k_bits, v_bits=wl.v_bits, group_size=wl.group_size,
                              residual_length=wl.residual_length)
        del k, v
        ks.append(pk)
        vs.append(pv)
        qs.append(workloads.make_query(wl, layer, device=device))
    geom = _geometry(qs[0], ks[0], vs[0])
    step_bytes = workloads.layer_bytes(wl)["total"] * wl.layers
    stream = torch.cuda.Stream(device)
    peak = _hbm_peak()
    rows, first = [], None
    for engine in ENGINES:
        outs = [torch.empty_like(q) for q in qs]
        ptrs = [_layer_ptrs(q, o, k, v) for q, o, k, v in zip(qs, outs, ks, vs)]
        cls = DecodeLaunch if engine == "tensor" else SimtDecodeLaunch
        launches = [cls(geom, ptrs[i:i + _lib.KVR_MAX_LAYERS], device, stream=stream.cuda_stream)
                    for i in range(0, wl.layers, _lib.KVR_MAX_LAYERS)]

        def step():
            for launch in launches:
                launch()

        with torch.cuda.stream(stream):
            for _ in range(max(3, warmup)):
                step()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            for _ in range(max(3, warmup)):
                g.replay()
            start.record(stream)
            for _ in range(steps):
                g.replay()
            end.record(stream)
        torch.cuda.synchronize()
        us = start.elapsed_time(end) * 1e3 / steps
        del g
        out = torch.stack(outs).float()
        if first is None:
            first = out
        gbs = step_bytes / us / 1e3
        rows.append({"workload": wl.name, "engine": engine, "us_per_step": round(us, 2), "gbps": round(gbs, 1),
                     "frac_of_measured_hbm": round(gbs / peak, 4), "launches_per_step": len(launches),
                     "max_abs_diff_vs_tensor": float((out - first).abs().max())})
    return rows


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--configs", default="2,4", help="workload keys (kv_reduce_b200.workloads.CONFIGS)")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args()
    for key in args.configs.split(","):
        for row in measure(key, args.steps, args.warmup):
            print(json.dumps(row), flush=True)
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
