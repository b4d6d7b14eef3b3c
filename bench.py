#!/usr/bin/env python3
"""Packed-KV decode attention benchmark (B200).

One step = decode attention for every layer of the workload's packed cache
(default: the Qwen2.5-1.5B-geometry draft cache, 28 layers x 32K tokens,
K4V4, key group 32, 128-token BF16 residual window, batch 1).

  value  : achieved algorithmic HBM GB/s of the step (all ranks), inputs
           resident in HBM, all layers of the step in one launch (layer
           index in the grid), replayed as a CUDA graph.  Layers rotate
           through 273 MB of distinct buffers, more than the 126 MB L2, so
           no flush is needed.  `per_layer` times the same step as one
           launch per layer (28 launches in a CUDA graph).
  e2e    : the same metric through the public Python API with the queries
           copied host->device and the outputs device->host every step.

  workloads : the other benchmark workloads on the same kernel, each with
           its own clock record: Llama-3.2-1B geometry batch 32 x 8K K8V4 and
           K4V8, Qwen geometry batch 64 x 16K K2V2 (one launch per step), and
           the speculative draft loop (batch 128 x 4K, four steps of append +
           decode per round, replayed as a CUDA graph).  At N > 1 their global
           batch is sharded across the ranks.

With --gpus N (torchrun) each rank holds its own batch-1 sequence for the
headline (weak scaling, batch sharding, no collective on the data path); the
step time is the max over ranks.  At N > 1 the line also carries
`split_sequence`: ONE batch-1 32K sequence with its tokens split across the
ranks (partial decode + the fused NVLink exchange and LSE merge kernel).
``--impl reference`` times the reference's unfused CPU path (unpack + SDPA)
on the host cores: the reference's own code from its install under
baseline/_ref, or its restatement in oracle/cpu_baseline.py when that is
absent.

Tools on the same workloads (not part of the driver's line):
  --engine-ab     tensor cores vs CUDA cores for the decode (one JSON line per
                  workload and engine)
  --all-kernels   every library kernel once per round, for a profiler's
                  launch list
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "packed-KV decode attn µs/step & achieved HBM GB/s (K4V4, 32K ctx) at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", default="2", help="workload key in kv_reduce_b200.workloads.CONFIGS")
    p.add_argument("--split-tokens", type=int, default=0)
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU-baseline sample length")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--exchange", choices=["best", "delivered", "owner", "push", "nccl"], default="best",
                   help="sequence split's exchange: the decode stores its rows into the peers and one kernel "
                        "waits and merges (delivered); the decode stores each row into its owner rank, which "
                        "merges it and sends the merged row to every rank (owner); one kernel pushes, signals "
                        "and merges (push); or an NCCL all-gather plus the LSE merge launch (nccl); best: "
                        "delivered and owner both timed, the faster reported")
    p.add_argument("--nccl-exchange", action="store_true", help="same as --exchange nccl")
    p.add_argument("--draft-loop", action="store_true",
                   help="speculative draft loop on the streaming cache (use with --config 5)")
    p.add_argument("--split-sequence", action="store_true",
                   help="N>1: split ONE batch-1 sequence's tokens across the ranks (strong scaling, "
                        "partial decode + NCCL all-gather + LSE merge) instead of one sequence per rank")
    p.add_argument("--no-workloads", action="store_true", help="headline workload only")
    p.add_argument("--workload-steps", type=int, default=10, help="timed steps per extra workload")
    p.add_argument("--engine-ab", action="store_true", help="tool: tensor cores vs CUDA cores (see --configs)")
    p.add_argument("--configs", default="2,4", help="--engine-ab workloads")
    p.add_argument("--all-kernels", action="store_true", help="tool: run every library kernel (see --repeat)")
    p.add_argument("--repeat", type=int, default=2, help="--all-kernels rounds after one warm-up round")
    return p.parse_args()


# ------------------------------------------------------------------ helpers
def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    return world, rank, local


def measured_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            d = json.loads(path.read_text())
            return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, burst copy)"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback 6.65 TB/s"


def profiled_traffic(workload: str):
    """Per-launch DRAM bytes of the decode kernel from the committed ncu summary."""
    path = ROOT / "profiles" / "decode_traffic.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 2 and parts[0] == workload:
            try:
                return int(parts[1])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device):
        self.proc = None
        self.file = None
        try:
            self.uuid = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            self.uuid = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.file is None:
            return None
        self.file.flush()
        rows = []
        with open(self.file.name) as f:
            for line in f:
                cols = [c.strip() for c in line.split(",")]
                if len(cols) < 9 or (self.uuid and cols[0] != self.uuid):
                    continue
                rows.append(cols)
        os.unlink(self.file.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "samples": len(rows), "reasons": reasons}


# ------------------------------------------------------------ CPU baseline
REF_DIR = ROOT / "baseline" / "_ref"   # the reference package, installed offline (pip --target)


def reference_cpu_step(wl):
    """One step of the reference's unfused decode on host cores for one
    layer of `wl`: (kind, step function, description).

    kind "reference": the reference's own code, imported from its install
    under baseline/_ref -- pack_kivi_kv once (kv_reduce/packed_kv_cache.py:256-275),
    then per step gqa_attention(query, packed_keys.unpack(), packed_values.unpack())
    (kv_reduce/experiments/benchmark_packed_kv_attention.py:58-76, :236-240).
    kind "port": the same operator sequence restated by oracle/cpu_baseline.py
    (pinned to the reference's outputs), when the install is absent."""
    import numpy as np

    from kv_reduce_b200 import workloads

    k, v = workloads.make_layer_kv(wl, 0, device="cpu")
    q = workloads.make_query(wl, 0, device="cpu")
    if (REF_DIR / "kv_reduce" / "packed_kv_cache.py").exists():
        if str(REF_DIR) not in sys.path:
            sys.path.insert(0, str(REF_DIR))
        from kv_reduce.experiments.benchmark_packed_kv_attention import gqa_attention
        from kv_reduce.packed_kv_cache import pack_kivi_kv

        pk, pv = pack_kivi_kv(k, v, k_bits=wl.k_bits, v_bits=wl.v_bits, group_size=wl.group_size,
                              residual_length=wl.residual_length)
        return ("reference", lambda: gqa_attention(q, pk.unpack(), pv.unpack()),
                "the reference's own PackedKVComponent.unpack() x2 + gqa_attention (SDPA, bf16), "
                "kv_reduce installed under baseline/_ref")
    from oracle import cpu_baseline

    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    pk, pv = cpu_baseline.pack_cpu(bits(k), bits(v), wl.k_bits, wl.v_bits, wl.group_size, wl.residual_length)
    return ("port", lambda: cpu_baseline.unfused_decode(q, pk, pv),
            "unpack + SDPA in bf16, the reference's unfused path restated by the oracle port")


def cpu_baseline_sample(wl, seconds: float, layer_bytes: int):
    """Reference unfused path (unpack K, unpack V, SDPA) on host cores, one
    layer repeated for about `seconds`."""
    torch.set_num_threads(os.cpu_count() or 1)
    kind, step, what = reference_cpu_step(wl)
    step()   # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        step()
        n += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = (time.perf_counter() - t0) / n
    return {"value": layer_bytes / dt / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": kind,
            "sample": f"{n} x one {wl.seq_len}-token layer of the {wl.name} workload ({what})",
            "ms_per_layer": dt * 1e3, "ms_per_step_extrapolated": dt * 1e3 * wl.layers}


def workload_config(wl, world, args, batch_sharded_global=False):
    """The `config` object of a line, the same for our arm and the reference arm."""
    from kv_reduce_b200 import workloads

    step_bytes = workloads.layer_bytes(wl)["total"] * wl.layers
    per_gpu = wl.batch if not batch_sharded_global else -(-wl.batch // world)
    glob = wl.batch * world if not batch_sharded_global else wl.batch
    return {"workload": wl.name, "layers": wl.layers, "batch_per_gpu": per_gpu, "global_batch": glob,
            "seq_len": wl.seq_len, "q_heads": wl.q_heads, "kv_heads": wl.kv_heads, "head_dim": wl.head_dim,
            "kv_bits": f"K{wl.k_bits}V{wl.v_bits}", "group_size": wl.group_size, "residual": wl.residual_length,
            "parallelism": f"batch-sharded x{world}", "split_tokens": args.split_tokens,
            "l2": f"inputs {step_bytes / 1e6:.0f} MB per step > 126 MB L2; layers rotate, no flush"}


def run_reference(args, wl, world, rank):
    from kv_reduce_b200 import workloads

    if rank != 0:
        return
    lb = workloads.layer_bytes(wl)["total"]
    torch.set_num_threads(os.cpu_count() or 1)
    kind, step, what = reference_cpu_step(wl)
    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    dt = sum(times) / len(times)
    value = lb / dt / 1e9
    sample = f"one {wl.seq_len}-token layer per step (of {wl.layers}), {what}"
    line = {"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt * 1e3 * wl.layers,
            "ms_per_step_note": "extrapolated: layer time x layers",
            "us_per_step": dt * 1e6 * wl.layers,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "impl": "reference",
            "config": workload_config(wl, world, args),
            "cpu_baseline": {"value": value, "unit": "GB/s", "cores": torch.get_num_threads(), "kind": kind,
                             "sample": sample},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm
def build_cache(wl, device, rank, batch_range=None):
    """Packed caches, queries of every layer.  batch_range=(a, b) keeps the
    sequences [a, b) of the workload's batch (the data of a sequence does not
    depend on how the batch is sharded)."""
    import kv_reduce_b200 as kvr
    from kv_reduce_b200 import workloads

    seed_wl = wl.scaled(seed=wl.seed + 100 * rank) if batch_range is None else wl
    ks, vs, qs = [], [], []
    for layer in range(wl.layers):
        k, v = workloads.make_layer_kv(seed_wl, layer, device=device)
        q = workloads.make_query(seed_wl, layer, device=device)
        if batch_range is not None:
            a, b = batch_range
            k, v, q = k[a:b].contiguous(), v[a:b].contiguous(), q[a:b].contiguous()
        pk, pv = kvr.pack_kivi_kv(k, v, k_bits=wl.k_bits, v_bits=wl.v_bits, group_size=wl.group_size,
                                  residual_length=wl.residual_length)
        del k, v
        ks.append(pk)
        vs.append(pv)
        qs.append(q)
    torch.cuda.synchronize(device)
    return ks, vs, qs


def time_graph(fn, stream, steps, warmup, world, pg_sync):
    """Capture `fn` (enqueues one step on `stream`) in a CUDA graph; time
    `steps` replays with CUDA events on that stream; max over ranks."""
    with torch.cuda.stream(stream):
        for _ in range(max(warmup, 3)):
            fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    with torch.cuda.stream(stream):
        for _ in range(max(warmup, 3)):
            g.replay()
    torch.cuda.synchronize()
    pg_sync()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(steps):
            g.replay()
        end.record(stream)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    pg_sync()
    del g
    return ms


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def fused_launches(ks, vs, qs, device, stream, split_tokens):
    """All layers of a step in one launch per <= 32 layers (layer index in the grid)."""
    from kv_reduce_b200.packed_kv_attention import DecodeLaunch, _geometry, _layer_ptrs

    outs = [torch.empty_like(q) for q in qs]
    geom = _geometry(qs[0], ks[0], vs[0])
    ptrs = [_layer_ptrs(q, o, k, v) for q, o, k, v in zip(qs, outs, ks, vs)]
    launches = [DecodeLaunch(geom, ptrs[i:i + 32], device, split_tokens=split_tokens, stream=stream.cuda_stream)
                for i in range(0, len(ptrs), 32)]
    return launches, outs, geom, ptrs


def measure_workload(args, key, world, rank, device, pg_sync):
    """One extra workload on the fused kernel, its global batch sharded over
    the ranks; returns its sub-dict (rank 0) with its own clock record."""
    from kv_reduce_b200 import distributed as kd
    from kv_reduce_b200 import workloads

    wl = workloads.CONFIGS[key]
    a, b = kd.batch_shard(wl.batch, world, rank)
    ks, vs, qs = build_cache(wl, device, rank, batch_range=(a, b))
    stream = torch.cuda.Stream(device)
    # the outputs must outlive the captured graph: torch.cuda.graph empties the
    # allocator cache before capture, so a dropped output would be unmapped
    launches, outs, _, _ = fused_launches(ks, vs, qs, device, stream, args.split_tokens)

    def step():
        for launch in launches:
            launch()

    steps = max(1, args.workload_steps)
    with ClockSampler(device) as clocks:
        ms = time_graph(step, stream, steps, max(args.warmup, 3), world, pg_sync)
    ms = max_over_ranks(ms, world, device)
    step_ms = ms / steps
    my_bytes = workloads.layer_bytes(wl, batch=b - a)["total"] * wl.layers
    total_bytes = sum_over_ranks(my_bytes, world, device)
    peak, _ = measured_peak()
    gbs = total_bytes / (step_ms * 1e-3) / 1e9
    res = {"workload": wl.name, "layers": wl.layers, "global_batch": wl.batch, "batch_per_gpu": b - a,
           "seq_len": wl.seq_len, "kv_bits": f"K{wl.k_bits}V{wl.v_bits}", "head_dim": wl.head_dim,
           "q_heads": wl.q_heads, "kv_heads": wl.kv_heads,
           "us_per_step": step_ms * 1e3, "gbps": gbs, "frac": gbs / world / peak, "frac_note": "of measured, per GPU",
           "bytes_per_step": total_bytes, "num_splits": launches[0].num_splits, "steps": steps,
           "scaling": "strong (global batch fixed, sharded by batch)" if world > 1 else "n/a",
           "timing": "all layers per launch, CUDA graph, CUDA events, max over ranks; inputs > L2",
           "gpu_launches": steps * len(launches), "clocks": clocks.summary()}
    del launches, outs, ks, vs, qs
    torch.cuda.empty_cache()
    return res


def measure_draft_loop(args, world, rank, device, pg_sync):
    """The speculative draft loop (batch 128 x 4K, K4V4, 4 steps of append +
    decode per round) on the streaming cache, the batch sharded over the
    ranks; µs per draft step of the replayed CUDA graph."""
    import kv_reduce_b200 as kvr
    from kv_reduce_b200 import distributed as kd
    from kv_reduce_b200 import workloads
    from kv_reduce_b200.draft import DraftLoop

    wl = workloads.CONFIGS["5"]
    a, b = kd.batch_shard(wl.batch, world, rank)
    steps = max(1, wl.draft_steps or 4)
    cache = kvr.PackedKVCache(wl.layers, b - a, wl.kv_heads, wl.head_dim, k_bits=wl.k_bits, v_bits=wl.v_bits,
                              group_size=wl.group_size, residual_length=wl.residual_length,
                              capacity=wl.seq_len + 64, device=device)
    for i, layer in enumerate(cache.layers):
        k, v = workloads.make_layer_kv(wl, i, device=device)
        layer.prefill(k[a:b].contiguous(), v[a:b].contiguous())
        del k, v
    loop = DraftLoop(cache, q_heads=wl.q_heads, steps=steps, split_tokens=args.split_tokens)
    g = torch.Generator(device=device).manual_seed(1234 + rank)
    for t in (loop.q, loop.k, loop.v):
        t.copy_(torch.randn(t.shape, generator=g, device=device).to(torch.bfloat16))
    start = cache.get_seq_length()
    rounds = max(1, args.workload_steps)

    def timed(fn, n):
        ev = []
        for i in range(max(args.warmup, 3) + n):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            cache.crop(start)
            if i >= max(args.warmup, 3):
                ev.append((e0, e1))
        torch.cuda.synchronize()
        return sum(x.elapsed_time(y) for x, y in ev) / len(ev)

    pg_sync()
    with ClockSampler(device) as clocks:
        graph_ms = timed(loop.replay, rounds)
    graph_ms = max_over_ranks(graph_ms, world, device)
    errors = int(sum_over_ranks(loop.errors(), world, device))
    wl_b = wl.scaled(batch=b - a)
    my_bytes = sum(workloads.layer_bytes(wl_b, seq_len=start + t + 1)["total"] for t in range(steps)) / steps
    my_bytes = my_bytes * wl.layers + wl.layers * (b - a) * wl.kv_heads * (
        2 * wl.head_dim + wl.head_dim * wl.v_bits // 8 + 4)
    total_bytes = sum_over_ranks(my_bytes, world, device)
    us_step = graph_ms * 1e3 / steps
    peak, _ = measured_peak()
    gbs = total_bytes / (us_step * 1e-6) / 1e9
    res = {"workload": wl.name, "layers": wl.layers, "global_batch": wl.batch, "batch_per_gpu": b - a,
           "seq_len": start, "draft_steps": steps, "kv_bits": f"K{wl.k_bits}V{wl.v_bits}",
           "us_per_draft_step": us_step, "gbps": gbs, "frac": gbs / world / peak,
           "frac_note": "of measured, per GPU", "bytes_per_draft_step": total_bytes, "rounds": rounds,
           "append_errors": errors,
           "scaling": "strong (global batch fixed, sharded by batch)" if world > 1 else "n/a",
           "timing": "CUDA graph of one round of draft steps (one append+decode launch per layer and step, "
                     "device-side lengths), CUDA events per round, rolled back between rounds, max over ranks",
           "gpu_launches": rounds * steps * wl.layers, "clocks": clocks.summary()}
    del loop, cache
    torch.cuda.empty_cache()
    return res


def measure_split_sequence(args, wl, world, rank, device, mode="delivered"):
    """One batch-1 sequence, its tokens split across the ranks (strong scaling).

    Each rank packs every layer and keeps its 32-token-aligned token shard
    (kv_reduce_b200.distributed.shard_component); a step is one partial
    decode launch over all layers of the shard and one exchange kernel.
    mode "delivered": the decode stores each finished row of (m, l, o)
    partials into every peer over NVLink as (value, epoch) words; the
    exchange kernel reads them until every word carries the step's epoch,
    and merges.  "push": the decode
    writes its partials locally; the exchange kernel stores them into every
    peer, signals and merges.  "nccl": an NCCL all-gather and the LSE merge
    kernel.  The step time is the max over ranks; the result counts the
    whole sequence's bytes once.  Returns the sub-dict (rank 0) and the
    exchange error count.
    """
    import torch.distributed as dist

    import kv_reduce_b200 as kvr
    from kv_reduce_b200 import distributed as kd
    from kv_reduce_b200 import workloads
    from kv_reduce_b200.packed_kv_attention import DecodeLaunch, _geometry, _layer_ptrs

    a, b = kd.token_shards(wl.seq_len, world, align=wl.group_size)[rank]
    ks, vs, qs = [], [], []
    for layer in range(wl.layers):
        k, v = workloads.make_layer_kv(wl, layer, device=device)
        pk, pv = kvr.pack_kivi_kv(k, v, k_bits=wl.k_bits, v_bits=wl.v_bits, group_size=wl.group_size,
                                  residual_length=wl.residual_length)
        sk, sv = kd.shard_component(pk, pv, a, b)
        del k, v, pk, pv
        ks.append(sk)
        vs.append(sv)
        qs.append(workloads.make_query(wl, layer, device=device))
    torch.cuda.synchronize()
    rows = wl.layers * wl.batch * wl.q_heads
    dummy = [torch.empty_like(q) for q in qs]
    geom = _geometry(qs[0], ks[0], vs[0])
    launch = DecodeLaunch(geom, [_layer_ptrs(q, o, k, v) for q, o, k, v in zip(qs, dummy, ks, vs)], device,
                          split_tokens=args.split_tokens)
    out = torch.empty(rows, wl.head_dim, dtype=torch.bfloat16, device=device)
    p2p = world > 1 and mode != "nccl"
    delivered = mode in ("delivered", "owner")
    owner = mode == "owner"
    if p2p:
        xchg = kd.PeerExchange(rows, wl.head_dim, device)

        def step():
            if delivered:
                xchg.step_delivered(launch, owner=owner)
            else:
                xchg.step(launch.partial)
    else:
        dec = kd.SequenceShardDecoder(rows, wl.head_dim, world, device, partial_fn=launch.partial,
                                      merge_fn=lambda ml, o: kvr.lse_merge(ml, o, out=out))

        def step():
            dec.step()

    for _ in range(2 * ((max(args.warmup, 3) + 1) // 2)):   # an even number: the graph pairs steps
        step()
    torch.cuda.synchronize()
    graph = None
    if p2p:
        # both steps of a pair (one per receive half) in one CUDA graph, the
        # partial launch bound to the capture stream
        side = torch.cuda.Stream(device)
        launch_g = DecodeLaunch(geom, [_layer_ptrs(q, o, k, v) for q, o, k, v in zip(qs, dummy, ks, vs)], device,
                                split_tokens=args.split_tokens, stream=side.cuda_stream)
        graph = xchg.capture_pair(launch_g if delivered else launch_g.partial, side, delivered=delivered,
                                  owner=owner)
        for _ in range(2):
            xchg.replay_pair(graph)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    pairs = max(1, args.steps // 2)
    n_steps = 2 * pairs if graph is not None else args.steps
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device) as clocks:
        s0.record()
        if graph is not None:
            for _ in range(pairs):
                xchg.replay_pair(graph)
        else:
            for _ in range(args.steps):
                step()
        s1.record()
        torch.cuda.synchronize()
    ms = max_over_ranks(s0.elapsed_time(s1) / n_steps, world, device)
    errors = xchg.errors() if p2p else 0
    errors = int(sum_over_ranks(errors, world, device))
    lb = workloads.layer_bytes(wl)
    step_bytes = lb["total"] * wl.layers
    peak, peak_src = measured_peak()
    value = step_bytes / (ms * 1e-3) / 1e9
    res = {"workload": wl.name, "layers": wl.layers, "global_batch": wl.batch, "seq_len": wl.seq_len,
           "parallelism": f"token-split x{world}", "shard_tokens": b - a, "num_splits": launch.num_splits,
           "us_per_step": ms * 1e3, "gbps": value, "tokens_per_s": wl.batch / (ms * 1e-3),
           "frac_per_gpu": value / world / peak, "frac_note": "of measured, per GPU", "steps": n_steps,
           "exchange": ("the decode stores each partial row into its owner rank over NVLink as (value, epoch) "
                        "words; the owner merges it and stores the merged bf16 row into every rank; a gather "
                        "kernel collects them" if p2p and owner else
                        "the decode stores its partial rows into every peer over NVLink as (value, epoch) "
                        "words; one wait-and-merge kernel"
                        if p2p and delivered else
                        "one kernel: NVLink peer stores + signal + LSE merge" if p2p else
                        "NCCL all-gather + LSE merge launch" if world > 1 else "none"),
           "exchange_errors": errors, "scaling": "strong (one sequence)",
           "timing": ("CUDA graph of two steps (partial decode of all layers + fused exchange)"
                      if graph is not None else
                      "eager: partial decode (all layers, one launch) + exchange/merge per step")
                     + ", CUDA events, max over ranks",
           "exchange_mode": mode if world > 1 else "none",
           "gpu_launches": n_steps * (3 if p2p and owner else 2), "clocks": clocks.summary()}
    del graph
    if p2p:
        xchg.close()
    del launch, ks, vs, qs
    torch.cuda.empty_cache()
    return res, errors


def init_pg(world, device):
    if world > 1:
        import torch.distributed as dist

        # the exchange's peer loads and stores are plain; keep NCCL's own
        # collectives (barriers, timing reductions) off NVLink multicast too
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
        return lambda: (dist.barrier(), torch.cuda.synchronize())
    return lambda: torch.cuda.synchronize()


def close_pg(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def run_ours(args, wl, world, rank, local):
    import kv_reduce_b200 as kvr
    from kv_reduce_b200 import workloads
    from kv_reduce_b200.packed_kv_attention import DecodeLaunch

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    pg_sync = init_pg(world, device)

    ks, vs, qs = build_cache(wl, device, rank)
    stream = torch.cuda.Stream(device)
    fused, outs, geom, ptrs = fused_launches(ks, vs, qs, device, stream, args.split_tokens)
    # one launch per layer, as a model calls it
    per_layer = [DecodeLaunch(geom, [p], device, split_tokens=args.split_tokens, stream=stream.cuda_stream)
                 for p in ptrs]
    torch.cuda.synchronize()
    lb = workloads.layer_bytes(wl)
    step_bytes = lb["total"] * wl.layers

    def step_fused():
        for launch in fused:
            launch()

    def step_per_layer():
        for launch in per_layer:
            launch()

    with ClockSampler(device) as clocks:
        ms_fused = time_graph(step_fused, stream, args.steps, args.warmup, world, pg_sync)
    ms_fused = max_over_ranks(ms_fused, world, device)
    ms_layers = max_over_ranks(time_graph(step_per_layer, stream, args.steps, args.warmup, world, pg_sync),
                               world, device)

    step_ms = ms_fused / args.steps
    value = step_bytes * world / (step_ms * 1e-3) / 1e9
    layer_step_ms = ms_layers / args.steps
    peak, peak_src = measured_peak()
    launch_us = step_ms * 1e3 / len(fused)
    bytes_per_launch = step_bytes / len(fused)
    achieved = bytes_per_launch / (launch_us * 1e-6) / 1e9

    # ---------------------------------------------------------------- e2e
    e2e = None
    e2e_per_layer = None
    e2e_layers_call = None
    if not args.no_e2e:
        q_host = [q.cpu().pin_memory() for q in qs]
        o_host = [torch.empty_like(h).pin_memory() for h in q_host]
        q_dev = [torch.empty_like(q) for q in qs]
        io_bytes = sum(q.numel() * q.element_size() for q in qs)
        # the decode loop's shape of the call: all layers' queries of the step
        # staged in one pinned buffer, one H2D copy, one decoder call, one D2H copy
        q_host_all = torch.stack([q.cpu() for q in qs]).pin_memory()
        o_host_all = torch.empty_like(q_host_all).pin_memory()
        decoder = kvr.PackedDecoder(ks, vs, q_heads=wl.q_heads, split_tokens=args.split_tokens)

        def e2e_decoder():
            decoder.host_step(q_host_all, o_host_all)

        def e2e_layers():
            for i in range(wl.layers):
                q_dev[i].copy_(q_host[i], non_blocking=True)
            res = kvr.packed_kv_decode_attention_layers(q_dev, ks, vs, split_tokens=args.split_tokens)
            for i in range(wl.layers):
                o_host[i].copy_(res[i], non_blocking=True)
            torch.cuda.current_stream().synchronize()

        def e2e_calls():
            res = []
            for i in range(wl.layers):
                q_dev[i].copy_(q_host[i], non_blocking=True)
                res.append(kvr.packed_kv_decode_attention(q_dev[i], ks[i], vs[i], split_tokens=args.split_tokens))
            for i in range(wl.layers):
                o_host[i].copy_(res[i], non_blocking=True)
            torch.cuda.current_stream().synchronize()

        def time_host(fn):
            for _ in range(max(args.warmup, 3)):
                fn()
            pg_sync()
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0 = time.perf_counter()
            s0.record()
            for _ in range(args.steps):
                fn()
            s1.record()
            torch.cuda.synchronize()
            wall_ms = (time.perf_counter() - t0) * 1e3
            return max_over_ranks(max(s0.elapsed_time(s1), wall_ms) / args.steps, world, device)

        e2e_ms = time_host(e2e_decoder)
        e2e = {"value": step_bytes * world / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
               "h2d_bytes_per_step": io_bytes, "d2h_bytes_per_step": io_bytes, "ms_per_step": e2e_ms,
               "path": "kv_reduce_b200.PackedDecoder.host_step (planned once) each step on the step's stacked "
                       "pinned host queries: the decode of all layers reads them in place (one CTA per (layer, "
                       "b, kv head) across PCIe, shared over distributed shared memory; an H2D copy when the "
                       "plan has no clusters) and its final merge writes the outputs into the pinned host "
                       "buffer, replayed as one CUDA graph, then a wait for the outputs",
               "queries_in_place": bool(decoder._host and decoder._host.get("queries_in_place"))}
        e2e_l_ms = time_host(e2e_layers)
        e2e_layers_call = {"value": step_bytes * world / (e2e_l_ms * 1e-3) / 1e9, "unit": "GB/s",
                           "ms_per_step": e2e_l_ms,
                           "path": "kv_reduce_b200.packed_kv_decode_attention_layers (validates every layer "
                                   "every call), per-layer query/output copies"}
        e2e_pl_ms = time_host(e2e_calls)
        e2e_per_layer = {"value": step_bytes * world / (e2e_pl_ms * 1e-3) / 1e9, "unit": "GB/s",
                         "ms_per_step": e2e_pl_ms,
                         "path": "kv_reduce_b200.packed_kv_decode_attention once per layer (the reference's call)"}
        del decoder

    num_splits = fused[0].num_splits
    per_layer_splits = per_layer[0].num_splits
    n_fused = len(fused)
    del fused, per_layer, outs, ptrs, ks, vs, qs
    torch.cuda.empty_cache()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample(wl, args.cpu_seconds, lb["total"])

    extra = None
    if not args.no_workloads:
        extra = {}
        for key in ("3a", "3b", "4"):
            extra[key] = measure_workload(args, key, world, rank, device, pg_sync)
        extra["5"] = measure_draft_loop(args, world, rank, device, pg_sync)

    split = None
    split_errors = 0
    if world > 1 and not args.no_workloads:
        pg_sync()
        split, split_errors = measure_split_best(args, wl, world, rank, device)

    if rank == 0:
        config = workload_config(wl, world, args)
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "us_per_step": step_ms * 1e3,
            "tokens_per_s": wl.batch * world / (step_ms * 1e-3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "u4 codes; f16/bf16 mma, fp32 accumulate and softmax",
            "data": "synthetic (seeded N(0,1) K/V/Q, outlier key channels)",
            "config": config,
            "plan": {"num_splits": num_splits, "per_layer_num_splits": per_layer_splits},
            "timing": "all layers of the step in one launch, CUDA graph, CUDA events, max over ranks",
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": profiled_traffic(wl.name),
                         "kernel": "kvr::dec::decode_kernel, all layers of the step per launch",
                         "bytes_per_launch": bytes_per_launch, "launch_us": launch_us, "peak_source": peak_src,
                         "frac_note": "of measured" if "measured" in peak_src else "of fallback"},
            "per_layer": {"ms_per_step": layer_step_ms, "us_per_layer": layer_step_ms * 1e3 / wl.layers,
                          "gbps": step_bytes * world / (layer_step_ms * 1e-3) / 1e9,
                          "num_splits": per_layer_splits,
                          "timing": "one launch per layer, 28 launches replayed as a CUDA graph"},
            "e2e": e2e, "e2e_layers_call": e2e_layers_call, "e2e_per_layer_calls": e2e_per_layer,
            "cpu_baseline": cpu,
            "workloads": extra,
            "split_sequence": split,
            "gpu_launches": args.steps * n_fused,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    close_pg(world)
    if split_errors:
        raise SystemExit(f"{split_errors} exchange wait(s) timed out in the sequence split")


def exchange_mode(args) -> str:
    return "nccl" if args.nccl_exchange else args.exchange


def measure_split_best(args, wl, world, rank, device):
    """The sequence split in the requested exchange mode; with "best", the
    delivered and the owner mode are both timed (same steps, same ranks)
    and the faster one is reported, with every mode's time beside it."""
    mode = exchange_mode(args)
    if mode != "best" or world == 1:
        return measure_split_sequence(args, wl, world, rank, device, mode="delivered" if mode == "best" else mode)
    results = {}
    errors = 0
    for m in ("delivered", "owner"):
        res, err = measure_split_sequence(args, wl, world, rank, device, mode=m)
        results[m] = res
        errors += err
    if rank != 0:
        return None, errors
    best = min(results, key=lambda m: results[m]["us_per_step"])
    out = dict(results[best])
    out["us_per_step_by_mode"] = {m: r["us_per_step"] for m, r in results.items()}
    return out, errors


def run_split_sequence(args, wl, world, rank, local):
    """--split-sequence: the sequence split as the whole line."""
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    init_pg(world, device)
    res, errors = measure_split_best(args, wl, world, rank, device)
    if rank == 0:
        line = {"metric": METRIC, "value": res["gbps"], "unit": "GB/s", "n_gpus": world, "steps": res["steps"],
                "warmup": args.warmup, "ms_per_step": res["us_per_step"] / 1e3, "us_per_step": res["us_per_step"],
                "tokens_per_s": res["tokens_per_s"], "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "u4 codes; f16/bf16 mma, fp32 accumulate and softmax",
                "data": "synthetic (seeded N(0,1) K/V/Q, outlier key channels)",
                "config": {"workload": wl.name, "layers": wl.layers, "global_batch": wl.batch,
                           "seq_len": wl.seq_len, "parallelism": res["parallelism"],
                           "shard_tokens": res["shard_tokens"], "num_splits": res["num_splits"],
                           "exchange": res["exchange"], "timing": res["timing"],
                           "us_per_step_by_mode": res.get("us_per_step_by_mode")},
                "per_gpu_fraction_of_peak": res["frac_per_gpu"], "exchange_errors": errors,
                "gpu_launches": res["gpu_launches"], "clocks": res["clocks"]}
        print(json.dumps(line), flush=True)
    close_pg(world)
    if errors:
        raise SystemExit(f"{errors} exchange wait(s) timed out")


def run_draft_loop(args, wl, world, rank, local):
    """--draft-loop: the speculative draft loop (workload 5) as the whole line."""
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    pg_sync = init_pg(world, device)
    res = measure_draft_loop(args, world, rank, device, pg_sync)
    if rank == 0:
        line = {"metric": "draft loop: us per draft step (append + decode, all layers)",
                "value": res["us_per_draft_step"], "unit": "us/step", "n_gpus": world, "steps": res["rounds"],
                "warmup": args.warmup, "higher_is_better": False,
                "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
                "dtype": "u4 codes; f16/bf16 mma, fp32 accumulate and softmax",
                "data": "synthetic (seeded N(0,1) K/V/Q, outlier key channels)",
                "config": {k: res[k] for k in ("workload", "layers", "global_batch", "batch_per_gpu", "seq_len",
                                               "draft_steps", "kv_bits")},
                "achieved_gbs": res["gbps"], "frac_of_peak_per_gpu": res["frac"],
                "append_errors": res["append_errors"], "timing": res["timing"],
                "gpu_launches": res["gpu_launches"], "clocks": res["clocks"]}
        print(json.dumps(line), flush=True)
    close_pg(world)


# ------------------------------------------------------------------- tools
def run_engine_ab(args):
    """Tensor cores vs CUDA cores for the packed decode attention.

    The decode kernel runs its GQA-group x token tiles on the tensor cores
    (kvr_decode_attention: mma.sync, codes as fp16 operands).  The
    alternative is the same computation on the CUDA cores
    (kvr_decode_attention_simt: fp32 FMA, same packed layout, split-K and LSE
    merge, every packed byte shared by the group's query heads).  One JSON
    line per workload and engine: all layers of a decode step, one launch per
    32 layers, replayed as a CUDA graph, CUDA events; every workload's packed
    cache is larger than the 126 MB L2, so no flush.
    """
    from kv_reduce_b200 import workloads
    from kv_reduce_b200.packed_kv_attention import DecodeLaunch, SimtDecodeLaunch, _geometry, _layer_ptrs

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    peak, _ = measured_peak()
    for key in args.configs.split(","):
        wl = workloads.CONFIGS[key]
        ks, vs, qs = build_cache(wl, device, 0)
        geom = _geometry(qs[0], ks[0], vs[0])
        step_bytes = workloads.layer_bytes(wl)["total"] * wl.layers
        stream = torch.cuda.Stream(device)
        first = None
        for engine, cls in (("tensor", DecodeLaunch), ("simt", SimtDecodeLaunch)):
            outs = [torch.empty_like(q) for q in qs]
            ptrs = [_layer_ptrs(q, o, k, v) for q, o, k, v in zip(qs, outs, ks, vs)]
            launches = [cls(geom, ptrs[i:i + 32], device, stream=stream.cuda_stream)
                        for i in range(0, wl.layers, 32)]

            def step():
                for launch in launches:
                    launch()

            ms = time_graph(step, stream, args.steps, args.warmup, 1, torch.cuda.synchronize)
            us = ms * 1e3 / args.steps
            out = torch.stack(outs).float()
            if first is None:
                first = out
            gbs = step_bytes / us / 1e3
            print(json.dumps({"workload": wl.name, "engine": engine, "us_per_step": round(us, 2),
                              "gbps": round(gbs, 1), "frac_of_measured_hbm": round(gbs / peak, 4),
                              "launches_per_step": len(launches),
                              "max_abs_diff_vs_tensor": float((out - first).abs().max())}), flush=True)
        del ks, vs, qs, first
        torch.cuda.empty_cache()


def run_all_kernels(args):
    """Every library kernel once per round at one layer of the 32K
    Qwen2.5-1.5B geometry (B=1, 2 KV heads, 12 query heads, D=128, K4V4,
    group 32, residual 128), for a profiler's launch list.  The packing
    kernels run on 8 sequences at once (134 MB of bf16 keys + values, more
    than the 126 MB L2)."""
    import kv_reduce_b200 as kvr
    from kv_reduce_b200 import workloads

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    wl = workloads.CONFIGS["2"]
    k8, v8 = workloads.make_layer_kv(wl, 0, device=dev, batch=8)
    k1, v1 = k8[:1].contiguous(), v8[:1].contiguous()
    q = workloads.make_query(wl, 0, device=dev)
    for _ in range(1 + args.repeat):
        pk8, pv8 = kvr.pack_kivi_kv(k8, v8, k_bits=4, v_bits=4, group_size=32, residual_length=128)
        pk8.unpack()
        pv8.unpack()
        pk, pv = kvr.pack_kivi_kv(k1, v1, k_bits=4, v_bits=4, group_size=32, residual_length=128)
        kvr.packed_kv_decode_attention(q, pk, pv)
        layer = kvr.PackedKVCacheLayer(1, wl.kv_heads, wl.head_dim, capacity=wl.seq_len + 256, device=dev)
        layer.prefill(k1, v1)
        for t in range(32):
            layer.append(k1[:, :, t:t + 1], v1[:, :, t:t + 1])
        layer.commit()
        rows = wl.layers * wl.q_heads
        ml = torch.zeros(4, rows, 2, device=dev)
        o = torch.randn(4, rows, wl.head_dim, device=dev)
        kvr.lse_merge(ml, o)
        codes = torch.randint(0, 16, (k8.numel(),), dtype=torch.uint8, device=dev)
        payload = kvr.pack_unsigned(codes, 4)
        kvr.unpack_unsigned(payload, 4, codes.numel())
        torch.cuda.synchronize()
        del pk8, pv8, pk, pv, layer


def main():
    args = parse_args()
    from kv_reduce_b200 import workloads

    if args.engine_ab:
        run_engine_ab(args)
        return
    if args.all_kernels:
        run_all_kernels(args)
        return
    if args.config not in workloads.CONFIGS:
        raise SystemExit(f"unknown --config {args.config}; choose from {sorted(workloads.CONFIGS)}")
    wl = workloads.CONFIGS[args.config]
    world, rank, local = dist_setup(args.gpus)
    if args.impl == "reference":
        run_reference(args, wl, world, rank)
        return
    if args.split_sequence:
        run_split_sequence(args, wl, world, rank, local)
        return
    if args.draft_loop:
        run_draft_loop(args, wl, world, rank, local)
        return
    run_ours(args, wl, world, rank, local)


if __name__ == "__main__":
    main()
