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

With --gpus N (torchrun) each rank holds its own batch-1 sequence (weak
scaling, batch sharding, no collective on the data path); the step time is
the max over ranks.  ``--impl reference`` times the reference's unfused CPU
path (unpack + SDPA, restated in oracle/cpu_baseline.py) on the host cores.
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
    p.add_argument("--nccl-exchange", action="store_true",
                   help="--split-sequence: exchange partials with NCCL all-gather instead of the fused kernel")
    p.add_argument("--draft-loop", action="store_true",
                   help="speculative draft loop on the streaming cache (use with --config 5)")
    p.add_argument("--split-sequence", action="store_true",
                   help="N>1: split ONE batch-1 sequence's tokens across the ranks (strong scaling, "
                        "partial decode + NCCL all-gather + LSE merge) instead of one sequence per rank")
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
def cpu_baseline_sample(wl, seconds: float, layer_bytes: int):
    """Reference unfused path (unpack K, unpack V, SDPA) on host cores, one
    32K-token layer repeated for about `seconds`."""
    import numpy as np

    from kv_reduce_b200 import workloads
    from oracle import cpu_baseline

    torch.set_num_threads(os.cpu_count() or 1)
    k, v = workloads.make_layer_kv(wl, 0, device="cpu")
    q = workloads.make_query(wl, 0, device="cpu")
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    pk, pv = cpu_baseline.pack_cpu(bits(k), bits(v), wl.k_bits, wl.v_bits, wl.group_size, wl.residual_length)
    cpu_baseline.unfused_decode(q, pk, pv)   # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        cpu_baseline.unfused_decode(q, pk, pv)
        n += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = (time.perf_counter() - t0) / n
    return {"value": layer_bytes / dt / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{n} x one {wl.seq_len}-token layer of the {wl.name} workload (unpack + SDPA, bf16)",
            "ms_per_layer": dt * 1e3, "ms_per_step_extrapolated": dt * 1e3 * wl.layers}


def run_reference(args, wl, world, rank):
    from kv_reduce_b200 import workloads

    if rank != 0:
        return
    lb = workloads.layer_bytes(wl)["total"]
    torch.set_num_threads(os.cpu_count() or 1)
    import numpy as np

    from oracle import cpu_baseline

    k, v = workloads.make_layer_kv(wl, 0, device="cpu")
    q = workloads.make_query(wl, 0, device="cpu")
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    pk, pv = cpu_baseline.pack_cpu(bits(k), bits(v), wl.k_bits, wl.v_bits, wl.group_size, wl.residual_length)
    for _ in range(args.warmup):
        cpu_baseline.unfused_decode(q, pk, pv)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        cpu_baseline.unfused_decode(q, pk, pv)
        times.append(time.perf_counter() - t0)
    dt = sum(times) / len(times)
    value = lb / dt / 1e9
    sample = f"one {wl.seq_len}-token layer per step (of {wl.layers}), unpack + SDPA in bf16 on host cores"
    line = {"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt * 1e3 * wl.layers, "ms_per_step_note": "extrapolated: layer time x layers",
            "us_per_step": dt * 1e6 * wl.layers,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": wl.name, "layers": wl.layers, "batch": wl.batch, "seq_len": wl.seq_len,
                       "q_heads": wl.q_heads, "kv_heads": wl.kv_heads, "head_dim": wl.head_dim,
                       "kv_bits": f"K{wl.k_bits}V{wl.v_bits}", "group_size": wl.group_size,
                       "residual": wl.residual_length},
            "cpu_baseline": {"value": value, "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm
def build_cache(wl, device, rank):
    import kv_reduce_b200 as kvr
    from kv_reduce_b200 import workloads

    seed_wl = wl.scaled(seed=wl.seed + 100 * rank)
    ks, vs, qs = [], [], []
    for layer in range(wl.layers):
        k, v = workloads.make_layer_kv(seed_wl, layer, device=device)
        pk, pv = kvr.pack_kivi_kv(k, v, k_bits=wl.k_bits, v_bits=wl.v_bits, group_size=wl.group_size,
                                  residual_length=wl.residual_length)
        del k, v
        ks.append(pk)
        vs.append(pv)
        qs.append(workloads.make_query(seed_wl, layer, device=device))
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


def run_ours(args, wl, world, rank, local):
    import kv_reduce_b200 as kvr
    from kv_reduce_b200 import workloads
    from kv_reduce_b200.packed_kv_attention import DecodeLaunch, _geometry, _layer_ptrs

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
        pg_sync = lambda: (dist.barrier(), torch.cuda.synchronize())  # noqa: E731
    else:
        pg_sync = lambda: torch.cuda.synchronize()  # noqa: E731

    ks, vs, qs = build_cache(wl, device, rank)
    outs = [torch.empty_like(q) for q in qs]
    geom = _geometry(qs[0], ks[0], vs[0])
    stream = torch.cuda.Stream(device)
    ptrs = [_layer_ptrs(q, o, k, v) for q, o, k, v in zip(qs, outs, ks, vs)]
    # the whole step in one launch per <= 32 layers (layer index in the grid)
    fused = [DecodeLaunch(geom, ptrs[i:i + 32], device, split_tokens=args.split_tokens, stream=stream.cuda_stream)
             for i in range(0, wl.layers, 32)]
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
                       "pinned host queries: H2D copy, decode of all layers and D2H copy of the outputs replayed "
                       "as one CUDA graph, then a wait for the outputs"}
        e2e_l_ms = time_host(e2e_layers)
        e2e_layers_call = {"value": step_bytes * world / (e2e_l_ms * 1e-3) / 1e9, "unit": "GB/s",
                           "ms_per_step": e2e_l_ms,
                           "path": "kv_reduce_b200.packed_kv_decode_attention_layers (validates every layer "
                                   "every call), per-layer query/output copies"}
        e2e_pl_ms = time_host(e2e_calls)
        e2e_per_layer = {"value": step_bytes * world / (e2e_pl_ms * 1e-3) / 1e9, "unit": "GB/s",
                         "ms_per_step": e2e_pl_ms,
                         "path": "kv_reduce_b200.packed_kv_decode_attention once per layer (the reference's call)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample(wl, args.cpu_seconds, lb["total"])

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "us_per_step": step_ms * 1e3,
            "tokens_per_s": wl.batch * world / (step_ms * 1e-3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "u4 codes; f16/bf16 mma, fp32 accumulate and softmax",
            "data": "synthetic (seeded N(0,1) K/V/Q, outlier key channels)",
            "config": {"workload": wl.name, "layers": wl.layers, "batch_per_gpu": wl.batch,
                       "global_batch": wl.batch * world, "seq_len": wl.seq_len, "q_heads": wl.q_heads,
                       "kv_heads": wl.kv_heads, "head_dim": wl.head_dim, "kv_bits": f"K{wl.k_bits}V{wl.v_bits}",
                       "group_size": wl.group_size, "residual": wl.residual_length,
                       "parallelism": f"batch-sharded x{world}", "split_tokens": args.split_tokens,
                       "num_splits": fused[0].num_splits,
                       "l2": f"inputs {step_bytes / 1e6:.0f} MB per step > 126 MB L2; layers rotate, no flush",
                       "timing": "all layers of the step in one launch, CUDA graph, CUDA events, max over ranks"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": profiled_traffic(wl.name),
                         "kernel": "kvr::dec::decode_kernel, all layers of the step per launch",
                         "bytes_per_launch": bytes_per_launch, "launch_us": launch_us, "peak_source": peak_src,
                         "frac_note": "of measured" if "measured" in peak_src else "of fallback"},
            "per_layer": {"ms_per_step": layer_step_ms, "us_per_layer": layer_step_ms * 1e3 / wl.layers,
                          "gbps": step_bytes * world / (layer_step_ms * 1e-3) / 1e9,
                          "num_splits": per_layer[0].num_splits,
                          "timing": "one launch per layer, 28 launches replayed as a CUDA graph"},
            "e2e": e2e, "e2e_layers_call": e2e_layers_call, "e2e_per_layer_calls": e2e_per_layer,
            "cpu_baseline": cpu,
            "gpu_launches": args.steps * len(fused),
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def run_split_sequence(args, wl, world, rank, local):
    """One batch-1 sequence, its tokens split across the ranks (strong scaling).

    Each rank packs every layer and keeps its 32-token-aligned token shard
    (kv_reduce_b200.distributed.shard_component); a step is one partial
    decode launch over all layers of the shard and one exchange kernel that
    stores the (m, l, o) partials into every peer over NVLink and merges
    them (--nccl-exchange: an NCCL all-gather and the LSE merge kernel).  The step time is the max
    over ranks; `value` counts the whole sequence's bytes once.
    """
    import torch.distributed as dist

    import kv_reduce_b200 as kvr
    from kv_reduce_b200 import distributed as kd
    from kv_reduce_b200 import workloads
    from kv_reduce_b200.packed_kv_attention import DecodeLaunch, _geometry, _layer_ptrs

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
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
    p2p = world > 1 and not args.nccl_exchange
    if p2p:
        xchg = kd.PeerExchange(rows, wl.head_dim, device)

        def step():
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
        graph = xchg.capture_pair(launch_g.partial, side)
        for _ in range(2):
            xchg.replay_pair(graph)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    pairs = max(1, args.steps // 2)
    n_steps = 2 * pairs if graph is not None else args.steps
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    if graph is not None:
        for _ in range(pairs):
            xchg.replay_pair(graph)
    else:
        for _ in range(args.steps):
            step()
    s1.record()
    torch.cuda.synchronize()
    ms = s0.elapsed_time(s1) / n_steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    lb = workloads.layer_bytes(wl)
    step_bytes = lb["total"] * wl.layers
    if rank == 0:
        peak, peak_src = measured_peak()
        value = step_bytes / (ms * 1e-3) / 1e9
        line = {"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": n_steps,
                "warmup": args.warmup, "ms_per_step": ms, "us_per_step": ms * 1e3,
                "tokens_per_s": wl.batch / (ms * 1e-3), "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "u4 codes; f16/bf16 mma, fp32 accumulate and softmax",
                "data": "synthetic (seeded N(0,1) K/V/Q, outlier key channels)",
                "config": {"workload": wl.name, "layers": wl.layers, "global_batch": wl.batch,
                           "seq_len": wl.seq_len, "parallelism": f"token-split x{world}",
                           "shard_tokens": b - a, "num_splits": launch.num_splits,
                           "exchange": ("one kernel: NVLink peer stores + signal + LSE merge" if p2p else
                                        "NCCL all-gather + LSE merge launch" if world > 1 else "none"),
                           "timing": ("CUDA graph of two steps (partial decode of all layers + fused exchange)"
                                      if graph is not None else
                                      "eager: partial decode (all layers, one launch) + exchange/merge per step")
                                     + ", CUDA events, max over ranks"},
                "per_gpu_fraction_of_peak": value / world / peak, "peak_source": peak_src,
                "gpu_launches": args.steps * 2}
        print(json.dumps(line), flush=True)
    if p2p:
        errors = xchg.errors()
        del graph
        xchg.close()
        if errors:
            raise SystemExit(f"rank {rank}: {errors} exchange wait(s) timed out")
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_draft_loop(args, wl, world, rank, local):
    """Speculative draft loop on the streaming cache (default workload 5):
    rounds of `draft_steps` steps, each step appending one token to every
    layer and decoding over it.  Times the CUDA-graph replay of a round
    (device-side lengths, one capture) against issuing the same launches
    eagerly; each round is rolled back to the starting length so every round
    sees the same cache.  Per rank: its own batch (weak scaling)."""
    import torch.distributed as dist

    import kv_reduce_b200 as kvr
    from kv_reduce_b200 import workloads
    from kv_reduce_b200.draft import DraftLoop

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    steps = max(1, wl.draft_steps or 4)
    cache = kvr.PackedKVCache(wl.layers, wl.batch, wl.kv_heads, wl.head_dim, k_bits=wl.k_bits, v_bits=wl.v_bits,
                              group_size=wl.group_size, residual_length=wl.residual_length,
                              capacity=wl.seq_len + 64, device=device)
    seed_wl = wl.scaled(seed=wl.seed + 100 * rank)
    for i, layer in enumerate(cache.layers):
        k, v = workloads.make_layer_kv(seed_wl, i, device=device)
        layer.prefill(k, v)
        del k, v
    loop = DraftLoop(cache, q_heads=wl.q_heads, steps=steps, split_tokens=args.split_tokens)
    g = torch.Generator(device=device).manual_seed(1234 + rank)
    for t in (loop.q, loop.k, loop.v):
        t.copy_(torch.randn(t.shape, generator=g, device=device).to(torch.bfloat16))
    start = cache.get_seq_length()

    def timed(fn):
        ev = []
        for i in range(max(args.warmup, 3) + args.steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            cache.crop(start)
            if i >= max(args.warmup, 3):
                ev.append((e0, e1))
        torch.cuda.synchronize()
        ms = sum(a.elapsed_time(b) for a, b in ev) / len(ev)
        return max_over_ranks(ms, world, device)

    graph_ms = timed(loop.replay)
    eager_ms = timed(loop.run_eager)
    errors = loop.errors()
    # algorithmic bytes per draft step: the decode's bytes at the step's length
    # plus the appended token (key row, value codes and metadata) per layer
    step_bytes = sum(workloads.layer_bytes(wl, seq_len=start + t + 1)["total"] for t in range(steps)) / steps
    step_bytes = step_bytes * wl.layers + wl.layers * wl.batch * wl.kv_heads * (
        2 * wl.head_dim + wl.head_dim * wl.v_bits // 8 + 4)
    us_step = graph_ms * 1e3 / steps
    if rank == 0:
        peak, peak_src = measured_peak()
        line = {"metric": "draft loop: us per draft step (append + decode, all layers)", "value": us_step,
                "unit": "us/step", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
                "dtype": "u4 codes; f16/bf16 mma, fp32 accumulate and softmax",
                "data": "synthetic (seeded N(0,1) K/V/Q, outlier key channels)",
                "config": {"workload": wl.name, "layers": wl.layers, "batch_per_gpu": wl.batch,
                           "seq_len": start, "draft_steps": steps, "kv_bits": f"K{wl.k_bits}V{wl.v_bits}",
                           "timing": "CUDA graph of one round (device-side lengths) vs the same launches "
                                     "issued eagerly; CUDA events per round, rolled back between rounds"},
                "graph_us_per_draft_step": us_step, "eager_us_per_draft_step": eager_ms * 1e3 / steps,
                "achieved_gbs": step_bytes / (us_step * 1e-6) / 1e9 * world,
                "frac_of_peak_per_gpu": step_bytes / (us_step * 1e-6) / 1e9 / peak, "peak_source": peak_src,
                "append_errors": errors,
                # one launch per layer and draft step: the decode appends the token itself
                "gpu_launches": args.steps * steps * wl.layers}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse_args()
    from kv_reduce_b200 import workloads

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
