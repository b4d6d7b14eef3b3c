"""The sequence split's fused NVLink exchange + merge kernels
(kvr_exchange_merge, and the delivered mode: kvr_decode_partial_exchange +
kvr_exchange_merge_delivered, or + kvr_exchange_merge_owned +
kvr_exchange_gather_owned in owner mode).

On one GPU: the kernel's time-limited wait for a peer that never signals
runs out, sets the error flag and returns, and the next step completes; the
delivered mode with 2, 3 and 8 ranks emulated on one GPU (every launch
serialised on one stream, so each wait finds its words already written)
stores each rank's partials bit-identical to kvr_decode_partial and merges
bit-identical to kvr_lse_merge, and its wait for ranks that skip a step
runs out the same way.
On two GPUs (skipped with fewer): the split against the single-GPU decode of
the whole sequence, eagerly and as the replayed CUDA graph the benchmark
times, at the benchmarked 28-layer 32K shape, in every mode.
"""
import ctypes
import os
import socket
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result, seq_len, layers, graph_steps, mode):
    import torch.distributed as dist

    import kv_reduce_b200 as kvr
    from kv_reduce_b200 import distributed as kd
    from kv_reduce_b200 import workloads
    from kv_reduce_b200.packed_kv_attention import DecodeLaunch, _geometry, _layer_ptrs

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=device)
    try:
        wl = workloads.CONFIGS["2"].scaled(seq_len=seq_len, layers=layers)
        a, b = kd.token_shards(wl.seq_len, world, align=wl.group_size)[rank]
        ks, vs, qs, full = [], [], [], []
        for layer in range(wl.layers):
            k, v = workloads.make_layer_kv(wl, layer, device=device)
            pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=128)
            q = workloads.make_query(wl, layer, device=device)
            full.append(kvr.packed_kv_decode_attention(q, pk, pv, out_dtype=torch.float32))
            sk, sv = kd.shard_component(pk, pv, a, b)
            ks.append(sk), vs.append(sv), qs.append(q)
        dummy = [torch.empty_like(q) for q in qs]
        geom = _geometry(qs[0], ks[0], vs[0])
        launch = DecodeLaunch(geom, [_layer_ptrs(q, o, k, v) for q, o, k, v in zip(qs, dummy, ks, vs)], device)
        rows = wl.layers * wl.batch * wl.q_heads
        xchg = kd.PeerExchange(rows, wl.head_dim, device, timeout_s=5.0)
        ref = torch.cat([f.reshape(-1, wl.head_dim) for f in full])
        worst = 0.0
        for _ in range(4):   # both halves of the receive buffers, twice
            out = (xchg.step(launch.partial) if mode == "push"
                   else xchg.step_delivered(launch, owner=mode == "owner")).float()
            torch.cuda.synchronize()
            worst = max(worst, float((out - ref).abs().max()))
        if graph_steps:
            # the benchmark's form: both steps of a pair in one CUDA graph
            side = torch.cuda.Stream(device)
            launch_g = DecodeLaunch(geom, [_layer_ptrs(q, o, k, v) for q, o, k, v in zip(qs, dummy, ks, vs)],
                                    device, stream=side.cuda_stream)
            graph = xchg.capture_pair(launch_g.partial if mode == "push" else launch_g, side,
                                      delivered=mode != "push", owner=mode == "owner")
            for _ in range(graph_steps):
                xchg.replay_pair(graph)
                torch.cuda.synchronize()
                worst = max(worst, float((xchg.out.float() - ref).abs().max()))
            del graph
        errors = xchg.errors()
        xchg.close()
        result[rank] = (worst, errors, float(ref.abs().max()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("mode", ["push", "delivered", "owner"])
@pytest.mark.parametrize("seq_len,layers,graph_steps", [(5000, 3, 0), (32768, 28, 3)])
def test_two_gpu_sequence_split_fused_exchange(built_lib, seq_len, layers, graph_steps, mode):
    import torch.multiprocessing as mp

    world = 2
    with mp.get_context("spawn").Manager() as manager:
        result = manager.dict()
        mp.spawn(_worker, args=(world, _free_port(), result, seq_len, layers, graph_steps, mode),
                 nprocs=world, join=True)
        for rank in range(world):
            worst, errors, scale = result[rank]
            assert errors == 0
            # bf16 output of the merge vs the fp32 single-GPU result
            assert worst <= 2e-3 + scale * 2.0 ** -8, (rank, worst)


def test_exchange_wait_times_out_without_peer(built_lib):
    """World 2 emulated on one GPU: both receive buffers are local and only
    rank 0 runs, so its wait for rank 1's signal has nothing to end it but
    the 50 ms limit.  The kernel must return, raise the error flag, still
    have pushed its own partials and signal to the peer's buffer, and the
    next step -- with the peer's signal and an empty partial in place --
    must complete without error and equal rank 0's partial normalised."""
    from kv_reduce_b200 import _lib

    lib = _lib.load()
    world, rows, D = 2, 24, 128
    slot = rows * (2 + D)
    data_floats = 2 * world * slot
    bufs = [torch.zeros(data_floats + 64, dtype=torch.float32, device="cuda") for _ in range(world)]
    recv = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device="cuda")
    signal = recv + data_floats * 4
    state = torch.zeros(4, dtype=torch.int32, device="cuda")     # epoch, counter, error
    out = torch.empty(rows, D, dtype=torch.bfloat16, device="cuda")
    st = state.data_ptr()
    args = _lib.ExchangeArgs(world, 0, rows, D, recv.data_ptr(), signal.data_ptr(), st, st + 4, st + 8,
                             out.data_ptr(), 50_000_000)
    g = torch.Generator(device="cuda").manual_seed(11)

    def view(buf, parity, src):
        base = (parity * world + src) * slot
        return buf[base:base + 2 * rows].view(rows, 2), buf[base + 2 * rows:base + slot].view(rows, D)

    def fill_partial(parity):
        ml, o = view(bufs[0], parity, 0)
        ml[:, 0] = torch.randn(rows, generator=g, device="cuda")
        ml[:, 1] = torch.rand(rows, generator=g, device="cuda") + 0.5
        o.copy_(torch.randn(rows, D, generator=g, device="cuda"))
        return ml, o

    stream = torch.cuda.current_stream().cuda_stream
    fill_partial(1)                       # step 1 (epoch 1) uses receive half 1
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    assert lib.kvr_exchange_merge(ctypes.byref(args), stream) == _lib.KVR_OK
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert state[2].item() == 1, "the time-out did not raise the error flag"
    assert state[0].item() == 1 and state[1].item() == 0
    assert 0.04 <= waited < 5.0, waited
    ml1, o1 = view(bufs[0], 1, 0)
    pml, po = view(bufs[1], 1, 0)          # rank 0's slot in the peer's buffer
    assert torch.equal(pml, ml1) and torch.equal(po, o1)
    assert bufs[1].view(torch.int32)[data_floats].item() == 1    # rank 0 signalled epoch 1 to the peer

    # step 2: the peer has arrived with an empty partial (no tokens)
    state[2] = 0
    ml, o = fill_partial(0)
    eml, eo = view(bufs[0], 0, 1)
    eml[:, 0] = float("-inf")
    eml[:, 1] = 0.0
    eo.zero_()
    bufs[0].view(torch.int32)[data_floats + 1] = 2                 # rank 1's signal for epoch 2
    torch.cuda.synchronize()
    assert lib.kvr_exchange_merge(ctypes.byref(args), stream) == _lib.KVR_OK
    torch.cuda.synchronize()
    assert state[2].item() == 0 and state[0].item() == 2
    expect = o / ml[:, 1:2]
    assert torch.allclose(out.float(), expect, rtol=2.0 ** -8, atol=1e-6)


@pytest.mark.parametrize("owner", [False, True], ids=["to-all", "owner"])
@pytest.mark.parametrize("world", [2, 3, 8])
def test_delivered_exchange_ranks_on_one_gpu(built_lib, world, owner):
    """Delivered mode, `world` ranks emulated on one GPU, rows sent to every
    rank or (owner) only to the rank that merges them, which then sends the
    merged rows to every rank.  Every receive
    buffer and every rank's exchange state is local; the launches run in
    order on one stream (the decodes of ranks 0..world-1, then their
    merges), so every word a merge waits for was written by a decode that
    has already completed.  Per step: each rank's slot in EVERY receive
    area, as (value, epoch) words, is bit-identical to kvr_decode_partial
    over its shard, every word carries the step's epoch, every merge is
    bit-identical to kvr_lse_merge of all partials, and the result is the
    single-GPU decode of the whole sequence within the bf16 bound.  In owner
    mode each rank's area holds every source's words of the rows it owns,
    and its final area every other owner's merged rows, tagged.  Then rank 0
    alone takes a step and its bounded wait for the others runs out."""
    import kv_reduce_b200 as kvr
    from kv_reduce_b200 import _lib
    from kv_reduce_b200 import distributed as kd
    from kv_reduce_b200 import workloads
    from kv_reduce_b200.packed_kv_attention import DecodeLaunch, _geometry, _layer_ptrs

    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    wl = workloads.CONFIGS["2"].scaled(seq_len=5000, layers=3)
    D = wl.head_dim
    rows = wl.layers * wl.batch * wl.q_heads
    shards = kd.token_shards(wl.seq_len, world, align=wl.group_size)
    launches, full, keep = [], [], []
    per_rank = [([], [], []) for _ in range(world)]
    for layer in range(wl.layers):
        k, v = workloads.make_layer_kv(wl, layer, device="cuda")
        pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=128)
        q = workloads.make_query(wl, layer, device="cuda")
        full.append(kvr.packed_kv_decode_attention(q, pk, pv, out_dtype=torch.float32))
        for r, (a, b) in enumerate(shards):
            sk, sv = kd.shard_component(pk, pv, a, b)
            assert torch.equal(sk.scale_pairs, kvr.key_scale_pairs(sk.scale, 4))
            per_rank[r][0].append(sk), per_rank[r][1].append(sv), per_rank[r][2].append(q)
    for ks, vs, qs in per_rank:
        dummy = [torch.empty_like(q) for q in qs]
        keep.append(dummy)
        launches.append(DecodeLaunch(_geometry(qs[0], ks[0], vs[0]),
                                     [_layer_ptrs(q, o, k, v) for q, o, k, v in zip(qs, dummy, ks, vs)], dev))
    ref = torch.cat([f.reshape(-1, D) for f in full])
    # each rank's partials from the plain partial entry point
    parts = []
    for ln in launches:
        ml = torch.empty(rows, 2, dtype=torch.float32, device="cuda")
        o = torch.empty(rows, D, dtype=torch.float32, device="cuda")
        ln.partial(ml, o)
        parts.append((ml, o))
    merged = kvr.lse_merge(torch.stack([p[0] for p in parts]), torch.stack([p[1] for p in parts]))

    slot = rows * (2 + D)
    data_floats = 2 * world * slot
    bufs = [torch.zeros(data_floats + 64 + 2 * data_floats + 2 * rows * D, dtype=torch.float32, device="cuda")
            for _ in range(world)]
    recv = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device="cuda")
    signal = recv + data_floats * 4
    states = [torch.zeros(4, dtype=torch.int32, device="cuda") for _ in range(world)]
    outs = [torch.empty(rows, D, dtype=torch.bfloat16, device="cuda") for _ in range(world)]

    def xargs(r, timeout_ns=1_000_000_000):
        st = states[r].data_ptr()
        return _lib.ExchangeArgs(world, r, rows, D, recv.data_ptr(), signal.data_ptr(), st, st + 4, st + 8,
                                 outs[r].data_ptr(), timeout_ns, 1 if owner else 0)

    def merge(a):
        if owner:
            return (lib.kvr_exchange_merge_owned(ctypes.byref(a), stream),
                    lib.kvr_exchange_gather_owned(ctypes.byref(a), stream))
        return (lib.kvr_exchange_merge_delivered(ctypes.byref(a), stream),)

    args = [xargs(r) for r in range(world)]
    stream = torch.cuda.current_stream().cuda_stream
    for step in range(1, 5):   # both receive halves, twice
        for r, ln in enumerate(launches):
            assert lib.kvr_decode_partial_exchange(ln.args, ln.token_begin, ln.token_end, ctypes.byref(args[r]),
                                                   stream) == _lib.KVR_OK
        if owner:   # every owner merges before any rank gathers
            for fn in (lib.kvr_exchange_merge_owned, lib.kvr_exchange_gather_owned):
                for r in range(world):
                    assert fn(ctypes.byref(args[r]), stream) == _lib.KVR_OK
        else:
            for r in range(world):
                assert merge(args[r]) == (_lib.KVR_OK,)
        torch.cuda.synchronize()
        par = step & 1
        for r in range(world):
            assert states[r][2].item() == 0, "a wait timed out"
            assert states[r][0].item() == step and states[r][1].item() == 0
            words = bufs[r].view(torch.int32)[data_floats + 64:data_floats + 64 + 2 * data_floats]
            words = words.view(2, world, rows, 2 + D, 2)
            mine = torch.arange(rows, device="cuda") % world == r if owner else slice(None)
            for src in range(world):
                w = words[par, src][mine]
                assert bool((w[..., 1] == step).all()), "a word does not carry the step's epoch"
                assert torch.equal(w[:, :2, 0], parts[src][0][mine].view(torch.int32)), (step, r, src)
                assert torch.equal(w[:, 2:, 0], parts[src][1][mine].view(torch.int32)), (step, r, src)
            if owner:
                fin = bufs[r].view(torch.int32)[data_floats + 64 + 2 * data_floats:].view(2, rows, D // 2, 2)[par]
                others = torch.arange(rows, device="cuda") % world != r
                assert bool((fin[others][..., 1] == step).all())
                assert torch.equal(fin[others][..., 0], merged[others].view(torch.int32))
            assert torch.equal(outs[r], merged), (step, r)
        err = (outs[0].float() - ref).abs().max().item()
        assert err <= 2e-3 + ref.abs().max().item() * 2.0 ** -8, err
    # the other ranks do not take step 5: rank 0's merge finds their words
    # still tagged with step 3, its 50 ms wait runs out, the error flag is
    # raised and the kernel returns
    short = xargs(0, 50_000_000)
    ln = launches[0]
    assert lib.kvr_decode_partial_exchange(ln.args, ln.token_begin, ln.token_end, ctypes.byref(short),
                                           stream) == _lib.KVR_OK
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    assert all(st == _lib.KVR_OK for st in merge(short))
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert states[0][2].item() == 1, "the time-out did not raise the error flag"
    assert states[0][0].item() == 5 and states[0][1].item() == 0
    assert 0.04 <= waited < 5.0, waited
    # the exchange's rows must be the launch's layers x batch x q_heads
    bad = _lib.ExchangeArgs(world, 0, rows + 1, D, recv.data_ptr(), signal.data_ptr(), states[0].data_ptr(),
                            states[0].data_ptr() + 4, states[0].data_ptr() + 8, outs[0].data_ptr(), 1, int(owner))
    assert lib.kvr_decode_partial_exchange(launches[0].args, launches[0].token_begin, launches[0].token_end,
                                           ctypes.byref(bad), stream) == _lib.KVR_ERR_INVALID_ARGUMENT
