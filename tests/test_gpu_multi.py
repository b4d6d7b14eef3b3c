"""Sequence split across 2 GPUs with the fused NVLink exchange + merge kernel
(kvr_exchange_merge) against the single-GPU decode of the whole sequence.
Runs only where at least two GPUs are visible."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result):
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
        wl = workloads.CONFIGS["2"].scaled(seq_len=5000, layers=3)
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
            out = xchg.step(launch.partial).float()
            torch.cuda.synchronize()
            worst = max(worst, float((out - ref).abs().max()))
        errors = xchg.errors()
        xchg.close()
        result[rank] = (worst, errors, float(ref.abs().max()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_sequence_split_fused_exchange(built_lib):
    import torch.multiprocessing as mp

    world = 2
    with mp.get_context("spawn").Manager() as manager:
        result = manager.dict()
        mp.spawn(_worker, args=(world, _free_port(), result), nprocs=world, join=True)
        for rank in range(world):
            worst, errors, scale = result[rank]
            assert errors == 0
            # bf16 output of the merge vs the fp32 single-GPU result
            assert worst <= 2e-3 + scale * 2.0 ** -8, (rank, worst)
