"""World-size-2 gloo tests of the multi-GPU host logic, on CPU.

The GPU partial-decode kernel is replaced by the oracle's partials for the
rank's token shard; the sharding, the collective steps and the LSE merge are
the production code.  Failure handling: a rank that never joins makes the
others' collective end with an error after the process-group timeout.
"""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kv_reduce_b200 import distributed as kd
from oracle import attention


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _data(seq_len=1000, hq=12, hkv=2, d=64):
    rng = np.random.default_rng(42)
    q = rng.standard_normal((1, hq, d))
    k = rng.standard_normal((1, hkv, seq_len, d))
    v = rng.standard_normal((1, hkv, seq_len, d))
    return q, k, v


def _seq_split_worker(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    q, k, v = _data()
    a, b = kd.token_shards(k.shape[2], world)[rank]

    def partial_fn(ml, o):
        if b <= a:
            kd.empty_partial(ml, o)
            return
        m, l, oo = attention.partials(q, k[:, :, a:b], v[:, :, a:b])
        ml[:, 0] = torch.from_numpy(m.reshape(-1))
        ml[:, 1] = torch.from_numpy(l.reshape(-1))
        o.copy_(torch.from_numpy(oo.reshape(-1, q.shape[-1])))

    dec = kd.SequenceShardDecoder(rows=12, head_dim=64, world=world, device=torch.device("cpu"),
                                  partial_fn=partial_fn)
    out = dec.step()
    full = attention.decode_attention(q, k, v).reshape(12, 64)
    out_q.put((rank, float(np.abs(out.numpy() - full).max())))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sequence_split_gloo(world):
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_seq_split_worker, args=(r, world, port, out_q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    errs = dict(out_q.get(timeout=5) for _ in range(world))
    assert all(e < 1e-5 for e in errs.values()), errs


def _absent_peer_worker(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    if rank == 1:
        dist.destroy_process_group()   # leaves between steps, joins no collective
        out_q.put((rank, "left"))
        return
    try:
        t = torch.zeros(4)
        dist.all_reduce(t)
        out_q.put((rank, "completed"))
    except Exception as e:  # the collective ends with an error, it does not hang
        out_q.put((rank, "error:" + type(e).__name__))


def test_absent_rank_raises_not_hangs():
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_absent_peer_worker, args=(r, 2, port, out_q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    res = dict(out_q.get(timeout=5) for _ in range(2))
    assert res[1] == "left"
    assert res[0].startswith("error:")


def test_token_and_batch_shards():
    assert kd.token_shards(32768, 8) == [(i * 4096, (i + 1) * 4096) for i in range(8)]
    sh = kd.token_shards(1057, 4)
    assert sh[0][0] == 0 and sh[-1][1] == 1057
    assert all(a % 32 == 0 for a, _ in sh)
    assert all(b1 == a2 for (_, b1), (a2, _) in zip(sh, sh[1:]))
    assert kd.token_shards(40, 4)[-1][1] == 40
    assert [kd.batch_shard(128, 8, r) for r in (0, 7)] == [(0, 16), (112, 128)]
    assert kd.batch_shard(10, 4, 3) == (8, 10)


def test_merge_partials_torch_matches_oracle():
    q, k, v = _data(seq_len=500)
    parts = [attention.partials(q, k[:, :, a:b], v[:, :, a:b]) for a, b in ((0, 128), (128, 160), (160, 500))]
    ml = torch.stack([torch.stack([torch.from_numpy(m.reshape(-1)), torch.from_numpy(l.reshape(-1))], -1)
                      for m, l, _ in parts])
    o = torch.stack([torch.from_numpy(oo.reshape(-1, 64)) for _, _, oo in parts])
    empty_ml = torch.tensor([[float("-inf"), 0.0]] * 12, dtype=ml.dtype)[None]
    ml = torch.cat([ml, empty_ml])
    o = torch.cat([o, torch.zeros(1, 12, 64, dtype=o.dtype)])
    out = kd.merge_partials(ml, o)
    full = attention.decode_attention(q, k, v).reshape(12, 64)
    assert np.abs(out.numpy() - full).max() < 1e-10
