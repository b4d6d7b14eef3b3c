"""Multi-GPU layouts of the packed decode path (one process per GPU).

Two partitions, both from the build's partitioning of batch x KV-head x
tokens:

* batch sharding (weak scaling): each rank owns whole sequences; decode is
  rank-local and needs no collective.  ``batch_shard`` picks a rank's slice.
* sequence split (one long sequence, batch 1): each rank owns a contiguous,
  32-token-aligned range of every layer's tokens.  A step is a partial
  decode per rank -- unnormalised (m, l, o) per query head, m in log2 units
  -- an all-gather of those partials (NCCL over NVLink, a few KB per
  layer), and an LSE merge.  ``shard_component`` cuts a rank's token range
  out of a packed component; ``SequenceShardDecoder`` runs the step.

The reference has no multi-GPU path (its only multi-device use places the
target and draft models on different GPUs,
kv_reduce/experiments/benchmark_spec_kv_quantization.py:1157-1158).
"""
from __future__ import annotations

from typing import Callable, List, Tuple

import torch

from .packed_kv_cache import PackedKVComponent

CHUNK = 32


def batch_shard(batch: int, world: int, rank: int) -> Tuple[int, int]:
    """[begin, end) of the sequences rank `rank` owns (near-equal split)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, extra = divmod(batch, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def token_shards(seq_len: int, world: int, align: int = CHUNK) -> List[Tuple[int, int]]:
    """Contiguous token ranges, boundaries multiples of `align`, the last
    range ending at seq_len.  Ranks past the end get empty ranges."""
    if world < 1 or align < 1:
        raise ValueError("bad world/align")
    units = -(-seq_len // align)
    out = []
    for r in range(world):
        a = (units * r // world) * align
        b = min(seq_len, (units * (r + 1) // world) * align)
        out.append((min(a, seq_len), max(min(a, seq_len), b)))
    return out


def shard_component(k: PackedKVComponent, v: PackedKVComponent, begin: int, end: int
                    ) -> Tuple[PackedKVComponent, PackedKVComponent]:
    """Tokens [begin, end) of a packed (keys, values) pair as a compact pair.

    `begin` must be a multiple of the key group size; the shard's quantized
    prefix is the part of [begin, end) below the global prefix, and only a
    shard reaching past the prefix holds BF16 residual rows.
    """
    B, H, S, D = (int(s) for s in k.shape)
    G, P = int(k.group_size), int(k.prefix_length)
    if not (0 <= begin < end <= S) or begin % G:
        raise ValueError("shard bounds must satisfy 0 <= begin < end <= S with begin % group_size == 0")
    if begin < P and end < P and end % G:
        raise ValueError("a shard ending inside the prefix must end on a group boundary")
    kb, vb = int(k.bits), int(v.bits)
    p_end = min(end, P)
    n_pref = max(0, p_end - begin)
    rbk, rbv = D * kb // 8, D * vb // 8
    kp = k.payload.reshape(B, H, P, rbk)[:, :, begin:begin + n_pref].contiguous().reshape(-1)
    ks = k.scale.reshape(B, H, P // G, 1, D)[:, :, begin // G:(begin + n_pref) // G].contiguous()
    ko = k.offset.reshape(B, H, P // G, 1, D)[:, :, begin // G:(begin + n_pref) // G].contiguous()
    # the decode's fp16 scale pairs are per group: the shard keeps its groups' rows
    ksp = (k.scale_pairs.reshape(B, H, P // G, 1, D)[:, :, begin // G:(begin + n_pref) // G].contiguous()
           if k.scale_pairs is not None else None)
    r0, r1 = max(begin, P) - P, max(end, P) - P
    res = k.residual[:, :, r0:r1].contiguous() if k.residual is not None else None
    vp = v.payload.reshape(B, H, S, rbv)[:, :, begin:end].contiguous().reshape(-1)
    vs = v.scale.reshape(B, H, S, 1)[:, :, begin:end].contiguous()
    vo = v.offset.reshape(B, H, S, 1)[:, :, begin:end].contiguous()
    shape = (B, H, end - begin, D)
    ks_out = PackedKVComponent(kp, ks, ko, res, shape, kb, k.layout, k.output_dtype, G, n_pref, scale_pairs=ksp)
    vs_out = PackedKVComponent(vp, vs, vo, None, shape, vb, v.layout, v.output_dtype)
    return ks_out, vs_out


def merge_partials(ml: torch.Tensor, o: torch.Tensor) -> torch.Tensor:
    """Reference LSE merge on any device: ml [N, rows, 2], o [N, rows, D] -> [rows, D] fp32."""
    m, l = ml[..., 0], ml[..., 1]
    M = m.max(dim=0).values
    w = torch.where(torch.isinf(m), torch.zeros_like(m), torch.exp2(m - M))
    L = (w * l).sum(0)
    out = (w[..., None] * o).sum(0)
    return torch.where(L[:, None] > 0, out / L.clamp_min(1e-30)[:, None], torch.zeros_like(out))


class SequenceShardDecoder:
    """One rank's side of a sequence-split decode step.

    partial_fn() fills this rank's (ml [rows, 2], o [rows, D]) partials;
    the step all-gathers them over the process group and merges them with
    merge_fn (the GPU kvr_lse_merge kernel in production; the torch
    reference merge in CPU tests).  Every rank takes the same collective
    steps in the same order.
    """

    def __init__(self, rows: int, head_dim: int, world: int, device: torch.device,
                 partial_fn: Callable[[torch.Tensor, torch.Tensor], None],
                 merge_fn: Callable[[torch.Tensor, torch.Tensor], torch.Tensor] | None = None,
                 group=None) -> None:
        self.rows, self.head_dim, self.world = rows, head_dim, world
        self.partial_fn = partial_fn
        self.merge_fn = merge_fn or merge_partials
        self.group = group
        self.ml = torch.empty(rows, 2, dtype=torch.float32, device=device)
        self.o = torch.empty(rows, head_dim, dtype=torch.float32, device=device)
        self.ml_all = torch.empty(world, rows, 2, dtype=torch.float32, device=device)
        self.o_all = torch.empty(world, rows, head_dim, dtype=torch.float32, device=device)

    def step(self) -> torch.Tensor:
        import torch.distributed as dist

        self.partial_fn(self.ml, self.o)
        if self.world > 1:
            if dist.get_backend(self.group) == "nccl":
                # one NCCL all-gather per buffer straight into the stacked output
                dist.all_gather_into_tensor(self.ml_all, self.ml, group=self.group)
                dist.all_gather_into_tensor(self.o_all, self.o, group=self.group)
            else:
                # gloo has no stacked form: gather into views of the same buffers
                dist.all_gather(list(self.ml_all.unbind(0)), self.ml, group=self.group)
                dist.all_gather(list(self.o_all.unbind(0)), self.o, group=self.group)
        else:
            self.ml_all[0].copy_(self.ml)
            self.o_all[0].copy_(self.o)
        return self.merge_fn(self.ml_all, self.o_all)


def empty_partial(ml: torch.Tensor, o: torch.Tensor) -> None:
    """Partials of a rank that owns no tokens: no mass (m = -inf, l = 0)."""
    ml[:, 0].fill_(float("-inf"))
    ml[:, 1].zero_()
    o.zero_()


class _DeviceMemory:
    """A raw device range seen by torch.as_tensor (no copy, no ownership)."""

    def __init__(self, ptr: int, shape: Tuple[int, ...], typestr: str) -> None:
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerExchange:
    """Fused cross-GPU exchange + LSE merge of sequence-split partials.

    Every rank allocates a receive buffer, shares its CUDA IPC handle over the
    process group and maps every peer's buffer.  A step writes this rank's
    partials (partial_fn(ml [rows, 2], o [rows, D]), e.g. a DecodeLaunch's
    ``partial``) into its own buffer, then ``kvr_exchange_merge`` pushes them
    into every peer over NVLink, signals, waits for the peers (bounded by
    ``timeout_s``) and merges all ranks into the bf16 output -- one kernel in
    place of an all-gather collective and a merge launch.  All ranks make the
    same calls in the same order; ``close()`` is collective too.

    ``step_delivered(launch)`` is the fused form for a DecodeLaunch over this
    rank's token shard: the decode kernel itself stores every finished row
    of partials into each rank's receive area as (value, epoch) words
    (kvr_decode_partial_exchange), so the rows cross NVLink while the
    decode is still running and nothing is fenced; the exchange kernel
    (kvr_exchange_merge_delivered) reads the words until every one carries
    the step's epoch, and merges.  ``step_delivered(launch, owner=True)``
    sends each row only to its owner rank (row % world), which merges it
    (kvr_exchange_merge_owned) and sends the merged bf16 row to every rank
    as tagged words (kvr_exchange_gather_owned collects them): a
    reduce-scatter and an all-gather, about 1/world of the bytes for one
    more hop.
    """

    def __init__(self, rows: int, head_dim: int, device: torch.device, group=None,
                 timeout_s: float = 2.0) -> None:
        import ctypes

        import torch.distributed as dist

        from . import _lib

        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.rows, self.head_dim, self.device, self.group = int(rows), int(head_dim), device, group
        slot = self.rows * (2 + self.head_dim)
        data_bytes = 2 * self.world * slot * 4
        ll_bytes = 2 * data_bytes   # delivered mode: (value, epoch) words after the signal area
        final_bytes = 8 * self.rows * self.head_dim   # owner mode: merged rows as (bf16 pair, epoch) words
        own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        _lib.call("kvr_exchange_alloc", data_bytes + 256 + ll_bytes + final_bytes, ctypes.byref(own), handle)
        self._own = own.value
        mine = torch.tensor(list(handle.raw), dtype=torch.uint8, device=device)
        handles = torch.empty(self.world, 64, dtype=torch.uint8, device=device)
        if dist.get_backend(group) == "nccl":
            dist.all_gather_into_tensor(handles, mine, group=group)
        else:
            dist.all_gather(list(handles.unbind(0)), mine, group=group)
        handles = handles.cpu()
        self._peers: List[int] = []
        for r in range(self.world):
            if r == self.rank:
                self._peers.append(self._own)
                continue
            p = ctypes.c_void_p()
            _lib.call("kvr_exchange_open", bytes(handles[r].tolist()), ctypes.byref(p))
            self._peers.append(p.value)
        self.recv_ptrs = torch.tensor(self._peers, dtype=torch.int64, device=device)
        self.signal_ptrs = self.recv_ptrs + data_bytes
        self.state = torch.zeros(4, dtype=torch.int32, device=device)   # epoch, counter, error
        self.out = torch.empty(self.rows, self.head_dim, dtype=torch.bfloat16, device=device)
        self._views = []
        for parity in (0, 1):
            base = self._own + ((parity * self.world + self.rank) * slot) * 4
            ml = torch.as_tensor(_DeviceMemory(base, (self.rows, 2), "<f4"), device=device)
            o = torch.as_tensor(_DeviceMemory(base + 2 * self.rows * 4, (self.rows, self.head_dim), "<f4"),
                                device=device)
            self._views.append((ml, o))
        st = self.state.data_ptr()
        self._args = _lib.ExchangeArgs(self.world, self.rank, self.rows, self.head_dim, self.recv_ptrs.data_ptr(),
                                       self.signal_ptrs.data_ptr(), st, st + 4, st + 8, self.out.data_ptr(),
                                       int(timeout_s * 1e9), 0)
        self._args_owner = _lib.ExchangeArgs.from_buffer_copy(self._args)
        self._args_owner.mode = 1
        self.steps = 0
        torch.cuda.synchronize(device)
        dist.barrier(group=group)

    def step(self, partial_fn: Callable[[torch.Tensor, torch.Tensor], None]) -> torch.Tensor:
        from . import _lib

        n = self.steps + 1
        ml, o = self._views[n & 1]
        partial_fn(ml, o)
        _lib.call("kvr_exchange_merge", self._args, _lib.stream_ptr(self.device))
        self.steps = n
        return self.out

    def step_delivered(self, launch, owner: bool = False) -> torch.Tensor:
        """One step of the delivered mode on ``launch``'s stream: the decode
        over launch's token range with its rows stored into every rank's
        receive buffer, then the wait-and-merge kernel; with ``owner``, the
        rows go to their owner ranks only, then the owner merge and the
        gather of the merged rows."""
        import ctypes

        from . import _lib

        if launch.geom.head_dim != self.head_dim or len(launch.layers) * launch.geom.batch * launch.geom.q_heads != self.rows:
            raise ValueError("the launch's rows (layers x batch x q_heads) and head_dim must match the exchange")
        lib = _lib.load()
        x = self._args_owner if owner else self._args
        _lib.check("kvr_decode_partial_exchange", lib.kvr_decode_partial_exchange(
            launch.args, launch.token_begin, launch.token_end, ctypes.byref(x), launch.stream))
        if owner:
            _lib.check("kvr_exchange_merge_owned", lib.kvr_exchange_merge_owned(x, launch.stream))
            _lib.check("kvr_exchange_gather_owned", lib.kvr_exchange_gather_owned(x, launch.stream))
        else:
            _lib.check("kvr_exchange_merge_delivered", lib.kvr_exchange_merge_delivered(x, launch.stream))
        self.steps += 1
        return self.out

    def capture_pair(self, partial_fn: Callable[[torch.Tensor, torch.Tensor], None],
                     stream: torch.cuda.Stream, delivered: bool = False, owner: bool = False) -> torch.cuda.CUDAGraph:
        """Record two consecutive steps -- one per receive half -- into a CUDA
        graph on `stream` (partial_fn must launch on the current stream; with
        ``delivered``, partial_fn is a DecodeLaunch bound to `stream` and the
        steps are ``step_delivered(partial_fn, owner)``).  The exchange kernels read their epoch
        from device memory, so the graph can be replayed any number of times
        with ``replay_pair``; every rank records and replays its pair in step
        with the others."""
        if self.steps % 2:
            raise ValueError("capture after an even number of steps")
        g = torch.cuda.CUDAGraph()
        torch.cuda.synchronize(self.device)
        with torch.cuda.graph(g, stream=stream):
            for _ in range(2):
                if delivered:
                    self.step_delivered(partial_fn, owner)
                else:
                    self.step(partial_fn)
        self.steps -= 2   # they run when the graph is replayed
        return g

    def replay_pair(self, graph: torch.cuda.CUDAGraph) -> torch.Tensor:
        graph.replay()
        self.steps += 2
        return self.out

    def errors(self) -> int:
        """Non-zero if a wait for a peer timed out (synchronises)."""
        return int(self.state[2].item())

    def close(self) -> None:
        import torch.distributed as dist

        from . import _lib

        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for r, p in enumerate(self._peers):
            if r != self.rank:
                _lib.call("kvr_exchange_close", p)
        dist.barrier(group=self.group)
        _lib.call("kvr_exchange_free", self._own)
        self._peers = []
