"""Draft loop captured once in a CUDA graph and replayed at growing lengths.

A speculative-decoding round runs a few draft steps; each step appends the
new token's key/value to every layer of the packed cache and decodes over it
(packed_review.py:23-31 + :76-78, one launch each per layer and step in the
reference).  ``DraftLoop`` records ``steps`` such steps for all layers of a
``PackedKVCache`` in one CUDA graph: per layer and step an append that
also advances the layer's device-side length, and a decode, both reading
the lengths from device memory, so the same graph replays at any length the
capacity allows (the append moves the length on itself once every block
has written).  Queries and new keys/values are read from (and outputs
written to) the loop's static buffers ``q``, ``k``, ``v``, ``out``.

Host-side ``commit`` / ``crop`` between rounds keep the device lengths in
step; the layers pin their residual buffer so the graph's addresses hold.
A capacity change (growth) needs a new capture, which ``replay`` does.
"""
from __future__ import annotations

from typing import List, Tuple

import torch

from . import _lib
from .packed_kv_attention import CacheGeometry, DecodeLaunch
from .streaming import PackedKVCache, PackedKVCacheLayer


class DraftLoop:
    def __init__(self, cache: PackedKVCache, *, q_heads: int, steps: int, split_tokens: int = 0) -> None:
        if steps < 1:
            raise ValueError("steps must be >= 1")
        self.cache, self.steps, self.q_heads = cache, int(steps), int(q_heads)
        self.split_tokens = int(split_tokens)
        l0 = cache.layers[0]
        L, B, H, D = len(cache.layers), l0.batch, l0.kv_heads, l0.head_dim
        if self.q_heads % H or self.q_heads // H > 8:
            raise ValueError("q_heads must be a multiple of the KV heads, at most 8 per KV head.")
        dev = l0.device
        bf = torch.bfloat16
        self.q = torch.zeros(self.steps, L, B, self.q_heads, 1, D, dtype=bf, device=dev)
        self.k = torch.zeros(self.steps, L, B, H, 1, D, dtype=bf, device=dev)
        self.v = torch.zeros_like(self.k)
        self.out = torch.zeros_like(self.q)
        for layer in cache.layers:
            layer.pin_residual = True
            layer.device_lengths()
        self.graph: torch.cuda.CUDAGraph | None = None
        self._signature: Tuple = ()
        self._keep: List = []

    # ----------------------------------------------------------- launches
    @staticmethod
    def _buffers(layer: PackedKVCacheLayer) -> Tuple:
        return (layer.key_payload.data_ptr(), layer.key_residual[layer._cur].data_ptr(),
                layer.value_payload.data_ptr(), layer.capacity, layer.cap_residual)

    def _decode_launch(self, layer: PackedKVCacheLayer, q: torch.Tensor, out: torch.Tensor,
                       stream: int) -> DecodeLaunch:
        res = layer.key_residual[layer._cur]
        geom = CacheGeometry(layer.batch, self.q_heads, layer.kv_heads, layer.head_dim, layer.capacity,
                             layer.cap_prefix, layer.group_size, layer.k_bits, layer.v_bits,
                             layer.key_payload.stride(1), layer.key_scale.stride(1), res.stride(1),
                             layer.value_payload.stride(1), layer.value_scale.stride(1))
        ptrs = _lib.LayerPtrs(layer.key_payload.data_ptr(), layer.key_scale.data_ptr(), layer.key_offset.data_ptr(),
                              res.data_ptr(), layer.value_payload.data_ptr(), layer.value_scale.data_ptr(),
                              layer.value_offset.data_ptr(), q.data_ptr(), out.data_ptr(),
                              _lib.ptr(layer.key_scale_pairs))
        return DecodeLaunch(geom, [ptrs], layer.device, split_tokens=self.split_tokens, stream=stream)

    def _append_args(self, layer: PackedKVCacheLayer, k: torch.Tensor, v: torch.Tensor) -> _lib.AppendArgs:
        res = layer.key_residual[layer._cur]
        a = _lib.AppendArgs()
        a.k, a.v = k.data_ptr(), v.data_ptr()
        a.key_residual, a.key_residual_bh_stride = res.data_ptr(), res.stride(1)
        a.value_payload, a.value_payload_bh_stride = layer.value_payload.data_ptr(), layer.value_payload.stride(1)
        a.value_scale, a.value_offset = layer.value_scale.data_ptr(), layer.value_offset.data_ptr()
        a.value_meta_bh_stride = layer.value_scale.stride(1)
        a.bh, a.n, a.seq_len, a.res_len = layer.batch * layer.kv_heads, 1, 0, 0
        a.res_capacity, a.seq_capacity = layer.cap_residual, layer.capacity
        a.head_dim, a.value_bits = layer.head_dim, layer.v_bits
        return a

    def _prepare(self, stream: int) -> List:
        """Argument blocks of every launch (planned and allocated here, never
        inside a stream capture)."""
        work = []
        for t in range(self.steps):
            for li, layer in enumerate(self.cache.layers):
                work.append((self._append_args(layer, self.k[t, li], self.v[t, li]),
                             layer.device_lengths().data_ptr(),
                             self._decode_launch(layer, self.q[t, li], self.out[t, li], stream),
                             layer.cap_residual))
        return work

    @staticmethod
    def _issue(work: List, stream: int) -> None:
        lib = _lib.load()
        for a, dl, launch, res_cap in work:   # one token per step: the decode launch appends it
            _lib.check("kvr_decode_step", lib.kvr_decode_step(launch.args, a.k, a.v, dl, res_cap, stream))

    def capture(self) -> None:
        """Record the loop into a CUDA graph (the lengths do not move)."""
        dev = self.cache.layers[0].device
        side = torch.cuda.Stream(dev)
        work = self._prepare(side.cuda_stream)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            self._issue(work, side.cuda_stream)
        self.graph, self._keep = g, work
        self._signature = tuple(self._buffers(layer) for layer in self.cache.layers)

    def _check_room(self) -> None:
        for layer in self.cache.layers:
            if (layer.seq_len + self.steps > layer.capacity
                    or layer.residual_len + self.steps > layer.cap_residual):
                raise ValueError("not enough capacity for the draft steps: commit or grow the cache first")

    def replay(self) -> torch.Tensor:
        """Run the recorded steps; returns ``out`` [steps, layers, B, HQ, 1, D]."""
        self._check_room()
        if self.graph is None or tuple(self._buffers(layer) for layer in self.cache.layers) != self._signature:
            self.capture()
        self.graph.replay()
        for layer in self.cache.layers:
            layer.seq_len += self.steps
        return self.out

    def run_eager(self) -> torch.Tensor:
        """The same steps without the graph: one launch per append and decode."""
        self._check_room()
        stream = _lib.stream_ptr(self.cache.layers[0].device)
        self._issue(self._prepare(stream), stream)
        for layer in self.cache.layers:
            layer.seq_len += self.steps
        return self.out

    def errors(self) -> int:
        """Non-zero if an append ran past a capacity (synchronises)."""
        return int(sum(int(layer.device_lengths()[2].item()) for layer in self.cache.layers))
