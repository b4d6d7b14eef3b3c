"""Decode attention over bit-packed KV: the API of
kv_reduce/triton_packed_kv_attention.py on sm_100a.

``packed_kv_decode_attention`` keeps the reference signature, argument
meaning and ``ValueError`` preconditions (triton_packed_kv_attention.py:284-314)
and runs one CUDA launch (split-K decode + fused LSE merge) from libkvr.so,
through the C++ operator torch.ops.kvr.decode_attention (libkvr_torch.so).

Differences from the reference, stated where a caller could notice them:
  * bits: {2, 4, 8} are accepted (the reference: {4, 8});
  * geometry the kernel is built for: head_dim in {64, 128}, group_size a
    multiple of 16, at most 8 query heads per KV head, bf16 query and
    residual (other geometries raise ValueError instead of running);
  * ``split_tokens=0`` picks the split count for the GPU (the reference runs a
    single-pass kernel for 0); a positive value is honoured as the split
    size, rounded up to ``block_tokens`` and then to 32 tokens.  Results agree
    with every split choice to fp32 rounding.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Dict, List, Sequence, Tuple

import torch

from . import _lib
from .packed_kv_cache import PackedKVComponent, _bh_stride

SUPPORTED_BITS = {2, 4, 8}
SUPPORTED_HEAD_DIMS = {64, 128}
MAX_GQA = 8


def theoretical_attention_flops(query: torch.Tensor, seq_len: int) -> int:
    """Dot-product + value-accumulation FLOPs of one decode query (:392-395)."""
    batch, query_heads, _, head_dim = query.shape
    return int(4 * batch * query_heads * seq_len * head_dim)


def _validate(query: torch.Tensor, packed_keys: PackedKVComponent, packed_values: PackedKVComponent,
              block_tokens: int) -> None:
    # Reference preconditions, same order and messages (:293-314).
    if not query.is_cuda:
        raise ValueError("Packed attention requires a CUDA query tensor.")
    if query.ndim != 4 or query.shape[-2] != 1:
        raise ValueError("query must have shape [batch, query_heads, 1, head_dim].")
    if packed_keys.layout != "per_channel_grouped_affine":
        raise ValueError("keys must use the grouped per-channel affine layout.")
    if packed_values.layout != "per_token_affine":
        raise ValueError("values must use the per-token affine layout.")
    if packed_keys.bits not in SUPPORTED_BITS or packed_values.bits not in SUPPORTED_BITS:
        raise ValueError("The fused kernel supports only 2-, 4- and 8-bit K/V payloads.")
    if tuple(packed_keys.shape) != tuple(packed_values.shape):
        raise ValueError("Packed key and value shapes must match.")
    if tuple(query.shape[:1]) != tuple(packed_keys.shape[:1]):
        raise ValueError("Query and cache batch dimensions must match.")
    if query.shape[-1] != packed_keys.shape[-1]:
        raise ValueError("Query and cache head dimensions must match.")
    if query.shape[1] % packed_keys.shape[1] != 0:
        raise ValueError("Query heads must be divisible by KV heads.")
    if packed_keys.prefix_length <= 0:
        raise ValueError("The fused kernel requires a non-empty quantized key prefix.")
    if block_tokens not in {16, 32, 64}:
        raise ValueError("block_tokens must be one of 16, 32, or 64.")
    # Geometry this build's kernel covers.
    if len(packed_keys.shape) != 4:
        raise ValueError("packed K/V must have shape [batch, kv_heads, tokens, head_dim].")
    head_dim = int(packed_keys.shape[-1])
    if head_dim not in SUPPORTED_HEAD_DIMS:
        raise ValueError(f"head_dim must be one of {sorted(SUPPORTED_HEAD_DIMS)}.")
    if head_dim == 64 and packed_values.bits == 2:
        raise ValueError("2-bit values need head_dim 128.")
    if query.shape[1] // packed_keys.shape[1] > MAX_GQA:
        raise ValueError(f"At most {MAX_GQA} query heads per KV head are supported.")
    if packed_keys.group_size % 16 != 0:
        raise ValueError("group_size must be a multiple of 16 for the fused kernel.")
    if query.dtype != torch.bfloat16:
        raise ValueError("query must be bf16.")


@dataclass(frozen=True)
class CacheGeometry:
    batch: int
    q_heads: int
    kv_heads: int
    head_dim: int
    seq_len: int
    prefix_len: int
    group_size: int
    key_bits: int
    value_bits: int
    kp_bh: int
    km_bh: int
    kr_bh: int
    vp_bh: int
    vm_bh: int


def _geometry(query: torch.Tensor, k: PackedKVComponent, v: PackedKVComponent) -> CacheGeometry:
    batch, kv_heads, seq_len, head_dim = (int(s) for s in k.shape)
    P = int(k.prefix_length)
    kb, vb = int(k.bits), int(v.bits)
    for t, what in ((k.scale, "key scale"), (k.offset, "key offset"), (v.scale, "value scale"),
                    (v.offset, "value offset")):
        if t is None or t.dtype != torch.bfloat16:
            raise ValueError(f"{what} must be bf16.")
    kp_bh = _bh_stride(k.payload, P * head_dim * kb // 8, "key payload")
    km_bh = _bh_stride(k.scale, (P // k.group_size) * head_dim, "key scale")
    if _bh_stride(k.offset, (P // k.group_size) * head_dim, "key offset") != km_bh:
        raise ValueError("key scale and offset must share strides.")
    kr_bh = 0
    if seq_len > P:
        if k.residual is None or k.residual.dtype != torch.bfloat16:
            raise ValueError("key residual must be bf16.")
        kr_bh = _bh_stride(k.residual, (seq_len - P) * head_dim, "key residual")
    vp_bh = _bh_stride(v.payload, seq_len * head_dim * vb // 8, "value payload")
    vm_bh = _bh_stride(v.scale, seq_len, "value scale")
    if _bh_stride(v.offset, seq_len, "value offset") != vm_bh:
        raise ValueError("value scale and offset must share strides.")
    return CacheGeometry(batch, int(query.shape[1]), kv_heads, head_dim, seq_len, P, int(k.group_size),
                         kb, vb, kp_bh, km_bh, kr_bh, vp_bh, vm_bh)


def _check_device(dev_index: int, k: PackedKVComponent, v: PackedKVComponent) -> None:
    """Every cache tensor must live on the query's GPU (the kernel reads them
    through device pointers; a host tensor's address would be read as one)."""
    for t in (k.payload, k.scale, k.offset, k.residual, k.scale_pairs, v.payload, v.scale, v.offset):
        if t is not None and (not t.is_cuda or t.get_device() != dev_index):
            raise ValueError("Packed K/V tensors must be on the query's CUDA device.")


def _layer_ptrs(query: torch.Tensor | None, out: torch.Tensor | None, k: PackedKVComponent,
                v: PackedKVComponent) -> _lib.LayerPtrs:
    """Device pointers of one layer; query/out may be filled in later (None)."""
    _check_device(query.get_device() if query is not None else k.payload.get_device(), k, v)
    res = k.residual if (k.residual is not None and k.residual.numel()) else None
    return _lib.LayerPtrs(
        _lib.ptr(k.payload), _lib.ptr(k.scale), _lib.ptr(k.offset), _lib.ptr(res),
        _lib.ptr(v.payload), _lib.ptr(v.scale), _lib.ptr(v.offset),
        query.data_ptr() if query is not None else None, out.data_ptr() if out is not None else None,
        _lib.ptr(scale_pairs_of(k)),
    )


def scale_pairs_of(k: PackedKVComponent) -> torch.Tensor | None:
    """The component's key-scale pair table when it matches its scales'
    shape and strides (the decode indexes both alike), else None."""
    t = k.scale_pairs
    if t is None or k.scale is None or t.shape != k.scale.shape or t.stride() != k.scale.stride():
        return None
    return t


# Split-merge counters: zero on entry, left zero by every completed launch,
# so one array per (device, stream) serves all launches on that stream.  The
# split-partial workspace is scratch that stream-ordered launches can share
# the same way.  A launch object keeps references to the buffers it was
# built with, so growing a cached buffer never frees memory still in use.
_COUNTERS: Dict[Tuple[int, int], torch.Tensor] = {}
_WORKSPACE: Dict[Tuple[int, int], torch.Tensor] = {}
_PLANS: Dict[tuple, Tuple[int, int, int]] = {}
_SMS: Dict[int, int] = {}


def _dev_index(device: torch.device) -> int:
    return device.index if device.index is not None else torch.cuda.current_device()


def _counters(device: torch.device, stream: int, n: int) -> torch.Tensor:
    key = (_dev_index(device), stream)
    buf = _COUNTERS.get(key)
    if buf is None or buf.numel() < n:
        buf = torch.zeros(max(n, 1024), dtype=torch.int32, device=device)
        _COUNTERS[key] = buf
    return buf


def _workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    key = (_dev_index(device), stream)
    buf = _WORKSPACE.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        _WORKSPACE[key] = buf
    return buf


def _num_sms(device: torch.device) -> int:
    idx = _dev_index(device)
    if idx not in _SMS:
        _SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SMS[idx]


class DecodeLaunch:
    """A prepared decode launch over one or more layers of equal geometry.

    Holds the ctypes argument block, the split plan and the workspace, so a
    repeated call (a decode loop, a benchmark, a CUDA-graph capture) costs
    one C call.  Pointers are fixed at construction: the tensors must stay
    alive and in place.
    """

    def __init__(self, geom: CacheGeometry, layers: Sequence[_lib.LayerPtrs], device: torch.device,
                 split_tokens: int = 0, stream: int | None = None,
                 token_begin: int = 0, token_end: int | None = None, out_fp32: bool = False) -> None:
        if not 1 <= len(layers) <= _lib.KVR_MAX_LAYERS:
            raise ValueError(f"1..{_lib.KVR_MAX_LAYERS} layers per launch.")
        self.geom = geom
        self.device = device
        self.stream = _lib.stream_ptr(device) if stream is None else stream
        self._layers = (_lib.LayerPtrs * len(layers))(*layers)
        self.layers = self._layers   # per-layer pointers; PackedDecoder rewrites query/out in place
        a = _lib.DecodeArgs()
        a.layers = ctypes.cast(self._layers, ctypes.POINTER(_lib.LayerPtrs))
        a.n_layers = len(layers)
        a.batch, a.q_heads, a.kv_heads, a.head_dim = geom.batch, geom.q_heads, geom.kv_heads, geom.head_dim
        a.seq_len, a.prefix_len, a.group_size = geom.seq_len, geom.prefix_len, geom.group_size
        a.key_bits, a.value_bits = geom.key_bits, geom.value_bits
        a.key_payload_bh_stride, a.key_meta_bh_stride = geom.kp_bh, geom.km_bh
        a.key_residual_bh_stride, a.value_payload_bh_stride = geom.kr_bh, geom.vp_bh
        a.value_meta_bh_stride = geom.vm_bh
        a.out_dtype = 1 if out_fp32 else 0
        a.split_tokens = int(split_tokens)
        a.num_sms = _num_sms(device)
        key = (geom, len(layers), a.split_tokens, _dev_index(device), int(token_begin),
               geom.seq_len if token_end is None else int(token_end))
        plan = _PLANS.get(key)
        if plan is None:
            ns, wsb, ncnt = ctypes.c_int(0), ctypes.c_size_t(0), ctypes.c_size_t(0)
            _lib.check("kvr_decode_plan", _lib.load().kvr_decode_plan(a, ctypes.byref(ns), ctypes.byref(wsb),
                                                                     ctypes.byref(ncnt)))
            plan = (ns.value, int(wsb.value), int(ncnt.value))
            _PLANS[key] = plan
        self.num_splits, ws_bytes, n_counters = plan
        self.workspace = _workspace(device, self.stream, ws_bytes)
        self.counters = _counters(device, self.stream, n_counters)
        a.workspace, a.workspace_bytes = self.workspace.data_ptr(), self.workspace.numel()
        a.counters = self.counters.data_ptr()
        self.args = a
        self.token_begin = int(token_begin)
        self.token_end = geom.seq_len if token_end is None else int(token_end)

    def __call__(self) -> None:
        _lib.check("kvr_decode_attention", _lib.load().kvr_decode_attention(self.args, self.stream))

    @property
    def cluster(self) -> int:
        """Cluster size of the launch on this device (kvr_decode_cluster):
        1, or the split count when each (layer, b, kv head)'s splits form one
        thread-block cluster."""
        n = ctypes.c_int(1)
        _lib.check("kvr_decode_cluster", _lib.load().kvr_decode_cluster(self.args, ctypes.byref(n)))
        return int(n.value)

    def partial(self, part_ml: torch.Tensor, part_o: torch.Tensor) -> None:
        """Unnormalised (m, l, o) over tokens [token_begin, token_end)."""
        _lib.check("kvr_decode_partial", _lib.load().kvr_decode_partial(
            self.args, self.token_begin, self.token_end, part_ml.data_ptr(), part_o.data_ptr(), self.stream))


class SimtDecodeLaunch(DecodeLaunch):
    """A prepared decode launch on the CUDA-core engine
    (kvr_decode_attention_simt: fp32 FMA instead of tensor cores, same
    packed layout, split-K and LSE merge).  It is the measured alternative
    to the tensor-core kernel, kept as a library entry point so the A/B
    (``bench.py --engine-ab``) runs against a tested implementation."""

    def __init__(self, geom: CacheGeometry, layers: Sequence[_lib.LayerPtrs], device: torch.device,
                 split_tokens: int = 0, stream: int | None = None, out_fp32: bool = False) -> None:
        super().__init__(geom, layers, device, split_tokens=split_tokens, stream=stream, out_fp32=out_fp32)
        n = int(_lib.load().kvr_decode_simt_workspace(self.args))
        if n == 0:
            raise ValueError("this geometry is not supported by the CUDA-core engine")
        self.simt_workspace = torch.empty(n, dtype=torch.uint8, device=device)
        self.args.workspace, self.args.workspace_bytes = self.simt_workspace.data_ptr(), n

    def __call__(self) -> None:
        _lib.check("kvr_decode_attention_simt", _lib.load().kvr_decode_attention_simt(self.args, self.stream))


def _effective_split(split_tokens: int, block_tokens: int) -> int:
    if split_tokens <= 0:
        return 0
    return -(-int(split_tokens) // int(block_tokens)) * int(block_tokens)


def packed_kv_decode_attention(
    query: torch.Tensor,
    packed_keys: PackedKVComponent,
    packed_values: PackedKVComponent,
    *,
    block_tokens: int = 32,
    split_tokens: int = 0,
    out_dtype: torch.dtype | None = None,
) -> torch.Tensor:
    """One-token GQA attention straight from the packed cache.

    Drop-in for triton_packed_kv_attention.packed_kv_decode_attention
    (:284-389): returns a tensor like ``query``.  ``out_dtype=torch.float32``
    (an addition) returns the fp32 result before the cast to the query dtype.
    The checks (the reference's, same order and messages), the stride and
    pointer work and the launch run in C++ (torch.ops.kvr.decode_attention).
    """
    if out_dtype not in (None, query.dtype, torch.float32):
        raise ValueError("out_dtype must be None, the query dtype or torch.float32.")
    k, v = packed_keys, packed_values
    ks, vs = k.shape, v.shape
    if len(ks) != 4 or len(vs) != 4:
        _validate(query, k, v, block_tokens)   # raises the reference's error for this input
    if _decode_op is None:
        _bind_ops()
    layouts = (k.layout == "per_channel_grouped_affine") | ((v.layout == "per_token_affine") << 1)
    return _decode_op(query, k.payload, k.scale, k.offset, k.residual, v.payload, v.scale, v.offset, ks[2],
                      k.bits, v.bits, k.group_size, k.prefix_length, split_tokens, block_tokens,
                      out_dtype == torch.float32, (*ks, *vs), layouts, scale_pairs_of(k))


_decode_op = None


def _bind_ops() -> None:
    global _decode_op
    _lib.load_torch_ops()
    _decode_op = torch.ops.kvr.decode_attention.default


def packed_kv_decode_attention_simt(
    query: torch.Tensor,
    packed_keys: PackedKVComponent,
    packed_values: PackedKVComponent,
    *,
    split_tokens: int = 0,
    out_dtype: torch.dtype | None = None,
) -> torch.Tensor:
    """packed_kv_decode_attention computed by the CUDA-core engine (fp32 FMA).

    Same arguments, preconditions and result (to fp32 rounding) as the
    tensor-core path; geometries the engine does not cover raise ValueError.
    """
    _validate(query, packed_keys, packed_values, 32)
    if out_dtype not in (None, query.dtype, torch.float32):
        raise ValueError("out_dtype must be None, the query dtype or torch.float32.")
    query = query.contiguous()
    geom = _geometry(query, packed_keys, packed_values)
    out_fp32 = out_dtype == torch.float32
    out = torch.empty_like(query, dtype=torch.float32) if out_fp32 else torch.empty_like(query)
    launch = SimtDecodeLaunch(geom, [_layer_ptrs(query, out, packed_keys, packed_values)], query.device,
                              split_tokens=_effective_split(split_tokens, 32), out_fp32=out_fp32)
    launch()
    return out


def packed_kv_decode_attention_layers(
    queries: Sequence[torch.Tensor],
    packed_keys: Sequence[PackedKVComponent],
    packed_values: Sequence[PackedKVComponent],
    *,
    split_tokens: int = 0,
    out: torch.Tensor | None = None,
) -> List[torch.Tensor]:
    """Decode attention for several layers of equal geometry in one launch.

    Each layer is independent (its own query, cache and output); the result
    equals calling packed_kv_decode_attention per layer.  ``out`` (optional,
    [L, *query.shape], the query dtype or fp32) receives all layers' outputs;
    the returned list holds its per-layer views.
    """
    n = len(queries)
    if not (n == len(packed_keys) == len(packed_values)) or not n:
        raise ValueError("queries, packed_keys and packed_values must be non-empty and equally long.")
    q0 = queries[0]
    _validate(q0, packed_keys[0], packed_values[0], 32)
    geom = _geometry(q0, packed_keys[0], packed_values[0])
    if out is None:
        out = torch.empty((n,) + tuple(q0.shape), dtype=q0.dtype, device=q0.device)
    elif (tuple(out.shape) != (n,) + tuple(q0.shape) or out.dtype not in (q0.dtype, torch.float32)
          or out.device != q0.device or not out.is_contiguous()):
        raise ValueError("out must be a contiguous [layers, *query.shape] tensor of the query dtype or fp32.")
    outs = list(out.unbind(0))
    ptrs = []
    for i, (q, k, v) in enumerate(zip(queries, packed_keys, packed_values)):
        if i:
            _validate(q, k, v, 32)
            if _geometry(q, k, v) != geom:
                raise ValueError("All layers of one launch must share geometry and strides.")
        ptrs.append(_layer_ptrs(q.contiguous(), outs[i], k, v))
    for start in range(0, n, _lib.KVR_MAX_LAYERS):
        DecodeLaunch(geom, ptrs[start:start + _lib.KVR_MAX_LAYERS], q0.device, split_tokens=split_tokens,
                     out_fp32=out.dtype == torch.float32)()
    return outs


class PackedDecoder:
    """Plan once, run every decode step: attention for all layers of a cache.

    Construction validates every layer (the same preconditions and messages
    as packed_kv_decode_attention), resolves the cache pointers and the split
    plan, and builds the launch argument blocks.  A call then takes the
    step's stacked queries [L, B, HQ, 1, D] (bf16) and writes all layers'
    outputs with one library call per 32 layers; the cache pointers are
    not re-derived, so the per-step host cost does not grow with the number
    of layers.  The cache tensors must stay alive and in place (a streaming
    cache that appends or reallocates needs a new decoder).  Launches go to
    the CUDA stream current at the first call.
    """

    def __init__(self, packed_keys: Sequence[PackedKVComponent], packed_values: Sequence[PackedKVComponent],
                 *, q_heads: int, split_tokens: int = 0, out_dtype: torch.dtype = torch.bfloat16) -> None:
        n = len(packed_keys)
        if n == 0 or n != len(packed_values):
            raise ValueError("packed_keys and packed_values must be non-empty and equally long.")
        if out_dtype not in (torch.bfloat16, torch.float32):
            raise ValueError("out_dtype must be torch.bfloat16 or torch.float32.")
        k0 = packed_keys[0]
        if k0.payload is None or not k0.payload.is_cuda:
            raise ValueError("Packed attention requires CUDA cache tensors.")
        device = k0.payload.device
        batch, _, _, head_dim = (int(x) for x in k0.shape)
        # a query of the step's shape: the reference's checks take one
        probe = torch.empty(batch, int(q_heads), 1, head_dim, dtype=torch.bfloat16, device=device)
        geom, layers = None, []
        dev_index = probe.get_device()
        for k, v in zip(packed_keys, packed_values):
            _validate(probe, k, v, 32)
            _check_device(dev_index, k, v)
            g = _geometry(probe, k, v)
            if geom is None:
                geom = g
            elif g != geom:
                raise ValueError("All layers must share geometry and strides.")
            layers.append(_layer_ptrs(None, None, k, v))
        self.geom, self.device, self.n_layers = geom, device, n
        self.q_shape = (n,) + tuple(probe.shape)
        self.out_dtype = out_dtype
        self.split_tokens = int(split_tokens)
        self._keep = (list(packed_keys), list(packed_values))
        self._layers = layers
        self._launches: List[DecodeLaunch] = []   # built at the first call, with real query/out pointers
        self._q_step = head_dim * int(q_heads) * batch * 2
        self._o_step = head_dim * int(q_heads) * batch * (4 if out_dtype == torch.float32 else 2)
        self._bases = (0, 0)
        self._host = None   # host_step's recorded graph and buffers

    @property
    def num_splits(self) -> int:
        if not self._launches:
            raise RuntimeError("the split plan is made at the first call")
        return self._launches[0].num_splits

    def _build(self, qb: int, ob: int) -> None:
        for i, layer in enumerate(self._layers):
            layer.query = qb + i * self._q_step
            layer.out = ob + i * self._o_step
        self._launches = [DecodeLaunch(self.geom, self._layers[s:s + _lib.KVR_MAX_LAYERS], self.device,
                                       split_tokens=self.split_tokens, out_fp32=self.out_dtype == torch.float32)
                          for s in range(0, self.n_layers, _lib.KVR_MAX_LAYERS)]

    def __call__(self, queries: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if (tuple(queries.shape) != self.q_shape or queries.dtype != torch.bfloat16 or queries.device != self.device
                or not queries.is_contiguous()):
            raise ValueError(f"queries must be a contiguous bf16 tensor of shape {self.q_shape} on {self.device}.")
        if out is None:
            out = torch.empty(self.q_shape, dtype=self.out_dtype, device=self.device)
        elif (tuple(out.shape) != self.q_shape or out.dtype != self.out_dtype or out.device != self.device
              or not out.is_contiguous()):
            raise ValueError(f"out must be a contiguous {self.out_dtype} tensor of shape {self.q_shape}.")
        bases = (queries.data_ptr(), out.data_ptr())
        if not self._launches:
            self._build(*bases)
            self._bases = bases
        elif bases != self._bases:
            qb, ob = bases
            for li, launch in enumerate(self._launches):
                for j in range(launch.args.n_layers):
                    layer = li * _lib.KVR_MAX_LAYERS + j
                    launch.layers[j].query = qb + layer * self._q_step
                    launch.layers[j].out = ob + layer * self._o_step
            self._bases = bases
        for launch in self._launches:
            launch()
        return out

    def host_step(self, queries: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """One decode step from and to host memory.

        For loops whose queries are produced on the host and whose outputs
        are read there (a CPU-side draft controller, a caller that keeps no
        device buffers of its own).  ``queries`` and ``out`` are pinned host
        tensors of the step's shape ([L, B, HQ, 1, D]; bf16 and the decoder's
        output dtype).  When the GPU addresses ``out`` directly (pinned memory
        under unified addressing, kvr_host_mapped) the decode's final merge
        writes the outputs straight into it, otherwise a copy brings them
        back.  Mapped queries are read in place when every launch runs in
        thread-block clusters (kvr_decode_cluster): one CTA per (layer, b, kv
        head) reads them across PCIe and shares them with the other splits
        over distributed shared memory (query_host_mapped); otherwise the
        step copies them in (one copy).  (Every split reading its own query
        across PCIe measured slower than the copy, and so did a copy kernel
        reading them ahead of the decode.)  The first call with a
        pair of buffers runs the step eagerly and records it as a CUDA graph
        on a private stream; every call replays that graph and waits for it.
        Returns ``out`` holding this step's outputs.  The host buffers must
        stay alive and in place; passing another pair records a new graph.
        """
        hs = self._host
        if (hs is not None and hs["q"] is queries and hs["o"] is out and queries.data_ptr() == hs["qp"]
                and out.data_ptr() == hs["op"] and queries.shape == hs["shape"] and out.shape == hs["shape"]
                and queries.dtype == torch.bfloat16 and out.dtype == self.out_dtype):
            hs["graph"].replay()
            torch.cuda.current_stream(self.device).synchronize()
            return out
        if (tuple(queries.shape) != self.q_shape or queries.dtype != torch.bfloat16 or queries.is_cuda
                or not queries.is_pinned() or not queries.is_contiguous()):
            raise ValueError(f"queries must be a contiguous pinned host bf16 tensor of shape {self.q_shape}.")
        if (tuple(out.shape) != self.q_shape or out.dtype != self.out_dtype or out.is_cuda
                or not out.is_pinned() or not out.is_contiguous()):
            raise ValueError(f"out must be a contiguous pinned host {self.out_dtype} tensor of shape {self.q_shape}.")
        self._host = None
        zero_copy = _lib.host_mapped(out.data_ptr())   # outputs written in place
        o_buf = out if zero_copy else torch.empty(self.q_shape, dtype=self.out_dtype, device=self.device)
        stream = torch.cuda.Stream(self.device)

        def make_launches(q_base: int) -> List[DecodeLaunch]:
            layers = []
            for i, layer in enumerate(self._layers):
                copy = _lib.LayerPtrs.from_buffer_copy(layer)
                copy.query = q_base + i * self._q_step
                copy.out = o_buf.data_ptr() + i * self._o_step
                layers.append(copy)
            return [DecodeLaunch(self.geom, layers[s:s + _lib.KVR_MAX_LAYERS], self.device,
                                 split_tokens=self.split_tokens, stream=stream.cuda_stream,
                                 out_fp32=self.out_dtype == torch.float32)
                    for s in range(0, self.n_layers, _lib.KVR_MAX_LAYERS)]

        # mapped queries read in place when every launch runs in clusters
        # (one read per (layer, b, kv head), shared over distributed shared
        # memory); otherwise one H2D copy into a device buffer per step
        q_buf = None
        launches = []
        if _lib.host_mapped(queries.data_ptr()):
            launches = make_launches(queries.data_ptr())
            for launch in launches:
                launch.args.query_host_mapped = 1
            if not all(launch.cluster > 1 for launch in launches):
                launches = []
        if not launches:
            q_buf = torch.empty(self.q_shape, dtype=torch.bfloat16, device=self.device)
            launches = make_launches(q_buf.data_ptr())

        def step():
            if q_buf is not None:
                q_buf.copy_(queries, non_blocking=True)
            for launch in launches:
                launch()
            if not zero_copy:
                out.copy_(o_buf, non_blocking=True)

        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            step()
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        self._host = {"q": queries, "o": out, "qp": queries.data_ptr(), "op": out.data_ptr(),
                      "shape": queries.shape, "graph": graph, "buffers": (q_buf, o_buf),
                      "launches": launches, "stream": stream, "zero_copy": zero_copy,
                      "queries_in_place": q_buf is None}
        return out


def check_finite_outputs(device: torch.device | int | None = None, *, clear: bool = True) -> None:
    """Raise FloatingPointError if a decode on ``device`` has written a
    non-finite output since the last check (kvr_decode_nonfinite;
    synchronises the device).

    The reference computes attention in fp32; this kernel feeds the tensor
    cores fp16 operands.  It scales large queries by an exact power of two
    (|q| < 64), but a key scale, a scaled query times a key scale, or a
    value scale at or above 65504 does not fit, and such a decode writes
    inf/NaN.  Caches whose key or value ranges reach about 1e6 (4-bit codes)
    are outside the kernel's range: call this after their decodes.
    """
    if device is not None:
        with torch.cuda.device(device):
            _check_finite(clear)
    else:
        _check_finite(clear)


def _check_finite(clear: bool) -> None:
    flag = ctypes.c_int(0)
    _lib.call("kvr_decode_nonfinite", ctypes.byref(flag), 1 if clear else 0)
    if flag.value:
        raise FloatingPointError("a packed-KV decode wrote non-finite outputs: a key scale, query x key scale "
                                 "or value scale exceeded the fp16 range of the kernel's tensor-core operands")


def lse_merge(part_ml: torch.Tensor, part_o: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Merge per-shard partials: part_ml [n_parts, rows, 2] (m in log2 units, l),
    part_o [n_parts, rows, D] -> bf16 [rows, D]."""
    if part_ml.dim() != 3 or part_ml.shape[-1] != 2 or part_o.dim() != 3:
        raise ValueError("part_ml must be [n_parts, rows, 2] and part_o [n_parts, rows, D].")
    n_parts, rows, head_dim = (int(s) for s in part_o.shape)
    if tuple(part_ml.shape[:2]) != (n_parts, rows):
        raise ValueError("part_ml and part_o disagree on [n_parts, rows].")
    dev = _lib.require_cuda(part_ml, part_o)
    part_ml = part_ml.float().contiguous()
    part_o = part_o.float().contiguous()
    if out is None:
        out = torch.empty(rows, head_dim, dtype=torch.bfloat16, device=dev)
    _lib.call("kvr_lse_merge", part_ml.data_ptr(), part_o.data_ptr(), n_parts, rows, head_dim, out.data_ptr(),
              _lib.stream_ptr(dev))
    return out
