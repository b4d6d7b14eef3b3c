"""Streaming packed draft-KV cache with in-place append / commit / crop.

The reference keeps the draft cache in ``PackedLayer``
(kv_reduce/experiments/packed_review.py:17-63) and grows every tensor with
``torch.cat`` on each token, an O(S) copy per token and layer.  Here each
layer owns preallocated capacity buffers:

    key payload   uint8 [B, H, capP, D*kb/8]     key scale/offset bf16 [B, H, capP/G, 1, D]
    key residual  bf16  2 x [B, H, capR, D]      (double buffer, swapped on commit)
    value payload uint8 [B, H, cap, D*vb/8]      value scale/offset bf16 [B, H, cap, 1]

and the packed components handed to attention are strided views of them,
so append writes one token row, commit quantizes whole groups in place, and
crop only moves the length.  Semantics follow packed_review.py:
  * append (:23-31): keys join the BF16 residual window; values are
    quantized per token at once;
  * commit (:32-41): floor((res - R)/G) full groups of the residual are
    quantized and promoted to the packed prefix;
  * crop (:42-49): roll back inside the uncommitted tail (P <= length <= S).
Capacity grows by reallocation when exceeded.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch

from . import _lib
from .packed_kv_attention import packed_kv_decode_attention
from .packed_kv_cache import PackedKVComponent, _quantized_prefix_length, key_scale_pairs, tensor_bytes


def _round_up(x: int, m: int) -> int:
    return -(-x // m) * m


_step_op = None
_step_out_op = None


def _bind_ops() -> None:
    global _step_op, _step_out_op
    _lib.load_torch_ops()
    _step_op = torch.ops.kvr.decode_step.default
    _step_out_op = torch.ops.kvr.decode_step.out


class PackedKVCacheLayer:
    """One layer of the preallocated packed cache."""

    def __init__(self, batch: int, kv_heads: int, head_dim: int, *, k_bits: int = 4, v_bits: int = 4,
                 group_size: int = 32, residual_length: int = 128, capacity: int = 4096,
                 spec_capacity: int = 64, device: torch.device | str = "cuda") -> None:
        for b in (k_bits, v_bits):
            if b < 2 or b > 8 or (head_dim * b) % 8:
                raise ValueError("streaming cache needs 2..8-bit codes with byte-aligned rows (D*bits % 8 == 0).")
        if group_size <= 0 or residual_length < 0:
            raise ValueError("group_size must be positive and residual_length non-negative.")
        self.batch, self.kv_heads, self.head_dim = int(batch), int(kv_heads), int(head_dim)
        self.k_bits, self.v_bits = int(k_bits), int(v_bits)
        self.group_size, self.residual_length = int(group_size), int(residual_length)
        self.spec_capacity = int(spec_capacity)
        self.device = torch.device(device)
        self.seq_len = 0
        self.prefix_len = 0
        self._cur = 0
        # True: commit keeps the live residual in the same buffer (a captured
        # CUDA graph holds its address); lengths mirrored on the device
        self.pin_residual = False
        self._dev_len: Optional[torch.Tensor] = None
        self._alloc(_round_up(max(int(capacity), 64), 64))

    # ------------------------------------------------------------ storage
    def _alloc(self, capacity: int) -> None:
        B, H, D, G = self.batch, self.kv_heads, self.head_dim, self.group_size
        dev = self.device
        cap_p = (capacity // G) * G
        cap_r = _round_up(self.residual_length + G + self.spec_capacity, 8)
        self.capacity, self.cap_prefix, self.cap_residual = capacity, cap_p, cap_r
        self.key_payload = torch.zeros(B, H, cap_p, D * self.k_bits // 8, dtype=torch.uint8, device=dev)
        self.key_scale = torch.zeros(B, H, max(cap_p // G, 1), 1, D, dtype=torch.bfloat16, device=dev)
        self.key_offset = torch.zeros_like(self.key_scale)
        # the decode's fp16 scale pairs (key_scale_pairs), kept in step with key_scale
        self.key_scale_pairs = (torch.zeros(self.key_scale.shape, dtype=torch.int16, device=dev)
                                if D in (64, 128) and self.k_bits in (2, 4, 8) else None)
        self.key_residual = [torch.zeros(B, H, cap_r, D, dtype=torch.bfloat16, device=dev) for _ in range(2)]
        self.value_payload = torch.zeros(B, H, capacity, D * self.v_bits // 8, dtype=torch.uint8, device=dev)
        self.value_scale = torch.zeros(B, H, capacity, 1, dtype=torch.bfloat16, device=dev)
        self.value_offset = torch.zeros_like(self.value_scale)

    def _grow(self, need_seq: int, need_res: int) -> None:
        old = (self.key_payload, self.key_scale, self.key_offset, self.key_residual[self._cur],
               self.value_payload, self.value_scale, self.value_offset, self.key_scale_pairs)
        S, P, R = self.seq_len, self.prefix_len, self.seq_len - self.prefix_len
        cap = self.capacity
        while cap < need_seq:
            cap *= 2
        spec = self.spec_capacity
        while self.residual_length + self.group_size + spec < need_res:
            spec *= 2
        self.spec_capacity = spec
        self._alloc(_round_up(cap, 64))
        self._cur = 0
        G = self.group_size
        self.key_payload[:, :, :P].copy_(old[0][:, :, :P])
        self.key_scale[:, :, :P // G].copy_(old[1][:, :, :P // G])
        self.key_offset[:, :, :P // G].copy_(old[2][:, :, :P // G])
        if self.key_scale_pairs is not None:
            self.key_scale_pairs[:, :, :P // G].copy_(old[7][:, :, :P // G])
        self.key_residual[0][:, :, :R].copy_(old[3][:, :, :R])
        self.value_payload[:, :, :S].copy_(old[4][:, :, :S])
        self.value_scale[:, :, :S].copy_(old[5][:, :, :S])
        self.value_offset[:, :, :S].copy_(old[6][:, :, :S])

    @property
    def residual_len(self) -> int:
        return self.seq_len - self.prefix_len

    def _stream(self) -> int:
        return _lib.stream_ptr(self.device)

    def _check_kv(self, k: torch.Tensor, v: torch.Tensor) -> None:
        want = (self.batch, self.kv_heads)
        if k.shape != v.shape or k.dim() != 4 or tuple(k.shape[:2]) != want or k.shape[-1] != self.head_dim:
            raise ValueError(f"k/v must be [{self.batch}, {self.kv_heads}, n, {self.head_dim}].")
        if k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
            raise ValueError("k/v must be bf16.")
        _lib.require_cuda(k, v)

    # ------------------------------------------------------------ operations
    def prefill(self, keys: torch.Tensor, values: torch.Tensor) -> None:
        """Pack a prefilled [B, H, S, D] cache (pack_kivi_kv semantics)."""
        self._check_kv(keys, values)
        S = int(keys.shape[2])
        P = _quantized_prefix_length(S, self.group_size, self.residual_length)
        if S > self.capacity or S - P > self.cap_residual:
            self._grow(S, S - P)
        D, G = self.head_dim, self.group_size
        keys, values = keys.contiguous(), values.contiguous()
        bh = self.batch * self.kv_heads
        if P > 0:
            a = _lib.GroupQuantArgs()
            a.x, a.x_bh_stride, a.x_row_stride = keys.data_ptr(), S * D, D
            a.payload, a.payload_bh_stride = self.key_payload.data_ptr(), self.key_payload.stride(1)
            a.scale, a.offset = self.key_scale.data_ptr(), self.key_offset.data_ptr()
            a.meta_bh_stride = self.key_scale.stride(1)
            a.bh, a.groups, a.group0, a.group_size, a.head_dim, a.bits = bh, P // G, 0, G, D, self.k_bits
            _lib.call("kvr_quantize_grouped", a, self._stream())
            self._pairs(0, P // G)
        self._cur = 0
        self.key_residual[0][:, :, :S - P].copy_(keys[:, :, P:])
        if S > 0:
            a = _lib.TokenQuantArgs()
            a.x, a.x_bh_stride, a.x_row_stride = values.data_ptr(), S * D, D
            a.payload, a.payload_bh_stride = self.value_payload.data_ptr(), self.value_payload.stride(1)
            a.scale, a.offset = self.value_scale.data_ptr(), self.value_offset.data_ptr()
            a.meta_bh_stride = self.value_scale.stride(1)
            a.bh, a.rows, a.row0, a.head_dim, a.bits = bh, S, 0, D, self.v_bits
            _lib.call("kvr_quantize_per_token", a, self._stream())
        self.seq_len, self.prefix_len = S, P
        self._sync_lengths()

    def append(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """Append n tokens: keys to the BF16 window, values quantized now."""
        self._check_kv(k, v)
        n = int(k.shape[2])
        if n == 0:
            return
        if self.seq_len + n > self.capacity or self.residual_len + n > self.cap_residual:
            self._grow(self.seq_len + n, self.residual_len + n)
        k, v = k.contiguous(), v.contiguous()
        res = self.key_residual[self._cur]
        a = _lib.AppendArgs()
        a.k, a.v = k.data_ptr(), v.data_ptr()
        a.key_residual, a.key_residual_bh_stride = res.data_ptr(), res.stride(1)
        a.value_payload, a.value_payload_bh_stride = self.value_payload.data_ptr(), self.value_payload.stride(1)
        a.value_scale, a.value_offset = self.value_scale.data_ptr(), self.value_offset.data_ptr()
        a.value_meta_bh_stride = self.value_scale.stride(1)
        a.bh, a.n, a.seq_len, a.res_len = self.batch * self.kv_heads, n, self.seq_len, self.residual_len
        a.res_capacity, a.seq_capacity = self.cap_residual, self.capacity
        a.head_dim, a.value_bits = self.head_dim, self.v_bits
        _lib.call("kvr_append", a, self._stream())
        self.seq_len += n
        self._sync_lengths()

    def commit(self) -> int:
        """Promote full key groups out of the residual window; returns tokens promoted."""
        res_len = self.residual_len
        promoted = _quantized_prefix_length(res_len, self.group_size, self.residual_length)
        if promoted == 0:
            return 0
        if self.prefix_len + promoted > self.cap_prefix:
            self._grow(self.prefix_len + promoted + self.group_size, res_len)
        src, dst = self.key_residual[self._cur], self.key_residual[1 - self._cur]
        a = _lib.FlushArgs()
        a.residual_in, a.residual_out, a.residual_bh_stride = src.data_ptr(), dst.data_ptr(), src.stride(1)
        a.key_payload, a.key_payload_bh_stride = self.key_payload.data_ptr(), self.key_payload.stride(1)
        a.key_scale, a.key_offset = self.key_scale.data_ptr(), self.key_offset.data_ptr()
        a.key_meta_bh_stride = self.key_scale.stride(1)
        a.bh, a.res_len, a.groups = self.batch * self.kv_heads, res_len, promoted // self.group_size
        a.prefix_len, a.prefix_capacity = self.prefix_len, self.cap_prefix
        a.group_size, a.head_dim, a.key_bits = self.group_size, self.head_dim, self.k_bits
        _lib.call("kvr_flush_groups", a, self._stream())
        self._pairs(self.prefix_len // self.group_size, promoted // self.group_size)
        self.prefix_len += promoted
        if self.pin_residual:
            rest = res_len - promoted
            src[:, :, :rest].copy_(dst[:, :, :rest])
        else:
            self._cur = 1 - self._cur
        self._sync_lengths()
        return promoted

    def _pairs(self, group0: int, groups: int) -> None:
        """Refresh the scale pair table for key groups [group0, group0 + groups)."""
        if self.key_scale_pairs is not None and groups > 0:
            key_scale_pairs(self.key_scale, self.k_bits, out=self.key_scale_pairs, group0=group0, groups=groups)

    def crop(self, length: int) -> None:
        """Roll back to `length` tokens inside the uncommitted tail."""
        if not (self.prefix_len <= length <= self.seq_len):
            raise ValueError(f"crop({length}) outside [{self.prefix_len}, {self.seq_len}].")
        self.seq_len = int(length)
        self._sync_lengths()

    # ------------------------------------------------- device-side lengths
    def device_lengths(self) -> torch.Tensor:
        """int32[4] on the device: (sequence length, prefix length, error
        flag, scratch), kept equal to the host lengths by every host-side operation;
        the graph-replayable append / advance / decode read and move it."""
        if self._dev_len is None:
            self._dev_len = torch.zeros(4, dtype=torch.int32, device=self.device)
            self._sync_lengths()
        return self._dev_len

    def _sync_lengths(self) -> None:
        if self._dev_len is not None:
            _lib.call("kvr_set_lengths", self._dev_len.data_ptr(), self.seq_len, self.prefix_len, self._stream())

    def get_seq_length(self) -> int:
        return self.seq_len

    # --------------------------------------------------------------- views
    @property
    def k(self) -> PackedKVComponent:
        B, H, D = self.batch, self.kv_heads, self.head_dim
        P, S, G = self.prefix_len, self.seq_len, self.group_size
        return PackedKVComponent(
            payload=self.key_payload[:, :, :P], scale=self.key_scale[:, :, :P // G],
            offset=self.key_offset[:, :, :P // G], residual=self.key_residual[self._cur][:, :, :S - P],
            shape=(B, H, S, D), bits=self.k_bits, layout="per_channel_grouped_affine",
            output_dtype=torch.bfloat16, group_size=G, prefix_length=P,
            scale_pairs=None if self.key_scale_pairs is None else self.key_scale_pairs[:, :, :P // G],
        )

    @property
    def v(self) -> PackedKVComponent:
        B, H, D, S = self.batch, self.kv_heads, self.head_dim, self.seq_len
        return PackedKVComponent(
            payload=self.value_payload[:, :, :S], scale=self.value_scale[:, :, :S],
            offset=self.value_offset[:, :, :S], residual=None, shape=(B, H, S, D), bits=self.v_bits,
            layout="per_token_affine", output_dtype=torch.bfloat16,
        )

    def attention(self, query: torch.Tensor, *, split_tokens: int = 0,
                  out_dtype: torch.dtype | None = None) -> torch.Tensor:
        return packed_kv_decode_attention(query, self.k, self.v, split_tokens=split_tokens, out_dtype=out_dtype)

    def decode_step(self, query: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, split_tokens: int = 0,
                    out: torch.Tensor | None = None) -> torch.Tensor:
        """append(k, v) then attention(query): for one new token a single
        decode launch that stores the token before attending
        (kvr_decode_step, through the C++ operator torch.ops.kvr.decode_step),
        else an append and a decode call.

        Both forms read the lengths from the layer's device-side copy and
        move it on themselves, so the host only rewrites the query,
        new-token and output pointers of argument blocks prepared once per
        buffer layout (and the calls can be captured in a CUDA graph).  The
        decode is planned for the buffers' capacity.  The residual buffer is
        pinned (commit copies the live rows back) so the prepared addresses
        hold across commits.
        """
        n = int(k.shape[2]) if k.dim() == 4 else -1
        if (n == 1 and self.seq_len > 0 and self.seq_len < self.capacity
                and self.seq_len - self.prefix_len < self.cap_residual):
            # one token, room in the buffers: the C++ operator checks the
            # tensors and launches the fused append + decode
            self.pin_residual = True
            geom = (self.capacity, self.cap_prefix, self.cap_residual, self.k_bits, self.v_bits, self.group_size,
                    int(split_tokens))
            bufs = (self.key_payload, self.key_scale, self.key_offset, self.key_residual[self._cur],
                    self.value_payload, self.value_scale, self.value_offset, self.device_lengths())
            if _step_op is None:
                _bind_ops()
            if out is None:
                out = _step_op(query, k, v, *bufs, geom, self.key_scale_pairs)
            else:
                _step_out_op(query, k, v, *bufs, geom, self.key_scale_pairs, out=out)
            self.seq_len += 1
            return out
        if (k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16 or k.shape != v.shape or n < 1
                or tuple(k.shape[:2]) != (self.batch, self.kv_heads) or k.shape[3] != self.head_dim):
            raise ValueError(f"k/v must be bf16 [{self.batch}, {self.kv_heads}, n, {self.head_dim}].")
        if (query.dim() != 4 or query.dtype != torch.bfloat16 or query.shape[0] != self.batch
                or query.shape[2] != 1 or query.shape[3] != self.head_dim or query.shape[1] % self.kv_heads):
            raise ValueError(f"query must be bf16 [{self.batch}, q_heads, 1, {self.head_dim}].")
        _lib.require_cuda(query, k, v)
        if self.seq_len + n > self.capacity or self.residual_len + n > self.cap_residual:
            self._grow(self.seq_len + n, self.residual_len + n)
        if self.seq_len == 0:
            raise ValueError("decode_step needs a prefilled layer.")
        self.pin_residual = True
        k, v, query = k.contiguous(), v.contiguous(), query.contiguous()
        if out is None:
            out = torch.empty_like(query)
        stream = self._stream()
        key = (int(query.shape[1]), int(split_tokens), stream, self.key_payload.data_ptr(),
               self.key_residual[self._cur].data_ptr(), self.capacity)
        prep = getattr(self, "_step_prep", None)
        if prep is None or prep[0] != key:
            prep = (key,) + self._prepare_step(int(query.shape[1]), int(split_tokens), stream, query, out)
            self._step_prep = prep
        _, app, launch = prep
        app.k, app.v, app.n = k.data_ptr(), v.data_ptr(), n
        launch.layers[0].query, launch.layers[0].out = query.data_ptr(), out.data_ptr()
        dl = self.device_lengths().data_ptr()
        lib = _lib.load()
        if n == 1:   # the decode launch appends the token itself
            _lib.check("kvr_decode_step", lib.kvr_decode_step(launch.args, k.data_ptr(), v.data_ptr(), dl,
                                                              self.cap_residual, stream))
        else:
            _lib.check("kvr_append_lengths", lib.kvr_append_lengths(app, dl, 1, stream))
            _lib.check("kvr_decode_attention_lengths",
                       lib.kvr_decode_attention_lengths(launch.args, dl, self.cap_residual, stream))
        self.seq_len += n
        return out

    def _prepare_step(self, q_heads: int, split_tokens: int, stream: int, query: torch.Tensor,
                      out: torch.Tensor):
        from .packed_kv_attention import CacheGeometry, DecodeLaunch

        res = self.key_residual[self._cur]
        a = _lib.AppendArgs()
        a.key_residual, a.key_residual_bh_stride = res.data_ptr(), res.stride(1)
        a.value_payload, a.value_payload_bh_stride = self.value_payload.data_ptr(), self.value_payload.stride(1)
        a.value_scale, a.value_offset = self.value_scale.data_ptr(), self.value_offset.data_ptr()
        a.value_meta_bh_stride = self.value_scale.stride(1)
        a.bh, a.seq_len, a.res_len = self.batch * self.kv_heads, 0, 0
        a.res_capacity, a.seq_capacity = self.cap_residual, self.capacity
        a.head_dim, a.value_bits = self.head_dim, self.v_bits
        geom = CacheGeometry(self.batch, q_heads, self.kv_heads, self.head_dim, self.capacity, self.cap_prefix,
                             self.group_size, self.k_bits, self.v_bits, self.key_payload.stride(1),
                             self.key_scale.stride(1), res.stride(1), self.value_payload.stride(1),
                             self.value_scale.stride(1))
        ptrs = _lib.LayerPtrs(self.key_payload.data_ptr(), self.key_scale.data_ptr(), self.key_offset.data_ptr(),
                              res.data_ptr(), self.value_payload.data_ptr(), self.value_scale.data_ptr(),
                              self.value_offset.data_ptr(), query.data_ptr(), out.data_ptr(),
                              _lib.ptr(self.key_scale_pairs))
        return a, DecodeLaunch(geom, [ptrs], self.device, split_tokens=split_tokens, stream=stream)

    def breakdown(self) -> Dict[str, int]:
        """Byte accounting with the keys of packed_review.py:50-54."""
        k, v = self.k, self.v
        return {"k_payload": tensor_bytes(k.payload), "v_payload": tensor_bytes(v.payload),
                "k_scales": tensor_bytes(k.scale), "v_scales": tensor_bytes(v.scale),
                "k_offsets": tensor_bytes(k.offset), "v_offsets": tensor_bytes(v.offset),
                "key_residual": tensor_bytes(k.residual)}


class PackedKVCache:
    """All layers of a draft model's packed cache (batch-uniform lengths)."""

    def __init__(self, num_layers: int, batch: int, kv_heads: int, head_dim: int, **kw) -> None:
        self.layers: List[PackedKVCacheLayer] = [
            PackedKVCacheLayer(batch, kv_heads, head_dim, **kw) for _ in range(num_layers)]

    def commit(self) -> None:
        for layer in self.layers:
            layer.commit()

    def crop(self, length: int) -> None:
        for layer in self.layers:
            layer.crop(length)

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self.layers[layer_idx].get_seq_length()

    def breakdown(self) -> Dict[str, int]:
        parts = [layer.breakdown() for layer in self.layers]
        return {key: sum(p[key] for p in parts) for key in parts[0]}


class PackedLayer(PackedKVCacheLayer):
    """Shim with the constructor of packed_review.PackedLayer (:17-22):
    K4V4, group 32, from a prefilled [B, H, S, D] cache."""

    def __init__(self, k: torch.Tensor, v: torch.Tensor, residual: int, *, k_bits: int = 4, v_bits: int = 4,
                 group_size: int = 32, capacity: Optional[int] = None) -> None:
        B, H, S, D = (int(s) for s in k.shape)
        super().__init__(B, H, D, k_bits=k_bits, v_bits=v_bits, group_size=group_size,
                         residual_length=residual, capacity=capacity or S + 2048, device=k.device)
        self.prefill(k, v)


class PackedCache(PackedKVCache):
    """Shim of packed_review.PackedCache (:56-63) over (k, v) pairs per layer."""

    def __init__(self, cache, residual: int, **kw) -> None:
        self.layers = [PackedLayer(k, v, residual, **kw) for k, v in cache]
