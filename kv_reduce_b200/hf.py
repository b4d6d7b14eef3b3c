"""Draft-model integration with transformers: a packed Cache and the
attention hook.

Mirrors kv_reduce/experiments/packed_review.py:17-80:

* ``PackedDraftCache`` plays the role of the reference's ``PackedCache``
  (a ``DynamicCache`` whose layers hold the packed K/V; :56-63), built from a
  prefilled cache, with ``commit()`` (promote full key groups out of the
  BF16 residual window, :32-41, :61-62) and ``breakdown()`` (:50-54, :63).
  Its layers are the preallocated streaming layers of
  ``kv_reduce_b200.streaming``, so a decode step appends one token in place
  instead of the reference's ``torch.cat`` of the whole payload.
* ``PackedDraftCache.empty(num_layers, residual)`` packs each layer during
  the prompt forward itself (streaming prefill): the full BF16 cache the
  reference builds first and packs afterwards never exists.
* ``install(model)`` patches every decoder layer's attention (:65-80): with
  a ``PackedDraftCache`` and a one-token step, it projects q/k/v, applies the
  rotary embedding and runs ``decode_step`` on the packed layer (append
  in place + fused decode, two library calls from device-side lengths); any
  other call goes to the original forward.

Written against the Qwen2 attention module of transformers 5.x (q/k/v/o
projections, ``head_dim``, ``layer_idx``, rotary ``position_embeddings``).
"""
from __future__ import annotations

import types
from typing import Dict, Iterable, Tuple

import torch
from transformers.cache_utils import DynamicCache, DynamicLayer
from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

from .streaming import PackedKVCacheLayer, PackedLayer


class PackedDraftLayer(DynamicLayer):
    """A transformers cache layer over one streaming packed layer.

    Built over an already packed layer, or empty: then the prompt forward's
    ``update`` packs the layer's K/V as soon as they are produced (streaming
    prefill) and passes the BF16 tensors on to that layer's attention only,
    so the model never holds a BF16 copy of more than one layer's cache.
    """

    def __init__(self, packed: PackedKVCacheLayer | None = None, *, residual: int = 128,
                 spare_capacity: int = 2048, **kw) -> None:
        super().__init__()
        self.packed = packed
        self._residual, self._spare, self._kw = int(residual), int(spare_capacity), kw
        self.is_initialized = True

    def get_seq_length(self) -> int:
        return 0 if self.packed is None else self.packed.get_seq_length()

    def get_mask_sizes(self, query_length: int) -> Tuple[int, int]:
        return self.get_seq_length() + int(query_length), 0

    def crop(self, max_length: int) -> None:
        # transformers semantics: a negative length removes tokens from the end
        n = self.get_seq_length()
        self.packed.crop(n + max_length if max_length < 0 else min(max_length, n))

    def update(self, key_states, value_states, *args, **kwargs):
        if self.get_seq_length() == 0:
            # streaming prefill: pack this layer now (pack_kivi_kv semantics)
            B, H, S, D = (int(x) for x in key_states.shape)
            if self.packed is None:
                self.packed = PackedKVCacheLayer(B, H, D, residual_length=self._residual,
                                                 capacity=S + self._spare, device=key_states.device, **self._kw)
            self.packed.prefill(key_states, value_states)
            return key_states, value_states
        raise RuntimeError("a packed draft cache is extended by the installed attention hook, one token per step "
                           "(call kv_reduce_b200.hf.install(model) first)")


def _legacy_pairs(cache) -> Iterable[Tuple[torch.Tensor, torch.Tensor]]:
    if isinstance(cache, DynamicCache):
        return [(layer.keys, layer.values) for layer in cache.layers]
    return list(cache)


class PackedDraftCache(DynamicCache):
    """Packed draft cache built from a prefilled cache (a ``DynamicCache`` or
    (k, v) pairs of [B, H, S, D] bf16 per layer)."""

    def __init__(self, cache, residual: int, **kw) -> None:
        super().__init__()
        self.layers = [PackedDraftLayer(PackedLayer(k, v, residual, **kw)) for k, v in _legacy_pairs(cache)]

    @classmethod
    def empty(cls, num_layers: int, residual: int, *, spare_capacity: int = 2048, **kw) -> "PackedDraftCache":
        """A cache to run the prompt forward into: each layer is packed as the
        forward produces it (streaming prefill), then decoded through the hook.
        ``kw`` are PackedKVCacheLayer options (k_bits, v_bits, group_size)."""
        self = cls([], residual)
        self.layers = [PackedDraftLayer(None, residual=residual, spare_capacity=spare_capacity, **kw)
                       for _ in range(int(num_layers))]
        return self

    def commit(self) -> None:
        for layer in self.layers:
            if layer.packed is not None:
                layer.packed.commit()

    def breakdown(self) -> Dict[str, int]:
        parts = [layer.packed.breakdown() for layer in self.layers if layer.packed is not None]
        return {key: sum(p[key] for p in parts) for key in parts[0]}


def install(model, *, split_tokens: int = 0) -> None:
    """Route one-token attention steps over a ``PackedDraftCache`` through the
    packed decode kernel (packed_review.py:65-80).  ``split_tokens`` is
    passed to the kernel (0: the library's split plan; the reference used
    512)."""
    for layer in model.model.layers:
        attn = layer.self_attn
        original = attn.forward

        def forward(self, hidden_states, position_embeddings, attention_mask, past_key_values=None,
                    _original=original, **kwargs):
            if (not isinstance(past_key_values, PackedDraftCache)
                    or past_key_values.layers[self.layer_idx].get_seq_length() == 0):
                # other caches, and the prompt forward of an empty packed cache
                # (its update() packs the layer: streaming prefill)
                return _original(hidden_states, position_embeddings, attention_mask, past_key_values, **kwargs)
            if hidden_states.shape[1] != 1:
                raise ValueError("the packed draft cache decodes one token per step")
            shape = hidden_states.shape[:-1]
            view = (*shape, -1, self.head_dim)
            q = self.q_proj(hidden_states).view(view).transpose(1, 2)
            k = self.k_proj(hidden_states).view(view).transpose(1, 2)
            v = self.v_proj(hidden_states).view(view).transpose(1, 2)
            q, k = apply_rotary_pos_emb(q, k, *position_embeddings)
            packed = past_key_values.layers[self.layer_idx].packed
            out = packed.decode_step(q, k, v, split_tokens=split_tokens)
            return self.o_proj(out.transpose(1, 2).reshape(*shape, -1).contiguous()), None

        attn.forward = types.MethodType(forward, attn)
