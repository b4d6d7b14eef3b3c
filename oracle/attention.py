"""Attention oracle -- test infrastructure only.

One-token GQA decode attention over the fp32-dequantized cache, computed in
float64: softmax(q K^T / sqrt(D)) V per query head, query head h reading KV
head h // (HQ/HKV).  This is what the reference kernels compute
(kv_reduce/triton_packed_kv_attention.py:27-131 and :134-281) and what its
own check compares them with (SDPA over PackedKVComponent.unpack(),
kv_reduce/experiments/packed_review.py:93).
"""
from __future__ import annotations

import numpy as np


def decode_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """q [B, HQ, D], k/v [B, HKV, S, D] (any float) -> [B, HQ, D] float64."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    B, HQ, D = q.shape
    HKV = k.shape[1]
    rep = HQ // HKV
    kk = np.repeat(k, rep, axis=1)          # [B, HQ, S, D]
    vv = np.repeat(v, rep, axis=1)
    s = np.einsum("bhd,bhsd->bhs", q, kk) / np.sqrt(D)
    s -= s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("bhs,bhsd->bhd", p, vv)


def partials(q: np.ndarray, k: np.ndarray, v: np.ndarray):
    """(m, l, o) of a token shard in log2 units: m = max_t s_t*log2(e),
    l = sum 2^(s*log2e - m), o = sum 2^(...) v  -- for LSE-merge tests."""
    q = np.asarray(q, dtype=np.float64)
    B, HQ, D = q.shape
    rep = HQ // k.shape[1]
    kk = np.repeat(np.asarray(k, np.float64), rep, axis=1)
    vv = np.repeat(np.asarray(v, np.float64), rep, axis=1)
    s = np.einsum("bhd,bhsd->bhs", q, kk) / np.sqrt(D) * np.log2(np.e)
    m = s.max(axis=-1)
    w = np.exp2(s - m[..., None])
    return m, w.sum(-1), np.einsum("bhs,bhsd->bhd", w, vv)
