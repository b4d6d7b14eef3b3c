"""ctypes binding of libkvr.so (the C ABI declared in include/kvr.h).

This module is the only place that touches the shared library.  It fails
loudly when the library is missing or when a tensor is not on a CUDA device:
there is no CPU fallback for any operation of the package.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, Structure, c_int, c_int64, c_size_t, c_void_p, c_char_p
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("KVR_LIB", _PKG / "libkvr.so"))
TORCH_OPS_PATH = _PKG / "libkvr_torch.so"

KVR_OK = 0
KVR_ERR_INVALID_ARGUMENT = 1
KVR_ERR_UNSUPPORTED = 2
KVR_ERR_MISALIGNED = 3
KVR_ERR_CUDA = 4
KVR_ERR_CAPACITY = 5
KVR_ERR_WORKSPACE = 6
KVR_MAX_LAYERS = 32

# Every symbol include/kvr.h declares; tests check the library exports them.
EXPORTED_SYMBOLS = (
    "kvr_version",
    "kvr_status_string",
    "kvr_last_error",
    "kvr_host_mapped",
    "kvr_pack_unsigned",
    "kvr_unpack_unsigned",
    "kvr_quantize_per_token",
    "kvr_quantize_grouped",
    "kvr_dequantize",
    "kvr_append",
    "kvr_flush_groups",
    "kvr_decode_plan",
    "kvr_decode_cluster",
    "kvr_decode_attention",
    "kvr_decode_attention_simt",
    "kvr_decode_simt_workspace",
    "kvr_lse_merge",
    "kvr_decode_partial",
    "kvr_decode_attention_noalloc",
    "kvr_append_lengths",
    "kvr_advance_lengths",
    "kvr_set_lengths",
    "kvr_decode_attention_lengths",
    "kvr_decode_step",
    "kvr_key_scale_pairs",
    "kvr_decode_nonfinite",
    "kvr_exchange_merge",
    "kvr_exchange_merge_delivered",
    "kvr_exchange_merge_owned",
    "kvr_exchange_gather_owned",
    "kvr_decode_partial_exchange",
    "kvr_exchange_alloc",
    "kvr_exchange_open",
    "kvr_exchange_close",
    "kvr_exchange_free",
)


class KvrError(RuntimeError):
    """A libkvr call returned a non-zero status."""

    def __init__(self, fn: str, status: int, text: str, cuda: str = "") -> None:
        msg = f"{fn} failed: {text} (status {status})"
        if cuda:
            msg += f": {cuda}"
        super().__init__(msg)
        self.status = status


class TokenQuantArgs(Structure):
    _fields_ = [
        ("x", c_void_p), ("x_bh_stride", c_int64), ("x_row_stride", c_int64),
        ("payload", c_void_p), ("payload_bh_stride", c_int64),
        ("scale", c_void_p), ("offset", c_void_p), ("meta_bh_stride", c_int64),
        ("bh", c_int), ("rows", c_int), ("row0", c_int), ("head_dim", c_int), ("bits", c_int),
        ("codes_scratch", c_void_p),
    ]


class GroupQuantArgs(Structure):
    _fields_ = [
        ("x", c_void_p), ("x_bh_stride", c_int64), ("x_row_stride", c_int64),
        ("payload", c_void_p), ("payload_bh_stride", c_int64),
        ("scale", c_void_p), ("offset", c_void_p), ("meta_bh_stride", c_int64),
        ("bh", c_int), ("groups", c_int), ("group0", c_int), ("group_size", c_int),
        ("head_dim", c_int), ("bits", c_int),
        ("codes_scratch", c_void_p),
    ]


class DequantArgs(Structure):
    _fields_ = [
        ("payload", c_void_p), ("payload_bh_stride", c_int64),
        ("scale", c_void_p), ("offset", c_void_p), ("meta_bh_stride", c_int64),
        ("residual", c_void_p), ("residual_bh_stride", c_int64),
        ("out", c_void_p), ("out_dtype", c_int), ("bh", c_int), ("seq_len", c_int),
        ("prefix_len", c_int), ("group_size", c_int), ("head_dim", c_int), ("bits", c_int),
    ]


class AppendArgs(Structure):
    _fields_ = [
        ("k", c_void_p), ("v", c_void_p),
        ("key_residual", c_void_p), ("key_residual_bh_stride", c_int64),
        ("value_payload", c_void_p), ("value_payload_bh_stride", c_int64),
        ("value_scale", c_void_p), ("value_offset", c_void_p), ("value_meta_bh_stride", c_int64),
        ("bh", c_int), ("n", c_int), ("seq_len", c_int), ("res_len", c_int),
        ("res_capacity", c_int), ("seq_capacity", c_int), ("head_dim", c_int), ("value_bits", c_int),
    ]


class FlushArgs(Structure):
    _fields_ = [
        ("residual_in", c_void_p), ("residual_out", c_void_p), ("residual_bh_stride", c_int64),
        ("key_payload", c_void_p), ("key_payload_bh_stride", c_int64),
        ("key_scale", c_void_p), ("key_offset", c_void_p), ("key_meta_bh_stride", c_int64),
        ("bh", c_int), ("res_len", c_int), ("groups", c_int), ("prefix_len", c_int),
        ("prefix_capacity", c_int), ("group_size", c_int), ("head_dim", c_int), ("key_bits", c_int),
    ]


class LayerPtrs(Structure):
    _fields_ = [
        ("key_payload", c_void_p), ("key_scale", c_void_p), ("key_offset", c_void_p),
        ("key_residual", c_void_p), ("value_payload", c_void_p), ("value_scale", c_void_p),
        ("value_offset", c_void_p), ("query", c_void_p), ("out", c_void_p),
        ("key_scale_pairs", c_void_p),
    ]


class ScalePairsArgs(Structure):
    _fields_ = [
        ("scale", c_void_p), ("scale_bh_stride", c_int64),
        ("pairs", c_void_p), ("pairs_bh_stride", c_int64),
        ("bh", c_int), ("groups", c_int), ("group0", c_int), ("head_dim", c_int), ("key_bits", c_int),
    ]


class ExchangeArgs(Structure):
    _fields_ = [
        ("world", c_int), ("rank", c_int), ("rows", c_int), ("head_dim", c_int),
        ("recv", c_void_p), ("signal", c_void_p), ("epoch", c_void_p), ("counter", c_void_p),
        ("error", c_void_p), ("out", c_void_p), ("timeout_ns", ctypes.c_longlong), ("mode", c_int),
    ]


class DecodeArgs(Structure):
    _fields_ = [
        ("layers", POINTER(LayerPtrs)), ("n_layers", c_int),
        ("batch", c_int), ("q_heads", c_int), ("kv_heads", c_int), ("head_dim", c_int),
        ("seq_len", c_int), ("prefix_len", c_int), ("group_size", c_int),
        ("key_bits", c_int), ("value_bits", c_int),
        ("key_payload_bh_stride", c_int64), ("key_meta_bh_stride", c_int64),
        ("key_residual_bh_stride", c_int64), ("value_payload_bh_stride", c_int64),
        ("value_meta_bh_stride", c_int64),
        ("out_dtype", c_int), ("split_tokens", c_int), ("num_sms", c_int),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("counters", c_void_p), ("query_host_mapped", c_int),
    ]


_lib = None


def load() -> ctypes.CDLL:
    """Load libkvr.so once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m kv_reduce_b200.build` "
            "(kv_reduce_b200 has no CPU fallback)"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    lib.kvr_version.restype = c_int
    lib.kvr_status_string.restype = c_char_p
    lib.kvr_status_string.argtypes = [c_int]
    lib.kvr_last_error.restype = c_char_p
    lib.kvr_pack_unsigned.argtypes = [c_void_p, c_int64, c_int, c_void_p, c_void_p]
    lib.kvr_unpack_unsigned.argtypes = [c_void_p, c_int64, c_int, c_void_p, c_void_p]
    lib.kvr_quantize_per_token.argtypes = [POINTER(TokenQuantArgs), c_void_p]
    lib.kvr_quantize_grouped.argtypes = [POINTER(GroupQuantArgs), c_void_p]
    lib.kvr_dequantize.argtypes = [POINTER(DequantArgs), c_void_p]
    lib.kvr_append.argtypes = [POINTER(AppendArgs), c_void_p]
    lib.kvr_flush_groups.argtypes = [POINTER(FlushArgs), c_void_p]
    lib.kvr_decode_plan.argtypes = [POINTER(DecodeArgs), POINTER(c_int), POINTER(c_size_t), POINTER(c_size_t)]
    lib.kvr_decode_cluster.argtypes = [POINTER(DecodeArgs), POINTER(c_int)]
    lib.kvr_decode_attention.argtypes = [POINTER(DecodeArgs), c_void_p]
    lib.kvr_decode_partial.argtypes = [POINTER(DecodeArgs), c_int, c_int, c_void_p, c_void_p, c_void_p]
    lib.kvr_lse_merge.argtypes = [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]
    lib.kvr_decode_attention_noalloc.argtypes = [POINTER(DecodeArgs), c_void_p]
    lib.kvr_decode_attention_simt.argtypes = [POINTER(DecodeArgs), c_void_p]
    lib.kvr_decode_simt_workspace.argtypes = [POINTER(DecodeArgs)]
    lib.kvr_append_lengths.argtypes = [POINTER(AppendArgs), c_void_p, c_int, c_void_p]
    lib.kvr_advance_lengths.argtypes = [c_void_p, c_int, c_void_p]
    lib.kvr_set_lengths.argtypes = [c_void_p, c_int, c_int, c_void_p]
    lib.kvr_decode_attention_lengths.argtypes = [POINTER(DecodeArgs), c_void_p, c_int, c_void_p]
    lib.kvr_decode_step.argtypes = [POINTER(DecodeArgs), c_void_p, c_void_p, c_void_p, c_int, c_void_p]
    lib.kvr_key_scale_pairs.argtypes = [POINTER(ScalePairsArgs), c_void_p]
    lib.kvr_host_mapped.argtypes = [c_void_p, POINTER(c_int)]
    lib.kvr_decode_nonfinite.argtypes = [POINTER(c_int), c_int]
    lib.kvr_exchange_merge.argtypes = [POINTER(ExchangeArgs), c_void_p]
    lib.kvr_exchange_merge_delivered.argtypes = [POINTER(ExchangeArgs), c_void_p]
    lib.kvr_exchange_merge_owned.argtypes = [POINTER(ExchangeArgs), c_void_p]
    lib.kvr_exchange_gather_owned.argtypes = [POINTER(ExchangeArgs), c_void_p]
    lib.kvr_decode_partial_exchange.argtypes = [POINTER(DecodeArgs), c_int, c_int, POINTER(ExchangeArgs), c_void_p]
    lib.kvr_exchange_alloc.argtypes = [c_size_t, POINTER(c_void_p), ctypes.c_char_p]
    lib.kvr_exchange_open.argtypes = [ctypes.c_char_p, POINTER(c_void_p)]
    lib.kvr_exchange_close.argtypes = [c_void_p]
    lib.kvr_exchange_free.argtypes = [c_void_p]
    for name in EXPORTED_SYMBOLS:
        if name not in ("kvr_version", "kvr_status_string", "kvr_last_error"):
            getattr(lib, name).restype = c_int
    lib.kvr_decode_simt_workspace.restype = c_size_t
    _lib = lib
    return lib


_torch_ops = False


def load_torch_ops() -> None:
    """Register the C++ operators torch.ops.kvr.decode_attention /
    decode_step / lse_merge (libkvr_torch.so over libkvr.so); raise if the
    library has not been built."""
    global _torch_ops
    if _torch_ops:
        return
    load()
    if not TORCH_OPS_PATH.exists():
        raise RuntimeError(
            f"{TORCH_OPS_PATH} is missing: build it with `python -m kv_reduce_b200.build` "
            "(kv_reduce_b200 has no CPU fallback)"
        )
    torch.ops.load_library(str(TORCH_OPS_PATH))
    _torch_ops = True


def check(fn: str, status: int) -> None:
    if status == KVR_OK:
        return
    lib = load()
    text = lib.kvr_status_string(status).decode()
    cuda = lib.kvr_last_error().decode() if status == KVR_ERR_CUDA else ""
    raise KvrError(fn, status, text, cuda)


def call(fn: str, *args) -> None:
    check(fn, getattr(load(), fn)(*args))


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def host_mapped(ptr_value: int) -> bool:
    """True when a kernel can read and write this pinned host address
    directly (kvr_host_mapped)."""
    flag = c_int(0)
    call("kvr_host_mapped", ptr_value, ctypes.byref(flag))
    return bool(flag.value)


def stream_ptr(device: torch.device) -> int:
    """cudaStream_t of the current stream on `device` (as an int)."""
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    if t is None or t.numel() == 0:
        return None
    return t.data_ptr()


def require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("kv_reduce_b200 operates on CUDA tensors only (no CPU fallback).")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("All tensors must be on the same CUDA device.")
    if dev is None:
        raise ValueError("No CUDA tensor given.")
    return dev
