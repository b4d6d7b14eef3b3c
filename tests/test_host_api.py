"""Host-side checks that need no GPU: the C-ABI library loads and exports
every declared symbol, argument validation, byte accounting."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def test_library_exports_header_symbols(built_lib):
    from kv_reduce_b200 import _lib

    header = (ROOT / "include" / "kvr.h").read_text()
    declared = set(re.findall(r"^(?:int|size_t|const char\*)\s+(kvr_\w+)\(", header, flags=re.M))
    assert declared == set(_lib.EXPORTED_SYMBOLS)
    lib = _lib.load()
    for name in declared:
        assert hasattr(lib, name), name
    assert lib.kvr_version() >= 100
    assert lib.kvr_status_string(0) == b"ok"
    assert lib.kvr_status_string(6) == b"workspace too small"


def test_c_abi_validation_without_gpu(built_lib):
    """Bad arguments are rejected before any CUDA call."""
    from kv_reduce_b200 import _lib

    lib = _lib.load()
    assert lib.kvr_pack_unsigned(None, 10, 0, None, None) == _lib.KVR_ERR_INVALID_ARGUMENT
    assert lib.kvr_pack_unsigned(None, 0, 4, None, None) == _lib.KVR_OK
    assert lib.kvr_unpack_unsigned(None, 10, 9, None, None) == _lib.KVR_ERR_INVALID_ARGUMENT
    a = _lib.DecodeArgs()
    layer = (_lib.LayerPtrs * 1)(_lib.LayerPtrs(16, 16, 16, 16, 16, 16, 16, 16, 16))
    a.layers = ctypes.cast(layer, ctypes.POINTER(_lib.LayerPtrs))
    a.n_layers, a.batch, a.q_heads, a.kv_heads, a.head_dim = 1, 1, 12, 2, 128
    a.seq_len, a.prefix_len, a.group_size, a.key_bits, a.value_bits = 32768, 32640, 32, 4, 4
    a.key_payload_bh_stride, a.key_meta_bh_stride = 32640 * 64, 1020 * 128
    a.key_residual_bh_stride, a.value_payload_bh_stride, a.value_meta_bh_stride = 128 * 128, 32768 * 64, 32768
    a.num_sms = 148
    ns, ws, nc = ctypes.c_int(), ctypes.c_size_t(), ctypes.c_size_t()
    assert lib.kvr_decode_plan(a, ctypes.byref(ns), ctypes.byref(ws), ctypes.byref(nc)) == _lib.KVR_OK
    assert 1 <= ns.value <= 256
    g1 = -(-ns.value // 16)                       # first-level merge groups of 16 splits
    assert nc.value == 2 * (g1 + 1)
    assert ws.value == (2 * (ns.value + (g1 if g1 > 1 else 0)) * 8 * 130 * 4 if ns.value > 1 else 0)
    a.key_bits = 3
    assert lib.kvr_decode_plan(a, None, None, None) == _lib.KVR_ERR_UNSUPPORTED
    a.key_bits, a.head_dim = 4, 96
    assert lib.kvr_decode_plan(a, None, None, None) == _lib.KVR_ERR_UNSUPPORTED
    a.head_dim, a.q_heads = 128, 13
    assert lib.kvr_decode_plan(a, None, None, None) == _lib.KVR_ERR_INVALID_ARGUMENT
    a.q_heads, a.value_payload_bh_stride = 12, 32768 * 64 + 8
    assert lib.kvr_decode_plan(a, None, None, None) == _lib.KVR_ERR_MISALIGNED
    a.value_payload_bh_stride, a.n_layers = 32768 * 64, 33
    assert lib.kvr_decode_plan(a, None, None, None) == _lib.KVR_ERR_INVALID_ARGUMENT
    # a workspace smaller than the plan is refused before launching
    a.n_layers, a.workspace, a.workspace_bytes, a.counters = 1, 256, 16, 256
    if ns.value > 1:
        assert lib.kvr_decode_attention(a, None) == _lib.KVR_ERR_WORKSPACE


def test_python_validation_without_gpu(built_lib):
    import kv_reduce_b200 as kvr
    from kv_reduce_b200.packed_kv_cache import _quantized_prefix_length

    assert _quantized_prefix_length(32768, 32, 128) == 32640
    with pytest.raises(ValueError):
        _quantized_prefix_length(10, 0, 0)
    assert kvr.packed_num_bytes(37, 3) == 14
    with pytest.raises(ValueError):
        kvr.packed_num_bytes(1, 9)
    with pytest.raises(ValueError):
        kvr.pack_unsigned(torch.zeros(4, dtype=torch.uint8), 0)
    with pytest.raises(ValueError):   # CPU tensors: no CPU fallback, fail loudly
        kvr.pack_unsigned(torch.zeros(4, dtype=torch.uint8), 4)
    with pytest.raises(ValueError):
        kvr.pack_per_token_affine(torch.zeros(1, 1, 4, 8, dtype=torch.bfloat16), 4)
    with pytest.raises(ValueError):
        kvr.pack_per_token_affine(torch.zeros(1, 1, 4, 8, dtype=torch.bfloat16), 1)
    native = kvr.pack_per_channel_grouped_affine(torch.zeros(1, 1, 4, 8, dtype=torch.bfloat16), 16)
    assert native.layout == "native" and native.storage_bytes == 64
    q = torch.zeros(1, 12, 1, 128, dtype=torch.bfloat16)
    comp = kvr.PackedKVComponent(torch.zeros(1, dtype=torch.uint8), None, None, None, (1, 2, 8, 128), 4,
                                 "per_channel_grouped_affine", torch.bfloat16, 32, 0)
    with pytest.raises(ValueError, match="CUDA query"):
        kvr.packed_kv_decode_attention(q, comp, comp)


def test_byte_accounting_matches_reference_numbers():
    from kv_reduce_b200 import workloads

    b = workloads.layer_bytes(workloads.CONFIGS["2"])
    assert b["cache"] == 9_744_384                  # results/packed JSON packed_cache_bytes_one_layer
    assert b["total"] == 9_750_528
    assert 28 * b["total"] == 273_014_784
    assert workloads.layer_bytes(workloads.CONFIGS["1"])["total"] == 309_248
    assert workloads.layer_bytes(workloads.CONFIGS["4"])["total"] == 179_961_856
    assert workloads.layer_bytes(workloads.CONFIGS["3a"])["total"] == 228_589_568
