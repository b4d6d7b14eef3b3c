"""The allocation-free decode entry point, through the C ABI.

Callers such as an FFI host without a CUDA allocator or a serving loop that
must not call cudaMalloc use kvr_decode_attention_noalloc, whose split
scratch is a fixed array inside the library instead of a caller workspace.
It takes the same plan, kernel and merge order as kvr_decode_attention, so
on the same inputs it must give the same bits, on repeated calls (the shared
array keeps the previous call's contents), and it must refuse a problem
larger than its fixed scratch.  This file is collected last
so that a run stopping at the first failure has run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(kvr, seq_len, residual, seed):
    from kv_reduce_b200 import workloads
    from kv_reduce_b200.packed_kv_attention import DecodeLaunch, _geometry, _layer_ptrs

    wl = workloads.CONFIGS["2"].scaled(seq_len=seq_len, residual_length=residual, seed=seed)
    k, v = workloads.make_layer_kv(wl, 0)
    q = workloads.make_query(wl, 0)
    pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=residual)
    geom = _geometry(q, pk, pv)
    out_ref = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    ref = DecodeLaunch(geom, [_layer_ptrs(q, out_ref, pk, pv)], q.device, out_fp32=True)
    return q, pk, pv, geom, out_ref, ref, _layer_ptrs


def _noalloc_args(ref_launch, layers_arr):
    from kv_reduce_b200 import _lib

    a = _lib.DecodeArgs()
    ctypes.pointer(a)[0] = ref_launch.args          # same geometry, strides, split plan inputs
    a.layers = ctypes.cast(layers_arr, ctypes.POINTER(_lib.LayerPtrs))
    a.workspace, a.workspace_bytes, a.counters = None, 0, None   # the entry point uses its own scratch
    return a


@pytest.mark.parametrize("seq_len,residual", [(32768, 128), (1024, 0)])
def test_noalloc_matches_allocating_entry_point(built_lib, seq_len, residual):
    import kv_reduce_b200 as kvr
    from kv_reduce_b200 import _lib

    lib = _lib.load()
    q, pk, pv, geom, out_ref, ref, layer_ptrs = _setup(kvr, seq_len, residual, seed=3)
    ref()
    torch.cuda.synchronize()
    out = torch.empty_like(out_ref)
    layers_arr = (_lib.LayerPtrs * 1)(layer_ptrs(q, out, pk, pv))
    args = _noalloc_args(ref, layers_arr)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):                    # second call reuses the scratch left by the first
        out.fill_(float("nan"))
        st = lib.kvr_decode_attention_noalloc(ctypes.byref(args), stream)
        assert st == _lib.KVR_OK, lib.kvr_status_string(st)
        torch.cuda.synchronize()
        assert torch.equal(out, out_ref), f"call {call}: max abs diff {(out - out_ref).abs().max().item():.3e}"


def test_noalloc_refuses_problem_larger_than_scratch(built_lib):
    import kv_reduce_b200 as kvr
    from kv_reduce_b200 import _lib

    lib = _lib.load()
    q, pk, pv, geom, out_ref, ref, layer_ptrs = _setup(kvr, 32768, 128, seed=4)
    out = torch.empty_like(out_ref)
    layers_arr = (_lib.LayerPtrs * 1)(layer_ptrs(q, out, pk, pv))
    args = _noalloc_args(ref, layers_arr)
    args.split_tokens = 32          # 1024 splits requested -> capped at 256, ~2 MB of partials x 2 heads
    args.batch = 1
    # 32 layers sharing one geometry need 32x the partials: over the 4 MiB limit
    many = (_lib.LayerPtrs * 32)(*([layer_ptrs(q, out, pk, pv)] * 32))
    args.layers = ctypes.cast(many, ctypes.POINTER(_lib.LayerPtrs))
    args.n_layers = 32
    st = lib.kvr_decode_attention_noalloc(ctypes.byref(args), torch.cuda.current_stream().cuda_stream)
    assert st == _lib.KVR_ERR_WORKSPACE
