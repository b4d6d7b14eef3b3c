"""The benchmarked launches themselves, at full size, against the oracle.

bench.py times one decode launch per step over all layers of each workload
with the automatic split plan (for the 28-layer 32K Qwen2.5-1.5B step: 10
splits per (layer, KV head), merged in thread-block clusters; for the
batched workloads: multi-wave plans of 1 to 4 splits with the global
merge).  These tests build the same caches with the same code
(bench.build_cache, bench.fused_launches), run the same launches with fp32
outputs, and compare whole layers with the oracle (fp32 dequantize +
softmax attention of the reference, in float64) at the path's tolerance:
max |err| <= 2e-3, mean |err| <= 1e-3.  The bf16 launch that the benchmark
times must equal that fp32 result rounded to bf16, bit for bit.
"""
import numpy as np
import pytest
import torch

import bench
from conftest import bits_of
from oracle import attention, packing

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-3, 1e-3


@pytest.fixture(scope="module")
def kvr(built_lib):
    import kv_reduce_b200

    return kv_reduce_b200


def oracle_layer(wl, layer, seqs):
    """Oracle output [len(seqs), HQ, D] of one layer for the given sequences
    (the workload data is generated on the GPU, as the benchmark does)."""
    from kv_reduce_b200 import workloads

    k, v = workloads.make_layer_kv(wl, layer, device="cuda")
    q = workloads.make_query(wl, layer, device="cuda")
    outs = []
    for b in seqs:
        kb, vb, qb = k[b:b + 1], v[b:b + 1], q[b:b + 1]
        kq = packing.quantize_grouped(bits_of(kb), wl.k_bits, wl.group_size, wl.residual_length)
        vq = packing.quantize_per_token(bits_of(vb), wl.v_bits)
        K = packing.dequant_grouped(kq["payload"], kq["scale"], kq["offset"], kq["residual"], wl.k_bits,
                                    tuple(kb.shape), kq["P"], wl.group_size)
        V = packing.dequant_per_token(vq["payload"], vq["scale"], vq["offset"], wl.v_bits, tuple(vb.shape))
        outs.append(attention.decode_attention(packing.bf16_to_f32(bits_of(qb))[:, :, 0], K, V)[0])
    del k, v, q
    return np.stack(outs)


def run_benchmarked(kvr, key, check_layers, check_seqs):
    from kv_reduce_b200 import workloads
    from kv_reduce_b200.packed_kv_attention import DecodeLaunch

    wl = workloads.CONFIGS[key]
    device = torch.device("cuda", 0)
    ks, vs, qs = bench.build_cache(wl, device, 0)
    stream = torch.cuda.Stream(device)
    launches, outs, geom, ptrs = bench.fused_launches(ks, vs, qs, device, stream, 0)
    outs32 = [torch.empty(q.shape, dtype=torch.float32, device=device) for q in qs]
    ptrs32 = []
    for p, o in zip(ptrs, outs32):
        c = type(p).from_buffer_copy(p)
        c.out = o.data_ptr()
        ptrs32.append(c)
    launches32 = [DecodeLaunch(geom, ptrs32[i:i + 32], device, stream=stream.cuda_stream, out_fp32=True)
                  for i in range(0, len(ptrs32), 32)]
    assert [x.num_splits for x in launches32] == [x.num_splits for x in launches]
    with torch.cuda.stream(stream):
        for x in launches:
            x()
        for x in launches32:
            x()
    torch.cuda.synchronize()
    for o, o32 in zip(outs, outs32):
        assert torch.equal(o, o32.to(torch.bfloat16)), "the timed bf16 launch differs from the fp32 launch"
    errs = []
    for layer in check_layers:
        ref = oracle_layer(wl, layer, check_seqs)
        got = outs32[layer][list(check_seqs), :, 0, :].cpu().numpy()
        err = np.abs(got - ref)
        assert err.max() <= MAX_ABS, f"{wl.name} layer {layer}: max abs err {err.max():.3e}"
        assert err.mean() <= MEAN_ABS, f"{wl.name} layer {layer}: mean abs err {err.mean():.3e}"
        errs.append(float(err.max()))
    splits = launches[0].num_splits
    del launches, launches32, ks, vs, qs, outs, outs32
    torch.cuda.empty_cache()
    return splits, errs


def test_benchmarked_qwen_32k_step(kvr):
    """The headline launch: 28 layers x 32K tokens, batch 1, K4V4, automatic
    plan; three whole layers (both KV heads, all 12 query heads) checked."""
    splits, _ = run_benchmarked(kvr, "2", (0, 13, 27), (0,))
    assert splits > 1


@pytest.mark.parametrize("key", ["3a", "3b"])
def test_benchmarked_llama_8k_batch32(kvr, key):
    """Llama-3.2-1B geometry (D=64, GQA 4), batch 32 x 8K, 16 layers, K8V4
    and K4V8 -- the benchmarked multi-wave plan; sequences 0, 17 and 31 of
    layers 0 and 15 checked."""
    run_benchmarked(kvr, key, (0, 15), (0, 17, 31))


def test_benchmarked_kivi2_16k_batch64(kvr):
    """K2V2 stress: batch 64 x 16K, 28 layers -- the benchmarked multi-wave
    few-split plan with the global merge; sequences 0 and 63 of layers 0 and
    27 checked."""
    splits, _ = run_benchmarked(kvr, "4", (0, 27), (0, 63))
    assert splits >= 1
