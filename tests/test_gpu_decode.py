"""GPU parity of the split-K packed decode attention against the oracle.

Tolerance (floating point, stated by the path's spec): max |err| <= 2e-3 and
mean |err| <= 1e-3 against the fp32 dequantize + softmax attention of the
reference, computed by the oracle in float64.  The tolerance applies to the
kernel's fp32 result (out_dtype=torch.float32); the default bf16 output is
that result rounded to bf16, checked bit-for-bit against the fp32 output and
against the oracle with the bf16 half-ulp (2^-8 |x|) added.
"""
import numpy as np
import pytest
import torch

from conftest import bf16_from_bits, bits_of
from oracle import attention, packing

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-3, 1e-3


@pytest.fixture(scope="module")
def kvr(built_lib):
    import kv_reduce_b200

    return kv_reduce_b200


def oracle_out(keys, values, query, kb, vb, G, R):
    kq = packing.quantize_grouped(bits_of(keys), kb, G, R)
    vq = packing.quantize_per_token(bits_of(values), vb)
    K = packing.dequant_grouped(kq["payload"], kq["scale"], kq["offset"], kq["residual"], kb, tuple(keys.shape),
                                kq["P"], G)
    V = packing.dequant_per_token(vq["payload"], vq["scale"], vq["offset"], vb, tuple(values.shape))
    q = packing.bf16_to_f32(bits_of(query))[:, :, 0, :]
    return attention.decode_attention(q, K, V)


def check(out, ref, what=""):
    assert out.dtype == torch.float32, "the tolerance applies to the fp32 result"
    got = out.cpu().numpy()[:, :, 0, :]
    err = np.abs(got - ref)
    assert err.max() <= MAX_ABS, f"{what}: max abs err {err.max():.3e}"
    assert err.mean() <= MEAN_ABS, f"{what}: mean abs err {err.mean():.3e}"
    return err


def check_bf16(out, ref, what=""):
    assert out.dtype == torch.bfloat16
    got = out.float().cpu().numpy()[:, :, 0, :]
    bound = MAX_ABS + np.abs(ref) * 2.0 ** -8
    assert np.all(np.abs(got - ref) <= bound), f"{what}: bf16 output outside tolerance"


F32 = torch.float32


def make(shape, hq, kb, vb, G, R, seed, q_scale=1.0, outliers=4):
    g = torch.Generator(device="cuda").manual_seed(seed)
    B, H, S, D = shape
    k = torch.randn(shape, generator=g, device="cuda")
    chans = torch.randperm(D, generator=torch.Generator().manual_seed(seed))[:outliers]
    k[..., chans] *= 10
    v = torch.randn(shape, generator=g, device="cuda")
    q = torch.randn(B, hq, 1, D, generator=g, device="cuda") * q_scale
    return k.to(torch.bfloat16), v.to(torch.bfloat16), q.to(torch.bfloat16)


def test_golden_attention(kvr, golden):
    """Kernel vs the reference's own fp32 unpack + SDPA result."""
    for name in (str(c) for c in golden["kv_cases"]):
        p = f"kv_{name}_"
        if p + "query" not in golden.files:
            continue
        kb, vb, G, R, P = (int(v) for v in golden[p + "params"])
        keys, values = bf16_from_bits(golden[p + "keys"]), bf16_from_bits(golden[p + "values"])
        q = bf16_from_bits(golden[p + "query"])
        pk, pv = kvr.pack_kivi_kv(keys, values, k_bits=kb, v_bits=vb, group_size=G, residual_length=R)
        out = kvr.packed_kv_decode_attention(q, pk, pv, out_dtype=F32)
        assert out.shape == q.shape
        check(out, golden[p + "attn_f32"][:, :, 0, :], name)
        out_bf16 = kvr.packed_kv_decode_attention(q, pk, pv)
        assert out_bf16.dtype == q.dtype and torch.equal(out_bf16, out.to(q.dtype))
        check_bf16(out_bf16, golden[p + "attn_f32"][:, :, 0, :], name)


@pytest.mark.parametrize("split", [0, 32, 64, 96, 512, 1 << 20])
def test_config1_all_splits(kvr, split):
    from kv_reduce_b200 import workloads

    wl = workloads.CONFIGS["1"]
    k, v = workloads.make_layer_kv(wl, 0)
    q = workloads.make_query(wl, 0)
    pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=0)
    out = kvr.packed_kv_decode_attention(q, pk, pv, split_tokens=split, out_dtype=F32)
    check(out, oracle_out(k, v, q, 4, 4, 32, 0), f"split={split}")


@pytest.mark.parametrize("shape,hq,kb,vb,G,R", [
    ((1, 2, 1026, 128), 12, 4, 4, 32, 0),     # after crop in the reference unit test
    ((1, 2, 1057, 128), 12, 4, 4, 32, 128),   # group boundary + residual
    ((2, 2, 4099, 128), 12, 2, 2, 32, 128),   # K2V2 ragged
    ((2, 2, 2000, 128), 12, 8, 4, 32, 128),
    ((2, 2, 2000, 128), 12, 4, 8, 32, 128),
    ((1, 2, 777, 128), 12, 8, 8, 16, 64),     # G=16: two groups per chunk
    ((1, 2, 777, 128), 16, 4, 2, 64, 33),     # GQA 8, G=64, odd residual
    ((3, 8, 1500, 64), 32, 8, 4, 32, 128),    # Llama geometry, K8V4
    ((3, 8, 1500, 64), 32, 4, 8, 32, 128),    # K4V8
    ((1, 4, 300, 64), 4, 2, 4, 32, 0),        # GQA 1
    ((1, 2, 33, 128), 12, 4, 4, 32, 0),       # one group + 1 residual token
])
def test_shapes_match_oracle(kvr, shape, hq, kb, vb, G, R):
    k, v, q = make(shape, hq, kb, vb, G, R, seed=sum(shape) + kb + vb + G + R)
    pk, pv = kvr.pack_kivi_kv(k, v, k_bits=kb, v_bits=vb, group_size=G, residual_length=R)
    ref = oracle_out(k, v, q, kb, vb, G, R)
    for split in (0, 64):
        out = kvr.packed_kv_decode_attention(q, pk, pv, split_tokens=split, out_dtype=F32)
        check(out, ref, f"{shape} k{kb}v{vb} G{G} R{R} split={split}")


def test_peaked_attention(kvr):
    """A query 6x larger: near one-hot softmax, largest fp16 operand rounding."""
    k, v, q = make((1, 2, 2048, 128), 12, 4, 4, 32, 128, seed=99, q_scale=6.0)
    pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=128)
    out = kvr.packed_kv_decode_attention(q, pk, pv, out_dtype=F32)
    check(out, oracle_out(k, v, q, 4, 4, 32, 128), "peaked")


def test_full_size_config2_layer(kvr):
    """One full 32K-token layer, checked against the oracle."""
    from kv_reduce_b200 import workloads

    wl = workloads.CONFIGS["2"]
    k, v = workloads.make_layer_kv(wl, 3)
    q = workloads.make_query(wl, 3)
    pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=128)
    out = kvr.packed_kv_decode_attention(q, pk, pv, out_dtype=F32)
    ref = oracle_out(k, v, q, 4, 4, 32, 128)
    check(out, ref, "32K")
    # the reference's own launch choice (split 512, block 32)
    out512 = kvr.packed_kv_decode_attention(q, pk, pv, split_tokens=512, out_dtype=F32)
    check(out512, ref, "32K split 512")
    check_bf16(kvr.packed_kv_decode_attention(q, pk, pv), ref, "32K bf16")


def test_multi_layer_launch_equals_per_layer(kvr):
    from kv_reduce_b200 import workloads

    wl = workloads.CONFIGS["2"].scaled(seq_len=3000, layers=5)
    qs, ks, vs = [], [], []
    for layer in range(wl.layers):
        k, v = workloads.make_layer_kv(wl, layer)
        pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=128)
        qs.append(workloads.make_query(wl, layer))
        ks.append(pk)
        vs.append(pv)
    outs = kvr.packed_kv_decode_attention_layers(qs, ks, vs, split_tokens=512)
    for q, pk, pv, o in zip(qs, ks, vs, outs):
        single = kvr.packed_kv_decode_attention(q, pk, pv, split_tokens=512)
        assert torch.equal(single, o)


@pytest.mark.parametrize("split,layers", [(256, 8), (512, 32)])
def test_cluster_merge_equals_global_merge(kvr, split, layers):
    """A launch whose CTAs each take one split, with at most 16 splits per
    (layer, b, kv head), merges them inside a thread-block cluster over
    distributed shared memory (4096 tokens, batch 4: split 256 -> 16
    splits, split 512 -> 8).  The same layer repeated in a multi-layer
    launch has more items than resident CTAs and merges through global
    memory.  Same partials in the same order, so bit-identical; and within
    the oracle's tolerance."""
    from kv_reduce_b200 import workloads

    wl = workloads.CONFIGS["2"].scaled(seq_len=4096, layers=1)
    k, v = workloads.make_layer_kv(wl, 0, batch=4)
    q = workloads.make_query(wl, 0, batch=4)
    pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=128)
    single = kvr.packed_kv_decode_attention(q, pk, pv, split_tokens=split)
    many = kvr.packed_kv_decode_attention_layers([q] * layers, [pk] * layers, [pv] * layers, split_tokens=split)
    for o in many:
        assert torch.equal(o, single)
    out32 = kvr.packed_kv_decode_attention(q, pk, pv, split_tokens=split, out_dtype=F32)
    check(out32, oracle_out(k, v, q, 4, 4, 32, 128), f"split {split}")


def test_token_shards_merge_to_full(kvr):
    """Partial decode over token shards + LSE merge == full decode (the
    cross-GPU split of one long sequence, emulated on one GPU)."""
    from kv_reduce_b200.packed_kv_attention import DecodeLaunch, _geometry, _layer_ptrs, lse_merge

    k, v, q = make((1, 2, 5000, 128), 12, 4, 4, 32, 128, seed=5)
    pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=128)
    full = kvr.packed_kv_decode_attention(q, pk, pv)
    geom = _geometry(q, pk, pv)
    bounds = [0, 1024, 2048, 4096, 5000]
    mls, os_ = [], []
    for a, b in zip(bounds[:-1], bounds[1:]):
        ml = torch.empty(12, 2, device="cuda")
        o = torch.empty(12, 128, device="cuda")
        dummy = torch.empty_like(q)
        DecodeLaunch(geom, [_layer_ptrs(q, dummy, pk, pv)], q.device, token_begin=a, token_end=b).partial(ml, o)
        mls.append(ml)
        os_.append(o)
    merged = lse_merge(torch.stack(mls), torch.stack(os_)).reshape(1, 12, 1, 128)
    ref = oracle_out(k, v, q, 4, 4, 32, 128)
    check_bf16(merged, ref, "shards")
    check_bf16(full, ref, "full")
    from kv_reduce_b200.distributed import merge_partials
    merged32 = merge_partials(torch.stack(mls), torch.stack(os_)).reshape(1, 12, 1, 128)
    check(merged32, ref, "shards fp32")


def test_api_errors(kvr):
    k, v, q = make((1, 2, 256, 128), 12, 4, 4, 32, 0, seed=1)
    pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=0)
    with pytest.raises(ValueError):
        kvr.packed_kv_decode_attention(q.cpu(), pk, pv)
    with pytest.raises(ValueError):
        kvr.packed_kv_decode_attention(q[:, :, :, :64], pk, pv)
    with pytest.raises(ValueError):
        kvr.packed_kv_decode_attention(q, pv, pk)
    with pytest.raises(ValueError):
        kvr.packed_kv_decode_attention(q, pk, pv, block_tokens=48)
    with pytest.raises(ValueError):
        kvr.packed_kv_decode_attention(q[:, :11], pk, pv)
    empty_k, empty_v = kvr.pack_kivi_kv(k[:, :, :100], v[:, :, :100], k_bits=4, v_bits=4, residual_length=128)
    with pytest.raises(ValueError):
        kvr.packed_kv_decode_attention(q, empty_k, empty_v)
    k3, v3 = kvr.pack_kivi_kv(k, v, k_bits=3, v_bits=4, group_size=32, residual_length=0)
    with pytest.raises(ValueError):
        kvr.packed_kv_decode_attention(q, k3, v3)


def test_value_metadata_in_padded_rows(kvr):
    """Value scale/offset rows padded to a multiple of 8 tokens (a capacity
    buffer) with a ragged sequence end: whole 8-token pieces travel with the
    chunk's copies, the tail is read directly, and the NaN padding past the
    sequence must not reach the output."""
    import dataclasses

    S, cap = 1001, 1008
    k, v, q = make((2, 2, S, 128), 12, 4, 4, 32, 128, seed=17)
    pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=128)

    def padded(t):
        shape = list(t.shape)
        shape[2] = cap
        buf = torch.full(shape, float("nan"), dtype=t.dtype, device=t.device)
        buf[:, :, :S] = t
        return buf[:, :, :S]

    pv_cap = dataclasses.replace(pv, scale=padded(pv.scale), offset=padded(pv.offset))
    ref = oracle_out(k, v, q, 4, 4, 32, 128)
    for split in (0, 64):
        dense = kvr.packed_kv_decode_attention(q, pk, pv, split_tokens=split, out_dtype=F32)
        strided = kvr.packed_kv_decode_attention(q, pk, pv_cap, split_tokens=split, out_dtype=F32)
        check(strided, ref, f"padded value metadata split={split}")
        assert torch.equal(dense, strided)



def test_packed_decoder_equals_per_layer_calls(kvr):
    """PackedDecoder (planned once, stacked queries) == packed_kv_decode_attention
    per layer, bit for bit; moving the query/output buffers re-points the launch."""
    from kv_reduce_b200 import workloads

    wl = workloads.CONFIGS["2"].scaled(seq_len=2100, layers=35)   # > 32 layers: two launches
    ks, vs, qs = [], [], []
    for layer in range(wl.layers):
        k, v = workloads.make_layer_kv(wl, layer)
        pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=128)
        ks.append(pk)
        vs.append(pv)
        qs.append(workloads.make_query(wl, layer))
    # a fixed split makes the merge order, hence the rounding, independent of
    # how many layers share a launch (the default plan depends on it)
    dec = kvr.PackedDecoder(ks, vs, q_heads=wl.q_heads, split_tokens=512)
    q_all = torch.stack(qs)
    out = dec(q_all)
    for i in range(wl.layers):
        assert torch.equal(out[i], kvr.packed_kv_decode_attention(qs[i], ks[i], vs[i], split_tokens=512))
    q_moved = q_all.clone()
    out2 = torch.empty_like(out)
    assert dec(q_moved, out=out2) is out2
    assert torch.equal(out2, out)
    outs = kvr.packed_kv_decode_attention_layers(qs, ks, vs, split_tokens=512, out=torch.empty_like(out))
    for i in range(wl.layers):
        assert torch.equal(outs[i], out[i])
    dec32 = kvr.PackedDecoder(ks[:3], vs[:3], q_heads=wl.q_heads, out_dtype=F32)
    ref = oracle_out(*workloads.make_layer_kv(wl, 1), qs[1], 4, 4, 32, 128)
    check(dec32(q_all[:3])[1], ref, "decoder fp32")
    with pytest.raises(ValueError):
        dec(q_all[:, :, :6].contiguous())
    with pytest.raises(ValueError):
        dec(q_all.float())


@pytest.mark.parametrize("layers,out_dtype", [(3, torch.bfloat16), (35, torch.float32)])
def test_packed_decoder_host_step(kvr, layers, out_dtype):
    """PackedDecoder.host_step (pinned host queries in, pinned host outputs
    out; the first call eager, later calls a replayed CUDA graph of the query
    copy and the decode, whose merge writes the outputs into the pinned
    buffer directly) == the device-buffer call, bit for bit, across steps
    with new query values written into the same host buffer; 35 layers take
    two launches per step."""
    from kv_reduce_b200 import workloads

    wl = workloads.CONFIGS["2"].scaled(seq_len=2100, layers=layers)
    ks, vs = [], []
    for layer in range(wl.layers):
        k, v = workloads.make_layer_kv(wl, layer)
        pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=128)
        ks.append(pk)
        vs.append(pv)
    dec = kvr.PackedDecoder(ks, vs, q_heads=wl.q_heads, out_dtype=out_dtype)
    q_host = torch.empty(dec.q_shape, dtype=torch.bfloat16).pin_memory()
    o_host = torch.empty(dec.q_shape, dtype=out_dtype).pin_memory()
    for step in range(3):
        q = torch.stack([workloads.make_query(wl, layer, step=step) for layer in range(wl.layers)])
        q_host.copy_(q.cpu())
        assert dec.host_step(q_host, o_host) is o_host
        assert torch.equal(o_host, dec(q).cpu()), f"step {step}"
    assert dec._host["zero_copy"]   # pinned memory is device-addressable here
    with pytest.raises(ValueError):
        dec.host_step(torch.empty(dec.q_shape, dtype=torch.bfloat16), o_host)


@pytest.mark.parametrize("split_tokens", [0, 128])
def test_host_mapped_queries(kvr, split_tokens):
    """Queries in pinned host memory, read by the decode in place
    (kvr_decode_args.query_host_mapped): with the automatic plan the launch
    runs in clusters and only rank 0 of each cluster reads the query (the
    others copy its staged words over distributed shared memory); with
    128-token splits (32 splits, no clusters) every split reads it.  Both
    are bit-identical to the decode of the same queries in device memory.
    host_step reads mapped queries in place when its launches are clustered."""
    from kv_reduce_b200 import workloads
    from kv_reduce_b200.packed_kv_attention import DecodeLaunch, _geometry, _layer_ptrs

    wl = workloads.CONFIGS["2"].scaled(seq_len=4096, layers=4)
    ks, vs, qs = [], [], []
    for layer in range(wl.layers):
        k, v = workloads.make_layer_kv(wl, layer)
        pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=128)
        ks.append(pk), vs.append(pv), qs.append(workloads.make_query(wl, layer))
    q_host = [q.cpu().pin_memory() for q in qs]
    dev = qs[0].device
    geom = _geometry(qs[0], ks[0], vs[0])
    o_dev = [torch.full_like(q, float("nan")) for q in qs]
    o_map = [torch.full_like(q, float("nan")) for q in qs]
    ref_l = DecodeLaunch(geom, [_layer_ptrs(q, o, k, v) for q, o, k, v in zip(qs, o_dev, ks, vs)], dev,
                         split_tokens=split_tokens)
    lps = [_layer_ptrs(q, o, k, v) for q, o, k, v in zip(qs, o_map, ks, vs)]
    for lp, qh in zip(lps, q_host):
        lp.query = qh.data_ptr()
    map_l = DecodeLaunch(geom, lps, dev, split_tokens=split_tokens)
    map_l.args.query_host_mapped = 1
    ref_l()
    map_l()
    torch.cuda.synchronize()
    assert (map_l.cluster > 1) == (split_tokens == 0), (map_l.cluster, map_l.num_splits)
    for a, b in zip(o_map, o_dev):
        assert torch.equal(a, b)
    if split_tokens == 0:
        dec = kvr.PackedDecoder(ks, vs, q_heads=wl.q_heads)
        qh = torch.stack(qs).cpu().pin_memory()
        oh = torch.empty_like(qh).pin_memory()
        for _ in range(2):
            dec.host_step(qh, oh)
        assert dec._host["queries_in_place"]
        assert torch.equal(oh, dec(torch.stack(qs)).cpu())


def test_cache_on_another_device_is_rejected(kvr):
    k, v, q = make((1, 2, 256, 128), 12, 4, 4, 32, 0, seed=2)
    pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=0)
    import dataclasses

    cpu_v = dataclasses.replace(pv, payload=pv.payload.cpu())
    with pytest.raises(ValueError):
        kvr.packed_kv_decode_attention(q, pk, cpu_v)
    with pytest.raises(ValueError):
        kvr.PackedDecoder([pk], [cpu_v], q_heads=12)


def _key_dlocal(kb, r, e):
    rpw = 2 * (8 // kb)
    return (r // rpw) * (32 // kb) + r % rpw + e * (16 // kb)


def scale_pairs_oracle(scale_bits, kb, D):
    """numpy restatement of the fp16 scale pair table: word t4*D/8 + r of a
    group = fp16 of the bf16 scales of channels t4*D/4 + dlocal(r, 0/1),
    low half first."""
    s = packing.bf16_to_f32(scale_bits.reshape(-1, D)).astype(np.float32)
    out = np.empty((s.shape[0], D // 2), dtype=np.uint32)
    for t4 in range(4):
        for r in range(D // 8):
            d0, d1 = t4 * D // 4 + _key_dlocal(kb, r, 0), t4 * D // 4 + _key_dlocal(kb, r, 1)
            lo = s[:, d0].astype(np.float16).view(np.uint16).astype(np.uint32)
            hi = s[:, d1].astype(np.float16).view(np.uint16).astype(np.uint32)
            out[:, t4 * D // 8 + r] = lo | (hi << 16)
    return out


@pytest.mark.parametrize("kb,D", [(4, 128), (2, 128), (8, 128), (4, 64), (8, 64)])
def test_scale_pair_table_layout(kvr, kb, D):
    """kvr_key_scale_pairs: every word equals the numpy restatement (fp16 of
    the bf16 scale, channels of the decode's register order), including
    scales below fp16's normal range."""
    k, v, q = make((2, 2, 640, D), 12, kb, 4, 32, 0, seed=kb + D)
    k[0, 0, :, 3] = 0            # constant channel: scale 1e-8/levels, a flushed fp16
    k[1, 1, :, 5] *= 1e-4        # scales in fp16's subnormal range
    pk, _ = kvr.pack_kivi_kv(k, v, k_bits=kb, v_bits=4, group_size=32, residual_length=0)
    got = pk.scale_pairs.contiguous().cpu().numpy().view(np.uint16).reshape(-1, D).view(np.uint32)
    want = scale_pairs_oracle(bits_of(pk.scale), kb, D)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("kb,vb,D,hq", [(4, 4, 128, 12), (2, 2, 128, 12), (8, 4, 64, 32), (4, 8, 64, 32)])
def test_scale_pair_table_is_bit_identical(kvr, kb, vb, D, hq):
    """The decode with the pair table equals the decode converting the bf16
    scales per chunk, bit for bit (full and ragged chunks, residual window)."""
    import dataclasses

    k, v, q = make((2, hq // 6 if D == 128 else 8, 3001, D), hq, kb, vb, 32, 128, seed=11 + kb + vb)
    pk, pv = kvr.pack_kivi_kv(k, v, k_bits=kb, v_bits=vb, group_size=32, residual_length=128)
    assert pk.scale_pairs is not None
    bare = dataclasses.replace(pk, scale_pairs=None)
    for split in (0, 256):
        a = kvr.packed_kv_decode_attention(q, pk, pv, split_tokens=split, out_dtype=F32)
        b = kvr.packed_kv_decode_attention(q, bare, pv, split_tokens=split, out_dtype=F32)
        assert torch.equal(a, b), f"split {split}"


def test_single_split_full_length(kvr):
    """The longest accumulation a launch can make: one 32K-token layer in a
    single split (each warp sums 255 chunks into its tensor-core
    accumulators), still within the tolerance."""
    from kv_reduce_b200 import workloads

    wl = workloads.CONFIGS["2"]
    k, v = workloads.make_layer_kv(wl, 5)
    q = workloads.make_query(wl, 5)
    pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=128)
    out = kvr.packed_kv_decode_attention(q, pk, pv, split_tokens=1 << 20, out_dtype=F32)
    err = check(out, oracle_out(k, v, q, 4, 4, 32, 128), "32K one split")
    print(f"one split at 32K: max {err.max():.2e} mean {err.mean():.2e}")


def test_large_query_is_scaled_exactly(kvr):
    """Queries far beyond fp16's range (|q| ~ 1e5, about 2^17) are scaled by an
    exact power of two before they meet the tensor cores: the result matches
    the oracle, and no output is flagged non-finite."""
    k, v, q = make((1, 2, 1500, 128), 12, 4, 4, 32, 128, seed=41)
    q = (q.float() * 1e5).to(torch.bfloat16)
    pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=128)
    kvr.check_finite_outputs(clear=True)
    out = kvr.packed_kv_decode_attention(q, pk, pv, out_dtype=F32)
    check(out, oracle_out(k, v, q, 4, 4, 32, 128), "|q| ~ 1e5")
    kvr.check_finite_outputs()


def test_outlier_key_channels_x1000(kvr):
    """Key channels scaled x1000 (group ranges in the thousands): the per-group
    scales stay inside fp16, the result matches the oracle."""
    k, v, q = make((1, 2, 2048, 128), 12, 4, 4, 32, 128, seed=43, outliers=0)
    chans = torch.randperm(128, generator=torch.Generator().manual_seed(43))[:4].cuda()
    k = k.float()
    k[..., chans] *= 1000.0
    k = k.to(torch.bfloat16)
    pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=128)
    out = kvr.packed_kv_decode_attention(q, pk, pv, out_dtype=F32)
    check(out, oracle_out(k, v, q, 4, 4, 32, 128), "outliers x1000")
    kvr.check_finite_outputs()


def test_key_scale_beyond_fp16_is_flagged(kvr):
    """A key channel with a range of about 1e7 has a 4-bit scale above fp16's
    largest value: the decode cannot represent it, and instead of a silent
    inf/NaN the overflow is reported by check_finite_outputs."""
    k, v, q = make((1, 2, 1024, 128), 12, 4, 4, 32, 0, seed=47)
    k = k.float()
    k[..., 7] *= 3e6
    k = k.to(torch.bfloat16)
    pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=0)
    kvr.check_finite_outputs(clear=True)
    kvr.packed_kv_decode_attention(q, pk, pv, out_dtype=F32)
    with pytest.raises(FloatingPointError):
        kvr.check_finite_outputs()
    kvr.check_finite_outputs()   # the check cleared the flag
