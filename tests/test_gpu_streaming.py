"""Streaming cache: append / crop / commit keep the reference semantics
(kv_reduce/experiments/packed_review.py:17-98) on the preallocated layout."""
import numpy as np
import pytest
import torch

from conftest import bits_of
from oracle import attention, packing

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def kvr(built_lib):
    import kv_reduce_b200

    return kv_reduce_b200


def one_shot(keys, values, kb, vb, G, R):
    kq = packing.quantize_grouped(bits_of(keys), kb, G, R)
    vq = packing.quantize_per_token(bits_of(values), vb)
    return kq, vq


@pytest.mark.parametrize("residual", [0, 128])
def test_reference_unit_test_flow(kvr, residual):
    """packed_review.unit_test (:82-98): append x4, crop(1026), commit, attention;
    then 34 appends, crop(1057), commit."""
    g = torch.Generator(device="cuda").manual_seed(123 + residual)
    k = torch.randn(1, 2, 1024, 128, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(1, 2, 1024, 128, generator=g, device="cuda").to(torch.bfloat16)
    layer = kvr.PackedLayer(k, v, residual)
    original_prefix = layer.k.payload.clone()
    all_k, all_v = [k], [v]
    for _ in range(4):
        nk = torch.randn(1, 2, 1, 128, generator=g, device="cuda").to(torch.bfloat16)
        nv = torch.randn(1, 2, 1, 128, generator=g, device="cuda").to(torch.bfloat16)
        layer.append(nk, nv)
        all_k.append(nk)
        all_v.append(nv)
    layer.crop(1026)
    layer.commit()
    assert layer.get_seq_length() == 1026
    assert torch.equal(original_prefix, layer.k.payload[:, :, : original_prefix.shape[2]])
    K = torch.cat(all_k, dim=2)[:, :, :1026]
    V = torch.cat(all_v, dim=2)[:, :, :1026]
    kq, vq = one_shot(K, V, 4, 4, 32, residual)
    # incremental == one-shot, bit for bit (reference test_kivi_axis :58-82)
    assert layer.k.prefix_length == kq["P"]
    assert np.array_equal(layer.k.payload.cpu().numpy().reshape(-1), kq["payload"])
    assert np.array_equal(bits_of(layer.k.residual), kq["residual"])
    assert np.array_equal(layer.v.payload.cpu().numpy().reshape(-1), vq["payload"])
    q = torch.randn(1, 12, 1, 128, generator=g, device="cuda").to(torch.bfloat16)
    out = kvr.packed_kv_decode_attention(q, layer.k, layer.v, split_tokens=512, out_dtype=torch.float32)
    Kf = packing.dequant_grouped(kq["payload"], kq["scale"], kq["offset"], kq["residual"], 4, (1, 2, 1026, 128),
                                 kq["P"], 32)
    Vf = packing.dequant_per_token(vq["payload"], vq["scale"], vq["offset"], 4, (1, 2, 1026, 128))
    ref = attention.decode_attention(packing.bf16_to_f32(bits_of(q))[:, :, 0], Kf, Vf)
    err = np.abs(out.float().cpu().numpy()[:, :, 0] - ref)
    assert err.max() <= 2e-3 and err.mean() <= 1e-3
    # the reference's own check: kernel vs SDPA(unpack) at atol 5e-3 / rtol 5e-2
    expected = torch.nn.functional.scaled_dot_product_attention(
        q, layer.k.unpack().repeat_interleave(6, 1), layer.v.unpack().repeat_interleave(6, 1))
    out_bf16 = kvr.packed_kv_decode_attention(q, layer.k, layer.v, split_tokens=512)
    torch.testing.assert_close(out_bf16, expected, atol=5e-3, rtol=5e-2)
    for _ in range(34):
        layer.append(torch.randn(1, 2, 1, 128, generator=g, device="cuda").to(torch.bfloat16),
                     torch.randn(1, 2, 1, 128, generator=g, device="cuda").to(torch.bfloat16))
    layer.crop(1057)
    layer.commit()
    assert layer.k.prefix_length == ((1057 - residual) // 32) * 32


def test_draft_loop_matches_one_shot(kvr):
    """Config-5-style loop at small batch: prefill, rounds of 4 draft appends,
    rollback of the rejected tail, commit; state equals one-shot packing."""
    from kv_reduce_b200 import workloads

    wl = workloads.CONFIGS["5"].scaled(batch=3, seq_len=700)
    k, v = workloads.make_layer_kv(wl, 0)
    cache = kvr.PackedKVCacheLayer(3, 2, 128, k_bits=4, v_bits=4, group_size=32, residual_length=128, capacity=704)
    cache.prefill(k, v)
    keep_k, keep_v = [k], [v]
    g = torch.Generator(device="cuda").manual_seed(11)
    for rnd in range(12):
        start = cache.get_seq_length()
        drafted = []
        for step in range(4):
            nk = torch.randn(3, 2, 1, 128, generator=g, device="cuda").to(torch.bfloat16)
            nv = torch.randn(3, 2, 1, 128, generator=g, device="cuda").to(torch.bfloat16)
            cache.append(nk, nv)
            drafted.append((nk, nv))
            q = workloads.make_query(wl, 0, step=step, batch=3)
            cache.attention(q)
        accepted = rnd % 5   # 0..4 accepted, rest rolled back
        cache.crop(start + min(accepted, 4))
        for nk, nv in drafted[: min(accepted, 4)]:
            keep_k.append(nk)
            keep_v.append(nv)
        cache.commit()
    K, V = torch.cat(keep_k, 2), torch.cat(keep_v, 2)
    assert cache.get_seq_length() == K.shape[2]
    assert cache.capacity > 704   # grew by reallocation on the way
    kq, vq = one_shot(K, V, 4, 4, 32, 128)
    assert cache.prefix_len == kq["P"]
    assert np.array_equal(cache.k.payload.cpu().numpy().reshape(-1), kq["payload"])
    assert np.array_equal(bits_of(cache.k.scale).reshape(-1), kq["scale"].reshape(-1))
    # the decode's scale pair table, kept through prefill, commits and growth,
    # equals the table of a one-shot pack
    one = kvr.key_scale_pairs(cache.k.scale.contiguous(), 4)
    assert torch.equal(cache.k.scale_pairs, one)
    assert np.array_equal(bits_of(cache.k.residual), kq["residual"])
    assert np.array_equal(cache.v.payload.cpu().numpy().reshape(-1), vq["payload"])
    assert np.array_equal(bits_of(cache.v.scale).reshape(-1), vq["scale"].reshape(-1))
    q = workloads.make_query(wl, 0, step=9, batch=3)
    out = cache.attention(q, out_dtype=torch.float32)
    Kf = packing.dequant_grouped(kq["payload"], kq["scale"], kq["offset"], kq["residual"], 4, tuple(K.shape),
                                 kq["P"], 32)
    Vf = packing.dequant_per_token(vq["payload"], vq["scale"], vq["offset"], 4, tuple(V.shape))
    ref = attention.decode_attention(packing.bf16_to_f32(bits_of(q))[:, :, 0], Kf, Vf)
    err = np.abs(out.float().cpu().numpy()[:, :, 0] - ref)
    assert err.max() <= 2e-3 and err.mean() <= 1e-3
    bd = cache.breakdown()
    assert bd["k_payload"] == kq["payload"].size and bd["key_residual"] == kq["residual"].size * 2


def test_crop_bounds(kvr):
    k = torch.randn(1, 2, 200, 128, device="cuda").to(torch.bfloat16)
    layer = kvr.PackedLayer(k, k.clone(), 128)
    with pytest.raises(ValueError):
        layer.crop(layer.k.prefix_length - 1)
    with pytest.raises(ValueError):
        layer.crop(201)
