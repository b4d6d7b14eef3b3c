"""Graph-replayable draft loop (device-side lengths): a CUDA-graph replay of
append + decode steps equals the same launches issued eagerly bit for bit,
and matches the host-length path (PackedKVCacheLayer.append +
packed_kv_decode_attention per layer and step) within bf16 rounding, across
rounds separated by crop (rollback) and commit."""
import pytest
import torch

pytestmark = pytest.mark.gpu

B, H, HQ, D, L, S0 = 2, 2, 12, 128, 3, 700


@pytest.fixture(scope="module")
def kvr(built_lib):
    import kv_reduce_b200

    return kv_reduce_b200


def make_cache(kvr, seed=0, capacity=1024):
    g = torch.Generator(device="cuda").manual_seed(seed)
    cache = kvr.PackedKVCache(L, B, H, D, k_bits=4, v_bits=4, group_size=32, residual_length=128,
                              capacity=capacity, device="cuda")
    for layer in cache.layers:
        k = torch.randn(B, H, S0, D, generator=g, device="cuda").to(torch.bfloat16)
        v = torch.randn(B, H, S0, D, generator=g, device="cuda").to(torch.bfloat16)
        layer.prefill(k, v)
    return cache


def fill(loop, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    for t in (loop.q, loop.k, loop.v):
        t.copy_(torch.randn(t.shape, generator=g, device="cuda").to(torch.bfloat16))


def host_steps(kvr, cache, loop):
    outs = torch.empty_like(loop.out)
    for t in range(loop.steps):
        for li, layer in enumerate(cache.layers):
            layer.append(loop.k[t, li], loop.v[t, li])
            outs[t, li] = kvr.packed_kv_decode_attention(loop.q[t, li], layer.k, layer.v)
    return outs


def same_cache(a, b):
    for la, lb in zip(a.layers, b.layers):
        assert (la.seq_len, la.prefix_len) == (lb.seq_len, lb.prefix_len)
        S, P = la.seq_len, la.prefix_len
        assert torch.equal(la.value_payload[:, :, :S], lb.value_payload[:, :, :S])
        assert torch.equal(la.value_scale[:, :, :S], lb.value_scale[:, :, :S])
        assert torch.equal(la.value_offset[:, :, :S], lb.value_offset[:, :, :S])
        assert torch.equal(la.key_payload[:, :, :P], lb.key_payload[:, :, :P])
        assert torch.equal(la.k.residual, lb.k.residual)
        assert torch.equal(la.device_lengths()[:2].cpu(), torch.tensor([S, P], dtype=torch.int32))


def close(a, b):
    a, b = a.float(), b.float()
    assert torch.all((a - b).abs() <= 2e-3 + b.abs() * 2.0 ** -7)


def test_graph_replay_matches_eager_and_host_path(kvr):
    from kv_reduce_b200.draft import DraftLoop

    graph_cache, eager_cache, host_cache = make_cache(kvr), make_cache(kvr), make_cache(kvr)
    graph_loop = DraftLoop(graph_cache, q_heads=HQ, steps=4)
    eager_loop = DraftLoop(eager_cache, q_heads=HQ, steps=4)
    for rnd in range(3):
        fill(graph_loop, 10 + rnd)
        fill(eager_loop, 10 + rnd)
        got = graph_loop.replay().clone()
        assert torch.equal(got, eager_loop.run_eager())
        close(got, host_steps(kvr, host_cache, graph_loop))
        same_cache(graph_cache, host_cache)
        same_cache(graph_cache, eager_cache)
        # speculative rollback of two tokens, then promote full key groups
        for cache in (graph_cache, eager_cache, host_cache):
            cache.crop(cache.get_seq_length() - 2)
            cache.commit()
        same_cache(graph_cache, host_cache)
    assert graph_loop.errors() == 0


def test_capacity_is_checked_before_replay(kvr):
    from kv_reduce_b200.draft import DraftLoop

    cache = make_cache(kvr, capacity=704)      # 4 free value rows
    loop = DraftLoop(cache, q_heads=HQ, steps=8)
    with pytest.raises(ValueError):
        loop.replay()
    assert loop.errors() == 0


def test_decode_step_matches_append_then_attention(kvr):
    """PackedKVCacheLayer.decode_step (one token: one decode launch that
    appends it, lengths in device memory) == append +
    packed_kv_decode_attention: same cache bytes,
    outputs within bf16 rounding; across a commit and a capacity growth."""
    a_cache, b_cache = make_cache(kvr, seed=3, capacity=768), make_cache(kvr, seed=3, capacity=768)
    g = torch.Generator(device="cuda").manual_seed(21)
    for step in range(90):   # 700 + 90 > 768: the buffers grow on the way
        for la, lb in zip(a_cache.layers, b_cache.layers):
            q = torch.randn(B, HQ, 1, D, generator=g, device="cuda").to(torch.bfloat16)
            k = torch.randn(B, H, 1, D, generator=g, device="cuda").to(torch.bfloat16)
            v = torch.randn(B, H, 1, D, generator=g, device="cuda").to(torch.bfloat16)
            got = la.decode_step(q, k, v)
            lb.append(k, v)
            close(got, kvr.packed_kv_decode_attention(q, lb.k, lb.v))
        if step % 40 == 39:
            a_cache.commit()
            b_cache.commit()
    same_cache(a_cache, b_cache)
    with pytest.raises(ValueError):
        a_cache.layers[0].decode_step(q[:, :, :, :64], k, v)


def test_decode_step_two_tokens_and_capacity_flag(kvr):
    """decode_step with two new tokens (an append launch and a decode launch)
    == append + attention, cache bytes equal; and kvr_decode_step with the
    sequence already at capacity sets the error flag, leaves the lengths
    where they were and appends nothing."""
    from kv_reduce_b200 import _lib

    a_cache, b_cache = make_cache(kvr, seed=5), make_cache(kvr, seed=5)
    g = torch.Generator(device="cuda").manual_seed(8)
    la, lb = a_cache.layers[0], b_cache.layers[0]
    q = torch.randn(B, HQ, 1, D, generator=g, device="cuda").to(torch.bfloat16)
    k2 = torch.randn(B, H, 2, D, generator=g, device="cuda").to(torch.bfloat16)
    v2 = torch.randn(B, H, 2, D, generator=g, device="cuda").to(torch.bfloat16)
    got = la.decode_step(q, k2, v2)
    lb.append(k2, v2)
    close(got, kvr.packed_kv_decode_attention(q, lb.k, lb.v))
    same_cache(a_cache, b_cache)

    layer = a_cache.layers[1]
    k1, v1 = k2[:, :, :1].contiguous(), v2[:, :, :1].contiguous()
    out = torch.empty_like(q)
    stream = _lib.stream_ptr(q.device)
    _, launch = layer._prepare_step(HQ, 0, stream, q, out)
    dl = layer.device_lengths()
    dl[0] = layer.capacity                  # no room for one more token
    payload_before = layer.value_payload.clone()
    _lib.check("kvr_decode_step", _lib.load().kvr_decode_step(launch.args, k1.data_ptr(), v1.data_ptr(),
                                                              dl.data_ptr(), layer.cap_residual, stream))
    torch.cuda.synchronize()
    assert int(dl[2]) == 1 and int(dl[0]) == layer.capacity and int(dl[3]) == 0
    assert torch.equal(layer.value_payload, payload_before)
