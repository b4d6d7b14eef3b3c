"""Pin the CPU oracle to the reference: every golden vector was produced by
running kv_reduce/packed_kv_cache.py itself (tests/golden/make_golden.py)."""
import hashlib

import numpy as np
import pytest
import torch

from oracle import attention, cpu_baseline, packing


def sha(a: np.ndarray) -> np.ndarray:
    return np.frombuffer(hashlib.sha256(np.ascontiguousarray(a).tobytes()).digest(), dtype=np.uint8)


@pytest.mark.parametrize("bits", range(1, 9))
@pytest.mark.parametrize("case", ["ar37", "rnd1001"])
def test_pack_unsigned_matches_reference(golden, bits, case):
    codes = golden[f"u_{case}_b{bits}_codes"]
    payload = packing.pack_unsigned(codes, bits)
    assert np.array_equal(payload, golden[f"u_{case}_b{bits}_payload"])
    assert payload.size == packing.packed_num_bytes(codes.size, bits)
    assert np.array_equal(packing.unpack_unsigned(payload, bits, codes.size), codes)


def test_per_token_linspace_matches_reference(golden):
    x = golden["tok_linspace_x"]
    q = packing.quantize_per_token(x, 4)
    assert np.array_equal(q["payload"], golden["tok_linspace_payload"])
    assert np.array_equal(q["scale"].reshape(-1), golden["tok_linspace_scale"].reshape(-1))
    assert np.array_equal(q["offset"].reshape(-1), golden["tok_linspace_offset"].reshape(-1))
    deq = packing.dequant_per_token(q["payload"], q["scale"], q["offset"], 4, x.shape)
    assert np.array_equal(packing.f32_to_bf16(deq), golden["tok_linspace_unpack"])


def test_grouped_seed7_matches_reference(golden):
    x = golden["grp_seed7_x"]
    q = packing.quantize_grouped(x, 3, 4, 3)
    assert q["P"] == int(golden["grp_seed7_P"][0]) == 8
    assert np.array_equal(q["payload"], golden["grp_seed7_payload"])
    assert np.array_equal(q["scale"].reshape(-1), golden["grp_seed7_scale"].reshape(-1))
    assert np.array_equal(q["offset"].reshape(-1), golden["grp_seed7_offset"].reshape(-1))
    assert np.array_equal(q["residual"], golden["grp_seed7_residual"])
    deq = packing.dequant_grouped(q["payload"], q["scale"], q["offset"], q["residual"], 3, x.shape, 8, 4)
    assert np.array_equal(packing.f32_to_bf16(deq), golden["grp_seed7_unpack"])


def kv_cases(golden):
    return [str(c) for c in golden["kv_cases"]]


def test_kv_cases_match_reference(golden):
    for name in kv_cases(golden):
        p = f"kv_{name}_"
        kb, vb, G, R, P = (int(v) for v in golden[p + "params"])
        keys, values = golden[p + "keys"], golden[p + "values"]
        kq = packing.quantize_grouped(keys, kb, G, R)
        vq = packing.quantize_per_token(values, vb)
        assert kq["P"] == P, name
        assert np.array_equal(kq["payload"], golden[p + "k_payload"]), name
        assert np.array_equal(kq["scale"].reshape(-1), golden[p + "k_scale"].reshape(-1)), name
        assert np.array_equal(kq["offset"].reshape(-1), golden[p + "k_offset"].reshape(-1)), name
        assert np.array_equal(kq["residual"], golden[p + "k_residual"]), name
        assert np.array_equal(vq["payload"], golden[p + "v_payload"]), name
        assert np.array_equal(vq["scale"].reshape(-1), golden[p + "v_scale"].reshape(-1)), name
        assert np.array_equal(vq["offset"].reshape(-1), golden[p + "v_offset"].reshape(-1)), name
        K = packing.dequant_grouped(kq["payload"], kq["scale"], kq["offset"], kq["residual"], kb, keys.shape, P, G)
        V = packing.dequant_per_token(vq["payload"], vq["scale"], vq["offset"], vb, values.shape)
        assert np.array_equal(sha(K), golden[p + "k_unpack_f32_sha256"]), name
        assert np.array_equal(sha(V), golden[p + "v_unpack_f32_sha256"]), name
        assert np.array_equal(sha(packing.f32_to_bf16(K)), golden[p + "k_unpack_bf16_sha256"]), name
        assert np.array_equal(sha(packing.f32_to_bf16(V)), golden[p + "v_unpack_bf16_sha256"]), name
        if p + "query" in golden.files:
            q = packing.bf16_to_f32(golden[p + "query"])[:, :, 0, :]
            out = attention.decode_attention(q, K, V)
            ref = golden[p + "attn_f32"][:, :, 0, :]
            np.testing.assert_allclose(out, ref, atol=2e-5, rtol=1e-4, err_msg=name)


def test_cpu_baseline_restatement_matches_reference(golden):
    """The timed CPU baseline computes what the reference's unfused path computes."""
    torch.set_num_threads(2)
    for name in ("s200_k4v4", "s200_k2v2", "d64_k4v8_r0"):
        p = f"kv_{name}_"
        kb, vb, G, R, P = (int(v) for v in golden[p + "params"])
        k, v = cpu_baseline.pack_cpu(golden[p + "keys"], golden[p + "values"], kb, vb, G, R)
        Kb, Vb = cpu_baseline.unpack_keys(k), cpu_baseline.unpack_values(v)
        as_bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
        assert np.array_equal(sha(as_bits(Kb)), golden[p + "k_unpack_bf16_sha256"]), name
        assert np.array_equal(sha(as_bits(Vb)), golden[p + "v_unpack_bf16_sha256"]), name
        qbits = golden[p + "query"]
        q = torch.from_numpy(qbits.view(np.int16)).view(torch.bfloat16)
        out = cpu_baseline.unfused_decode(q, k, v).float().numpy()
        np.testing.assert_allclose(out, golden[p + "attn_f32"], atol=3e-2, rtol=3e-2)


def test_prefix_rule_cases():
    assert packing.quantized_prefix_length(64, 16, 20) == 32          # reference test_kivi_axis :44-56
    assert packing.quantized_prefix_length(1024, 32, 128) == 896      # :116-162 byte model
    assert packing.quantized_prefix_length(32768, 32, 128) == 32640
    assert packing.quantized_prefix_length(100, 32, 128) == 0
    assert packing.quantized_prefix_length(1057, 32, 0) == 1056
    with pytest.raises(ValueError):
        packing.quantized_prefix_length(10, 0, 1)


def test_oracle_partial_merge_equals_full():
    rng = np.random.default_rng(3)
    q = rng.standard_normal((1, 12, 128))
    k = rng.standard_normal((1, 2, 640, 128))
    v = rng.standard_normal((1, 2, 640, 128))
    full = attention.decode_attention(q, k, v)
    parts = [attention.partials(q, k[:, :, a:b], v[:, :, a:b]) for a, b in ((0, 96), (96, 500), (500, 640))]
    M = np.max([m for m, _, _ in parts], axis=0)
    L = sum(l * np.exp2(m - M) for m, l, _ in parts)
    O = sum(o * np.exp2(m - M)[..., None] for m, _, o in parts)
    np.testing.assert_allclose(O / L[..., None], full, atol=1e-12)
