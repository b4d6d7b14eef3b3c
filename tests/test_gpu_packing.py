"""GPU parity of quantize + pack + unpack: bit-exact against the reference's
golden vectors and against the oracle on larger seeded inputs."""
import hashlib

import numpy as np
import pytest
import torch

from conftest import bf16_from_bits, bits_of
from oracle import packing

pytestmark = pytest.mark.gpu


def sha(a: np.ndarray) -> np.ndarray:
    return np.frombuffer(hashlib.sha256(np.ascontiguousarray(a).tobytes()).digest(), dtype=np.uint8)


@pytest.fixture(scope="module")
def kvr(built_lib):
    import kv_reduce_b200

    return kv_reduce_b200


@pytest.mark.parametrize("bits", range(1, 9))
@pytest.mark.parametrize("case", ["ar37", "rnd1001"])
def test_pack_unsigned_golden(kvr, golden, bits, case):
    codes = torch.from_numpy(golden[f"u_{case}_b{bits}_codes"]).cuda()
    payload = kvr.pack_unsigned(codes, bits)
    assert np.array_equal(payload.cpu().numpy(), golden[f"u_{case}_b{bits}_payload"])
    back = kvr.unpack_unsigned(payload, bits, codes.numel())
    assert torch.equal(back, codes)


def test_pack_unsigned_errors(kvr):
    with pytest.raises(ValueError):
        kvr.pack_unsigned(torch.tensor([0, 16], dtype=torch.uint8, device="cuda"), 4)
    with pytest.raises(ValueError):
        kvr.unpack_unsigned(torch.zeros(3, dtype=torch.uint8, device="cuda"), 4, 7)
    assert kvr.pack_unsigned(torch.zeros(0, dtype=torch.uint8, device="cuda"), 3).numel() == 0


def test_per_token_linspace_golden(kvr, golden):
    """Reference test_per_token_affine_uses_actual_packed_storage input (D=7: flat stream path)."""
    x = bf16_from_bits(golden["tok_linspace_x"])
    c = kvr.pack_per_token_affine(x, 4)
    assert np.array_equal(c.payload.cpu().numpy(), golden["tok_linspace_payload"])
    assert np.array_equal(bits_of(c.scale), golden["tok_linspace_scale"])
    assert np.array_equal(bits_of(c.offset), golden["tok_linspace_offset"])
    assert np.array_equal(bits_of(c.unpack()), golden["tok_linspace_unpack"])
    assert c.payload.numel() == kvr.packed_num_bytes(x.numel(), 4)
    assert c.storage_bytes < x.numel() * x.element_size()


def test_grouped_seed7_golden(kvr, golden):
    """Reference test_grouped_keys_preserve_residual_tail_exactly input (3-bit, G=4, R=3)."""
    x = bf16_from_bits(golden["grp_seed7_x"])
    c = kvr.pack_per_channel_grouped_affine(x, 3, group_size=4, residual_length=3)
    assert c.prefix_length == 8
    assert np.array_equal(c.payload.cpu().numpy(), golden["grp_seed7_payload"])
    assert np.array_equal(bits_of(c.scale), golden["grp_seed7_scale"])
    assert np.array_equal(bits_of(c.offset), golden["grp_seed7_offset"])
    assert np.array_equal(bits_of(c.residual), golden["grp_seed7_residual"])
    restored = c.unpack()
    assert np.array_equal(bits_of(restored), golden["grp_seed7_unpack"])
    assert torch.equal(restored[..., 8:, :], x[..., 8:, :])


def test_kv_cases_golden(kvr, golden):
    for name in (str(c) for c in golden["kv_cases"]):
        p = f"kv_{name}_"
        kb, vb, G, R, P = (int(v) for v in golden[p + "params"])
        keys, values = bf16_from_bits(golden[p + "keys"]), bf16_from_bits(golden[p + "values"])
        pk, pv = kvr.pack_kivi_kv(keys, values, k_bits=kb, v_bits=vb, group_size=G, residual_length=R)
        assert pk.prefix_length == P
        assert np.array_equal(pk.payload.cpu().numpy(), golden[p + "k_payload"]), name
        assert np.array_equal(bits_of(pk.scale), golden[p + "k_scale"]), name
        assert np.array_equal(bits_of(pk.offset), golden[p + "k_offset"]), name
        assert np.array_equal(bits_of(pk.residual), golden[p + "k_residual"]), name
        assert np.array_equal(pv.payload.cpu().numpy(), golden[p + "v_payload"]), name
        assert np.array_equal(bits_of(pv.scale), golden[p + "v_scale"]), name
        assert np.array_equal(bits_of(pv.offset), golden[p + "v_offset"]), name
        assert np.array_equal(sha(bits_of(pk.unpack())), golden[p + "k_unpack_bf16_sha256"]), name
        assert np.array_equal(sha(bits_of(pv.unpack())), golden[p + "v_unpack_bf16_sha256"]), name
        pk.output_dtype = torch.float32
        pv.output_dtype = torch.float32
        assert np.array_equal(sha(pk.unpack().cpu().numpy()), golden[p + "k_unpack_f32_sha256"]), name
        assert np.array_equal(sha(pv.unpack().cpu().numpy()), golden[p + "v_unpack_f32_sha256"]), name


@pytest.mark.parametrize("shape,kb,vb,G,R", [
    ((1, 2, 1024, 128), 4, 4, 32, 0),          # config 1
    ((3, 2, 1057, 128), 2, 8, 32, 128),        # ragged S, 2-bit keys
    ((2, 8, 333, 64), 8, 4, 16, 128),          # D=64, G=16
    ((1, 1, 31, 128), 4, 4, 32, 0),            # shorter than one group: empty prefix
    ((2, 3, 40, 40), 6, 5, 8, 3),              # odd widths, byte-aligned rows
    ((2, 2, 50, 20), 5, 3, 7, 1),              # rows not byte-aligned: flat stream path
])
def test_pack_matches_oracle(kvr, shape, kb, vb, G, R):
    g = torch.Generator(device="cuda").manual_seed(sum(shape) + kb * 10 + vb)
    keys = (torch.randn(shape, generator=g, device="cuda") * 3).to(torch.bfloat16)
    values = torch.randn(shape, generator=g, device="cuda").to(torch.bfloat16)
    keys[..., 0, :] = 0  # a constant token / channel edge: range clamps to 1e-8
    values[..., 1, :] = 1.5
    pk, pv = kvr.pack_kivi_kv(keys, values, k_bits=kb, v_bits=vb, group_size=G, residual_length=R)
    kq = packing.quantize_grouped(bits_of(keys), kb, G, R)
    vq = packing.quantize_per_token(bits_of(values), vb)
    assert pk.prefix_length == kq["P"]
    assert np.array_equal(pk.payload.cpu().numpy(), kq["payload"])
    assert np.array_equal(bits_of(pk.scale).reshape(-1), kq["scale"].reshape(-1))
    assert np.array_equal(bits_of(pk.offset).reshape(-1), kq["offset"].reshape(-1))
    assert np.array_equal(bits_of(pk.residual), kq["residual"])
    assert np.array_equal(pv.payload.cpu().numpy(), vq["payload"])
    assert np.array_equal(bits_of(pv.scale).reshape(-1), vq["scale"].reshape(-1))
    assert np.array_equal(bits_of(pv.offset).reshape(-1), vq["offset"].reshape(-1))
    K = packing.dequant_grouped(kq["payload"], kq["scale"], kq["offset"], kq["residual"], kb, shape, kq["P"], G)
    V = packing.dequant_per_token(vq["payload"], vq["scale"], vq["offset"], vb, shape)
    pk.output_dtype = torch.float32
    pv.output_dtype = torch.float32
    assert np.array_equal(pk.unpack().cpu().numpy(), K)
    assert np.array_equal(pv.unpack().cpu().numpy(), V)


def test_pack_full_size_layer_matches_oracle(kvr):
    """One full 32K-token layer of the Qwen2.5-1.5B-geometry cache, bit-exact."""
    from kv_reduce_b200 import workloads

    wl = workloads.CONFIGS["2"]
    keys, values = workloads.make_layer_kv(wl, 0)
    pk, pv = kvr.pack_kivi_kv(keys, values, k_bits=4, v_bits=4, group_size=32, residual_length=128)
    kq = packing.quantize_grouped(bits_of(keys), 4, 32, 128)
    vq = packing.quantize_per_token(bits_of(values), 4)
    assert pk.prefix_length == 32640
    assert np.array_equal(pk.payload.cpu().numpy(), kq["payload"])
    assert np.array_equal(bits_of(pk.scale).reshape(-1), kq["scale"].reshape(-1))
    assert np.array_equal(bits_of(pk.offset).reshape(-1), kq["offset"].reshape(-1))
    assert np.array_equal(pv.payload.cpu().numpy(), vq["payload"])
    assert np.array_equal(bits_of(pv.scale).reshape(-1), vq["scale"].reshape(-1))
    assert pk.storage_bytes + pv.storage_bytes == 9_744_384   # reference JSON per-layer packed bytes


def test_pack_rejects(kvr):
    x = torch.zeros(1, 2, 64, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        kvr.pack_per_token_affine(x, 1)
    with pytest.raises(ValueError):
        kvr.pack_per_channel_grouped_affine(x, 9)
    with pytest.raises(ValueError):
        kvr.pack_per_channel_grouped_affine(x, 4, group_size=0)
    with pytest.raises(ValueError):
        kvr.pack_per_token_affine(x.float(), 4)
    native = kvr.pack_per_token_affine(x, 16)
    assert native.layout == "native" and native.unpack().shape == x.shape
