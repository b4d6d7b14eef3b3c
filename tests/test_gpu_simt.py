"""The CUDA-core decode engine (kvr_decode_attention_simt, the measured A/B
baseline for the tensor-core kernel) against the oracle, within the same
tolerance as the tensor-core kernel (max |err| <= 2e-3, mean <= 1e-3 of
the fp32 result), on every geometry it supports."""
import pytest
import torch

from test_gpu_decode import check, make, oracle_out

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def kvr(built_lib):
    import kv_reduce_b200

    return kv_reduce_b200


@pytest.mark.parametrize("shape,hq,kb,vb", [
    ((1, 2, 1000, 128), 12, 4, 4),
    ((2, 2, 700, 128), 12, 2, 2),
    ((1, 8, 900, 128), 32, 4, 4),
    ((2, 8, 600, 64), 32, 8, 4),
    ((1, 8, 800, 64), 32, 4, 8),
])
@pytest.mark.parametrize("split", [0, 64])
def test_simt_matches_oracle(kvr, shape, hq, kb, vb, split):
    k, v, q = make(shape, hq, kb, vb, 32, 128, seed=shape[2] + kb)
    pk, pv = kvr.pack_kivi_kv(k, v, k_bits=kb, v_bits=vb, group_size=32, residual_length=128)
    out = kvr.packed_kv_decode_attention_simt(q, pk, pv, split_tokens=split, out_dtype=torch.float32)
    check(out, oracle_out(k, v, q, kb, vb, 32, 128), f"simt {shape} K{kb}V{vb} split {split}")
    tensor = kvr.packed_kv_decode_attention(q, pk, pv, split_tokens=split, out_dtype=torch.float32)
    assert (out - tensor).abs().max().item() <= 2e-3


def test_simt_rejects_unsupported_geometry(kvr):
    k, v, q = make((1, 2, 300, 128), 12, 8, 8, 32, 128, seed=5)
    pk, pv = kvr.pack_kivi_kv(k, v, k_bits=8, v_bits=8, group_size=32, residual_length=128)
    with pytest.raises(ValueError):
        kvr.packed_kv_decode_attention_simt(q, pk, pv)
