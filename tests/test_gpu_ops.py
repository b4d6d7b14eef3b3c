"""torch.ops.kvr on the GPU: equal to the Python API, opcheck, and a
torch.compile trace through the operators (aot_eager: no generated kernels)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def kvr(built_lib):
    import kv_reduce_b200
    import kv_reduce_b200.ops  # noqa: F401

    return kv_reduce_b200


def _inputs(B=1, H=2, S=1057, D=128, HQ=12, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = torch.randn(B, H, S, D, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, H, S, D, generator=g, device="cuda").to(torch.bfloat16)
    q = torch.randn(B, HQ, 1, D, generator=g, device="cuda").to(torch.bfloat16)
    return k, v, q


def test_ops_equal_python_api(kvr):
    k, v, q = _inputs()
    pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=128)
    p, s, o, r = torch.ops.kvr.pack_grouped(k, 4, 32, 128)
    assert torch.equal(p, pk.payload) and torch.equal(s, pk.scale) and torch.equal(o, pk.offset)
    assert torch.equal(r, pk.residual)
    vp, vs, vo = torch.ops.kvr.pack_per_token(v, 4)
    assert torch.equal(vp, pv.payload) and torch.equal(vs, pv.scale) and torch.equal(vo, pv.offset)
    from kv_reduce_b200.ops import decode_attention_from

    out = decode_attention_from(q, pk, pv, split_tokens=512)
    assert torch.equal(out, kvr.packed_kv_decode_attention(q, pk, pv, split_tokens=512))


def test_opcheck(kvr):
    k, v, q = _inputs(S=700, seed=1)
    torch.library.opcheck(torch.ops.kvr.pack_grouped, (k, 4, 32, 128))
    torch.library.opcheck(torch.ops.kvr.pack_per_token, (v, 4))
    pk, pv = kvr.pack_kivi_kv(k, v, k_bits=4, v_bits=4, group_size=32, residual_length=128)
    args = (q, pk.payload, pk.scale, pk.offset, pk.residual, pv.payload, pv.scale, pv.offset, 700, 4, 4, 32,
            pk.prefix_length, 512)
    torch.library.opcheck(torch.ops.kvr.decode_attention, args)


def test_compile_traces_through_the_ops(kvr):
    k, v, q = _inputs(S=900, seed=2)

    def step(q, k, v):
        p, s, o, r = torch.ops.kvr.pack_grouped(k, 4, 32, 128)
        vp, vs, vo = torch.ops.kvr.pack_per_token(v, 4)
        out = torch.ops.kvr.decode_attention(q, p, s, o, r, vp, vs, vo, 900, 4, 4, 32, 768, 512)
        return out * 2

    compiled = torch.compile(step, backend="aot_eager", fullgraph=True)
    assert torch.equal(compiled(q, k, v), step(q, k, v))
