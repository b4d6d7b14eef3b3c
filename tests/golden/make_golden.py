"""Generate golden vectors by running the reference's own packed_kv_cache.py.

Run where a checkout of the reference exists, giving its path:

    python tests/golden/make_golden.py <path of the KV_Reduce checkout>

It imports kv_reduce.packed_kv_cache from that checkout (read-only), runs it
on seeded bf16 inputs -- including the exact inputs of the reference's own
tests (tests/test_packed_kv_cache.py:17-66) -- and stores inputs and outputs
as bit patterns in golden_packing.npz.  For attention it stores the fp32
reference result: PackedKVComponent.unpack() with output_dtype=float32, then
torch scaled_dot_product_attention with enable_gqa, the comparison the
reference's own GPU check makes (kv_reduce/experiments/packed_review.py:93).
"""
from __future__ import annotations

import copy
import hashlib
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

OUT = Path(__file__).resolve().parent / "golden_packing.npz"


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def digest(a: np.ndarray) -> np.ndarray:
    """SHA-256 of the array's raw bytes (C order), as uint8[32]."""
    return np.frombuffer(hashlib.sha256(np.ascontiguousarray(a).tobytes()).digest(), dtype=np.uint8)


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from kv_reduce import packed_kv_cache as ref  # noqa: E402

    data: dict[str, np.ndarray] = {}
    cases: list[str] = []

    # --- pack_unsigned: the reference test's values and random streams
    for bits in range(1, 9):
        for name, vals in (("ar37", torch.arange(37, dtype=torch.int64).remainder(1 << bits).to(torch.uint8)),
                           ("rnd1001", torch.randint(0, 1 << bits, (1001,),
                                                     generator=torch.Generator().manual_seed(bits)).to(torch.uint8))):
            key = f"u_{name}_b{bits}"
            data[key + "_codes"] = vals.numpy()
            data[key + "_payload"] = ref.pack_unsigned(vals, bits).numpy()

    def add_kv_case(name: str, keys: torch.Tensor, values: torch.Tensor, kb: int, vb: int, G: int, R: int,
                    query: torch.Tensor | None, full: bool = False) -> None:
        pk, pv = ref.pack_kivi_kv(keys, values, k_bits=kb, v_bits=vb, group_size=G, residual_length=R)
        p = f"kv_{name}_"
        data[p + "keys"] = bits16(keys)
        data[p + "values"] = bits16(values)
        data[p + "params"] = np.array([kb, vb, G, R, pk.prefix_length], dtype=np.int64)
        data[p + "k_payload"] = pk.payload.numpy()
        data[p + "k_scale"] = bits16(pk.scale)
        data[p + "k_offset"] = bits16(pk.offset)
        data[p + "k_residual"] = bits16(pk.residual)
        data[p + "v_payload"] = pv.payload.numpy()
        data[p + "v_scale"] = bits16(pv.scale)
        data[p + "v_offset"] = bits16(pv.offset)
        k32, v32 = copy.copy(pk), copy.copy(pv)
        k32.output_dtype = torch.float32
        v32.output_dtype = torch.float32
        K, V = k32.unpack(), v32.unpack()
        outs = {"k_unpack_bf16": bits16(pk.unpack()), "v_unpack_bf16": bits16(pv.unpack()),
                "k_unpack_f32": K.numpy(), "v_unpack_f32": V.numpy()}
        for key, arr in outs.items():
            if full:
                data[p + key] = arr
            data[p + key + "_sha256"] = digest(arr)
        if query is not None:
            out = F.scaled_dot_product_attention(query.float(), K, V, enable_gqa=True)
            data[p + "query"] = bits16(query)
            data[p + "attn_f32"] = out.numpy()
        cases.append(name)

    # reference tests' exact inputs (tests/test_packed_kv_cache.py)
    lin = torch.linspace(-2.0, 3.0, 2 * 3 * 5 * 7).reshape(2, 3, 5, 7).to(torch.bfloat16)
    pv = ref.pack_per_token_affine(lin, bits=4)
    data["tok_linspace_x"] = bits16(lin)
    data["tok_linspace_payload"] = pv.payload.numpy()
    data["tok_linspace_scale"] = bits16(pv.scale)
    data["tok_linspace_offset"] = bits16(pv.offset)
    data["tok_linspace_unpack"] = bits16(pv.unpack())

    torch.manual_seed(7)
    k7 = torch.randn(1, 2, 11, 8, dtype=torch.bfloat16)
    pk = ref.pack_per_channel_grouped_affine(k7, bits=3, group_size=4, residual_length=3)
    data["grp_seed7_x"] = bits16(k7)
    data["grp_seed7_payload"] = pk.payload.numpy()
    data["grp_seed7_scale"] = bits16(pk.scale)
    data["grp_seed7_offset"] = bits16(pk.offset)
    data["grp_seed7_residual"] = bits16(pk.residual)
    data["grp_seed7_unpack"] = bits16(pk.unpack())
    data["grp_seed7_P"] = np.array([pk.prefix_length])

    g = torch.Generator().manual_seed(2024)
    kk = torch.randn(1, 2, 32, 16, generator=g, dtype=torch.bfloat16)
    vv = torch.randn(1, 2, 32, 16, generator=g, dtype=torch.bfloat16)
    add_kv_case("kivi_g8r8", kk, vv, 4, 4, 8, 8, None, full=True)

    # seeded draft-cache-like cases with outlier key channels
    def synth(shape, seed, outliers, scale):
        gg = torch.Generator().manual_seed(seed)
        k = torch.randn(shape, generator=gg)
        chans = torch.randperm(shape[-1], generator=gg)[:outliers]
        k[..., chans] *= scale
        v = torch.randn(shape, generator=gg)
        B, H, _, D = shape
        q = torch.randn((B, H * 6, 1, D), generator=gg)
        return k.to(torch.bfloat16), v.to(torch.bfloat16), q.to(torch.bfloat16)

    for kb, vb in ((4, 4), (2, 2), (8, 8), (8, 4), (4, 8), (2, 4), (3, 5)):
        k, v, q = synth((1, 2, 200, 128), 100 + 10 * kb + vb, 4, 10.0)
        add_kv_case(f"s200_k{kb}v{vb}", k, v, kb, vb, 32, 64, q if kb in (2, 4, 8) and vb in (2, 4, 8) else None)
    k, v, q = synth((2, 2, 96, 64), 555, 8, 8.0)
    q = q[:, :8]  # 4 query heads per KV head
    add_kv_case("d64_k4v8_r0", k, v, 4, 8, 32, 0, q, full=True)

    data["kv_cases"] = np.array(cases)
    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(cases)} kv cases)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <path of the KV_Reduce checkout>")
    main(sys.argv[1])
