"""torch.ops.kvr registration and fake (meta) shapes, without a GPU."""
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import kv_reduce_b200.ops  # noqa: F401  (registers torch.ops.kvr.*)
from kv_reduce_b200.packed_kv_cache import packed_num_bytes


def test_ops_registered():
    for name in ("pack_per_token", "pack_grouped", "decode_attention", "lse_merge"):
        assert hasattr(torch.ops.kvr, name)


def test_fake_shapes_follow_the_packing_rules():
    with FakeTensorMode():
        k = torch.empty(2, 2, 1000, 128, dtype=torch.bfloat16, device="cuda")
        p, s, o, r = torch.ops.kvr.pack_grouped(k, 4, 32, 128)
        prefix = 864                      # floor((1000 - 128) / 32) * 32
        assert p.shape == (packed_num_bytes(4 * prefix * 128, 4),) and p.dtype == torch.uint8
        assert s.shape == o.shape == (2, 2, prefix // 32, 1, 128) and s.dtype == torch.bfloat16
        assert r.shape == (2, 2, 1000 - prefix, 128) and r.dtype == torch.bfloat16
        p0, s0, o0, r0 = torch.ops.kvr.pack_grouped(k[:, :, :100], 2, 32, 128)
        assert p0.numel() == s0.numel() == o0.numel() == 0 and r0.shape == (2, 2, 100, 128)
        pv, sv, ov = torch.ops.kvr.pack_per_token(k, 2)
        assert pv.shape == (packed_num_bytes(k.numel(), 2),) and sv.shape == ov.shape == (2, 2, 1000, 1)
        q = torch.empty(2, 12, 1, 128, dtype=torch.bfloat16, device="cuda")
        out = torch.ops.kvr.decode_attention(q, p, s, o, r, pv, sv, ov, 1000, 4, 2, 32, prefix, 0)
        assert out.shape == q.shape and out.dtype == q.dtype
        m = torch.ops.kvr.lse_merge(torch.empty(3, 24, 2, device="cuda"), torch.empty(3, 24, 128, device="cuda"))
        assert m.shape == (24, 128) and m.dtype == torch.bfloat16
