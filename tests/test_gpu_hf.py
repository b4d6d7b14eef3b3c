"""Draft-model integration (kv_reduce/experiments/packed_review.py:17-80) on a
small random-initialised Qwen2 model: the installed attention hook against
SDPA over the dequantized packed cache, a 40-step greedy decode with commits
against the same model on an unquantized cache, and streaming prefill (each
layer packed inside the prompt forward) against packing after the fact."""
import pytest
import torch

pytestmark = pytest.mark.gpu

transformers = pytest.importorskip("transformers")


def tiny_qwen2(seed=0):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    torch.manual_seed(seed)
    cfg = Qwen2Config(vocab_size=512, hidden_size=768, intermediate_size=1024, num_hidden_layers=2,
                      num_attention_heads=6, num_key_value_heads=2, max_position_embeddings=4096,
                      attn_implementation="sdpa")
    return Qwen2ForCausalLM(cfg).to(device="cuda", dtype=torch.bfloat16).eval()


@torch.inference_mode()
def test_installed_attention_matches_sdpa_over_dequantized_cache(built_lib):
    from kv_reduce_b200 import hf

    model = tiny_qwen2()
    prompt = torch.randint(0, 512, (1, 600), device="cuda", generator=torch.Generator("cuda").manual_seed(1))
    cache = model(prompt, use_cache=True).past_key_values
    packed = hf.PackedDraftCache(cache, residual=128)
    assert packed.get_seq_length() == 600
    hf.install(model)

    attn = model.model.layers[0].self_attn
    h = torch.randn(1, 1, 768, device="cuda", dtype=torch.bfloat16)
    pe = model.model.rotary_emb(h, torch.tensor([[600]], device="cuda"))
    got = attn(h, pe, None, past_key_values=packed)[0]
    assert packed.layers[0].get_seq_length() == 601

    view = (1, 1, -1, attn.head_dim)
    q = attn.q_proj(h).view(view).transpose(1, 2)
    k = attn.k_proj(h).view(view).transpose(1, 2)
    q, _ = hf.apply_rotary_pos_emb(q, k, *pe)
    layer = packed.layers[0].packed
    K = layer.k.unpack().float()
    V = layer.v.unpack().float()
    o = torch.nn.functional.scaled_dot_product_attention(q.float(), K, V, enable_gqa=True)
    want = attn.o_proj(o.to(torch.bfloat16).transpose(1, 2).reshape(1, 1, -1))
    rel = (got.float() - want.float()).norm() / want.float().norm()
    assert rel < 1e-2, f"relative error {rel:.3e}"


@torch.inference_mode()
def test_greedy_decode_with_commits_tracks_unquantized_model(built_lib):
    from transformers.cache_utils import DynamicCache

    from kv_reduce_b200 import hf

    model = tiny_qwen2(seed=3)
    prompt = torch.randint(0, 512, (1, 700), device="cuda", generator=torch.Generator("cuda").manual_seed(4))
    out = model(prompt, use_cache=True)
    ref_cache = out.past_key_values
    packed = hf.PackedDraftCache([(l.keys.clone(), l.values.clone()) for l in ref_cache.layers], residual=128)
    assert isinstance(ref_cache, DynamicCache)
    hf.install(model)
    token = out.logits[:, -1].argmax(-1, keepdim=True)
    p0 = packed.layers[0].packed.prefix_len
    for step in range(40):
        ref = model(token, past_key_values=ref_cache, use_cache=True).logits[:, -1].float()
        got = model(token, past_key_values=packed, use_cache=True).logits[:, -1].float()
        cos = torch.nn.functional.cosine_similarity(ref, got, dim=-1).item()
        assert cos > 0.98, f"step {step}: logits cosine {cos:.4f}"
        token = ref.argmax(-1, keepdim=True)
        if step % 8 == 7:
            packed.commit()
    layer = packed.layers[0].packed
    assert layer.get_seq_length() == 740
    assert layer.prefix_len > p0            # commits promoted key groups out of the residual window
    assert layer.seq_len - layer.prefix_len < 128 + 32 + 8
    assert set(packed.breakdown()) == {"k_payload", "v_payload", "k_scales", "v_scales", "k_offsets",
                                       "v_offsets", "key_residual"}


@torch.inference_mode()
def test_hook_leaves_other_caches_alone(built_lib):
    from kv_reduce_b200 import hf

    model = tiny_qwen2(seed=5)
    ids = torch.randint(0, 512, (1, 64), device="cuda", generator=torch.Generator("cuda").manual_seed(6))
    before = model(ids).logits
    hf.install(model)
    after = model(ids).logits
    assert torch.equal(before, after)
    packed = hf.PackedDraftCache(model(ids, use_cache=True).past_key_values, residual=0)
    with pytest.raises(ValueError):
        model(ids[:, :2], past_key_values=packed, use_cache=True)


@torch.inference_mode()
def test_streaming_prefill_packs_each_layer_bit_exact(built_lib):
    """An empty PackedDraftCache packs each layer inside the prompt forward:
    the prompt logits are the BF16 model's, the packed layers equal
    pack_kivi_kv of the BF16 cache bit for bit, and decoding continues
    through the hook exactly as from a cache packed after the fact."""
    import kv_reduce_b200 as kvr
    from kv_reduce_b200 import hf

    model = tiny_qwen2(seed=7)
    prompt = torch.randint(0, 512, (1, 777), device="cuda", generator=torch.Generator("cuda").manual_seed(8))
    ref = model(prompt, use_cache=True)
    hf.install(model)
    streamed = hf.PackedDraftCache.empty(num_layers=2, residual=128)
    out = model(prompt, past_key_values=streamed, use_cache=True)
    assert torch.equal(out.logits, ref.logits)
    after = hf.PackedDraftCache(ref.past_key_values, residual=128)
    for i, layer in enumerate(ref.past_key_values.layers):
        pk, pv = kvr.pack_kivi_kv(layer.keys, layer.values, k_bits=4, v_bits=4, group_size=32,
                                  residual_length=128)
        sk, sv = streamed.layers[i].packed.k, streamed.layers[i].packed.v
        assert sk.prefix_length == pk.prefix_length == 640
        assert torch.equal(sk.payload.reshape(-1), pk.payload.reshape(-1))
        assert torch.equal(sk.scale.reshape(-1), pk.scale.reshape(-1))
        assert torch.equal(sk.offset.reshape(-1), pk.offset.reshape(-1))
        assert torch.equal(sk.residual, pk.residual)
        assert torch.equal(sv.payload.reshape(-1), pv.payload.reshape(-1))
        assert torch.equal(sv.scale.reshape(-1), pv.scale.reshape(-1))
        assert torch.equal(sv.offset.reshape(-1), pv.offset.reshape(-1))
    token = ref.logits[:, -1].argmax(-1, keepdim=True)
    for _ in range(3):
        a = model(token, past_key_values=streamed, use_cache=True).logits
        b = model(token, past_key_values=after, use_cache=True).logits
        assert torch.equal(a, b)
        token = a[:, -1].argmax(-1, keepdim=True)
