"""CompressedAttentionKVCache: decode attention over compressed chunks + the
lazily encoded tail, against float64 attention over the same dequantised K/V
(the chunks decoded in fp32 by the CUDA codec, which the codec tests pin to
the oracle), and a tiny random Llama driven through the transformers hook against
the reference-semantics cache (materialised buffer).  Tolerance: attention
1e-3 of the row's max |o|; logits 2e-2 of the step's max |logit| (the hook
reads chunks with the fp16 scale, the materialised buffer holds the fp32-scale
values, as the reference's two paths do)."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref_attention(q, k, v, scaling):
    B, Hq, _, D = q.shape
    H = k.shape[1]
    qg = q.double().view(B, H, Hq // H, D)
    s = torch.einsum("bhgd,bhsd->bhgs", qg, k.double()) * scaling
    p = torch.softmax(s, -1)
    return torch.einsum("bhgs,bhsd->bhgd", p, v.double()).reshape(B, Hq, 1, D)


@pytest.mark.parametrize("D,S0,steps", [(128, 128, 70), (64, 256, 133)])
def test_decode_attention_over_chunks_and_tail(D, S0, steps):
    from latticequant_b200.llm.compressed_attention import CompressedAttentionKVCache

    torch.manual_seed(0)
    B, H, G = 2, 2, 4
    cache = CompressedAttentionKVCache(4, tail_tokens=64)
    k = torch.randn(B, H, S0, D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, H, S0, D, device="cuda", dtype=torch.bfloat16)
    kd, vd = cache.update(k, v, 0)
    assert kd.shape == k.shape
    worst = 0.0
    for step in range(steps):
        kt = torch.randn(B, H, 1, D, device="cuda", dtype=torch.bfloat16)
        vt = torch.randn(B, H, 1, D, device="cuda", dtype=torch.bfloat16)
        cache.update(kt, vt, 0)
        q = torch.randn(B, H * G, 1, D, device="cuda", dtype=torch.float32) / math.sqrt(D)
        o = cache.decode_attention(0, q)
        kk, vv = cache._materialise(cache._state[0], torch.float32)
        ref = _ref_attention(q, kk, vv, 1 / math.sqrt(D))
        err = ((o.double() - ref).abs().amax(-1) / ref.abs().amax(-1)).max().item()
        worst = max(worst, err)
    assert cache.flags() == 0
    assert worst <= 1e-3, worst
    st = cache._state[0]
    assert st.seq == S0 + steps
    # flushed tails are stored encoded and attended from the layer's dense tail
    assert len(st.parts) == 1 and st.n_tail == steps % 64 and st.n_tail_dense == (steps // 64) * 64
    assert cache.get_seq_length(0) == S0 + steps
    # the tail chunks hold exactly the reference's per-token quantisation
    # resident: only the fixed-size tail buffers, vs. the reference's whole dequantised K/V
    ref_resident = 2 * B * H * (S0 + steps) * D * 2
    assert cache.compressed_bytes() > 0 and cache.decompressed_resident_bytes() < ref_resident


def test_tiny_llama_decode_through_hook():
    from transformers import LlamaConfig, LlamaForCausalLM

    from latticequant_b200.llm.compressed_attention import CompressedAttentionKVCache
    from latticequant_b200.llm.compressed_kv_cache import CompressedKVCache

    torch.manual_seed(1)
    cfg = LlamaConfig(vocab_size=512, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=1024)
    model = LlamaForCausalLM(cfg).to("cuda", torch.bfloat16).eval()
    ids = torch.randint(0, 512, (2, 128), device="cuda")
    steps = 70
    with torch.no_grad():
        # reference semantics: materialised dequantised buffer, SDPA
        ref_cache = CompressedKVCache(4)
        out = model(ids, past_key_values=ref_cache, use_cache=True)
        toks, ref_logits = [], []
        nxt = out.logits[:, -1].argmax(-1, keepdim=True)
        for _ in range(steps):
            toks.append(nxt)
            out = model(nxt, past_key_values=ref_cache, use_cache=True)
            ref_logits.append(out.logits[:, -1].float())
            nxt = out.logits[:, -1].argmax(-1, keepdim=True)
        # the hook: decode steps attend over the compressed cache (teacher-forced on the same tokens)
        cache = CompressedAttentionKVCache(4, tail_tokens=64).bind(model)
        out2 = model(ids, past_key_values=cache, use_cache=True)
        # prefill keeps the reference's semantics (SDPA over update()'s dequantised K/V)
        assert (out2.logits.float() - out.logits.float()).abs().max().item() >= 0  # ran
        worst = 0.0
        for t in range(steps):
            o = model(toks[t], past_key_values=cache, use_cache=True)
            lg = o.logits[:, -1].float()
            worst = max(worst, ((lg - ref_logits[t]).abs().amax() / ref_logits[t].abs().amax()).item())
    assert cache.flags() == 0
    assert cache.get_seq_length(0) == 128 + steps
    assert worst < 2e-2, worst


def test_tails_past_the_dense_limit_become_encoded_parts(monkeypatch):
    """rANS layout: flushed tails are attended from the dense tail buffer up to
    TAIL_MERGE_MAX tokens per layer and from per-token-scale parts (recoded
    together as they arrive) beyond it; the attention over all of them stays
    within the bar of float64 attention over the same dequantised tokens."""
    import latticequant_b200.llm.compressed_attention as CA

    monkeypatch.setattr(CA, "TAIL_MERGE_MAX", 32)
    torch.manual_seed(6)
    B, H, G, S0, D, T = 2, 2, 4, 128, 128, 16
    steps = 4 * T + 3
    cache = CA.CompressedAttentionKVCache(4, tail_tokens=T)
    cache.update(torch.randn(B, H, S0, D, device="cuda", dtype=torch.bfloat16),
                 torch.randn(B, H, S0, D, device="cuda", dtype=torch.bfloat16), 0)
    worst = 0.0
    for _ in range(steps):
        cache.update(torch.randn(B, H, 1, D, device="cuda", dtype=torch.bfloat16),
                     torch.randn(B, H, 1, D, device="cuda", dtype=torch.bfloat16), 0)
        q = torch.randn(B, H * G, 1, D, device="cuda", dtype=torch.float32) / math.sqrt(D)
        o = cache.decode_attention(0, q)
        kk, vv = cache._materialise(cache._state[0], torch.float32)
        ref = _ref_attention(q, kk, vv, 1 / math.sqrt(D))
        worst = max(worst, ((o.double() - ref).abs().amax(-1) / ref.abs().amax(-1)).max().item())
    st = cache._state[0]
    assert st.n_tail_dense == 2 * T and st.n_tail == 3
    tails = [p for p in st.parts if p.per_token]
    assert len(tails) == 1 and tails[0].shape == (B, H, 2 * T, D)
    assert cache.get_seq_length(0) == S0 + steps
    assert cache.flags() == 0
    assert worst <= 1e-3, worst


@pytest.mark.parametrize("bits", [4, 3])
def test_compact_layout_decode_attention(bits):
    """layout="compact": the prefill chunk in the compact fixed-rate layout
    (llm/fused_triton_merge.py's format) attended with lq_attn_decode_compact,
    decode tokens in the exact tail, flushed tails kept dequantised; against
    float64 attention over every token dequantised (the merged fp16 values of
    the compact chunk, the tail's fp32-scale values)."""
    from latticequant_b200.llm.compressed_attention import CompressedAttentionKVCache

    torch.manual_seed(4)
    B, H, G, S0, D, steps = 2, 2, 4, 256, 128, 70
    cache = CompressedAttentionKVCache(bits, tail_tokens=64, layout="compact")
    k = torch.randn(B, H, S0, D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, H, S0, D, device="cuda", dtype=torch.bfloat16)
    cache.update(k, v, 0)
    worst = 0.0
    for _ in range(steps):
        cache.update(torch.randn(B, H, 1, D, device="cuda", dtype=torch.bfloat16),
                     torch.randn(B, H, 1, D, device="cuda", dtype=torch.bfloat16), 0)
        q = torch.randn(B, H * G, 1, D, device="cuda", dtype=torch.float32) / math.sqrt(D)
        o = cache.decode_attention(0, q)
        kk, vv = cache._materialise(cache._state[0], torch.float32)
        ref = _ref_attention(q, kk, vv, 1 / math.sqrt(D))
        worst = max(worst, ((o.double() - ref).abs().amax(-1) / ref.abs().amax(-1)).max().item())
    assert cache.flags() == 0
    assert worst <= 1e-3, worst
    st = cache._state[0]
    assert len(st.parts) == 1 and st.parts[0].layout == "compact"
    # the flushed tail is kept dequantised in the layer's growing tail buffer
    assert not st.dense_k and st.n_tail_dense == 64 and st.n_tail == steps - 64
    assert cache.get_seq_length(0) == S0 + steps
    with pytest.raises(ValueError):
        from latticequant_b200 import serialize

        serialize.cache_state(cache)
