"""Parity of the CUDA path against the C oracle at BASELINE sizes and on the
API rows whose older tests compared the CUDA path with itself.

  * one full config-2 chunk (8 heads x 8192 tokens x 128, bf16, K with
    log-normal channel scales and an outlier channel) and the full config-1
    chunk (262,144 vectors x 128 fp32, a scale per vector): scales, coset
    words, tables, every lane's words / bit count / final state and the
    decoded values byte-identical to oracle.compress_chunk / decompress_chunk
    (llm/compressed_kv_cache.py:176-332 restated in oracle/);
  * VariableRateKVCache (allocation/eval_alloc.py:87-145) at per-layer 3/4/5
    bits: update()'s returned K/V and every chunk's decode bit-exact;
  * CompressedAttentionKVCache: every decode token's update() output and every
    per-token-scale tail chunk bit-exact against the oracle's quantisation of
    that one-token update (llm/compressed_kv_cache.py:183-204 with S = 1), and
    decode attention against float64 attention over the oracle's values;
  * the outlier side channel: the tokens left in the streams decode to the
    oracle's lattice points, the extracted records hold the oracle's symbols;
  * config 3 at full shape: 256 sampled (batch, query head) rows of the fused
    attention against float64 attention over the oracle's dequantisation.

Bars: bit-exact for integers, bytes and dequantised values; attention
max |o - o_ref| <= 1e-3 * max |o_ref| per query row.
"""
import math

import numpy as np
import pytest
import torch

from oracle import lq_oracle as O

pytestmark = pytest.mark.gpu

RTOL = 1e-3


def _bf16_bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _u32(t):
    return t.detach().cpu().contiguous().numpy().view(np.uint32)


def _compare_lane_chunk(ch, ref):
    """Every stored field of a LaneChunk against the oracle's chunk."""
    assert np.array_equal(_u32(ch.scale_f32), ref.scale_f32.view(np.uint32))
    assert np.array_equal(ch.scale_f16.cpu().numpy().view(np.uint16), ref.scale_f16)
    n = ref.n_vectors
    assert np.array_equal(ch.coset_words.cpu().numpy().view(np.uint8)[: (n + 7) // 8], ref.coset_packed)
    assert np.array_equal(ch.tab_lo.cpu().numpy(), ref.tab_lo)
    assert np.array_equal(ch.tab_nsym.cpu().numpy(), ref.tab_nsym)
    fr = ch.tab_freq.cpu().numpy().view(np.uint16).astype(np.int32)
    for s in range(16):
        assert np.array_equal(fr[s, : ref.tab_nsym[s]], ref.tab_freq[s, : ref.tab_nsym[s]]), s
    assert np.array_equal(ch.tile_n0.cpu().numpy().astype(np.uint32), ref.tile_n0)
    assert ch.n_words == ref.words.size
    assert np.array_equal(_u32(ch.lane_off), ref.lane_off)
    assert np.array_equal(_u32(ch.lane_nbits), ref.lane_nbits)
    assert np.array_equal(_u32(ch.lane_state), ref.lane_state)
    assert np.array_equal(_u32(ch.words[: ch.n_words]), ref.words)


def _config2_chunk(kind, seed):
    g = torch.Generator().manual_seed(seed)
    H, S, D = 8, 8192, 128
    if kind == "K":  # per-channel log-normal(0,1) scales, one outlier channel x10 per head
        s_c = torch.exp(torch.randn(H, 1, D, generator=g))
        ch = torch.randint(0, D, (H,), generator=g)
        s_c[torch.arange(H), 0, ch] *= 10.0
        x = torch.randn(H, S, D, generator=g) * s_c
    else:
        x = torch.randn(H, S, D, generator=g)
    return x.to(torch.bfloat16).view(1, H, S, D)


@pytest.mark.parametrize("kind", ["K", "V"])
def test_full_config2_chunk_matches_oracle(kind):
    from latticequant_b200 import codec

    x = _config2_chunk(kind, 2024 if kind == "K" else 2025)
    ch, _ = codec.compress(x.cuda(), 4, tile_blocks=1024)
    out = codec.decompress(ch)
    xn = _bf16_bits(x)
    ref = O.compress_chunk(xn, O.DT_BF16, 8, 8192 * 16, 4, tile_blocks=1024, ties="stable")
    _compare_lane_chunk(ch, ref)
    rec = O.decompress_chunk(ref, out_dtype=O.DT_BF16)
    assert np.array_equal(_bf16_bits(out).reshape(-1), rec.reshape(-1))


def test_full_config1_chunk_matches_oracle():
    """Config 1: CompressedKVCache(4)._compress_tensor of the (1, 262144, 1, 128)
    view -- one fp16 scale per vector -- through the reference-facing API."""
    from latticequant_b200.llm.compressed_kv_cache import CompressedKVCache

    g = torch.Generator().manual_seed(101)
    x = torch.randn(262144, 128, generator=g) * torch.exp(0.5 * torch.randn(262144, 1, generator=g))
    cache = CompressedKVCache(4)
    chunk, deq = cache._compress_tensor(x.view(1, 262144, 1, 128).cuda())
    rec_dev = cache._decompress_chunk(chunk)
    xn = x.numpy()
    ref = O.compress_chunk(xn, O.DT_F32, 262144, 16, 4, tile_blocks=1024, ties="stable")
    _compare_lane_chunk(chunk.lanes, ref)
    rec = O.decompress_chunk(ref, out_dtype=O.DT_F32)
    assert np.array_equal(_u32(rec_dev).reshape(-1), rec.reshape(-1).view(np.uint32))
    # update()'s values use the fp32 scale (llm/compressed_kv_cache.py:204)
    _, _, _, deq_ref = O.quantize_chunk(xn, O.DT_F32, 262144, 16, ref.scale_f32, out_dtype=O.DT_F32)
    assert np.array_equal(_u32(deq).reshape(-1), deq_ref.reshape(-1).view(np.uint32))
    # accounting: words + coset bits + fp16 scales, as the reference counts them
    assert chunk.lanes.compressed_bytes() == 4 * ref.words.size + (262144 * 16 + 7) // 8 + 2 * 262144
    mse = float(((rec.astype(np.float64).reshape(-1, 128) - xn) ** 2).mean())
    assert 0 < mse < 0.02 * float((xn.astype(np.float64) ** 2).mean())


def _oracle_update_values(x, bits):
    """What the reference's update() returns for x (B, H, S, D) bf16 -- q times
    the fp32 head scale, in bf16 -- and the fp16-scale decode, as bf16 bits."""
    B, H, S, D = x.shape
    xn = _bf16_bits(x)
    _, s32, s16 = O.head_scales(xn, B * H, bits, O.DT_BF16)
    q, _, _, deq = O.quantize_chunk(xn, O.DT_BF16, B * H, S * D // 8, s32, out_dtype=O.DT_BF16)
    return deq.reshape(B, H, S, D), q, s32, s16


def test_variable_rate_cache_matches_oracle():
    """Per-layer K/V bit rates: every update()'s returned K/V (the concatenated
    fp32-scale values) and every stored chunk -- all fields and its decode --
    against the oracle at that layer's rate."""
    from latticequant_b200.allocation.eval_alloc import VariableRateKVCache

    sched = [{'K': 3, 'V': 5}, {'K': 5, 'V': 4}, {'K': 4, 'V': 3}]
    cache = VariableRateKVCache(sched, eval_only_no_entropy=False)
    g = torch.Generator().manual_seed(77)
    B, H, S, D = 1, 4, 64, 128
    for layer in range(3):
        inputs = {"K": [], "V": []}
        for step, s in enumerate((S, 1, 1)):
            k = (torch.randn(B, H, s, D, generator=g) * (1 + layer)).to(torch.bfloat16)
            v = torch.randn(B, H, s, D, generator=g).to(torch.bfloat16)
            inputs["K"].append(k)
            inputs["V"].append(v)
            k_full, v_full = cache.update(k.cuda(), v.cuda(), layer)
            for kind, got in (("K", k_full), ("V", v_full)):
                want = np.concatenate([_oracle_update_values(x, sched[layer][kind])[0] for x in inputs[kind]], 2)
                assert np.array_equal(_bf16_bits(got), want), (layer, step, kind)
        for kind, layers in (("K", cache._comp_keys), ("V", cache._comp_values)):
            bits = sched[layer][kind]
            assert len(layers[layer].chunks) == 3
            for chunk, x in zip(layers[layer].chunks, inputs[kind]):
                assert chunk.bits_per_dim == bits
                b, h, s, d = x.shape
                ref = O.compress_chunk(_bf16_bits(x), O.DT_BF16, b * h, s * d // 8, bits, tile_blocks=1024,
                                       ties="stable")
                _compare_lane_chunk(chunk.lanes, ref)
                rec = cache._decompress_chunk(chunk)
                want = O.decompress_chunk(ref, out_dtype=O.DT_BF16)
                assert np.array_equal(_bf16_bits(rec).reshape(-1), want.reshape(-1)), (layer, kind)
                assert chunk.lanes.compressed_bytes() == 4 * ref.words.size + (b * h * s * d // 8 + 7) // 8 + 2 * b * h


def test_compressed_attention_tails_match_oracle():
    """Decode tokens: update()'s output, the stored per-token-scale tail chunks,
    the dequantised tail the attention reads and the attention itself, all
    against the oracle."""
    from latticequant_b200 import codec
    from latticequant_b200.llm.compressed_attention import CompressedAttentionKVCache

    B, H, G, S0, D, T = 2, 2, 4, 128, 128, 16
    steps = 2 * T + 5  # two flushed tails and a partial one
    cache = CompressedAttentionKVCache(4, tail_tokens=T)
    g = torch.Generator().manual_seed(9)
    k0 = torch.randn(B, H, S0, D, generator=g).to(torch.bfloat16)
    v0 = torch.randn(B, H, S0, D, generator=g).to(torch.bfloat16)
    cache.update(k0.cuda(), v0.cuda(), 0)
    toks_k, toks_v = [], []
    for step in range(steps):
        kt = torch.randn(B, H, 1, D, generator=g).to(torch.bfloat16)
        vt = torch.randn(B, H, 1, D, generator=g).to(torch.bfloat16)
        kd, vd = cache.update(kt.cuda(), vt.cuda(), 0)
        assert np.array_equal(_bf16_bits(kd), _oracle_update_values(kt, 4)[0]), step
        assert np.array_equal(_bf16_bits(vd), _oracle_update_values(vt, 4)[0]), step
        toks_k.append(kt)
        toks_v.append(vt)
    st = cache._state[0]
    # the two flushed tails: stored as per-token-scale chunks, attended from
    # their dequantised tokens (update()'s values) in the layer's dense tail
    assert not [p for p in st.parts if p.per_token]
    assert st.n_tail_dense == 2 * T and st.n_tail == steps - 2 * T
    stored_k, stored_v = cache._comp_keys[0].chunks[1:], cache._comp_values[0].chunks[1:]
    assert len(stored_k) == len(stored_v) == 2

    def oracle_fp16_values(x):  # (B, H, S, D) -> q * fp16 scale per head, float64
        xb, q, s32, s16 = _oracle_update_values(x, 4)
        b, h, s, d = x.shape
        sc = s16.view(np.float16).astype(np.float64).reshape(b * h, 1, 1)
        return (q.astype(np.float64).reshape(b * h, s * d // 8, 8) * sc).reshape(b, h, s, d)

    for i in range(2):
        for chunk, toks in ((stored_k[i].lanes, toks_k), (stored_v[i].lanes, toks_v)):
            # a tail chunk holds the (B, H*T, 1, D) view: one head per token
            per_tok = torch.cat(toks[i * T:(i + 1) * T], 2).reshape(B, H * T, 1, D)
            _, _, s32, s16 = _oracle_update_values(per_tok, 4)
            assert np.array_equal(_u32(chunk.scale_f32), s32.view(np.uint32))
            assert np.array_equal(chunk.scale_f16.cpu().numpy().view(np.uint16), s16)
            dec = codec.decompress(chunk, out_dtype=torch.float32).double().cpu().numpy()
            assert np.array_equal(dec.reshape(-1), oracle_fp16_values(per_tok).reshape(-1))

    def update_bits(toks):  # tokens as their own update() quantised them: bf16 bits (B, H, n, D)
        n = len(toks)
        per_tok = torch.cat(toks, 2).reshape(B, H * n, 1, D)
        return _oracle_update_values(per_tok, 4)[0].reshape(B, H, n, D)

    def update_values(toks):
        return torch.from_numpy(update_bits(toks).view(np.int16)).view(torch.bfloat16).double().numpy()

    # the dense tail holds exactly update()'s values of the flushed tokens
    assert np.array_equal(_bf16_bits(st.tail_dense_k[:, :, :2 * T]), update_bits(toks_k[:2 * T]))
    assert np.array_equal(_bf16_bits(st.tail_dense_v[:, :, :2 * T]), update_bits(toks_v[:2 * T]))
    # attention against float64 attention over the oracle's values: the prefill
    # with its fp16 scales, every decode token as update() returned it
    K = np.concatenate([oracle_fp16_values(k0), update_values(toks_k)], 2)
    V = np.concatenate([oracle_fp16_values(v0), update_values(toks_v)], 2)
    gq = torch.Generator().manual_seed(10)
    q = torch.randn(B, H * G, 1, D, generator=gq) / math.sqrt(D)  # fp32: the output is fp32 too
    o = cache.decode_attention(0, q.cuda()).cpu().numpy().reshape(B, H * G, D)
    ref = O.decode_attention_f64(q.numpy().reshape(B, H * G, D), K, V, 1 / math.sqrt(D))
    err = (np.abs(o - ref).max(-1) / np.abs(ref).max(-1)).max()
    assert err <= RTOL, err
    assert cache.flags() == 0


def test_outlier_chunk_matches_oracle_lattice():
    """Tokens left in the streams decode to the oracle's lattice points times the
    fp16 scale; the extracted records are the oracle's (coset, symbols)."""
    from latticequant_b200 import codec

    g = torch.Generator().manual_seed(0)
    x = torch.randn(2, 2, 256, 128, generator=g)
    for b, h, s, d, v in ((0, 0, 5, 3, 66.0), (0, 0, 9, 7, -66.0), (1, 1, 100, 0, 4000.0)):
        x[b, h, s, d] = v
    x = x.to(torch.bfloat16)
    ch, _ = codec.compress(x.cuda(), 5, tile_blocks=1024)
    assert ch.n_outliers > 0 and ch.n_outliers % 16 == 0
    out, sym = codec.decompress(ch, out_dtype=torch.float32, want_symbols=True)
    xn = _bf16_bits(x)
    n_heads, bph = 4, 256 * 16
    _, s32, s16 = O.head_scales(xn, n_heads, 5, O.DT_BF16)
    assert np.array_equal(_u32(ch.scale_f32), s32.view(np.uint32))
    q, cos, osym, _ = O.quantize_chunk(xn, O.DT_BF16, n_heads, bph, s32)
    sc = s16.view(np.float16).astype(np.float32)
    # decoded values come from the symbols (symbols_to_e8, so zeros are +0)
    qs = O.symbols_to_e8(cos, osym)
    assert np.array_equal(qs, q)  # equal as numbers (q may hold -0)
    want = (qs.reshape(n_heads, bph, 8) * sc[:, None, None]).reshape(-1)
    assert np.array_equal(_u32(out).reshape(-1), want.view(np.uint32))
    assert np.array_equal(sym.cpu().numpy(), osym)
    rec = ch.outlier_rec.cpu().numpy()
    blk = rec[:, 0]
    assert np.array_equal(rec[:, 1], cos[blk].astype(np.int32))
    assert np.array_equal(rec[:, 2:], osym[blk])
    # the extracted blocks are whole tokens holding a symbol beyond the limit
    toks = np.unique(blk // 16)
    assert all(np.abs(osym[t * 16:(t + 1) * 16]).max() > codec.OUTLIER_LIMIT for t in toks)


def test_config3_full_shape_sampled_rows_match_oracle():
    """Config 3 (B16, 32 q / 8 kv heads, D128, ctx 32768, 4 b/dim): 64 of the 128
    (batch, kv head) pairs -- 256 query rows -- against float64 attention over
    the oracle's lattice points times the fp16 head scale."""
    from latticequant_b200 import attention, codec

    B, Hkv, G, S, D = 16, 8, 4, 32768, 128
    gen = torch.Generator(device="cuda").manual_seed(41)
    shape = (B, Hkv, S, D)

    def kv():
        return (torch.randn(shape, generator=gen, device="cuda") *
                torch.exp(0.5 * torch.randn(B, Hkv, S, 1, generator=gen, device="cuda"))).to(torch.bfloat16)

    k, v = kv(), kv()
    q = (torch.randn(B, Hkv * G, D, generator=gen, device="cuda") / math.sqrt(D)).to(torch.bfloat16)
    kc, _ = codec.compress(k, 4)
    vc, _ = codec.compress(v, 4)
    o = attention.decode_attention(q, kc, vc, out_dtype=torch.float32).cpu().numpy()
    rng = np.random.default_rng(3)
    pairs = rng.choice(B * Hkv, 64, replace=False)
    qn = q.float().cpu().numpy()
    worst = 0.0
    for hp in pairs:
        b, h = divmod(int(hp), Hkv)
        vals = []
        for x, ch in ((k, kc), (v, vc)):
            xn = _bf16_bits(x[b, h])
            s32 = ch.scale_f32[hp:hp + 1].cpu().numpy()  # the chunk's scale of this head
            qq, _, _, _ = O.quantize_chunk(xn, O.DT_BF16, 1, S * D // 8, s32)
            s16 = ch.scale_f16[hp:hp + 1].cpu().numpy().astype(np.float64)
            vals.append(qq.astype(np.float64).reshape(1, 1, S, D) * s16[0])
        ref = O.decode_attention_f64(qn[b:b + 1, h * G:(h + 1) * G], vals[0], vals[1], 1 / math.sqrt(D))
        got = o[b, h * G:(h + 1) * G]
        worst = max(worst, float((np.abs(got - ref[0]).max(-1) / np.abs(ref[0]).max(-1)).max()))
    assert worst <= RTOL, worst
    # the scales themselves are the oracle's for the sampled heads
    for hp in pairs[:8]:
        b, h = divmod(int(hp), Hkv)
        _, s32, _ = O.head_scales(_bf16_bits(k[b, h]), 1, 4, O.DT_BF16)
        assert kc.scale_f32[hp].cpu().numpy().view(np.uint32) == s32.view(np.uint32)[0]
