"""Fused dequant + decode attention (lq_attn_decode / lq_attn_merge) against
the oracle: K/V compressed by the CUDA codec, dequantised by the C oracle's
lane decoder (q * fp16 head scale, llm/compressed_kv_cache.py:289-332) and
attended in float64 with repeat_kv (oracle.decode_attention_f64).

Tolerance (merged attention outputs): max |o - o_ref| <= 1e-3 * max |o_ref|
per query row, fp32 output.
"""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

RTOL = 1e-3


def _kv(shape, seed, dtype):
    g = torch.Generator().manual_seed(seed)
    B, H, S, D = shape
    # config 1's distribution: N(0,1) times a log-normal(0, 0.5) magnitude per vector
    x = torch.randn(shape, generator=g) * torch.exp(0.5 * torch.randn(B, H, S, 1, generator=g))
    return x.to(dtype)


def _oracle_deq(x, chunk):
    from oracle import lq_oracle as O

    B, H, S, D = x.shape
    xf = x.numpy() if x.dtype == torch.float32 else x.view(torch.int16).numpy().view(np.uint16)
    dt = {torch.float32: O.DT_F32, torch.float16: O.DT_F16, torch.bfloat16: O.DT_BF16}[x.dtype]
    ch = O.compress_chunk(np.ascontiguousarray(xf), dt, B * H, S * D // 8, chunk.bits, chunk.geom.tile_blocks,
                          scale_f32=chunk.scale_f32.cpu().numpy())
    return O.decompress_chunk(ch, O.DT_F32).reshape(B, H, S, D)


def _check(o, ref):
    o = o.float().cpu().numpy().reshape(ref.shape)
    err = np.abs(o - ref).max(axis=-1)
    scale = np.abs(ref).max(axis=-1)
    assert np.all(err <= RTOL * scale), float((err / scale).max())


CASES = [
    # B, Hkv, G, S, D, tile_blocks, kv dtype, q dtype
    (2, 2, 4, 256, 128, 256, torch.bfloat16, torch.bfloat16),
    (1, 4, 7, 192, 128, 1024, torch.bfloat16, torch.bfloat16),   # odd tiles per head
    (3, 1, 1, 96, 64, 256, torch.float16, torch.float16),        # head_dim 64
    (2, 2, 8, 128, 64, 64, torch.float32, torch.float32),
    (1, 3, 2, 512, 128, 512, torch.float32, torch.bfloat16),
    (2, 1, 3, 64, 128, 1024, torch.bfloat16, torch.float16),    # one tile per head
]


@pytest.mark.parametrize("case", CASES, ids=[f"B{c[0]}H{c[1]}G{c[2]}S{c[3]}D{c[4]}T{c[5]}" for c in CASES])
def test_attention_matches_oracle(case):
    from oracle import lq_oracle as O

    from latticequant_b200 import attention, codec

    B, Hkv, G, S, D, TB, kvdt, qdt = case
    k = _kv((B, Hkv, S, D), 11, kvdt)
    v = _kv((B, Hkv, S, D), 12, kvdt)
    gq = torch.Generator().manual_seed(13)
    q = (torch.randn(B, Hkv * G, D, generator=gq) / math.sqrt(D)).to(qdt)
    kc, _ = codec.compress(k.cuda(), 4, tile_blocks=TB)
    vc, _ = codec.compress(v.cuda(), 4, tile_blocks=TB)
    o, lse = attention.decode_attention(q.cuda(), kc, vc, out_dtype=torch.float32, return_lse=True)
    kd, vd = _oracle_deq(k, kc), _oracle_deq(v, vc)
    sm = 1.0 / math.sqrt(D)
    ref = O.decode_attention_f64(q.float().numpy(), kd, vd, sm)
    _check(o, ref)
    # log-sum-exp of the scores
    qf = q.double().numpy()
    kf = np.repeat(kd.astype(np.float64), G, axis=1)
    s = np.einsum("bhd,bhsd->bhs", qf, kf) * sm
    mx = s.max(-1, keepdims=True)
    lref = (mx[..., 0] + np.log(np.exp(s - mx).sum(-1)))
    assert np.allclose(lse.cpu().numpy(), lref, rtol=0, atol=1e-4 * np.abs(lref).max() + 1e-5)


def test_attention_is_deterministic_and_4d_q():
    from latticequant_b200 import attention, codec

    B, Hkv, G, S, D = 2, 2, 4, 512, 128
    k = _kv((B, Hkv, S, D), 21, torch.bfloat16).cuda()
    v = _kv((B, Hkv, S, D), 22, torch.bfloat16).cuda()
    q = (torch.randn(B, Hkv * G, 1, D, generator=torch.Generator().manual_seed(23)) / math.sqrt(D)).to(
        torch.bfloat16).cuda()
    kc, _ = codec.compress(k, 4, tile_blocks=256)
    vc, _ = codec.compress(v, 4, tile_blocks=256)
    a = attention.decode_attention(q, kc, vc)
    b = attention.decode_attention(q, kc, vc)
    assert a.shape == q.shape and a.dtype == torch.bfloat16
    assert torch.equal(a, b)


def test_sequence_split_merge_matches_whole():
    """Sequence-sharded attention: each shard's (o, lse), merged, equals attention
    over the whole context (the multi-GPU all-gather + LSE merge path)."""
    from oracle import lq_oracle as O

    from latticequant_b200 import attention, codec

    B, Hkv, G, S, D = 2, 2, 4, 1024, 128
    k = _kv((B, Hkv, S, D), 31, torch.bfloat16)
    v = _kv((B, Hkv, S, D), 32, torch.bfloat16)
    q = (torch.randn(B, Hkv * G, D, generator=torch.Generator().manual_seed(33)) / math.sqrt(D)).to(torch.bfloat16)
    parts_o, parts_l, kd, vd = [], [], [], []
    for lo in range(0, S, S // 4):
        ks, vs = k[:, :, lo:lo + S // 4].contiguous(), v[:, :, lo:lo + S // 4].contiguous()
        kc, _ = codec.compress(ks.cuda(), 4, tile_blocks=256)
        vc, _ = codec.compress(vs.cuda(), 4, tile_blocks=256)
        o, l = attention.decode_attention(q.cuda(), kc, vc, out_dtype=torch.float32, return_lse=True)
        parts_o.append(o)
        parts_l.append(l)
        kd.append(_oracle_deq(ks, kc))
        vd.append(_oracle_deq(vs, vc))
    om, lm = attention.merge_attention(parts_o, parts_l, out_dtype=torch.float32)
    ref = O.decode_attention_f64(q.float().numpy(), np.concatenate(kd, 2), np.concatenate(vd, 2), 1 / math.sqrt(D))
    _check(om, ref)
    assert lm.shape == (B, Hkv * G)


def test_config3_shape_against_torch_fp32():
    """Config 3 (B=16, Hq=32, Hkv=8, D=128, ctx 32768, 4 bits/dim): the fused
    kernel against fp32 attention over the CUDA codec's own dequantised K/V."""
    from latticequant_b200 import attention, codec

    B, Hkv, G, S, D = 16, 8, 4, 32768, 128
    gen = torch.Generator(device="cuda").manual_seed(41)
    shape = (B, Hkv, S, D)
    k = (torch.randn(shape, generator=gen, device="cuda") *
         torch.exp(0.5 * torch.randn(B, Hkv, S, 1, generator=gen, device="cuda"))).to(torch.bfloat16)
    v = (torch.randn(shape, generator=gen, device="cuda") *
         torch.exp(0.5 * torch.randn(B, Hkv, S, 1, generator=gen, device="cuda"))).to(torch.bfloat16)
    q = (torch.randn(B, Hkv * G, D, generator=gen, device="cuda") / math.sqrt(D)).to(torch.bfloat16)
    kc, _ = codec.compress(k, 4)
    vc, _ = codec.compress(v, 4)
    del k, v
    o = attention.decode_attention(q, kc, vc, out_dtype=torch.float32)
    kd = codec.decompress(kc, torch.float32)
    vd = codec.decompress(vc, torch.float32)
    qf = q.float().view(B, Hkv, G, D)
    s = torch.einsum("bhgd,bhsd->bhgs", qf, kd) / math.sqrt(D)
    p = torch.softmax(s, dim=-1)
    ref = torch.einsum("bhgs,bhsd->bhgd", p, vd).reshape(B, Hkv * G, D)
    err = (o - ref).abs().amax(-1)
    scale = ref.abs().amax(-1)
    assert bool((err <= RTOL * scale).all()), float((err / scale).max())


def test_attention_rejects_bad_geometry():
    from latticequant_b200 import attention, codec

    k = _kv((1, 2, 40, 128), 51, torch.bfloat16).cuda()
    kc, _ = codec.compress(k, 4, tile_blocks=256)   # 640 blocks per head: tiles straddle heads
    q = torch.randn(1, 8, 128, device="cuda", dtype=torch.bfloat16)
    assert not attention.supports(kc, 4)
    with pytest.raises(ValueError):
        attention.decode_attention(q, kc, kc)
    kc2, _ = codec.compress(_kv((1, 2, 64, 128), 52, torch.bfloat16).cuda(), 4, tile_blocks=1024)
    with pytest.raises(ValueError):
        attention.decode_attention(torch.randn(1, 6, 64, device="cuda"), kc2, kc2)   # head_dim mismatch
    with pytest.raises(ValueError):
        attention.decode_attention(torch.randn(1, 7, 128, device="cuda"), kc2, kc2)  # 7 not a multiple of 2


def test_bulk_staged_tables_match_per_thread_staging():
    """The decode tables filled by one bulk copy (lq_stage_tables +
    cp.async.bulk) give bit-identical attention to the per-thread staging."""
    from latticequant_b200 import attention, codec

    B, Hkv, G, S, D = 2, 2, 4, 512, 128
    k = _kv((B, Hkv, S, D), 71, torch.bfloat16).cuda()
    v = _kv((B, Hkv, S, D), 72, torch.bfloat16).cuda()
    q = (torch.randn(B, Hkv * G, D, generator=torch.Generator().manual_seed(73)) / math.sqrt(D)).to(torch.bfloat16)
    kc, _ = codec.compress(k, 4, tile_blocks=1024)
    vc, _ = codec.compress(v, 4, tile_blocks=1024)
    op = attention.DecodeAttention(kc, vc, G)
    assert op.kv.staged_tab and op.vv.staged_tab
    o1 = torch.empty(B, Hkv * G, D, dtype=torch.float32, device="cuda")
    o2 = torch.empty_like(o1)
    op(q.cuda(), o1)
    op.kv.staged_tab = None
    op.vv.staged_tab = None
    op(q.cuda(), o2)
    assert op.flags() == 0
    assert torch.equal(o1, o2)
