"""Decode attention over the compact fixed-rate layout (lq_attn_decode_compact)
against the oracle: every block's value from the chunk -- the oracle's
unpack_e8 (core/compact_storage.py:140-222) times the fp32 head scale for a
representable block, the stored fp16 row for a fallback block -- attended in
float64 with repeat_kv (oracle.decode_attention_f64).  The reference's own
path merges the chunk into fp16 K/V first (llm/fused_triton_merge.py:137-177);
that rounding is the one difference, and the merged-fp16 attention is checked
against the same bar.

Tolerance: max |o - o_ref| <= 1e-3 * max |o_ref| per query row; lse within
1e-3 absolute.
"""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

RTOL = 1e-3


def _exact_values(chunk):
    from oracle import lq_oracle as O

    mask = chunk.repr_mask.cpu().numpy().astype(bool)
    n = mask.size
    out = np.zeros((n, 8), np.float64)
    q = O.unpack_e8(chunk.packed.cpu().numpy(), chunk.bits_per_dim)
    head = np.arange(n) // chunk.blocks_per_head
    sc = chunk.scales.cpu().numpy().astype(np.float64)
    out[mask] = q.astype(np.float64) * sc[head[mask]][:, None]
    out[~mask] = chunk.fallback.cpu().float().numpy()
    return out.reshape(chunk.orig_shape)


def _row_err(o, ref):
    err = np.abs(o - ref).max(axis=-1)
    scale = np.abs(ref).max(axis=-1)
    return float((err / scale).max())


def _kv(shape, seed):
    g = torch.Generator().manual_seed(seed)
    B, H, S, D = shape
    return (torch.randn(shape, generator=g) * torch.exp(0.5 * torch.randn(B, H, S, 1, generator=g))).to(torch.bfloat16)


CASES = [
    # B, Hkv, G, S, D, bits, q dtype  (head_dim 128 with G <= 4 runs the tensor-core kernel)
    (2, 2, 4, 256, 128, 4, torch.bfloat16),
    (1, 3, 2, 128, 64, 4, torch.float16),
    (2, 1, 1, 64, 128, 3, torch.float32),
    (1, 2, 8, 96, 128, 5, torch.bfloat16),
    (1, 4, 7, 1030, 128, 4, torch.bfloat16),   # tokens past the last full warp slab
    (1, 2, 4, 1030, 128, 4, torch.bfloat16),   # tensor cores: partial stage and CTA
    (2, 2, 3, 2050, 128, 4, torch.float16),    # three of four padded query heads
    (1, 3, 2, 300, 128, 5, torch.float32),
    (1, 1, 4, 4096, 128, 3, torch.bfloat16),   # four CTAs per head
]


@pytest.mark.parametrize("case", CASES, ids=[f"B{c[0]}H{c[1]}G{c[2]}S{c[3]}D{c[4]}b{c[5]}" for c in CASES])
def test_compact_attention_matches_merge_then_attention(case):
    from oracle import lq_oracle as O

    from latticequant_b200 import attention
    from latticequant_b200.llm.fused_triton_merge import compress_compact, fused_decompress_chunk

    B, Hkv, G, S, D, bits, qdt = case
    k = _kv((B, Hkv, S, D), 21).cuda()
    v = _kv((B, Hkv, S, D), 22).cuda()
    kc, _ = compress_compact(k, bits)
    vc, _ = compress_compact(v, bits)
    assert 0 < kc.oor_rate < 1 and 0 < vc.oor_rate < 1  # both paths of the kernel run
    gq = torch.Generator().manual_seed(23)
    q = (torch.randn(B, Hkv * G, D, generator=gq) / math.sqrt(D)).to(qdt)
    sm = 1.0 / math.sqrt(D)
    o, lse = attention.decode_attention_compact(q.cuda(), kc, vc, out_dtype=torch.float32, return_lse=True)
    kd, vd = _exact_values(kc), _exact_values(vc)
    ref = O.decode_attention_f64(q.float().numpy(), kd, vd, sm)
    o = o.cpu().numpy().reshape(ref.shape)
    assert _row_err(o, ref) <= RTOL, _row_err(o, ref)
    # and within the same bar of the reference's merge-then-attend path
    km = fused_decompress_chunk(kc).float().cpu().numpy()
    vm = fused_decompress_chunk(vc).float().cpu().numpy()
    assert _row_err(o, O.decode_attention_f64(q.float().numpy(), km, vm, sm)) <= RTOL
    qf = q.double().numpy()
    kf = np.repeat(kd.astype(np.float64), G, axis=1)
    s = np.einsum("bhd,bhsd->bhs", qf, kf) * sm
    mx = s.max(-1, keepdims=True)
    lref = mx[..., 0] + np.log(np.exp(s - mx).sum(-1))
    assert np.abs(lse.cpu().numpy() - lref).max() < 1e-3


def test_compact_attention_rejects_unaligned_heads():
    from latticequant_b200 import attention
    from latticequant_b200.llm.fused_triton_merge import compress_compact

    k = _kv((1, 1, 3, 128), 5).cuda()  # 48 blocks per head: not a multiple of 32
    kc, _ = compress_compact(k, 4)
    q = torch.randn(1, 1, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        attention.decode_attention_compact(q, kc, kc)


@pytest.mark.parametrize("how", ["rank_high", "rank_order", "mask_bits"])
def test_compact_attention_flags_inconsistent_index(how):
    """Mask words or ranks that disagree with the arrays (a damaged chunk) are
    caught by the kernel's range checks: the BITSTREAM flag, no stray access."""
    from latticequant_b200 import attention
    from latticequant_b200.llm.fused_triton_merge import compress_compact

    k = _kv((1, 2, 512, 128), 31).cuda()
    kc, _ = compress_compact(k, 4)
    vc, _ = compress_compact(_kv((1, 2, 512, 128), 32).cuda(), 4)
    words, rank = attention.compact_index(kc)
    words, rank = words.clone(), rank.clone()
    if how == "rank_high":
        rank[5:9] += 100000
    elif how == "rank_order":
        rank[40:] -= 7
    else:
        words[3:6] = -1  # every block representable: more codes than the ranks allow
    kc._lq_index = (words, rank)
    q = torch.randn(1, 8, 128, dtype=torch.bfloat16, device="cuda")
    from latticequant_b200._lib import LatticeQuantError

    with pytest.raises(LatticeQuantError, match="decode_attention_compact"):
        attention.decode_attention_compact(q, kc, vc)


def _force_fallback(chunk, force):
    """The same chunk with the blocks in `force` (bool, per block) stored as
    fp16 fallback rows (their merged values) instead of codes."""
    from latticequant_b200.llm.fused_triton_merge import CompressedChunk, fused_decompress_chunk

    vals = fused_decompress_chunk(chunk).reshape(-1, 8)
    mask = chunk.repr_mask.bool()
    keep = mask & ~force
    rank = torch.cumsum(mask.int(), 0) - mask.int()
    fb_rank = torch.cumsum((~mask).int(), 0) - (~mask).int()
    was_fb = (~mask)[~keep]
    old_rows = chunk.fallback[fb_rank[~keep].clamp(max=max(chunk.fallback.shape[0] - 1, 0)).long()] \
        if chunk.fallback.shape[0] else torch.zeros_like(vals[~keep])
    fb = torch.where(was_fb[:, None], old_rows, vals[~keep]).contiguous()
    return CompressedChunk(packed=chunk.packed[rank[keep].long()].contiguous(), fallback=fb, repr_mask=keep,
                           scales=chunk.scales, orig_shape=chunk.orig_shape, blocks_per_head=chunk.blocks_per_head,
                           bits_per_dim=chunk.bits_per_dim, orig_dtype=chunk.orig_dtype)


@pytest.mark.parametrize("bits", [4, 3])
def test_compact_attention_stage_beyond_staged_fallback_rows(bits):
    """A 128-token stage whose blocks are all fallback rows (more than the 768
    a tensor-core stage buffer holds): the rows past the staged ones are read
    from HBM; the result matches the reference as everywhere else."""
    from oracle import lq_oracle as O

    from latticequant_b200 import attention
    from latticequant_b200.llm.fused_triton_merge import compress_compact

    B, Hkv, G, S, D = 1, 2, 4, 512, 128
    k = _kv((B, Hkv, S, D), 61).cuda()
    v = _kv((B, Hkv, S, D), 62).cuda()
    kc, _ = compress_compact(k, bits)
    vc, _ = compress_compact(v, bits)
    bph = S * D // 8
    force = torch.zeros(B * Hkv * bph, dtype=torch.bool, device="cuda")
    force[128 * 16:256 * 16] = True             # head 0, tokens 128..255: one whole stage
    force[bph + 300 * 16:bph + 400 * 16] = True  # head 1: 100 tokens across two stages
    kc2, vc2 = _force_fallback(kc, force), _force_fallback(vc, force)
    assert kc2.fallback.shape[0] > kc.fallback.shape[0] + 1000
    q = (torch.randn(B, Hkv * G, D, generator=torch.Generator().manual_seed(63)) / math.sqrt(D)).to(torch.bfloat16)
    o = attention.decode_attention_compact(q.cuda(), kc2, vc2, out_dtype=torch.float32)
    ref = O.decode_attention_f64(q.float().numpy(), _exact_values(kc2), _exact_values(vc2), 1 / math.sqrt(D))
    assert _row_err(o.cpu().numpy().reshape(ref.shape), ref) <= RTOL
    # and the same numbers as the unforced chunks (the forced rows hold the merged values)
    o1 = attention.decode_attention_compact(q.cuda(), kc, vc, out_dtype=torch.float32)
    assert _row_err(o.cpu().numpy(), o1.cpu().numpy()) <= RTOL
