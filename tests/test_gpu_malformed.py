"""Malformed lane streams through the CUDA decoder.

The tile decoder runs its table-driven steps without a per-step bit check and
afterwards asks whether any lane read past its n_bits; such a warp decodes its
tiles again with the exact, checked steps.  Whatever path a lane takes, the
symbols must be those of the reference's literal decoder
(core/gpu_ans.py:146-168: stop reading at n_bits, state formula as written),
restated by the oracle's lqo_rans_decode, for truncated bit counts, flipped
bits and initial states outside [L, 2L) -- and the fused attention over such
chunks must equal attention over those symbols.

Bar: symbols bit-exact; attention max |o - o_ref| <= 1e-3 * max |o_ref| per row.
"""
import dataclasses
import math

import numpy as np
import pytest
import torch

from oracle import lq_oracle as O

pytestmark = pytest.mark.gpu

L = 1024
RTOL = 1e-3


def _chunk(shape, bits, seed, tile):
    from latticequant_b200 import codec

    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g) * torch.exp(0.5 * torch.randn(*shape[:-1], 1, generator=g))
    ch, _ = codec.compress(x.to(torch.bfloat16).cuda(), bits, tile_blocks=tile)
    return ch


def _corrupt(ch, kind, seed, frac=0.25):
    """A copy of the chunk with a fraction of its non-empty lanes damaged."""
    rng = np.random.default_rng(seed)
    nb = ch.lane_nbits.cpu().numpy().astype(np.int64)
    st = ch.lane_state.cpu().numpy().astype(np.int64)
    off = ch.lane_off.cpu().numpy().view(np.uint32).astype(np.int64)
    w = ch.words.cpu().numpy().view(np.uint32).copy()
    live = np.flatnonzero(nb > 0)
    pick = rng.choice(live, max(1, int(frac * live.size)), replace=False)
    for l in pick:
        if kind == "truncate":
            nb[l] -= int(rng.integers(1, min(nb[l], 160) + 1))
        elif kind == "flip":
            for _ in range(3):
                i = int(off[l] + rng.integers(0, off[l + 1] - off[l]))
                w[i] ^= np.uint32(1) << np.uint32(rng.integers(0, 32))
        elif kind == "state":
            st[l] = int(rng.choice([L - 3, 2 * L + 5, 7, 3 * L - 1]))
    dev = ch.words.device
    return dataclasses.replace(
        ch, lane_nbits=torch.from_numpy(nb.astype(np.int32)).to(dev),
        lane_state=torch.from_numpy(st.astype(np.int32)).to(dev),
        words=torch.from_numpy(w.view(np.int32)).to(dev), dec_tab=None)


def _oracle_symbols(ch):
    g = ch.geom
    n = g.n_heads * g.bph
    cos = O.unpack_coset_bits(ch.coset_words.cpu().numpy().view(np.uint8), n)
    fr = ch.tab_freq.cpu().numpy().view(np.uint16).astype(np.int32)
    sym = O.decode_lanes(cos, g.tile_blocks, ch.tab_lo.cpu().numpy(), ch.tab_nsym.cpu().numpy(), fr,
                         ch.words[:max(ch.n_words, 1)].cpu().numpy().view(np.uint32),
                         ch.lane_off.cpu().numpy().view(np.uint32), ch.lane_nbits.cpu().numpy().view(np.uint32),
                         ch.lane_state.cpu().numpy().view(np.uint32))
    return cos, sym


def _oracle_values(ch):
    """Dequantised values of the oracle's decode: E8 point * fp16 head scale in fp32."""
    g = ch.geom
    cos, sym = _oracle_symbols(ch)
    q = O.symbols_to_e8(cos, sym).astype(np.float32).reshape(g.n_heads, g.bph * 8)
    s = ch.scale_f16.cpu().float().numpy().reshape(g.n_heads, 1)
    return (q * s).reshape(ch.orig_shape)


@pytest.mark.parametrize("kind", ["truncate", "flip", "state"])
@pytest.mark.parametrize("tile", [64, 1024])
def test_decode_malformed_matches_literal_decoder(kind, tile):
    from latticequant_b200 import codec

    ch = _chunk((2, 3, 96, 128), 4, 21, tile)
    bad = _corrupt(ch, kind, 5)
    _, sym = codec.decompress(bad, want_symbols=True)
    _, ref = _oracle_symbols(bad)
    assert np.array_equal(sym.cpu().numpy(), ref)
    # the healthy chunk still decodes to its own symbols
    _, sym0 = codec.decompress(ch, want_symbols=True)
    _, ref0 = _oracle_symbols(ch)
    assert np.array_equal(sym0.cpu().numpy(), ref0)


@pytest.mark.parametrize("kind", ["truncate", "flip", "state"])
def test_attention_malformed_matches_literal_decoder(kind):
    from latticequant_b200 import attention

    B, Hkv, G, S, D = 2, 2, 4, 256, 128
    kc = _corrupt(_chunk((B, Hkv, S, D), 4, 31, 256), kind, 6)
    vc = _corrupt(_chunk((B, Hkv, S, D), 4, 32, 256), kind, 7)
    gq = torch.Generator().manual_seed(33)
    q = (torch.randn(B, Hkv * G, D, generator=gq) / math.sqrt(D)).to(torch.bfloat16)
    o = attention.decode_attention(q.cuda(), kc, vc, out_dtype=torch.float32)
    kd, vd = _oracle_values(kc), _oracle_values(vc)
    ref = O.decode_attention_f64(q.float().numpy(), kd, vd, 1.0 / math.sqrt(D))
    o = o.float().cpu().numpy().reshape(ref.shape)
    err = np.abs(o - ref).max(axis=-1)
    scale = np.abs(ref).max(axis=-1)
    assert np.all(err <= RTOL * scale), float((err / scale).max())
