"""Pin the CPU oracle to the reference's own outputs (committed fixtures).

The fixtures were produced by running yoon9728/LatticeQuant itself
(tests/golden/make_golden.py).  Everything here is CPU-only.
"""
import numpy as np
import pytest

from conftest import golden
from oracle import lq_oracle as O


def _bits16(a):
    return np.asarray(a).view(np.uint16)


# ---------------------------------------------------------------- E8 core
def test_e8_and_d8_bit_exact():
    g = golden("e8.npz")
    x = g["x"]
    assert np.array_equal(O.encode_d8(x).view(np.uint32), g["d8"].view(np.uint32))
    assert np.array_equal(O.encode_e8(x).view(np.uint32), g["e8"].view(np.uint32))


def test_tiebreaker_bits_match_torch():
    import torch

    t = (torch.arange(8, dtype=torch.float32) * 1e-7).numpy().view(np.uint32)
    assert [hex(v) for v in t] == ['0x0', '0x33d6bf95', '0x3456bf95', '0x34a10fb0', '0x34d6bf95', '0x350637bd',
                                   '0x35210fb0', '0x353be7a2']


def test_cascade_sum_matches_torch_rows():
    import torch

    torch.manual_seed(0)
    for rows, n in [(4, 8), (3, 24), (5, 136), (2, 1000), (4, 4096), (2, 70000), (2, 262144), (2, 1 << 20)]:
        a = (torch.randn(rows, n) * torch.exp(torch.randn(rows, n))).float() ** 2
        ref = a.sum(dim=1).numpy()
        for r in range(rows):
            assert O.cascade_sum_f32(a[r].numpy()).view(np.uint32) == ref[r:r + 1].view(np.uint32)[0], (rows, n, r)


@pytest.mark.parametrize("case,dt", [("f32", O.DT_F32), ("f16", O.DT_F16), ("bf16", O.DT_BF16),
                                     ("pervec", O.DT_F32), ("big", O.DT_BF16), ("hd64", O.DT_F32),
                                     ("zero", O.DT_F32)])
@pytest.mark.parametrize("bits", [3, 4, 5])
def test_head_scales_bit_exact(case, dt, bits):
    g = golden("scales.npz")
    x = g[f"{case}_x"]
    k = f"{case}_b{bits}"
    n_heads = x.shape[0] * x.shape[1]
    xin = x if dt == O.DT_F32 else x.view(np.uint16)
    s2, s32, s16 = O.head_scales(xin, n_heads, bits, dt)
    # sigma2: torch's CPU reduction tree, restated exactly
    assert np.array_equal(s2.view(np.uint32), g[k + "_sigma2"].view(np.uint32))
    # scale: IEEE sqrt here; torch's vectorised CPU sqrt (a vector-math library
    # on large tensors) is off by one ulp on a few heads, so allow 1 ulp there
    d = np.abs(s32.view(np.int32).astype(np.int64) - g[k + "_s32"].view(np.int32).astype(np.int64))
    assert d.max() <= 1 and (d == 0).mean() >= 0.99
    same = d == 0
    assert np.array_equal(s16[same], _bits16(g[k + "_s16"])[same])
    # quantise + dequantise with the reference's fp32 scale, as update() returns it
    bph = x.shape[2] * x.shape[3] // 8
    _, _, _, deq = O.quantize_chunk(xin, dt, n_heads, bph, g[k + "_s32"], out_dtype=dt)
    want = g[k + "_deq"]
    if dt == O.DT_F32:
        assert np.array_equal(deq.reshape(-1).view(np.uint32), want.reshape(-1).view(np.uint32))
    else:
        assert np.array_equal(deq.reshape(-1), _bits16(want).reshape(-1))


def test_symbols_roundtrip_bit_exact():
    g = golden("symbols.npz")
    cos, sym = O.e8_to_symbols(g["q"])
    assert np.array_equal(cos, g["coset"].astype(np.uint8))
    assert np.array_equal(sym[:, :7], g["free"])
    assert np.array_equal(sym[:, 7], g["c8h"])
    assert np.array_equal(O.symbols_to_e8(cos, sym), g["back"])


# ---------------------------------------------------------------- rANS
def test_rans_tables_streams_and_decode():
    g = golden("rans.npz")
    for i in range(int(g["n_cases"])):
        alphabet = list(g[f"c{i}_alphabet"])
        counts = g[f"c{i}_counts"]
        t = O.build_rans_table(counts, alphabet, ties="numpy")
        assert np.array_equal(t.freqs, g[f"c{i}_freqs"]), i
        assert np.array_equal(t.cumfreqs, g[f"c{i}_cumfreqs"]), i
        assert np.array_equal(t.lookup, g[f"c{i}_lookup"]), i
        bs, st, nb = O.rans_encode(g[f"c{i}_syms"], t)
        assert nb == int(g[f"c{i}_nbits"]) and st == int(g[f"c{i}_state"]), i
        assert np.array_equal(bs, g[f"c{i}_bitstream"]), i
        dec = O.rans_decode(bs, nb, st, t, len(g[f"c{i}_syms"]))
        assert np.array_equal(dec, g[f"c{i}_decoded"]), i
    t = O.build_rans_table(g["c0_counts"], list(g["c0_alphabet"]))
    dec = O.rans_decode(g["c0_bitstream"], int(g["trunc_nbits"]), int(g["c0_state"]), t, len(g["c0_syms"]))
    assert np.array_equal(dec, g["trunc_decoded"])


def test_stable_tables_differ_only_inside_ties():
    """The CUDA tie rule (ascending index) differs from numpy's only among equal keys."""
    g = golden("rans.npz")
    for i in range(int(g["n_cases"])):
        c = g[f"c{i}_counts"]
        a = O.normalize_freqs_numpy(c)
        b = O.normalize_freqs_stable(c)
        assert a.sum() == b.sum() == O.L
        assert sorted(a.tolist()) == sorted(b.tolist())  # same multiset of frequencies
        for j in np.nonzero(a != b)[0]:
            # every disagreeing symbol shares its count with another symbol
            assert (c == c[j]).sum() >= 2, (i, j)


def test_pipeline_streams_bit_exact():
    g = golden("pipeline.npz")
    for b in (3, 4, 5):
        k = f"b{b}"
        x = g[k + "_x"]
        q = O.encode_e8((x / np.float32(g[k + "_scale"])).astype(np.float32))
        assert np.array_equal(q, g[k + "_q"])
        cos, sym = O.e8_to_symbols(q)
        assert np.array_equal(cos, g[k + "_coset"])
        assert np.array_equal(sym, g[k + "_syms"])
        si = 0
        for c in (0, 1):
            m = cos == c
            if not m.any():
                continue
            for idx in range(8):
                col = sym[m, idx].astype(np.int64)
                alphabet, counts = O.stream_alphabet(col)
                assert alphabet[0] == int(g[f"{k}_s{si}_lo"])
                t = O.build_rans_table(counts, alphabet, ties="numpy")
                assert np.array_equal(t.freqs, g[f"{k}_s{si}_freqs"])
                bs, st, nb = O.rans_encode(col, t)
                assert nb == int(g[f"{k}_s{si}_nbits"]) and st == int(g[f"{k}_s{si}_state"])
                assert np.array_equal(bs, g[f"{k}_s{si}_bitstream"])
                si += 1
        assert si == int(g[k + "_nstreams"])


# ---------------------------------------------------------------- chunks
CHUNKS = ["chunk_cfg1.npz", "chunk_cfg2k.npz", "chunk_cfg2v.npz", "chunk_f16_b3.npz", "chunk_f16_b5.npz",
          "chunk_decode1.npz"]


def _chunk_input(g):
    dt = str(g["dtype"])
    code = O.dtype_code(dt)
    x = g["x"] if code == O.DT_F32 else g["x"].view(np.uint16)
    shape = tuple(int(v) for v in g["shape"])
    return code, x, shape


@pytest.mark.parametrize("name", CHUNKS)
def test_chunk_reference_layout_bit_exact(name):
    """_compress_tensor + _decompress_chunk, reference chunking (one tile), numpy ties."""
    g = golden(name)
    code, x, shape = _chunk_input(g)
    b, h, s, d = shape
    n_heads, bph = b * h, s * d // 8
    ch = O.compress_chunk(x, code, n_heads, bph, float(g["bits"]), tile_blocks=None, ties="numpy")
    assert np.array_equal(ch.scale_f16, _bits16(g["scales_f16"]))
    assert np.array_equal(ch.coset_packed, g["coset_packed"])
    # stream s of the reference == lane s of the single tile (empty cosets skipped there)
    ref_i = 0
    for s_ in range(16):
        if ch.tab_nsym[s_] == 0:
            continue
        assert ch.tab_lo[s_] == int(g[f"s{ref_i}_lo"])
        assert ch.tab_nsym[s_] == int(g[f"s{ref_i}_nsym"])
        assert np.array_equal(ch.tab_freq[s_, :ch.tab_nsym[s_]], g[f"s{ref_i}_freqs"])
        w = ch.words[ch.lane_off[s_]:ch.lane_off[s_ + 1]]
        ref_bs = g[f"s{ref_i}_bitstream"]
        assert np.array_equal(np.concatenate([w, np.zeros(1, np.uint32)]), ref_bs)
        assert ch.lane_nbits[s_] == int(g[f"s{ref_i}_nbits"])
        assert ch.lane_state[s_] == int(g[f"s{ref_i}_state"])
        ref_i += 1
    assert ref_i == int(g["n_streams"])
    rec = O.decompress_chunk(ch, out_dtype=code)
    want = g["rec"]
    if code == O.DT_F32:
        assert np.array_equal(rec.reshape(-1).view(np.uint32), want.reshape(-1).view(np.uint32))
    else:
        assert np.array_equal(rec.reshape(-1), _bits16(want).reshape(-1))


@pytest.mark.parametrize("name", CHUNKS)
@pytest.mark.parametrize("tile", [1, 7, 256, 1024])
def test_chunk_lane_layout_roundtrip(name, tile):
    """Tiled lanes decode to the same symbols; every lane is a reference stream."""
    g = golden(name)
    code, x, shape = _chunk_input(g)
    b, h, s, d = shape
    ch = O.compress_chunk(x, code, b * h, s * d // 8, float(g["bits"]), tile_blocks=tile)
    rec = O.decompress_chunk(ch, out_dtype=code)
    want = g["rec"]
    if code == O.DT_F32:
        assert np.array_equal(rec.reshape(-1).view(np.uint32), want.reshape(-1).view(np.uint32))
    else:
        assert np.array_equal(rec.reshape(-1), _bits16(want).reshape(-1))


# ---------------------------------------------------------------- compact layout
def test_compact_pack_unpack_bit_exact():
    g = golden("compact.npz")
    for b in (3, 4, 5):
        q = g[f"hand_b{b}_q"]
        assert np.array_equal(O.pack_e8(q, b), g[f"hand_b{b}_packed"])
        assert np.array_equal(O.unpack_e8(g[f"hand_b{b}_packed"], b), g[f"hand_b{b}_unpacked"])
        q = g[f"gauss_b{b}_q"][g[f"gauss_b{b}_inrange"]]
        assert np.array_equal(O.pack_e8(q, b), g[f"gauss_b{b}_packed"])
        assert np.array_equal(O.unpack_e8(g[f"gauss_b{b}_packed"], b), g[f"gauss_b{b}_unpacked"])
    out = O.unpack_e8_4bit_f16(g["gauss_b4_packed"], g["u4_scales"], g["u4_head"])
    assert np.array_equal(out.view(np.uint16), _bits16(g["u4_out"]))


def test_normalisation_needing_many_passes():
    """Many rare symbols: the reference's fix-up loop needs hundreds of passes (no early cap)."""
    counts = np.array([10 ** 6] + [1] * 600 + [3, 5, 9], dtype=np.int64)
    a = O.normalize_freqs_numpy(counts)
    b = O.normalize_freqs_stable(counts)
    assert a.sum() == O.L and np.array_equal(a, b)  # entries at 1 never move, so ties cannot matter
    counts = np.array([500, 400] + [1] * 1000 + [0, 0], dtype=np.int64)
    a = O.normalize_freqs_numpy(counts)
    assert a.sum() == O.L and np.array_equal(a, O.normalize_freqs_stable(counts))
