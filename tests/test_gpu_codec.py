"""CUDA path vs the CPU oracle and the reference-generated fixtures (needs a B200).

Bar: bit-exact for lattice points, symbols, coset bits, tables, bitstreams and
decoded values; fp32 scales within 1 ulp of the reference (torch's CPU sqrt
is not correctly rounded on large tensors; ours is IEEE, as is the oracle's).
"""
import ctypes

import math

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import lq_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lq():
    from latticequant_b200 import _lib, codec

    _lib.lib()
    return _lib, codec


def _u32(a):
    return np.asarray(a).view(np.uint32)


def _bits16(a):
    return np.asarray(a).view(np.uint16)


def _to_dev(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype=dtype).cuda() if dtype is not None else \
        torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _torch_input(x_np, code):
    if code == O.DT_F32:
        return torch.from_numpy(np.ascontiguousarray(x_np, np.float32)).cuda()
    t = torch.from_numpy(np.ascontiguousarray(x_np.view(np.int16)))
    return t.view(torch.float16 if code == O.DT_F16 else torch.bfloat16).cuda()


def test_library_loads_and_exports(lq):
    _lib, _ = lq
    lib = _lib.lib()
    for name in _lib.exported_symbols():
        assert hasattr(lib, name), name
    assert lib.lq_version() >= 100


def test_encode_e8_d8_golden(lq):
    _lib, _ = lq
    g = golden("e8.npz")
    x = torch.from_numpy(g["x"]).cuda()
    for d8, key in ((0, "e8"), (1, "d8")):
        out = torch.empty_like(x)
        _lib.check(_lib.lib().lq_encode_e8(_lib.ptr(x), x.shape[0], _lib.ptr(out), d8, _lib.stream_handle()), "e8")
        assert np.array_equal(_u32(out.cpu().numpy()), _u32(g[key]))


@pytest.mark.parametrize("case,code", [("f32", O.DT_F32), ("f16", O.DT_F16), ("bf16", O.DT_BF16),
                                       ("pervec", O.DT_F32), ("big", O.DT_BF16), ("hd64", O.DT_F32),
                                       ("zero", O.DT_F32)])
@pytest.mark.parametrize("bits", [3, 4, 5])
def test_head_scales_golden(lq, case, code, bits):
    _lib, codec = lq
    g = golden("scales.npz")
    x_np = g[f"{case}_x"]
    k = f"{case}_b{bits}"
    b, h, s, d = x_np.shape
    x = _torch_input(x_np, code)
    geom = codec.Geometry(1, b * h, s * d // 8, 1024)
    cd = codec.Codec(geom)
    cd.scales(x, bits)
    torch.cuda.synchronize()
    assert np.array_equal(_u32(cd.sigma2.cpu().numpy()), _u32(g[k + "_sigma2"]))
    s32 = cd.scale_f32.cpu().numpy()
    d_ = np.abs(s32.view(np.int32).astype(np.int64) - g[k + "_s32"].view(np.int32).astype(np.int64))
    assert d_.max() <= 1 and (d_ == 0).mean() >= 0.99
    # and exactly the oracle's (both IEEE sqrt of the same fp32 product)
    xin = x_np if code == O.DT_F32 else x_np.view(np.uint16)
    _, o32, o16 = O.head_scales(xin, b * h, bits, code)
    assert np.array_equal(_u32(s32), _u32(o32))
    assert np.array_equal(cd.scale_f16.cpu().numpy().view(np.uint16), o16)


def _oracle_chunk(x_np, code, n_heads, bph, bits, tile, s32=None):
    xin = x_np if code == O.DT_F32 else x_np.view(np.uint16)
    return O.compress_chunk(xin, code, n_heads, bph, bits, tile_blocks=tile, scale_f32=s32, ties="stable")


@pytest.mark.parametrize("shape,dt,bits", [((1, 8, 64, 128), torch.bfloat16, 4), ((2, 4, 33, 128), torch.float32, 3),
                                           ((1, 3, 17, 64), torch.float16, 5), ((1, 512, 1, 128), torch.float32, 4),
                                           ((1, 8, 1, 128), torch.float16, 4), ((1, 2, 5, 16), torch.bfloat16, 4)])
@pytest.mark.parametrize("tile", [32, 1024, None])
def test_compress_matches_oracle_bytes(lq, shape, dt, bits, tile):
    _lib, codec = lq
    torch.manual_seed(7)
    x = (torch.randn(*shape) * torch.exp(torch.randn(shape[0], shape[1], 1, 1))).to(dt)
    code = O.dtype_code(dt)
    b, h, s, d = shape
    n_heads, bph = b * h, s * d // 8
    x_np = x.float().numpy() if dt == torch.float32 else x.view(torch.int16).numpy()
    q_dev = torch.empty(n_heads * bph, 8, dtype=torch.float32, device="cuda")
    chunk, deq = codec.compress(x.cuda(), bits, tile_blocks=tile, keep_deq=True, q_out=q_dev)
    tb = chunk.geom.tile_blocks
    ref = _oracle_chunk(x_np, code, n_heads, bph, bits, tb)
    # scales, lattice points, coset bits
    assert np.array_equal(_u32(chunk.scale_f32.cpu().numpy()), _u32(ref.scale_f32))
    q_ref, cos_ref, sym_ref, deq_ref = O.quantize_chunk(x_np if code == O.DT_F32 else x_np.view(np.uint16), code,
                                                        n_heads, bph, ref.scale_f32, out_dtype=code)
    assert np.array_equal(_u32(q_dev.cpu().numpy()), _u32(q_ref))
    cw = chunk.coset_words.cpu().numpy().view(np.uint8)[: (n_heads * bph + 7) // 8]
    assert np.array_equal(cw, ref.coset_packed)
    dq = deq.reshape(-1).cpu()
    if dt == torch.float32:
        assert np.array_equal(_u32(dq.numpy()), _u32(deq_ref.reshape(-1)))
    else:
        assert np.array_equal(dq.view(torch.int16).numpy().view(np.uint16), deq_ref.reshape(-1))
    # tables (stable tie rule) and every lane byte for byte
    assert np.array_equal(chunk.tab_lo.cpu().numpy(), ref.tab_lo)
    assert np.array_equal(chunk.tab_nsym.cpu().numpy(), ref.tab_nsym)
    fr = chunk.tab_freq.cpu().numpy().view(np.uint16).astype(np.int32)
    for s_ in range(16):
        n = ref.tab_nsym[s_]
        assert np.array_equal(fr[s_, :n], ref.tab_freq[s_, :n]), s_
    assert np.array_equal(chunk.tile_n0.cpu().numpy(), ref.tile_n0.astype(np.int32))
    assert chunk.n_words == ref.words.size
    assert np.array_equal(_u32(chunk.lane_off.cpu().numpy()), ref.lane_off)
    assert np.array_equal(_u32(chunk.lane_nbits.cpu().numpy()), ref.lane_nbits)
    assert np.array_equal(_u32(chunk.lane_state.cpu().numpy()), ref.lane_state)
    assert np.array_equal(_u32(chunk.words[: chunk.n_words].cpu().numpy()), ref.words)
    # decode back: symbols and fp16-scaled values, bit-exact vs the oracle
    out, sym = codec.decompress(chunk, want_symbols=True)
    assert np.array_equal(sym.cpu().numpy(), sym_ref)
    rec_ref = O.decompress_chunk(ref, out_dtype=code)
    if dt == torch.float32:
        assert np.array_equal(_u32(out.reshape(-1).cpu().numpy()), _u32(rec_ref.reshape(-1)))
    else:
        assert np.array_equal(out.reshape(-1).cpu().view(torch.int16).numpy().view(np.uint16), rec_ref.reshape(-1))


CHUNKS = ["chunk_cfg1.npz", "chunk_cfg2k.npz", "chunk_cfg2v.npz", "chunk_f16_b3.npz", "chunk_f16_b5.npz",
          "chunk_decode1.npz"]


@pytest.mark.parametrize("name", CHUNKS)
def test_reference_streams_byte_identical(lq, name):
    """One tile per chunk + the reference's numpy tables: our lanes ARE the reference streams."""
    _lib, codec = lq
    g = golden(name)
    code = O.dtype_code(str(g["dtype"]))
    shape = tuple(int(v) for v in g["shape"])
    x = _torch_input(g["x"], code).reshape(shape)
    lo = np.zeros(16, np.int32)
    ns = np.zeros(16, np.int32)
    fr = np.zeros((16, O.L), np.int32)
    meta = g["stream_meta"]
    for i in range(int(g["n_streams"])):
        c, idx, _ = meta[i]
        s_ = 8 * c + idx
        lo[s_] = int(g[f"s{i}_lo"])
        ns[s_] = int(g[f"s{i}_nsym"])
        fr[s_, : ns[s_]] = g[f"s{i}_freqs"]
    chunk, _ = codec.compress(x, int(g["bits"]), tile_blocks=None, freqs=(lo, ns, fr))
    assert np.array_equal(chunk.scale_f16.cpu().numpy().view(np.uint16), _bits16(g["scales_f16"]))
    n = chunk.geom.n_vectors
    assert np.array_equal(chunk.coset_words.cpu().numpy().view(np.uint8)[: (n + 7) // 8], g["coset_packed"])
    words = _u32(chunk.words[: chunk.n_words].cpu().numpy())
    off = _u32(chunk.lane_off.cpu().numpy())
    nbits = _u32(chunk.lane_nbits.cpu().numpy())
    st = _u32(chunk.lane_state.cpu().numpy())
    for i in range(int(g["n_streams"])):
        c, idx, _ = meta[i]
        s_ = 8 * c + idx
        lane = np.concatenate([words[off[s_]:off[s_ + 1]], np.zeros(1, np.uint32)])
        assert np.array_equal(lane, g[f"s{i}_bitstream"]), (name, i)
        assert nbits[s_] == int(g[f"s{i}_nbits"]) and st[s_] == int(g[f"s{i}_state"])
    out = codec.decompress(chunk)
    want = g["rec"]
    if code == O.DT_F32:
        assert np.array_equal(_u32(out.reshape(-1).cpu().numpy()), _u32(want.reshape(-1)))
    else:
        assert np.array_equal(out.reshape(-1).cpu().view(torch.int16).numpy().view(np.uint16),
                              _bits16(want).reshape(-1))


def test_reference_streams_decode_golden(lq):
    """lq_rans_decode_streams == rans_decode_cpu on the reference's distributions."""
    _lib, _ = lq
    g = golden("rans.npz")
    n = int(g["n_cases"])
    tabs = [O.table_from_freqs(g[f"c{i}_freqs"], list(g[f"c{i}_alphabet"])) for i in range(n)]
    max_sym = max(t.n_symbols for t in tabs)
    words, boffs, nbits, states, ndec, outoffs = [], [], [], [], [], []
    lookup = np.zeros((n, O.L), np.int32)
    fr = np.zeros((n, max_sym), np.int32)
    cf = np.zeros((n, max_sym), np.int32)
    al = np.zeros((n, max_sym), np.int32)
    tot_w = tot_o = 0
    for i, t in enumerate(tabs):
        bs = g[f"c{i}_bitstream"]
        boffs.append(tot_w * 32)
        words.append(bs)
        tot_w += bs.size
        nbits.append(int(g[f"c{i}_nbits"]))
        states.append(int(g[f"c{i}_state"]))
        ndec.append(len(g[f"c{i}_syms"]))
        outoffs.append(tot_o)
        tot_o += ndec[-1]
        lookup[i] = t.lookup
        fr[i, : t.n_symbols] = t.freqs
        cf[i, : t.n_symbols] = t.cumfreqs[: t.n_symbols]
        al[i, : t.n_symbols] = t.alphabet
    dev = lambda a, dt: torch.from_numpy(np.ascontiguousarray(np.asarray(a).astype(dt))).cuda()
    w = dev(np.concatenate(words).view(np.int32), np.int32)
    out = torch.zeros(tot_o, dtype=torch.int64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    L_ = _lib.lib()
    P = _lib.ptr
    args = [dev(boffs, np.int64), dev(nbits, np.int64), dev(states, np.int64), dev(ndec, np.int64),
            dev(lookup, np.int32), dev(fr, np.int32), dev(cf, np.int32), dev(al, np.int32),
            dev(np.arange(n), np.int32)]
    oo = dev(outoffs, np.int64)
    _lib.check(L_.lq_rans_decode_streams(P(w), w.numel(), *[P(a) for a in args], max_sym, n, P(out), P(oo), P(err),
                                         _lib.stream_handle()), "streams")
    o = out.cpu().numpy()
    assert int(err.item()) == 0
    for i in range(n):
        assert np.array_equal(o[outoffs[i]:outoffs[i] + ndec[i]], g[f"c{i}_decoded"]), i


def test_compact_pack_unpack_golden(lq):
    _lib, _ = lq
    g = golden("compact.npz")
    L_ = _lib.lib()
    P = _lib.ptr
    for b in (3, 4, 5):
        for key in ("hand", "gauss"):
            q = g[f"{key}_b{b}_q"]
            if key == "gauss":
                q = q[g[f"gauss_b{b}_inrange"]]
            qd = torch.from_numpy(np.ascontiguousarray(q)).cuda()
            out = torch.empty(q.shape[0], b, dtype=torch.uint8, device="cuda")
            bad = torch.zeros(2, dtype=torch.int32, device="cuda")
            _lib.check(L_.lq_pack_e8(P(qd), q.shape[0], b, P(out), P(bad), _lib.stream_handle()), "pack")
            assert bad.tolist() == [0, 0]
            assert np.array_equal(out.cpu().numpy(), g[f"{key}_b{b}_packed"])
            back = torch.empty(q.shape[0], 8, dtype=torch.float32, device="cuda")
            _lib.check(L_.lq_unpack_e8(P(out), q.shape[0], b, None, None, P(back), None, _lib.stream_handle()),
                       "unpack")
            assert np.array_equal(back.cpu().numpy(), g[f"{key}_b{b}_unpacked"])
    p4 = torch.from_numpy(g["gauss_b4_packed"]).cuda()
    sc = torch.from_numpy(g["u4_scales"]).cuda()
    hi = torch.from_numpy(g["u4_head"]).cuda()
    o16 = torch.empty(p4.shape[0], 8, dtype=torch.float16, device="cuda")
    _lib.check(L_.lq_unpack_e8(P(p4), p4.shape[0], 4, P(sc), P(hi), None, P(o16), _lib.stream_handle()), "u4")
    assert np.array_equal(o16.cpu().view(torch.int16).numpy().view(np.uint16), _bits16(g["u4_out"]))
    # strict rejects
    bad_q = torch.from_numpy(g["bad_q"]).cuda()
    for i in range(bad_q.shape[0]):
        out = torch.empty(1, 4, dtype=torch.uint8, device="cuda")
        cnt = torch.zeros(2, dtype=torch.int32, device="cuda")
        _lib.check(L_.lq_pack_e8(P(bad_q[i:i + 1].contiguous()), 1, 4, P(out), P(cnt), _lib.stream_handle()), "p")
        assert (int(cnt.sum().item()) > 0) == bool(g["bad_rejected"][i])


def test_full_size_roundtrip_property(lq):
    """Config-2 geometry at full size: decode(encode(x)) reproduces every lattice point."""
    _lib, codec = lq
    torch.manual_seed(1)
    n_chunks, n_heads, seq, hd = 8, 8, 8192, 128
    x = torch.randn(n_chunks * n_heads, seq * hd // 8, 8, device="cuda").to(torch.bfloat16)
    geom = codec.Geometry(n_chunks, n_heads, seq * hd // 8, 1024)
    cd = codec.Codec(geom)
    q = torch.empty(n_chunks * n_heads * seq * hd // 8, 8, dtype=torch.float32, device="cuda")
    cd.scales(x, 4)
    cd.quantize(x, q_out=q)
    cd.build_tables()
    cd.expand_tables()
    cd.entropy_encode()
    out = torch.empty(q.numel(), dtype=torch.float32, device="cuda")
    cd.decode(out)
    assert cd.read_err() == 0
    sc = cd.scale_f16.float().repeat_interleave(seq * hd // 8)
    # symbols carry no sign of zero: decode (like the reference's _decompress_chunk)
    # rebuilds +0.0 where the quantiser's rint produced -0.0
    want = ((q + 0.0) * sc[:, None]).reshape(-1)
    assert torch.equal(out.view(torch.int32), want.view(torch.int32))
    bits_per_dim = (4 * cd.n_words() * 8) / (q.numel())
    assert 3.8 < bits_per_dim < 4.3


@pytest.mark.parametrize("case", ["rare_tail", "two_big_many_ones", "flat", "gaussian_large"])
def test_device_tables_match_oracle_rule(lq, case):
    """lq_build_tables == the oracle's stable-tie normalisation, including many-pass fix-ups."""
    _lib, codec = lq
    rng = np.random.default_rng(5)
    hist = np.zeros(1024, np.int64)
    if case == "rare_tail":
        hist[512] = 10 ** 6
        hist[512 - 300:512 + 300:1] += 1
    elif case == "two_big_many_ones":
        hist[100] = 500
        hist[101] = 400
        hist[102:1015] = 1
    elif case == "flat":
        hist[200:260] = 13
    else:
        v = np.clip(np.round(rng.standard_normal(2_000_000) * 40), -500, 500).astype(np.int64) + 512
        hist = np.bincount(v, minlength=1024).astype(np.int64)
    h = torch.from_numpy(hist.astype(np.int32)).cuda()
    lo = torch.empty(1, dtype=torch.int32, device="cuda")
    ns = torch.empty(1, dtype=torch.int32, device="cuda")
    fr = torch.empty(1, 1024, dtype=torch.int16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    P = _lib.ptr
    _lib.check(_lib.lib().lq_build_tables(P(h), 1, P(lo), P(ns), P(fr), P(err), _lib.stream_handle()), "tables")
    nz = np.nonzero(hist)[0]
    a, b = nz.min() - 2, nz.max() + 2
    counts = np.zeros(b - a + 1, np.int64)
    counts[:] = [hist[i] if 0 <= i < 1024 else 0 for i in range(a, b + 1)]
    want = O.normalize_freqs_stable(counts)
    assert int(err.item()) == 0
    assert int(lo.item()) == a - 512 and int(ns.item()) == len(counts)
    got = fr[0].cpu().numpy().view(np.uint16).astype(np.int32)[: len(counts)]
    assert np.array_equal(got, want)


@pytest.mark.parametrize("tile", [32, 1024])
def test_wide_symbols_take_the_escape_plane(lq, tile):
    """Symbols outside [-127, 127] (a few blocks ~60x the rest of their head)
    do not fit the int8 symbol columns between the quantiser and the lane
    encoder: they travel through the int16 plane of flagged tiles.  Lanes,
    words and decode stay byte-identical to the oracle, and -128 itself (the
    column's escape value) round-trips."""
    _lib, codec = lq
    g = torch.Generator().manual_seed(17)
    b, h, s, d = 1, 2, 256, 128
    x = torch.randn(b, h, s, d, generator=g)
    x[0, 0, 5] *= 60.0
    x[0, 1, 77] *= 60.0
    # one block of -128 in units of its head's scale: with the block's own
    # share in sigma^2, v^2 = c sigma^2 (c = 128^2 * 2 pi e / 4^4) and
    # sigma^2 = (S + 8 v^2) / n give sigma^2 = S / (n - 8c)
    hd = x[0, 1].double().clone()
    hd[200, :8] = 0.0
    c = 128.0 ** 2 * 2 * math.pi * math.e / 4 ** 4
    x[0, 1, 200, :8] = -math.sqrt(c * float((hd ** 2).sum()) / (hd.numel() - 8 * c))
    n_heads, bph = b * h, s * d // 8
    chunk, _ = codec.compress(x.cuda(), 4, tile_blocks=tile)
    ref = _oracle_chunk(x.numpy(), O.DT_F32, n_heads, bph, 4, chunk.geom.tile_blocks)
    _, _, sym_ref, _ = O.quantize_chunk(x.numpy(), O.DT_F32, n_heads, bph, ref.scale_f32, out_dtype=O.DT_F32)
    assert np.abs(sym_ref).max() > 127, "the case must hold symbols beyond the int8 range"
    assert (sym_ref == -128).any(), "and the column's escape value itself"
    assert np.array_equal(chunk.tab_lo.cpu().numpy(), ref.tab_lo)
    assert np.array_equal(chunk.tab_nsym.cpu().numpy(), ref.tab_nsym)
    assert chunk.n_words == ref.words.size
    assert np.array_equal(_u32(chunk.lane_nbits.cpu().numpy()), ref.lane_nbits)
    assert np.array_equal(_u32(chunk.lane_state.cpu().numpy()), ref.lane_state)
    assert np.array_equal(_u32(chunk.words[: chunk.n_words].cpu().numpy()), ref.words)
    out, sym = codec.decompress(chunk, want_symbols=True)
    assert np.array_equal(sym.cpu().numpy(), sym_ref)
    assert np.array_equal(_u32(out.reshape(-1).cpu().numpy()), _u32(O.decompress_chunk(ref, out_dtype=O.DT_F32).reshape(-1)))
