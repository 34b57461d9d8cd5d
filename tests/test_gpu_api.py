"""The reference-facing API (latticequant_b200.core / .llm / .allocation) on the GPU,
checked against fixtures produced by the reference itself."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import lq_oracle as O

pytestmark = pytest.mark.gpu


def _u32(a):
    return np.asarray(a).view(np.uint32)


def _bits16(t):
    return t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


# ---------------------------------------------------------------- core
def test_encode_and_quantize_e8():
    from latticequant_b200.core import e8_quantizer as E

    g = golden("e8.npz")
    x = torch.from_numpy(g["x"])
    assert np.array_equal(_u32(E.encode_e8(x).numpy()), _u32(g["e8"]))       # CPU in, CPU out
    assert np.array_equal(_u32(E.encode_d8(x.cuda()).cpu().numpy()), _u32(g["d8"]))
    p = golden("pipeline.npz")
    for b in (3, 4, 5):
        xb = torch.from_numpy(p[f"b{b}_x"]).cuda()
        sc = float(p[f"b{b}_scale"])
        xhat = E.quantize_e8(xb, sc)
        want = (torch.from_numpy(p[f"b{b}_q"]) * np.float32(sc)).numpy()
        assert np.array_equal(_u32(xhat.cpu().numpy()), _u32(want))


def test_symbols_roundtrip():
    from latticequant_b200.core import entropy_coder as EC

    g = golden("symbols.npz")
    cos, free, c8h = EC.e8_to_symbols(torch.from_numpy(g["q"]).cuda())
    assert np.array_equal(cos.cpu().numpy(), g["coset"])
    assert np.array_equal(free.cpu().numpy(), g["free"])
    assert np.array_equal(c8h.cpu().numpy(), g["c8h"])
    back = EC.symbols_to_e8(cos, free, c8h)
    assert np.array_equal(back.cpu().numpy(), g["back"])


def test_rans_streams_match_reference():
    from latticequant_b200.core import gpu_ans as G

    g = golden("rans.npz")
    streams, tables = [], []
    for i in range(int(g["n_cases"])):
        t = G.build_rans_table(g[f"c{i}_counts"], list(g[f"c{i}_alphabet"]))
        bs, st, nb = G.rans_encode(g[f"c{i}_syms"], t)
        assert nb == int(g[f"c{i}_nbits"]) and st == int(g[f"c{i}_state"]), i
        assert np.array_equal(bs, g[f"c{i}_bitstream"]), i
        dec = G.rans_decode_cpu(bs, nb, st, t, len(g[f"c{i}_syms"]))
        assert np.array_equal(dec, g[f"c{i}_decoded"]), i
        streams.append(G.RANSStream(bitstream=bs, n_bits=nb, initial_state=st, n_symbols=len(g[f"c{i}_syms"]),
                                    table=t))
    out = G.gpu_rans_decode(streams)
    for i, o in enumerate(out):
        assert np.array_equal(o, g[f"c{i}_decoded"]), i
    t = G.build_rans_table(g["c0_counts"], list(g["c0_alphabet"]))
    dec = G.rans_decode_cpu(g["c0_bitstream"], int(g["trunc_nbits"]), int(g["c0_state"]), t, len(g["c0_syms"]))
    assert np.array_equal(dec, g["trunc_decoded"])  # the reference's stop at n_bits


def test_pipeline_streams_through_api():
    from latticequant_b200.core import e8_quantizer as E
    from latticequant_b200.core import entropy_coder as EC
    from latticequant_b200.core import gpu_ans as G

    p = golden("pipeline.npz")
    for b in (3, 4, 5):
        k = f"b{b}"
        q = E.encode_e8(torch.from_numpy(p[k + "_x"]).cuda() / np.float32(p[k + "_scale"]))
        assert np.array_equal(q.cpu().numpy(), p[k + "_q"])
        cos, free, c8h = EC.e8_to_symbols(q)
        syms = torch.cat([free, c8h[:, None]], 1).cpu().numpy()
        cos = cos.cpu().numpy()
        si = 0
        cols, tabs = [], []
        for c in (0, 1):
            m = cos == c
            if not m.any():
                continue
            for idx in range(8):
                col = syms[m, idx]
                alphabet, counts = O.stream_alphabet(col)
                tabs.append(G.build_rans_table(counts, alphabet))
                cols.append(col)
        res = G.rans_encode_many(cols, tabs)
        for si, (bs, st, nb) in enumerate(res):
            assert np.array_equal(bs, p[f"{k}_s{si}_bitstream"]) and st == int(p[f"{k}_s{si}_state"])


def test_compact_api():
    from latticequant_b200.core import compact_storage as CS
    from latticequant_b200.core.triton_dequant import triton_unpack_e8_4bit

    g = golden("compact.npz")
    for b in (3, 4, 5):
        q = torch.from_numpy(g[f"hand_b{b}_q"])
        assert np.array_equal(CS.pack_e8(q, b).numpy(), g[f"hand_b{b}_packed"])
        assert np.array_equal(CS.unpack_e8(torch.from_numpy(g[f"hand_b{b}_packed"]), b).numpy(),
                              g[f"hand_b{b}_unpacked"])
        qg = torch.from_numpy(g[f"gauss_b{b}_q"]).cuda()
        ir = CS.check_representable(qg, b)
        assert np.array_equal(ir.cpu().numpy(), g[f"gauss_b{b}_inrange"])
        valid, coset = CS.validate_e8(qg)
        assert bool(valid.all())
    for i, qb in enumerate(g["bad_q"]):
        if g["bad_rejected"][i]:
            with pytest.raises(ValueError):
                CS.pack_e8(torch.from_numpy(qb[None]).cuda(), 4)
    p4 = torch.from_numpy(g["gauss_b4_packed"]).cuda()
    out = triton_unpack_e8_4bit(p4, torch.from_numpy(g["u4_scales"]).cuda(), torch.from_numpy(g["u4_head"]).cuda())
    assert np.array_equal(_bits16(out), g["u4_out"].view(np.uint16))


# ---------------------------------------------------------------- cache
def test_cache_update_sequence_matches_reference():
    """Prefill + decode steps on two layers: every returned K/V bit-identical to the reference."""
    from latticequant_b200.llm.compressed_kv_cache import CompressedKVCache

    g = golden("cache.npz")
    cache = CompressedKVCache(bits_per_dim=4)
    for i in range(int(g["n_steps"])):
        k = torch.from_numpy(g[f"u{i}_k"]).view(torch.float16).cuda()
        v = torch.from_numpy(g[f"u{i}_v"]).view(torch.float16).cuda()
        kf, vf = cache.update(k, v, layer_idx=int(g[f"u{i}_layer"]))
        assert np.array_equal(_bits16(kf), g[f"u{i}_kfull"].view(np.uint16)), i
        assert np.array_equal(_bits16(vf), g[f"u{i}_vfull"].view(np.uint16)), i
    assert cache.total_vectors == int(g["total_vectors"])
    assert cache.get_seq_length(0) == int(g["seq0"])
    assert cache.fp16_equivalent_bytes() == int(g["fp16_equivalent_bytes"])
    assert cache.decompressed_resident_bytes() == int(g["decompressed_resident_bytes"])
    # lane layout: no spare word per stream; within 2% of the reference's count
    assert abs(cache.compressed_bytes() - int(g["compressed_bytes"])) < 0.02 * int(g["compressed_bytes"])
    assert "CompressedKVCache Report" in cache.memory_report()


@pytest.mark.parametrize("name", ["chunk_cfg2k.npz", "chunk_cfg2v.npz", "chunk_f16_b3.npz", "chunk_f16_b5.npz",
                                  "chunk_decode1.npz", "chunk_cfg1.npz"])
def test_reference_layout_chunks(name):
    """tile_blocks=None + numpy tables: the reference's own chunk, byte for byte."""
    from latticequant_b200.llm.compressed_kv_cache import CompressedKVCache

    g = golden(name)
    code = O.dtype_code(str(g["dtype"]))
    shape = tuple(int(v) for v in g["shape"])
    if code == O.DT_F32:
        x = torch.from_numpy(g["x"]).reshape(shape).cuda()
    else:
        x = torch.from_numpy(g["x"]).view(torch.float16 if code == O.DT_F16 else torch.bfloat16).reshape(shape).cuda()
    cache = CompressedKVCache(bits_per_dim=int(g["bits"]), tile_blocks=None, table_mode="numpy")
    chunk, deq = cache._compress_tensor(x)
    # update()'s output uses the fp32 scale; torch's CPU sqrt is off by one ulp on a few heads of
    # large tensors (IEEE here), so compare per head: exact on >= 99% of heads, <= 2 ulp elsewhere
    want_deq = g["deq"]
    nh = shape[0] * shape[1]
    if code == O.DT_F32:
        got = deq.cpu().numpy().view(np.int32).reshape(nh, -1).astype(np.int64)
        ref = want_deq.view(np.int32).reshape(nh, -1).astype(np.int64)
    else:
        got = _bits16(deq).astype(np.int64).reshape(nh, -1)
        ref = want_deq.view(np.uint16).astype(np.int64).reshape(nh, -1)
    d = np.abs(got - ref).max(axis=1)
    assert (d == 0).mean() >= 0.99 and d.max() <= 2
    assert np.array_equal(_bits16(chunk.scales), g["scales_f16"].view(np.uint16))
    assert np.array_equal(chunk.coset_packed.cpu().numpy(), g["coset_packed"])
    assert len(chunk.streams) == int(g["n_streams"])
    for i, s in enumerate(chunk.streams):
        assert np.array_equal(s.bitstream, g[f"s{i}_bitstream"]), i
        assert s.n_bits == int(g[f"s{i}_nbits"]) and s.initial_state == int(g[f"s{i}_state"])
        assert tuple(chunk.stream_meta[i][:2]) == tuple(g["stream_meta"][i][:2])
    # the reference counts one spare word per stream
    ref_bytes = int(g["compressed_bytes"])
    ours = 4 * chunk.gpu_bitstream.numel() + chunk.coset_packed.numel() + 2 * chunk.scales.numel()
    assert ours + 4 * int(g["n_streams"]) == ref_bytes
    rec = cache._decompress_chunk(chunk)
    want = g["rec"]
    got = rec.cpu().numpy() if code == O.DT_F32 else _bits16(rec)
    assert np.array_equal(np.asarray(got).view(np.uint32 if code == O.DT_F32 else np.uint16).reshape(-1),
                          want.view(np.uint32 if code == O.DT_F32 else np.uint16).reshape(-1))


def test_tiled_chunks_decode_like_reference():
    """Default lane tiles: _decompress_chunk equals the reference's; lanes decode with rans_decode_cpu."""
    from latticequant_b200.core import gpu_ans as G
    from latticequant_b200.llm.compressed_kv_cache import CompressedKVCache

    g = golden("chunk_cfg2k.npz")
    x = torch.from_numpy(g["x"]).view(torch.bfloat16).reshape(tuple(int(v) for v in g["shape"])).cuda()
    cache = CompressedKVCache(bits_per_dim=4)
    chunk, _ = cache._compress_tensor(x)
    rec = cache._decompress_chunk(chunk)
    assert np.array_equal(_bits16(rec).reshape(-1), g["rec"].view(np.uint16).reshape(-1))
    for s, (c, idx, n) in list(zip(chunk.streams, chunk.stream_meta))[:40]:
        out = O.rans_decode(s.bitstream, s.n_bits, s.initial_state, O.table_from_freqs(s.table.freqs,
                                                                                     s.table.alphabet), n)
        assert np.array_equal(out, G.rans_decode_cpu(s.bitstream, s.n_bits, s.initial_state, s.table, n))


def test_decode_path_never_decompresses():
    """test_decode_no_redecompress (llm/compressed_kv_cache.py:623-660)."""
    from latticequant_b200.llm.compressed_kv_cache import CompressedKVCache

    calls = [0]
    orig = CompressedKVCache._decompress_chunk

    def counting(self, chunk):
        calls[0] += 1
        return orig(self, chunk)

    CompressedKVCache._decompress_chunk = counting
    try:
        cache = CompressedKVCache(bits_per_dim=4)
        torch.manual_seed(42)
        for layer in range(4):
            cache.update(torch.randn(1, 8, 64, 128, device="cuda", dtype=torch.float16),
                         torch.randn(1, 8, 64, 128, device="cuda", dtype=torch.float16), layer_idx=layer)
        calls[0] = 0
        for _ in range(8):
            for layer in range(4):
                k_out, _ = cache.update(torch.randn(1, 8, 1, 128, device="cuda", dtype=torch.float16),
                                        torch.randn(1, 8, 1, 128, device="cuda", dtype=torch.float16), layer)
    finally:
        CompressedKVCache._decompress_chunk = orig
    assert calls[0] == 0
    assert k_out.shape == (1, 8, 72, 128) and not torch.isnan(k_out).any()


def test_variable_rate_cache_and_uncompressible():
    from latticequant_b200.allocation.eval_alloc import VariableRateKVCache
    from latticequant_b200.llm.compressed_kv_cache import CompressedKVCache

    sched = [{'K': 3, 'V': 5}, {'K': 5, 'V': 4}]
    vc = VariableRateKVCache(sched, eval_only_no_entropy=False)
    torch.manual_seed(1)
    for layer in range(2):
        k = torch.randn(1, 4, 32, 128, device="cuda", dtype=torch.bfloat16)
        v = torch.randn(1, 4, 32, 128, device="cuda", dtype=torch.bfloat16)
        vc.update(k, v, layer)
        assert vc._comp_keys[layer].chunks[0].bits_per_dim == sched[layer]['K']
        assert vc._comp_values[layer].chunks[0].bits_per_dim == sched[layer]['V']
        rec = vc._decompress_chunk(vc._comp_keys[layer].chunks[0])
        assert rec.shape == k.shape
    c = CompressedKVCache(4)
    kf, _ = c.update(torch.randn(1, 2, 3, 12, device="cuda"), torch.randn(1, 2, 3, 12, device="cuda"), 0)
    assert kf.shape == (1, 2, 3, 12) and c.compressed_bytes() == 2 * 1 * 2 * 3 * 12 * 4


# ---------------------------------------------------------------- error paths
def test_alphabet_over_L():
    """The reference loops forever here.  With numpy tables (the reference's own
    normalisation) it is reported as ValueError; with device tables the chunk
    takes the outlier side channel and decodes exactly."""
    from latticequant_b200.llm.compressed_kv_cache import CompressedKVCache

    # one head of 1085 blocks, two spikes of +-1: they land on lattice values +-510 of the same
    # stream, whose alphabet [min-2, max+2] then has 1025 > L symbols (checked with the oracle)
    x = torch.zeros(1, 1, 1085, 8, device="cuda")
    x[0, 0, 0, 0] = 1.0
    x[0, 0, 1, 0] = -1.0
    with pytest.raises(ValueError):
        CompressedKVCache(bits_per_dim=5, table_mode="numpy")._compress_tensor(x)
    cache = CompressedKVCache(bits_per_dim=5)
    chunk, deq = cache._compress_tensor(x)
    assert chunk.lanes.n_outliers == 2  # head_dim 8: one block per token
    dec = cache._decompress_chunk(chunk)  # fp16 scale; update()'s deq uses the fp32 scale
    assert torch.allclose(dec, deq, rtol=1e-3, atol=0) and bool((dec.abs().amax() > 0.99).item())


def test_nonfinite_input_raises():
    from latticequant_b200._lib import LatticeQuantError
    from latticequant_b200.llm.compressed_kv_cache import CompressedKVCache

    x = torch.randn(1, 2, 8, 128, device="cuda")
    x[0, 1, 3, 5] = float("nan")
    with pytest.raises(LatticeQuantError):
        CompressedKVCache(4)._compress_tensor(x)


def test_corrupt_lane_metadata_is_reported():
    from latticequant_b200 import codec
    from latticequant_b200._lib import LatticeQuantError

    x = torch.randn(1, 2, 64, 128, device="cuda", dtype=torch.bfloat16)
    chunk, _ = codec.compress(x, 4, tile_blocks=256)
    chunk.lane_off[3] = chunk.n_words + 100  # points past the word buffer
    with pytest.raises(LatticeQuantError):
        codec.decompress(chunk)
