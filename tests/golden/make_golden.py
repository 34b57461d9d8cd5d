"""Generate golden fixtures by running the reference implementation itself.

Runs ONLY where a checkout of the reference is available; its path comes
from the LQ_REFERENCE environment variable (required).  The GPU box never
runs this script; it only reads the committed ``*.npz`` files.

    LQ_REFERENCE=<path to the reference checkout> python tests/golden/make_golden.py

Each fixture is produced by calling the reference's own functions on seeded
inputs (torch.manual_seed / np.random.seed as the reference's tests use):

  e8.npz        encode_d8 / encode_e8 (core/e8_quantizer.py:20-83) on
                random, integer, half-integer and tie-heavy blocks
  scales.npz    sigma2 / scale rule of _compress_tensor
                (llm/compressed_kv_cache.py:183-196) for fp32/fp16/bf16
  symbols.npz   e8_to_symbols / symbols_to_e8 (core/entropy_coder.py:46-89)
  rans.npz      build_rans_table / rans_encode / rans_decode_cpu on the
                distributions of core/gpu_ans.py:390-405 and :480-484
  pipeline.npz  the E8 -> symbols -> rANS pipeline of core/gpu_ans.py:579-655
                at 3/4/5 bits (CPU device)
  chunk_*.npz   CompressedKVCache._compress_tensor chunks (streams, tables,
                coset bits, scales, dequantised output) and their decode
  compact.npz   pack_e8 / unpack_e8 (core/compact_storage.py:87-222) on the
                handcrafted cases (:377-456) and a Gaussian round trip
  cache.npz     CompressedKVCache.update over a prefill + decode steps
  rht.npz       RHT signs, fast_hadamard_transform, RHT forward / inverse and
                LatticeQuantEncoder.encode (core/pipeline.py:33-239)

    python tests/golden/make_golden.py [fixture ...]   (default: all)
"""
import os
import sys

import numpy as np
import torch

REF = os.environ.get("LQ_REFERENCE")
if not REF or not os.path.isdir(REF):
    sys.exit("make_golden.py: set LQ_REFERENCE to the reference checkout (the directory holding core/ and llm/)")
OUT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REF, "core"))
sys.path.insert(0, os.path.join(REF, "llm"))

import e8_quantizer as ref_e8  # noqa: E402
import entropy_coder as ref_ec  # noqa: E402
import gpu_ans as ref_ans  # noqa: E402
import compact_storage as ref_cs  # noqa: E402
import compressed_kv_cache as ref_kv  # noqa: E402
import pipeline as ref_pipe  # noqa: E402


def save(name, **arrs):
    path = os.path.join(OUT, name)
    np.savez_compressed(path, **arrs)
    print(f"wrote {name}: {os.path.getsize(path)} B")


def e8_fixture():
    torch.manual_seed(42)
    parts = []
    parts.append(torch.randn(20000, 8) * 3.0)                      # generic
    parts.append(torch.randn(4000, 8) * 40.0)                      # wide range
    parts.append(torch.randint(-6, 7, (2000, 8)).float())          # exact integers (sign(0) path)
    parts.append(torch.randint(-6, 7, (2000, 8)).float() + 0.5)    # exact half-integers (round ties)
    base = torch.randint(-4, 5, (2000, 8)).float()
    frac = torch.randint(0, 5, (2000, 8)).float() * 0.25            # quarter grid: cost ties
    parts.append(base + frac)
    parts.append(torch.randn(2000, 8) * 1e-3)                      # near zero
    parts.append(torch.zeros(16, 8))
    x = torch.cat(parts).float()
    save("e8.npz", x=x.numpy(), d8=ref_e8.encode_d8(x.clone()).numpy(), e8=ref_e8.encode_e8(x.clone()).numpy())


def scales_fixture():
    torch.manual_seed(42)
    out = {}
    cases = [("f32", torch.float32, (2, 4, 37, 128)), ("f16", torch.float16, (1, 8, 64, 128)),
             ("bf16", torch.bfloat16, (1, 8, 64, 128)), ("pervec", torch.float32, (1, 512, 1, 128)),
             ("big", torch.bfloat16, (1, 3, 1024, 128)), ("hd64", torch.float32, (3, 2, 10, 64)),
             ("zero", torch.float32, (1, 2, 4, 16))]
    for name, dt, shape in cases:
        t = torch.randn(*shape) * torch.exp(torch.randn(shape[0], shape[1], 1, 1))
        if name == "zero":
            t[:, 0] = 0.0
        t = t.to(dt)
        for bits in (3, 4, 5):
            # llm/compressed_kv_cache.py:183-196, executed by torch exactly as written there
            batch, heads, seq, hd = t.shape
            bph = seq * (hd // 8)
            th = t.float().reshape(batch * heads, bph, 8)
            sigma2 = (th ** 2).mean(dim=(1, 2))
            tv = 2 * torch.pi * torch.e * sigma2 * (4.0 ** (-bits))
            s32 = torch.where(sigma2 < 1e-12, torch.ones_like(tv.sqrt()), tv.sqrt())
            cache = ref_kv.CompressedKVCache(bits_per_dim=bits, eval_only_no_entropy=True)
            chunk, deq = cache._compress_tensor(t)
            assert torch.equal(chunk.scales, s32.to(torch.float16))
            key = f"{name}_b{bits}"
            out[name + "_x"] = t.float().numpy() if dt == torch.float32 else t.view(torch.int16).numpy()
            out[key + "_sigma2"] = sigma2.numpy()
            out[key + "_s32"] = s32.numpy()
            out[key + "_s16"] = chunk.scales.view(torch.int16).numpy()
            out[key + "_deq"] = deq.numpy() if dt == torch.float32 else deq.view(torch.int16).numpy()
    save("scales.npz", **out)


def symbols_fixture():
    torch.manual_seed(42)
    x = torch.randn(20000, 8) * 5.0
    q = ref_e8.encode_e8(x)
    coset, free, c8h = ref_ec.e8_to_symbols(q)
    back = ref_ec.symbols_to_e8(coset, free, c8h)
    save("symbols.npz", q=q.numpy(), coset=coset.numpy(), free=free.numpy(), c8h=c8h.numpy(), back=back.numpy())


def rans_fixture():
    np.random.seed(42)
    cases = [
        (list(range(-5, 6)), np.array([1, 3, 10, 30, 50, 60, 50, 30, 10, 3, 1], dtype=np.int64), 2000),
        (list(range(5)), np.array([500, 10, 3, 2, 1], dtype=np.int64), 2000),
        (list(range(8)), np.array([13, 12, 13, 12, 13, 12, 13, 12], dtype=np.int64), 2000),
        ([0, 1], np.array([70, 30], dtype=np.int64), 2000),
        (list(range(-3, 4)), np.array([1, 1, 1, 200, 1, 1, 1], dtype=np.int64), 2000),
        (list(range(-15, 16)), np.array([max(1, int(50 * np.exp(-x ** 2 / 10))) for x in range(-15, 16)],
                                        dtype=np.int64), 2000),
        (list(range(-2, 3)), np.array([5, 10, 20, 10, 5], dtype=np.int64), 16),
    ]
    # core/gpu_ans.py:480-484 (the GPU-vs-CPU set), 4 streams each
    for alphabet, counts in [
        (list(range(-8, 9)), np.array([max(1, int(50 * np.exp(-x ** 2 / 6))) for x in range(-8, 9)], dtype=np.int64)),
        (list(range(4)), np.array([200, 20, 5, 1], dtype=np.int64)),
        (list(range(-3, 4)), np.array([5, 10, 20, 50, 20, 10, 5], dtype=np.int64)),
    ]:
        for _ in range(4):
            cases.append((alphabet, counts, 1000))
    # edge cases: single symbol stream, length 1, zero counts, out-of-alphabet symbols
    cases.append(([7], np.array([3], dtype=np.int64), 50))
    cases.append((list(range(-2, 3)), np.array([0, 0, 9, 0, 0], dtype=np.int64), 1))
    cases.append((list(range(3)), np.array([0, 0, 0], dtype=np.int64), 20))
    out = {}
    for i, (alphabet, counts, n) in enumerate(cases):
        table = ref_ans.build_rans_table(counts, alphabet)
        if counts.sum() > 0:
            syms = np.random.choice(alphabet, size=n, p=counts / counts.sum())
        else:
            syms = np.random.choice(alphabet, size=n)
        if i == len(cases) - 1:
            syms = syms.copy()
            syms[::5] = 9  # not in the alphabet: the encoder takes the nearest entry
        bs, state, n_bits = ref_ans.rans_encode(syms, table)
        dec = ref_ans.rans_decode_cpu(bs, n_bits, state, table, len(syms))
        out[f"c{i}_alphabet"] = np.array(alphabet, np.int64)
        out[f"c{i}_counts"] = counts
        out[f"c{i}_freqs"] = table.freqs
        out[f"c{i}_cumfreqs"] = table.cumfreqs
        out[f"c{i}_lookup"] = table.lookup
        out[f"c{i}_syms"] = np.asarray(syms, np.int64)
        out[f"c{i}_bitstream"] = bs
        out[f"c{i}_state"] = np.int64(state)
        out[f"c{i}_nbits"] = np.int64(n_bits)
        out[f"c{i}_decoded"] = dec
    # truncated stream: the reference decoder stops reading at n_bits
    t = 0
    table = ref_ans.build_rans_table(cases[t][1], cases[t][0])
    bs, state, n_bits = ref_ans.rans_encode(out["c0_syms"], table)
    cut = n_bits // 2
    out["trunc_nbits"] = np.int64(cut)
    out["trunc_decoded"] = ref_ans.rans_decode_cpu(bs, cut, state, table, len(out["c0_syms"]))
    out["n_cases"] = np.int64(len(cases))
    save("rans.npz", **out)


def _streams_of(q_cpu):
    coset, free, c8h = ref_ec.e8_to_symbols(q_cpu)
    cos_np = coset.numpy().astype(np.int32)
    all_syms = np.concatenate([free.numpy().astype(np.int64), c8h.numpy().astype(np.int64)[:, None]], axis=1)
    return cos_np, all_syms


def pipeline_fixture():
    # core/gpu_ans.py:579-655 on the CPU device
    torch.manual_seed(42)
    out = {}
    for bits in (3.0, 4.0, 5.0):
        scale = ref_e8.compute_scale(1.0, bits)
        x = torch.randn(10000, 8)
        q = ref_e8.encode_e8(x / scale)
        cos_np, all_syms = _streams_of(q)
        k = f"b{int(bits)}"
        out[k + "_x"] = x.numpy()
        out[k + "_scale"] = np.float64(scale)
        out[k + "_q"] = q.numpy()
        out[k + "_coset"] = cos_np.astype(np.uint8)
        out[k + "_syms"] = all_syms
        si = 0
        for c in (0, 1):
            mask = cos_np == c
            if mask.sum() == 0:
                continue
            for idx in range(8):
                col = all_syms[mask][:, idx]
                unique, ucounts = np.unique(col, return_counts=True)
                lo, hi = int(unique.min()) - 2, int(unique.max()) + 2
                alphabet = list(range(lo, hi + 1))
                cdict = dict(zip(unique.tolist(), ucounts.tolist()))
                counts = np.array([cdict.get(a, 0) for a in alphabet], dtype=np.int64)
                table = ref_ans.build_rans_table(counts, alphabet)
                bs, state, n_bits = ref_ans.rans_encode(col, table)
                out[f"{k}_s{si}_lo"] = np.int64(lo)
                out[f"{k}_s{si}_freqs"] = table.freqs
                out[f"{k}_s{si}_bitstream"] = bs
                out[f"{k}_s{si}_state"] = np.int64(state)
                out[f"{k}_s{si}_nbits"] = np.int64(n_bits)
                si += 1
        out[k + "_nstreams"] = np.int64(si)
    save("pipeline.npz", **out)


def _ref_decode_chunk(chunk):
    """_decompress_chunk (llm/compressed_kv_cache.py:289-332) with rans_decode_cpu per stream."""
    decoded = [ref_ans.rans_decode_cpu(s.bitstream, s.n_bits, s.initial_state, s.table, s.n_symbols)
               for s in chunk.streams]
    n = chunk.n_vectors
    cos_np = ref_kv.unpack_coset_bits(chunk.coset_packed, n).numpy().astype(np.int32)
    all_syms = np.zeros((n, 8), dtype=np.int64)
    si = 0
    for c in (0, 1):
        mask = cos_np == c
        if mask.sum() == 0:
            continue
        rows = np.where(mask)[0]
        for idx in range(8):
            all_syms[rows, idx] = decoded[si]
            si += 1
    q = ref_ec.symbols_to_e8(torch.tensor(cos_np, dtype=torch.long), torch.tensor(all_syms[:, :7]),
                             torch.tensor(all_syms[:, 7]))
    qh = q.reshape(chunk.n_heads, chunk.blocks_per_head, 8)
    res = torch.zeros_like(qh)
    for h in range(chunk.n_heads):
        res[h] = qh[h] * chunk.scales[h].float().item()
    return res.reshape(chunk.orig_shape).to(chunk.orig_dtype)


def chunk_fixture(name, t, bits):
    cache = ref_kv.CompressedKVCache(bits_per_dim=bits)
    chunk, deq = cache._compress_tensor(t)
    rec = _ref_decode_chunk(chunk)
    out = {"x": t.float().numpy() if t.dtype == torch.float32 else t.view(torch.int16).numpy(),
           "dtype": np.array(str(t.dtype)), "bits": np.int64(bits), "shape": np.array(t.shape, np.int64),
           "scales_f16": chunk.scales.view(torch.int16).numpy(), "coset_packed": chunk.coset_packed.numpy(),
           "deq": deq.numpy() if t.dtype == torch.float32 else deq.view(torch.int16).numpy(),
           "rec": rec.numpy() if t.dtype == torch.float32 else rec.view(torch.int16).numpy(), "gpu_bitstream": chunk.gpu_bitstream.numpy(),
           "word_offsets": np.array(chunk.stream_word_offsets, np.int64),
           "stream_meta": np.array(chunk.stream_meta, np.int64).reshape(-1, 3),
           "compressed_bytes": np.int64(cache.compressed_bytes() if False else
                                        4 * chunk.gpu_bitstream.numel() + chunk.coset_packed.numel() +
                                        2 * chunk.scales.numel())}
    for i, s in enumerate(chunk.streams):
        out[f"s{i}_lo"] = np.int64(s.table.alphabet[0])
        out[f"s{i}_nsym"] = np.int64(s.table.n_symbols)
        out[f"s{i}_freqs"] = s.table.freqs
        out[f"s{i}_bitstream"] = s.bitstream
        out[f"s{i}_state"] = np.int64(s.initial_state)
        out[f"s{i}_nbits"] = np.int64(s.n_bits)
        out[f"s{i}_nsymbols"] = np.int64(s.n_symbols)
    out["n_streams"] = np.int64(len(chunk.streams))
    save(name, **out)


def chunks():
    torch.manual_seed(42)
    # config-1 shape at reduced size: per-vector fp16 scale (n_heads = vectors, bph = 16)
    x = torch.randn(2048, 128) * torch.exp(torch.randn(2048, 1) * 0.5)
    chunk_fixture("chunk_cfg1.npz", x.view(1, 2048, 1, 128).float(), 4)
    # config-2 shape at reduced size: K with per-channel log-normal scales and 1 outlier channel x10
    torch.manual_seed(43)
    s_c = torch.exp(torch.randn(1, 8, 1, 128))
    s_c[..., 5] *= 10.0
    k = (torch.randn(1, 8, 64, 128) * s_c).to(torch.bfloat16)
    chunk_fixture("chunk_cfg2k.npz", k, 4)
    v = torch.randn(1, 8, 64, 128).to(torch.bfloat16)
    chunk_fixture("chunk_cfg2v.npz", v, 4)
    for bits in (3, 5):
        torch.manual_seed(44 + bits)
        chunk_fixture(f"chunk_f16_b{bits}.npz", torch.randn(1, 4, 32, 128).to(torch.float16), bits)
    torch.manual_seed(50)
    chunk_fixture("chunk_decode1.npz", torch.randn(1, 8, 1, 128).to(torch.float16), 4)  # one decode token


def compact_fixture():
    out = {}
    for bits in (3, 4, 5):
        R = 2 ** (bits - 1)
        lo, hi = -R, R - 1
        cases = [[0] * 8, [1, 1, 0, 0, 0, 0, 0, 0], [-1, 1, 0, 0, 0, 0, 0, 0], [1, 1, 1, 1, 0, 0, 0, 0], [1] * 8,
                 [1, 0, 0, 0, 0, 0, 0, 1], [2, 0, 0, 0, 0, 0, 0, 0], [-2, -2, 0, 0, 0, 0, 0, 0],
                 [hi, hi - 2, 0, 0, 0, 0, 0, 0], [lo, lo, 0, 0, 0, 0, 0, 0], [lo, hi - 1, 0, 0, 0, 0, 0, 0],
                 [0.5] * 8, [0.5, 0.5, -0.5, -0.5, 0.5, 0.5, -0.5, -0.5], [1.5, -0.5, 0.5, 0.5, 0.5, 0.5, 0.5, 0.5],
                 [-0.5] * 8]
        keep = []
        for c in cases:
            tq = torch.tensor([c], dtype=torch.float32)
            valid, _ = ref_cs.validate_e8(tq)
            if valid.all() and ref_cs.check_representable(tq, bits).all():
                keep.append(c)
        q = torch.tensor(keep, dtype=torch.float32)
        packed = ref_cs.pack_e8(q, bits)
        out[f"hand_b{bits}_q"] = q.numpy()
        out[f"hand_b{bits}_packed"] = packed.numpy()
        out[f"hand_b{bits}_unpacked"] = ref_cs.unpack_e8(packed, bits).numpy()
    torch.manual_seed(42)
    for bits in (3, 4, 5):
        scale = ref_e8.compute_scale(1.0, bits)
        x = torch.randn(10000, 8)
        q = ref_e8.encode_e8(x / scale)
        ir = ref_cs.check_representable(q, bits)
        packed = ref_cs.pack_e8(q[ir], bits)
        out[f"gauss_b{bits}_q"] = q.numpy()
        out[f"gauss_b{bits}_inrange"] = ir.numpy()
        out[f"gauss_b{bits}_packed"] = packed.numpy()
        out[f"gauss_b{bits}_unpacked"] = ref_cs.unpack_e8(packed, bits).numpy()
    # 4-bit GPU unpack semantics (core/triton_dequant.py:45-132): (c + 0.5*coset) * scale[head] -> fp16
    p4 = torch.tensor(out["gauss_b4_packed"])
    n = p4.shape[0]
    scales = torch.rand(7) * 0.5 + 0.1
    head = torch.randint(0, 7, (n,), dtype=torch.int32)
    ref = (ref_cs.unpack_e8(p4, 4) * scales[head.long()][:, None]).to(torch.float16)
    out["u4_scales"] = scales.numpy()
    out["u4_head"] = head.numpy()
    out["u4_out"] = ref.view(torch.int16).numpy()
    # strict rejects (core/compact_storage.py:459-489)
    R = 8
    bad = [[1.0, 0, 0, 0, 0, 0, 0, 0], [1.0, 0.5, 0, 0, 0, 0, 0, 0], [R + 5.0, -R - 5.0, 0, 0, 0, 0, 0, 0],
           [float(R), float(R), 0, 0, 0, 0, 0, 0], [-R - 1.0, -R - 1.0, 0, 0, 0, 0, 0, 0]]
    rej = []
    for b in bad:
        try:
            ref_cs.pack_e8(torch.tensor([b]), 4)
            rej.append(0)
        except ValueError:
            rej.append(1)
    out["bad_q"] = np.array(bad, np.float32)
    out["bad_rejected"] = np.array(rej, np.int64)
    save("compact.npz", **out)


def cache_fixture():
    # test_incremental_decode / test_multi_layer_decode shapes on CPU (llm/compressed_kv_cache.py:477-593)
    torch.manual_seed(42)
    cache = ref_kv.CompressedKVCache(bits_per_dim=4)
    out = {}
    steps = [(64, 0), (64, 1), (1, 0), (1, 1), (1, 0), (1, 1)]
    for i, (s, layer) in enumerate(steps):
        k = torch.randn(1, 8, s, 128, dtype=torch.float16)
        v = torch.randn(1, 8, s, 128, dtype=torch.float16)
        kf, vf = cache.update(k, v, layer_idx=layer)
        out[f"u{i}_k"] = k.view(torch.int16).numpy()
        out[f"u{i}_v"] = v.view(torch.int16).numpy()
        out[f"u{i}_kfull"] = kf.view(torch.int16).numpy()
        out[f"u{i}_vfull"] = vf.view(torch.int16).numpy()
        out[f"u{i}_layer"] = np.int64(layer)
    out["compressed_bytes"] = np.int64(cache.compressed_bytes())
    out["fp16_equivalent_bytes"] = np.int64(cache.fp16_equivalent_bytes())
    out["decompressed_resident_bytes"] = np.int64(cache.decompressed_resident_bytes())
    out["total_vectors"] = np.int64(cache.total_vectors)
    out["seq0"] = np.int64(cache.get_seq_length(0))
    out["n_steps"] = np.int64(len(steps))
    save("cache.npz", **out)


def rht_fixture():
    out = {}
    # signs of RHT(d, seed) (core/pipeline.py:81-101)
    for d in (8, 64, 128):
        for seed in (0, 7):
            out[f"signs_d{d}_s{seed}"] = ref_pipe.RHT(d, seed=seed).signs.numpy()
    torch.manual_seed(3)
    for d in (8, 64, 128, 256):
        x = torch.randn(32, d) * torch.exp(torch.randn(32, 1))
        out[f"fwht_x_d{d}"] = x.numpy()
        out[f"fwht_y_d{d}"] = ref_pipe.fast_hadamard_transform(x).numpy()
    r = ref_pipe.RHT(128, seed=0)
    v = torch.randn(64, 128)
    out["rht_v"] = v.numpy()
    out["rht_w"] = r.forward(v).numpy()
    out["rht_inv"] = r.inverse(r.forward(v)).numpy()
    # LatticeQuantEncoder.encode (core/pipeline.py:151-205)
    torch.manual_seed(42)
    for bits in (3, 4, 5):
        enc = ref_pipe.LatticeQuantEncoder(128, bits, rht_seed=0)
        v = torch.randn(256, 128)
        e = enc.encode(v)
        out[f"enc{bits}_v"] = v.numpy()
        for key in ("v_hat", "w", "w_hat", "coset", "free_coords", "coord8_half"):
            out[f"enc{bits}_{key}"] = e[key].numpy()
        out[f"enc{bits}_scale"] = np.float64(e["scale"])
        out[f"enc{bits}_sigma2"] = np.float64(e["sigma2"])
    save("rht.npz", **out)


FIXTURES = {"e8": e8_fixture, "scales": scales_fixture, "symbols": symbols_fixture, "rans": rans_fixture,
            "pipeline": pipeline_fixture, "chunks": chunks, "compact": compact_fixture, "cache": cache_fixture,
            "rht": rht_fixture}

if __name__ == "__main__":
    for name in (sys.argv[1:] or list(FIXTURES)):
        FIXTURES[name]()
