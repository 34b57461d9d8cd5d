"""CPU oracle for the LatticeQuant KV-cache hot path (TEST INFRASTRUCTURE).

This module is the checker, not the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
import it.  It wraps ``oracle/liblq_oracle.so`` (a C restatement of the
reference, see ``lq_oracle.c``) and adds the pieces that must call numpy
exactly as the reference does (table normalisation uses ``np.argsort``).

Reference citations are ``path:line`` inside yoon9728/LatticeQuant.
Parity is pinned against fixtures produced by running the reference itself
(``tests/golden/make_golden.py``), checked by ``tests/test_oracle_golden.py``.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import numpy as np

LOG2_L = 10
L = 1 << LOG2_L
DT_F32, DT_F16, DT_BF16 = 0, 1, 2

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liblq_oracle.so")
_lib = None


def build() -> str:
    """Compile the C oracle with its Makefile (gcc only)."""
    import subprocess

    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


def _p(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else None


def _declare(L_):
    vp, i64, i32, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
    L_.lqo_cascade_sum_f32.argtypes = [vp, i64]
    L_.lqo_cascade_sum_f32.restype = f32
    L_.lqo_head_scales.argtypes = [vp, i32, i64, i64, f32, vp, vp, vp]
    L_.lqo_encode_d8.argtypes = [vp, vp, i64]
    L_.lqo_encode_e8.argtypes = [vp, vp, i64]
    L_.lqo_e8_to_symbols.argtypes = [vp, i64, vp, vp]
    L_.lqo_symbols_to_e8.argtypes = [vp, vp, i64, vp]
    L_.lqo_quantize_chunk.argtypes = [vp, i32, i64, i64, vp, vp, vp, vp, vp, i32]
    L_.lqo_pack_coset_bits.argtypes = [vp, i64, vp]
    L_.lqo_unpack_coset_bits.argtypes = [vp, i64, vp]
    L_.lqo_normalize_freqs_stable.argtypes = [vp, i32, vp]
    L_.lqo_normalize_freqs_stable.restype = i32
    L_.lqo_table_from_freqs.argtypes = [vp, i32, vp, vp]
    L_.lqo_rans_encode.argtypes = [vp, i64, vp, vp, vp, i64, vp]
    L_.lqo_rans_encode.restype = i64
    L_.lqo_rans_decode.argtypes = [vp, i64, i64, i64, vp, vp, vp, i64, vp]
    L_.lqo_pack_e8.argtypes = [vp, i64, i32, vp]
    L_.lqo_unpack_e8.argtypes = [vp, i64, i32, vp]
    L_.lqo_unpack_e8_4bit_f16.argtypes = [vp, vp, vp, i64, vp]
    L_.lqo_chunk_tables.argtypes = [vp, vp, i64, vp, vp, vp, vp, vp, vp]
    L_.lqo_chunk_tables.restype = i32
    L_.lqo_lane_capacity_words.argtypes = [i64, i64]
    L_.lqo_lane_capacity_words.restype = i64
    L_.lqo_encode_lanes.argtypes = [vp, vp, i64, i64, vp, vp, vp, vp, i64, vp, vp, vp, vp]
    L_.lqo_encode_lanes.restype = i64
    L_.lqo_decode_lanes.argtypes = [vp, i64, i64, vp, vp, vp, vp, vp, vp, vp, vp]
    L_.lqo_dequant_symbols.argtypes = [vp, vp, i64, i64, vp, vp, i32]
    L_.lqo_codec_roundtrip_batch.argtypes = [vp, i32, i64, i64, i64, f32, i64, vp, i32, i32]
    L_.lqo_codec_roundtrip_batch.restype = i64


def dtype_code(dt) -> int:
    s = str(dt)
    if "bfloat16" in s:
        return DT_BF16
    if "float16" in s:
        return DT_F16
    if "float32" in s:
        return DT_F32
    raise ValueError(f"unsupported dtype {dt}")


def vol_mult(bits: float) -> np.float32:
    """fp32(4 ** -bits): the factor torch multiplies by (llm/compressed_kv_cache.py:192)."""
    return np.float32(4.0 ** (-bits))


# --------------------------------------------------------------------------
# numeric kernels
# --------------------------------------------------------------------------
def cascade_sum_f32(row: np.ndarray) -> np.float32:
    row = np.ascontiguousarray(row, dtype=np.float32)
    return np.float32(lib().lqo_cascade_sum_f32(_p(row), row.size))


def head_scales(x: np.ndarray, n_heads: int, bits: float, dtype: int = DT_F32):
    """Per-head (sigma2, scale_f32, scale_f16 bits): llm/compressed_kv_cache.py:183-196.

    ``x`` holds the raw elements (float32 array, or uint16 bit patterns for
    half / bfloat16 when ``dtype`` says so).
    """
    x = np.ascontiguousarray(x)
    eph = x.size // n_heads
    s2 = np.empty(n_heads, np.float32)
    s32 = np.empty(n_heads, np.float32)
    s16 = np.empty(n_heads, np.uint16)
    lib().lqo_head_scales(_p(x), dtype, n_heads, eph, ctypes.c_float(vol_mult(bits)), _p(s2), _p(s32), _p(s16))
    return s2, s32, s16


def encode_d8(x: np.ndarray) -> np.ndarray:
    """core/e8_quantizer.py:20-58."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, 8)
    out = np.empty_like(x)
    lib().lqo_encode_d8(_p(x), _p(out), x.shape[0])
    return out


def encode_e8(x: np.ndarray) -> np.ndarray:
    """core/e8_quantizer.py:61-83."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, 8)
    out = np.empty_like(x)
    lib().lqo_encode_e8(_p(x), _p(out), x.shape[0])
    return out


def e8_to_symbols(q: np.ndarray):
    """core/entropy_coder.py:46-68 -> (coset uint8 (N,), symbols int32 (N, 8))."""
    q = np.ascontiguousarray(q, dtype=np.float32).reshape(-1, 8)
    n = q.shape[0]
    cos = np.empty(n, np.uint8)
    sym = np.empty((n, 8), np.int32)
    lib().lqo_e8_to_symbols(_p(q), n, _p(cos), _p(sym))
    return cos, sym


def symbols_to_e8(coset: np.ndarray, sym: np.ndarray) -> np.ndarray:
    """core/entropy_coder.py:71-89."""
    coset = np.ascontiguousarray(coset, dtype=np.uint8)
    sym = np.ascontiguousarray(sym, dtype=np.int32).reshape(-1, 8)
    q = np.empty((sym.shape[0], 8), np.float32)
    lib().lqo_symbols_to_e8(_p(coset), _p(sym), sym.shape[0], _p(q))
    return q


def quantize_chunk(x: np.ndarray, dtype: int, n_heads: int, bph: int, scale_f32: np.ndarray, out_dtype: int = DT_F32):
    """x / scale -> E8 -> (q, coset, symbols, dequant): llm/compressed_kv_cache.py:198-228."""
    x = np.ascontiguousarray(x)
    n = n_heads * bph
    q = np.empty((n, 8), np.float32)
    cos = np.empty(n, np.uint8)
    sym = np.empty((n, 8), np.int32)
    deq = np.empty((n, 8), np.float32 if out_dtype == DT_F32 else np.uint16)
    sc = np.ascontiguousarray(scale_f32, dtype=np.float32)
    lib().lqo_quantize_chunk(_p(x), dtype, n_heads, bph, _p(sc), _p(q), _p(cos), _p(sym), _p(deq), out_dtype)
    return q, cos, sym, deq


def pack_coset_bits(coset: np.ndarray) -> np.ndarray:
    """llm/compressed_kv_cache.py:46-54."""
    coset = np.ascontiguousarray(coset, dtype=np.uint8)
    out = np.empty((coset.size + 7) // 8, np.uint8)
    lib().lqo_pack_coset_bits(_p(coset), coset.size, _p(out))
    return out


def unpack_coset_bits(packed: np.ndarray, n: int) -> np.ndarray:
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    out = np.empty(n, np.uint8)
    lib().lqo_unpack_coset_bits(_p(packed), n, _p(out))
    return out


# --------------------------------------------------------------------------
# rANS (core/gpu_ans.py)
# --------------------------------------------------------------------------
@dataclass
class Table:
    lookup: np.ndarray
    freqs: np.ndarray
    cumfreqs: np.ndarray
    alphabet: List[int]
    n_symbols: int


def normalize_freqs_numpy(counts: np.ndarray) -> np.ndarray:
    """core/gpu_ans.py:66-84 verbatim in behaviour, numpy argsort included.

    Raises ValueError where the reference would loop forever (n_sym > L).
    """
    n_sym = len(counts)
    if n_sym > L:
        raise ValueError(f"alphabet of {n_sym} symbols exceeds L={L}")
    total = counts.sum()
    if total == 0:
        freqs = np.ones(n_sym, dtype=np.int32)
    else:
        freqs = np.maximum((counts / total * L).astype(np.int32), 1)
    while freqs.sum() != L:
        diff = L - freqs.sum()
        if diff > 0:
            order = np.argsort(-counts)
            for j in range(abs(diff)):
                freqs[order[j % n_sym]] += 1
        else:
            order = np.argsort(-freqs)
            for j in range(abs(diff)):
                idx = order[j % n_sym]
                if freqs[idx] > 1:
                    freqs[idx] -= 1
    return freqs.astype(np.int32)


def normalize_freqs_stable(counts: np.ndarray) -> np.ndarray:
    """Same normalisation with ties broken by ascending index (the CUDA rule)."""
    counts = np.ascontiguousarray(counts, dtype=np.int64)
    out = np.empty(len(counts), np.int32)
    rc = lib().lqo_normalize_freqs_stable(_p(counts), len(counts), _p(out))
    if rc != 0:
        raise ValueError(f"alphabet of {len(counts)} symbols exceeds L={L}")
    return out


def table_from_freqs(freqs: np.ndarray, alphabet: Sequence[int]) -> Table:
    """core/gpu_ans.py:88-98."""
    freqs = np.ascontiguousarray(freqs, dtype=np.int32)
    n = len(freqs)
    cum = np.empty(n + 1, np.int32)
    lookup = np.empty(L, np.int32)
    lib().lqo_table_from_freqs(_p(freqs), n, _p(cum), _p(lookup))
    return Table(lookup=lookup, freqs=freqs, cumfreqs=cum, alphabet=list(alphabet), n_symbols=n)


def build_rans_table(counts: np.ndarray, alphabet: Sequence[int], ties: str = "numpy") -> Table:
    """core/gpu_ans.py:62-98 (ties='numpy' reproduces the reference on this host)."""
    counts = np.asarray(counts)
    f = normalize_freqs_numpy(counts) if ties == "numpy" else normalize_freqs_stable(counts)
    return table_from_freqs(f, alphabet)


def map_symbols(symbols: np.ndarray, alphabet: Sequence[int]) -> np.ndarray:
    """sym -> alphabet index; absent symbols take the nearest entry, first on ties (core/gpu_ans.py:115-119)."""
    lut = {v: i for i, v in enumerate(alphabet)}
    out = np.empty(len(symbols), np.int32)
    for k, s in enumerate(symbols):
        i = lut.get(int(s))
        if i is None:
            i = min(range(len(alphabet)), key=lambda j: abs(alphabet[j] - int(s)))
        out[k] = i
    return out


def rans_encode(symbols: np.ndarray, table: Table) -> Tuple[np.ndarray, int, int]:
    """core/gpu_ans.py:105-139 -> (words with the spare word, state, n_bits)."""
    idx = np.ascontiguousarray(map_symbols(np.asarray(symbols), table.alphabet))
    n = len(idx)
    cap = (10 * n + 31) // 32 + 2
    words = np.zeros(cap, np.uint32)
    st = np.zeros(1, np.uint32)
    nb = lib().lqo_rans_encode(_p(idx), n, _p(table.freqs), _p(table.cumfreqs), _p(words), cap, _p(st))
    nw = (nb + 31) // 32 + 1
    return words[:nw].copy(), int(st[0]), int(nb)


def rans_decode(bitstream: np.ndarray, n_bits: int, state: int, table: Table, n_symbols: int) -> np.ndarray:
    """core/gpu_ans.py:146-168 -> symbol values (int64)."""
    bs = np.ascontiguousarray(bitstream, dtype=np.uint32)
    out = np.empty(n_symbols, np.int32)
    lib().lqo_rans_decode(_p(bs), bs.size, n_bits, state, _p(table.lookup), _p(table.freqs), _p(table.cumfreqs),
                          n_symbols, _p(out))
    alpha = np.asarray(table.alphabet, dtype=np.int64)
    return alpha[out]


# --------------------------------------------------------------------------
# whole chunks
# --------------------------------------------------------------------------
def stream_alphabet(col: np.ndarray) -> Tuple[List[int], np.ndarray]:
    """llm/compressed_kv_cache.py:246-250: alphabet [min-2, max+2] and counts."""
    lo, hi = int(col.min()) - 2, int(col.max()) + 2
    counts = np.bincount(col - lo, minlength=hi - lo + 1).astype(np.int64)
    return list(range(lo, hi + 1)), counts


@dataclass
class LaneChunk:
    """A chunk in the tiled lane layout (see lq_oracle_codec.c)."""
    n_heads: int
    bph: int
    tile_blocks: int
    scale_f32: np.ndarray
    scale_f16: np.ndarray
    coset: np.ndarray
    coset_packed: np.ndarray
    tab_lo: np.ndarray
    tab_nsym: np.ndarray
    tab_freq: np.ndarray  # (16, L) int32
    words: np.ndarray
    lane_off: np.ndarray
    lane_nbits: np.ndarray
    lane_state: np.ndarray
    tile_n0: np.ndarray

    @property
    def n_vectors(self):
        return self.n_heads * self.bph


def chunk_tables(coset: np.ndarray, sym: np.ndarray, ties: str = "stable"):
    """Per-stream (lo, n_sym, freqs[L]) of a chunk (llm/compressed_kv_cache.py:236-253)."""
    lo = np.zeros(16, np.int32)
    ns = np.zeros(16, np.int32)
    fr = np.zeros((16, L), np.int32)
    for s in range(16):
        c, idx = s >> 3, s & 7
        col = sym[coset == c, idx]
        if col.size == 0:
            continue
        alphabet, counts = stream_alphabet(col.astype(np.int64))
        if len(alphabet) > L:
            raise ValueError(f"stream {s}: alphabet of {len(alphabet)} symbols exceeds L={L}")
        f = normalize_freqs_numpy(counts) if ties == "numpy" else normalize_freqs_stable(counts)
        lo[s] = alphabet[0]
        ns[s] = len(alphabet)
        fr[s, : len(f)] = f
    return lo, ns, fr


def encode_lanes(coset, sym, tile_blocks, tab_lo, tab_ns, tab_fr):
    n = coset.size
    cos = np.ascontiguousarray(coset, np.uint8)
    sy = np.ascontiguousarray(sym, np.int32)
    n_tiles = (n + tile_blocks - 1) // tile_blocks
    cap = lib().lqo_lane_capacity_words(n, tile_blocks)
    words = np.zeros(cap, np.uint32)
    loff = np.zeros(n_tiles * 16 + 1, np.uint32)
    lnb = np.zeros(n_tiles * 16, np.uint32)
    lst = np.zeros(n_tiles * 16, np.uint32)
    tn0 = np.zeros(n_tiles, np.uint32)
    fr = np.ascontiguousarray(tab_fr, np.int32)
    lo = np.ascontiguousarray(tab_lo, np.int32)
    ns = np.ascontiguousarray(tab_ns, np.int32)
    nw = lib().lqo_encode_lanes(_p(cos), _p(sy), n, tile_blocks, _p(lo), _p(ns), _p(fr), _p(words), cap, _p(loff),
                                _p(lnb), _p(lst), _p(tn0))
    if nw < 0:
        raise RuntimeError(f"oracle lane encode failed ({nw})")
    return words[:nw].copy(), loff, lnb, lst, tn0


def decode_lanes(coset, tile_blocks, tab_lo, tab_ns, tab_fr, words, loff, lnb, lst) -> np.ndarray:
    n = coset.size
    sym = np.zeros((n, 8), np.int32)
    w = np.ascontiguousarray(words, np.uint32) if words.size else np.zeros(1, np.uint32)
    lib().lqo_decode_lanes(_p(np.ascontiguousarray(coset, np.uint8)), n, tile_blocks,
                           _p(np.ascontiguousarray(tab_lo, np.int32)), _p(np.ascontiguousarray(tab_ns, np.int32)),
                           _p(np.ascontiguousarray(tab_fr, np.int32)), _p(w), _p(np.ascontiguousarray(loff)),
                           _p(np.ascontiguousarray(lnb)), _p(np.ascontiguousarray(lst)), _p(sym))
    return sym


def compress_chunk(x: np.ndarray, dtype: int, n_heads: int, bph: int, bits: float, tile_blocks: Optional[int] = None,
                   scale_f32: Optional[np.ndarray] = None, ties: str = "stable") -> LaneChunk:
    """CompressedKVCache._compress_tensor (llm/compressed_kv_cache.py:176-287) in the lane layout."""
    n = n_heads * bph
    tb = n if tile_blocks is None else tile_blocks
    if scale_f32 is None:
        _, s32, s16 = head_scales(x, n_heads, bits, dtype)
    else:
        s32 = np.ascontiguousarray(scale_f32, np.float32)
        s16 = np.array([lqo_f32_to_f16(v) for v in s32], np.uint16)
    _, cos, sym, _ = quantize_chunk(x, dtype, n_heads, bph, s32)
    lo, ns, fr = chunk_tables(cos, sym, ties)
    words, loff, lnb, lst, tn0 = encode_lanes(cos, sym, tb, lo, ns, fr)
    return LaneChunk(n_heads, bph, tb, s32, s16, cos, pack_coset_bits(cos), lo, ns, fr, words, loff, lnb, lst, tn0)


def decompress_chunk(ch: LaneChunk, out_dtype: int = DT_F32) -> np.ndarray:
    """CompressedKVCache._decompress_chunk (llm/compressed_kv_cache.py:289-332)."""
    sym = decode_lanes(ch.coset, ch.tile_blocks, ch.tab_lo, ch.tab_nsym, ch.tab_freq, ch.words, ch.lane_off,
                       ch.lane_nbits, ch.lane_state)
    n = ch.n_vectors
    out = np.empty((n, 8), np.float32 if out_dtype == DT_F32 else np.uint16)
    lib().lqo_dequant_symbols(_p(ch.coset), _p(sym), ch.n_heads, ch.bph, _p(np.ascontiguousarray(ch.scale_f16)),
                              _p(out), out_dtype)
    return out


def lqo_f32_to_f16(v: float) -> int:
    return int(np.float32(v).astype(np.float16).view(np.uint16))


def codec_roundtrip_batch(x: np.ndarray, dtype: int, n_chunks: int, n_heads: int, bph: int, bits: float,
                          tile_blocks: int, out_dtype: int, n_threads: int) -> Tuple[int, np.ndarray]:
    """CPU baseline: whole encode + decode of n_chunks chunks (pthreads over chunks)."""
    x = np.ascontiguousarray(x)
    n = n_chunks * n_heads * bph * 8
    out = np.empty(n, np.float32 if out_dtype == DT_F32 else np.uint16)
    total = lib().lqo_codec_roundtrip_batch(_p(x), dtype, n_chunks, n_heads, bph, ctypes.c_float(vol_mult(bits)),
                                            tile_blocks, _p(out), out_dtype, n_threads)
    if total < 0:
        raise RuntimeError(f"oracle codec failed ({total})")
    return int(total), out


# --------------------------------------------------------------------------
# compact layout (core/compact_storage.py) and its 4-bit GPU unpack
# --------------------------------------------------------------------------
def pack_e8(q: np.ndarray, b: int) -> np.ndarray:
    q = np.ascontiguousarray(q, np.float32).reshape(-1, 8)
    out = np.empty((q.shape[0], b), np.uint8)
    lib().lqo_pack_e8(_p(q), q.shape[0], b, _p(out))
    return out


def unpack_e8(packed: np.ndarray, b: int) -> np.ndarray:
    packed = np.ascontiguousarray(packed, np.uint8)
    q = np.empty((packed.shape[0], 8), np.float32)
    lib().lqo_unpack_e8(_p(packed), packed.shape[0], b, _p(q))
    return q


def unpack_e8_4bit_f16(packed: np.ndarray, scales: np.ndarray, head_idx: np.ndarray) -> np.ndarray:
    """core/triton_dequant.py:45-132 -> float16 (N, 8)."""
    packed = np.ascontiguousarray(packed, np.uint8)
    n = packed.shape[0]
    out = np.empty((n, 8), np.uint16)
    lib().lqo_unpack_e8_4bit_f16(_p(packed), _p(np.ascontiguousarray(scales, np.float32)),
                                 _p(np.ascontiguousarray(head_idx, np.int32)), n, _p(out))
    return out.view(np.float16)


# --------------------------------------------------------------------------
# attention over dequantised K/V (float64), the check for the fused kernel
# --------------------------------------------------------------------------
def decode_attention_f64(q: np.ndarray, k: np.ndarray, v: np.ndarray, sm_scale: float) -> np.ndarray:
    """softmax(q k^T * sm_scale) v with GQA (q heads grouped over kv heads).

    q: (B, Hq, D); k, v: (B, Hkv, S, D).  Returns (B, Hq, D) float64.
    Stands for HF attention over the reference's dequantised buffer with
    repeat_kv (llm/compressed_kv_cache.py:385-395 feeding transformers).
    """
    q = q.astype(np.float64)
    k = k.astype(np.float64)
    v = v.astype(np.float64)
    B, Hq, D = q.shape
    Hkv = k.shape[1]
    g = Hq // Hkv
    out = np.empty((B, Hq, D), np.float64)
    for b in range(B):
        for h in range(Hq):
            kh = k[b, h // g]
            s = kh @ q[b, h] * sm_scale
            s -= s.max()
            p = np.exp(s)
            out[b, h] = (p @ v[b, h // g]) / p.sum()
    return out
