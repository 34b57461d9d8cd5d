"""Bit-granular rANS (L = 1024) -- the API of core/gpu_ans.py on the B200.

Coding runs in the CUDA library: ``rans_encode`` / ``rans_decode_cpu`` /
``gpu_rans_decode`` produce and consume exactly the reference's streams
(LSB-first u32 words with one spare word, final state, bit count).
``rans_decode_cpu`` keeps its reference name for drop-in use; it runs on the
GPU like everything else here.

``build_rans_table`` normalises counts on the host with numpy exactly as the
reference does (``core/gpu_ans.py:62-98``): it is bookkeeping over at most
1024 counts, and numpy's argsort tie order is part of its result.  The
compressed KV cache builds its tables on the device (``lq_build_tables``).
Unlike the reference, an alphabet larger than L raises ValueError instead of
looping forever.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Tuple

import numpy as np
import torch

from .. import _dev, _lib
from .._lib import check, lib, ptr, raise_flags, stream_handle

LOG2_L = 10
L = 1 << LOG2_L


@dataclass
class RANSTable:
    """Precomputed rANS decode table (core/gpu_ans.py:53-59)."""
    lookup: np.ndarray      # (L,) int32 slot -> symbol index
    freqs: np.ndarray       # (n_symbols,) int32
    cumfreqs: np.ndarray    # (n_symbols+1,) int32
    alphabet: List[int]
    n_symbols: int


@dataclass
class RANSStream:
    """One encoded stream (core/gpu_ans.py:243-249)."""
    bitstream: np.ndarray
    n_bits: int
    initial_state: int
    n_symbols: int
    table: RANSTable


def build_rans_table(counts: np.ndarray, alphabet: List[int]) -> RANSTable:
    """Normalise counts to sum L and build the slot lookup (core/gpu_ans.py:62-98)."""
    n_sym = len(alphabet)
    if n_sym > L:
        raise ValueError(f"alphabet of {n_sym} symbols exceeds L={L} (the reference's normalisation never ends)")
    counts = np.asarray(counts)
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
    cumfreqs = np.zeros(n_sym + 1, dtype=np.int32)
    cumfreqs[1:] = np.cumsum(freqs)
    lookup = np.repeat(np.arange(n_sym, dtype=np.int32), freqs)
    return RANSTable(lookup=lookup.astype(np.int32), freqs=freqs.astype(np.int32), cumfreqs=cumfreqs,
                     alphabet=list(alphabet), n_symbols=n_sym)


def _enc_tables(tables: List[RANSTable], dev) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-table coder entries on the device (lq_expand_tables)."""
    n = len(tables)
    nsym = np.array([t.n_symbols for t in tables], np.int32)
    fr = np.zeros((n, L), np.uint16)
    for i, t in enumerate(tables):
        fr[i, : t.n_symbols] = t.freqs
    d_nsym = _dev.np_to_dev(nsym, np.int32, dev)
    d_fr = torch.from_numpy(fr.view(np.int16)).to(dev)
    enc = torch.empty(n * L, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    check(lib().lq_expand_tables(ptr(d_nsym), ptr(d_fr), n, ptr(enc), None, ptr(err), stream_handle(dev)),
          "lq_expand_tables")
    return d_nsym, enc


def _map_symbols(symbols: np.ndarray, alphabet: List[int], dev) -> torch.Tensor:
    sym = _dev.np_to_dev(np.asarray(symbols, dtype=np.int64).reshape(-1), np.int64, dev)
    alpha = np.asarray(alphabet, dtype=np.int64)
    contiguous = int(len(alpha) > 0 and np.array_equal(alpha, alpha[0] + np.arange(len(alpha))))
    d_alpha = _dev.np_to_dev(alpha, np.int64, dev)
    out = torch.empty(sym.numel(), dtype=torch.int32, device=dev)
    if sym.numel():
        check(lib().lq_map_symbols(ptr(sym), sym.numel(), ptr(d_alpha), len(alpha), contiguous, ptr(out),
                                   stream_handle(dev)), "lq_map_symbols")
    return out


def rans_encode_many(symbol_lists: List[np.ndarray], tables: List[RANSTable], device=None):
    """Encode independent streams on the device; each result is (bitstream, state, n_bits)
    exactly as core/gpu_ans.py:105-139 returns it."""
    dev = _dev.cuda_device() if device is None else torch.device(device)
    n_streams = len(symbol_lists)
    if n_streams == 0:
        return []
    uniq = {}
    tabs, tid = [], []
    for t in tables:
        if id(t) not in uniq:
            uniq[id(t)] = len(tabs)
            tabs.append(t)
        tid.append(uniq[id(t)])
    for t in tabs:
        if t.n_symbols > L:
            raise ValueError(f"alphabet of {t.n_symbols} symbols exceeds L={L}")
    d_nsym, enc = _enc_tables(tabs, dev)
    idx = [_map_symbols(s, t.alphabet, dev) for s, t in zip(symbol_lists, tables)]
    n_sym = np.array([int(i.numel()) for i in idx], np.int64)
    sym_off = np.concatenate([[0], np.cumsum(n_sym)[:-1]]).astype(np.int64)
    cap = (10 * n_sym + 31) // 32 + 1
    slot_off = np.concatenate([[0], np.cumsum(cap)]).astype(np.int64)
    all_idx = torch.cat(idx) if n_sym.sum() else torch.zeros(1, dtype=torch.int32, device=dev)
    slots = torch.zeros(int(slot_off[-1]) + 1, dtype=torch.int32, device=dev)
    nbits = torch.empty(n_streams, dtype=torch.int64, device=dev)
    state = torch.empty(n_streams, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    d_sym_off = _dev.np_to_dev(sym_off, np.int64, dev)
    d_n = _dev.np_to_dev(n_sym, np.int64, dev)
    d_tid = _dev.np_to_dev(np.array(tid, np.int32), np.int32, dev)
    d_slot = _dev.np_to_dev(slot_off, np.int64, dev)
    s = stream_handle(dev)
    check(lib().lq_rans_encode_streams(ptr(all_idx), ptr(d_sym_off), ptr(d_n), ptr(d_tid), ptr(d_nsym), ptr(enc),
                                       n_streams, ptr(d_slot), ptr(slots), ptr(nbits), ptr(state), ptr(err), s),
          "lq_rans_encode_streams")
    nb = nbits.cpu().numpy()
    raise_flags(int(err.item()) & 0xFFFFFFFF, "rans_encode")
    words = (nb + 31) // 32 + 1
    dst_off = np.concatenate([[0], np.cumsum(words)[:-1]]).astype(np.int64)
    dst = torch.empty(int(words.sum()), dtype=torch.int32, device=dev)
    check(lib().lq_rans_finish_streams(ptr(slots), ptr(d_slot), ptr(nbits), n_streams,
                                       ptr(_dev.np_to_dev(dst_off, np.int64, dev)), ptr(dst), s), "finish")
    host = dst.cpu().numpy().view(np.uint32)
    st = state.cpu().numpy().view(np.uint32)
    return [(host[dst_off[i]:dst_off[i] + words[i]].copy(), int(st[i]), int(nb[i])) for i in range(n_streams)]


def rans_encode(symbols: np.ndarray, table: RANSTable) -> Tuple[np.ndarray, int, int]:
    """Streaming rANS encode (core/gpu_ans.py:105-139): (bitstream u32, state, n_bits)."""
    return rans_encode_many([np.asarray(symbols)], [table])[0]


@dataclass
class PreparedGPUDecode:
    """Device tensors for decoding many streams (core/gpu_ans.py:252-271)."""
    d_bits: torch.Tensor
    d_bit_off: torch.Tensor
    d_nbits: torch.Tensor
    d_init: torch.Tensor
    d_ndec: torch.Tensor
    d_lookup: torch.Tensor
    d_freqs: torch.Tensor
    d_cumfreqs: torch.Tensor
    d_alphabet: torch.Tensor
    d_tid: torch.Tensor
    d_out: torch.Tensor
    d_out_off: torch.Tensor
    max_sym: int
    max_decode: int
    n_streams: int
    out_offsets: List[int]
    stream_lengths: List[int]


def prepare_gpu_decode(streams: List[RANSStream], device: str = "cuda") -> PreparedGPUDecode:
    """Stage streams and deduplicated tables on the device (core/gpu_ans.py:274-342)."""
    _lib.require_cuda()
    n_streams = len(streams)
    max_sym = max(s.table.n_symbols for s in streams)
    max_decode = max(s.n_symbols for s in streams)
    bit_offsets, words, total = [], [], 0
    for s in streams:
        bit_offsets.append(total)
        words.append(np.asarray(s.bitstream, dtype=np.uint32))
        total += len(s.bitstream) * 32
    flat = np.concatenate(words) if words else np.zeros(1, np.uint32)
    table_map, table_list, table_ids = {}, [], []
    for s in streams:
        if id(s.table) not in table_map:
            table_map[id(s.table)] = len(table_list)
            table_list.append(s.table)
        table_ids.append(table_map[id(s.table)])
    nt = len(table_list)
    lookup = np.zeros((nt, L), np.int32)
    fr = np.zeros((nt, max_sym), np.int32)
    cf = np.zeros((nt, max_sym), np.int32)
    al = np.zeros((nt, max_sym), np.int32)
    for ti, t in enumerate(table_list):
        lookup[ti] = t.lookup
        fr[ti, : t.n_symbols] = t.freqs
        cf[ti, : t.n_symbols] = t.cumfreqs[: t.n_symbols]
        al[ti, : t.n_symbols] = t.alphabet
    out_offsets, lengths, tot = [], [], 0
    for s in streams:
        out_offsets.append(tot)
        tot += s.n_symbols
        lengths.append(s.n_symbols)
    d = torch.device(device)
    t64 = lambda a: torch.tensor(np.asarray(a, dtype=np.int64), device=d)
    t32 = lambda a: torch.tensor(np.asarray(a, dtype=np.int32), device=d)
    return PreparedGPUDecode(
        d_bits=torch.from_numpy(flat.view(np.int32).copy()).to(d), d_bit_off=t64(bit_offsets),
        d_nbits=t64([s.n_bits for s in streams]), d_init=t64([s.initial_state for s in streams]),
        d_ndec=t64([s.n_symbols for s in streams]), d_lookup=t32(lookup.reshape(-1)), d_freqs=t32(fr.reshape(-1)),
        d_cumfreqs=t32(cf.reshape(-1)), d_alphabet=t32(al.reshape(-1)), d_tid=t32(table_ids),
        d_out=torch.zeros(max(tot, 1), dtype=torch.int64, device=d), d_out_off=t64(out_offsets), max_sym=max_sym,
        max_decode=max_decode, n_streams=n_streams, out_offsets=out_offsets, stream_lengths=lengths)


def run_gpu_decode_kernel(prep: PreparedGPUDecode, err: torch.Tensor | None = None):
    """Decode kernel only, no host copies (core/gpu_ans.py:345-354)."""
    dev = prep.d_bits.device
    check(lib().lq_rans_decode_streams(ptr(prep.d_bits), prep.d_bits.numel(), ptr(prep.d_bit_off), ptr(prep.d_nbits),
                                       ptr(prep.d_init), ptr(prep.d_ndec), ptr(prep.d_lookup), ptr(prep.d_freqs),
                                       ptr(prep.d_cumfreqs), ptr(prep.d_alphabet), ptr(prep.d_tid), prep.max_sym,
                                       prep.n_streams, ptr(prep.d_out), ptr(prep.d_out_off), ptr(err),
                                       stream_handle(dev)), "lq_rans_decode_streams")


def extract_gpu_results(prep: PreparedGPUDecode) -> List[np.ndarray]:
    out = prep.d_out.cpu().numpy()
    return [out[o:o + n] for o, n in zip(prep.out_offsets, prep.stream_lengths)]


def gpu_rans_decode(streams: List[RANSStream], device: str = "cuda") -> List[np.ndarray]:
    """Decode reference streams on the GPU (core/gpu_ans.py:364-370)."""
    if not streams:
        return []
    prep = prepare_gpu_decode(streams, device)
    err = torch.zeros(1, dtype=torch.int32, device=prep.d_bits.device)
    run_gpu_decode_kernel(prep, err)
    res = extract_gpu_results(prep)
    raise_flags(int(err.item()) & 0xFFFFFFFF, "gpu_rans_decode")
    return res


def rans_decode_cpu(bitstream: np.ndarray, n_bits: int, state: int, table: RANSTable, n_symbols: int) -> np.ndarray:
    """rANS decode of one stream with the reference's semantics (core/gpu_ans.py:146-168),
    including its stop at n_bits; computed by the GPU decoder."""
    s = RANSStream(bitstream=np.asarray(bitstream, dtype=np.uint32), n_bits=int(n_bits), initial_state=int(state),
                   n_symbols=int(n_symbols), table=table)
    if n_symbols == 0:
        return np.zeros(0, dtype=np.int64)
    return gpu_rans_decode([s], str(_dev.cuda_device()))[0].astype(np.int64)
