"""Entropy-coded E8 storage -- the API of core/entropy_storage.py on this
package's rANS coder.

The reference stores E8 lattice points as a coset stream plus 16 symbol
streams coded with the third-party coder constriction 0.4.2 (Rust; not
installed here, its byte format unpinned), with Laplace-smoothed
probabilities from a FrequencyModel (core/entropy_storage.py:137-246).  This
module keeps the same objects and accounting, and codes the same streams with
the reference-format bit-level rANS of core/gpu_ans.py on the GPU:
probabilities (count + 1) over the union of the model's and the data's
symbols, normalised to L = 1024 by build_rans_table.  Streams round-trip
exactly; no lattice point is out of range (alphabets above 1024 symbols per
stream are rejected, as build_rans_table rejects them).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Tuple

import numpy as np
import torch

from .e8_quantizer import compute_scale, encode_e8
from .entropy_coder import FrequencyModel, e8_to_symbols, symbols_to_e8
from .gpu_ans import RANSStream, build_rans_table, gpu_rans_decode, rans_encode_many

_COSET_SCALE = 1 << 20  # integer counts standing in for the coset probabilities


@dataclass
class CompressedE8Tensor:
    """Entropy-coded E8 points (core/entropy_storage.py:47-134)."""
    coset_stream: np.ndarray                 # rANS words of the coset bits
    symbol_streams: List[List[np.ndarray]]   # [coset][coord] rANS words
    freq_model: FrequencyModel
    scales: torch.Tensor
    num_vectors: int
    coset_counts: Tuple[int, int]
    bits_per_dim_target: float
    orig_shape: tuple
    group_size: int
    symbol_maps: List[List[dict]]            # [coset][coord] index -> symbol value
    streams: List[Optional[RANSStream]] = None  # coset stream, then [c][idx] row-major (decode state)

    @property
    def compressed_bits(self) -> int:
        total = len(self.coset_stream) * 32
        for c in range(2):
            for idx in range(8):
                if c < len(self.symbol_streams) and idx < len(self.symbol_streams[c]):
                    total += len(self.symbol_streams[c][idx]) * 32
        return total

    @property
    def compressed_bytes(self) -> int:
        return self.compressed_bits // 8

    @property
    def freq_table_bytes(self) -> int:
        return sum(len(t) for t in self.freq_model.tables.values()) * 16

    @property
    def scale_bytes(self) -> int:
        return self.scales.nelement() * self.scales.element_size()

    @property
    def total_bytes(self) -> int:
        return self.compressed_bytes + self.freq_table_bytes + self.scale_bytes

    @property
    def fp16_bytes(self) -> int:
        return self.num_vectors * 8 * 2

    @property
    def effective_bits_per_dim(self) -> float:
        return (self.total_bytes * 8) / (self.num_vectors * 8)

    @property
    def compression_ratio(self) -> float:
        return self.fp16_bytes / self.total_bytes

    def summary(self) -> str:
        return "\n".join([
            "CompressedE8Tensor (entropy-coded)",
            f"  Vectors: {self.num_vectors:,} x 8-dim",
            f"  Target rate: {self.bits_per_dim_target} bits/dim",
            f"  Compressed:  {self.compressed_bytes:,} B ({self.compressed_bytes/1024:.1f} KB)",
            f"  Freq tables: {self.freq_table_bytes:,} B ({self.freq_table_bytes/1024:.1f} KB)",
            f"  Scales:      {self.scale_bytes:,} B",
            f"  Total:       {self.total_bytes:,} B ({self.total_bytes/1024:.1f} KB)",
            f"  FP16 equiv:  {self.fp16_bytes:,} B ({self.fp16_bytes/1024:.1f} KB)",
            f"  Effective:   {self.effective_bits_per_dim:.3f} bits/dim",
            f"  Compression: {self.compression_ratio:.2f}x",
            "  OOR rate:    0.00% (entropy coding has no range limit)",
        ])


def _coset_table(model: FrequencyModel):
    p = np.array(model.coset_prob, dtype=np.float64)
    counts = np.maximum((p / p.sum() * _COSET_SCALE).astype(np.int64), 1)
    return build_rans_table(counts, [0, 1])


def _stream_table(model: FrequencyModel, key, col: np.ndarray):
    """Alphabet = model symbols | data symbols, counts + 1 (core/entropy_storage.py:186-201)."""
    table = model.tables.get(key, {})
    all_vals = sorted(set(table.keys()) | set(np.unique(col).tolist()))
    counts = np.array([table.get(s, 0) + 1 for s in all_vals], dtype=np.int64)
    return build_rans_table(counts, all_vals), {i: s for i, s in enumerate(all_vals)}


def compress_symbols(model: FrequencyModel, coset: np.ndarray, free_coords: np.ndarray, coord8_half: np.ndarray):
    """rANS streams [coset] + [c][idx] of the symbolised points (None for empty)
    and the index -> symbol maps of the 16 symbol streams."""
    cos = np.asarray(coset).astype(np.int64)
    all_symbols = np.concatenate([np.asarray(free_coords), np.asarray(coord8_half)[:, None]], axis=1).astype(np.int64)
    lists, tables, maps = [cos], [_coset_table(model)], []
    for c in (0, 1):
        syms_c = all_symbols[cos == c]
        for idx in range(8):
            if syms_c.shape[0] == 0:
                lists.append(None)
                tables.append(None)
                maps.append({})
                continue
            t, m = _stream_table(model, (c, idx), syms_c[:, idx])
            lists.append(syms_c[:, idx])
            tables.append(t)
            maps.append(m)
    live = [i for i, l in enumerate(lists) if l is not None and len(l)]
    enc = rans_encode_many([lists[i] for i in live], [tables[i] for i in live])
    streams: List[Optional[RANSStream]] = [None] * len(lists)
    for i, (words, state, nbits) in zip(live, enc):
        streams[i] = RANSStream(bitstream=words, n_bits=nbits, initial_state=state, n_symbols=len(lists[i]),
                                table=tables[i])
    return streams, maps


def compress_e8(q: torch.Tensor, bits_per_dim_target: float, scale: float,
                freq_model: Optional[FrequencyModel] = None) -> CompressedE8Tensor:
    """(N, 8) E8 lattice points -> CompressedE8Tensor (core/entropy_storage.py:137-246)."""
    N = q.shape[0]
    coset, free_coords, coord8_half = e8_to_symbols(q)
    cos_np = coset.cpu().numpy().astype(np.int32)
    free_np = free_coords.cpu().numpy().astype(np.int64)
    c8h_np = coord8_half.cpu().numpy().astype(np.int64)
    if freq_model is None:
        freq_model = FrequencyModel()
        freq_model.fit(cos_np, free_np, c8h_np)
    streams, maps = compress_symbols(freq_model, cos_np, free_np, c8h_np)
    empty = np.zeros(0, dtype=np.uint32)
    sym_streams = [[(streams[1 + 8 * c + i].bitstream if streams[1 + 8 * c + i] is not None else empty)
                    for i in range(8)] for c in (0, 1)]
    sym_maps = [[maps[8 * c + i] for i in range(8)] for c in (0, 1)]
    return CompressedE8Tensor(
        coset_stream=streams[0].bitstream if streams[0] is not None else empty, symbol_streams=sym_streams,
        freq_model=freq_model, scales=torch.tensor([scale], dtype=torch.float32), num_vectors=N,
        coset_counts=(int((cos_np == 0).sum()), int((cos_np == 1).sum())), bits_per_dim_target=bits_per_dim_target,
        orig_shape=(N, 8), group_size=N, symbol_maps=sym_maps, streams=streams)


def decompress_e8(compressed: CompressedE8Tensor, device: str = "cpu") -> torch.Tensor:
    """CompressedE8Tensor -> (N, 8) E8 lattice points (core/entropy_storage.py:249-323)."""
    N = compressed.num_vectors
    live = [s for s in compressed.streams if s is not None and s.n_symbols]
    dec = iter(gpu_rans_decode(live) if live else [])
    out = [next(dec) if (s is not None and s.n_symbols) else None for s in compressed.streams]
    cos_np = np.asarray(out[0], dtype=np.int64) if out[0] is not None else np.zeros(0, np.int64)
    if cos_np.shape[0] != N:
        raise ValueError("coset stream does not hold num_vectors symbols")
    all_symbols = np.zeros((N, 8), dtype=np.int64)
    for c in (0, 1):
        rows = np.where(cos_np == c)[0]
        if rows.size == 0:
            continue
        for idx in range(8):
            d = out[1 + 8 * c + idx]  # decoded symbol values (the decoder maps through the alphabet)
            if d is not None:
                all_symbols[rows, idx] = np.asarray(d, dtype=np.int64)
    coset_t = torch.tensor(cos_np, dtype=torch.long, device=device)
    free_t = torch.tensor(all_symbols[:, :7], dtype=torch.long, device=device)
    c8h_t = torch.tensor(all_symbols[:, 7], dtype=torch.long, device=device)
    return symbols_to_e8(coset_t, free_t, c8h_t)


def quantize_compress(x: torch.Tensor, bits_per_dim: float, sigma2: float,
                      freq_model: Optional[FrequencyModel] = None) -> CompressedE8Tensor:
    """Raw (N, 8) vectors -> E8 -> entropy-coded (core/entropy_storage.py:330-350)."""
    scale = compute_scale(sigma2, bits_per_dim)
    q = encode_e8(x / scale)
    return compress_e8(q, bits_per_dim, scale, freq_model)


def decompress_dequantize(compressed: CompressedE8Tensor, device: str = "cpu") -> torch.Tensor:
    """Decode and multiply by the scale (core/entropy_storage.py:353-362)."""
    q = decompress_e8(compressed, device)
    return q * compressed.scales[0].item()
