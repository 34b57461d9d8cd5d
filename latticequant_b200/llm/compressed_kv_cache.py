"""CompressedKVCache -- E8 + rANS KV storage with the API of llm/compressed_kv_cache.py.

Drop-in for the reference's HF ``DynamicCache`` subclass: ``update()``
quantises new keys/values on the GPU, entropy-codes them into rANS lanes
(every lane a reference-format stream), keeps the dequantised tokens for
attention exactly as the reference does (q * fp32 scale, in the model dtype),
and accounts memory with the reference's rule.  ``_decompress_chunk`` decodes
a chunk back with the fp16 scale, as the reference does.

Everything runs in liblq_b200.so; there is no CPU path.  Per ``_compress_tensor``
the host synchronises once, to read the kernel error word and the compressed
size.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, List, Optional, Tuple

import numpy as np
import torch
from transformers.cache_utils import DynamicCache

from .. import _dev, codec
from .._lib import check, lib, ptr, stream_handle
from ..core.gpu_ans import RANSStream, RANSTable


# ============================================================
# Coset bit-packing helpers (llm/compressed_kv_cache.py:46-63)
# ============================================================
def pack_coset_bits(coset: torch.Tensor) -> torch.Tensor:
    """(N,) coset bits -> ceil(N/8) bytes, bit i at byte i//8, bit i%8."""
    dev = _dev.cuda_device(coset)
    c = coset.to(device=dev, dtype=torch.uint8).contiguous()
    n = c.numel()
    out = torch.empty((n + 7) // 8, dtype=torch.uint8, device=dev)
    check(lib().lq_pack_bits(ptr(c), n, ptr(out), stream_handle(dev)), "lq_pack_bits")
    return _dev.back(out, coset.device)


def unpack_coset_bits(packed: torch.Tensor, n: int) -> torch.Tensor:
    """Packed bytes -> (n,) uint8 coset bits."""
    dev = _dev.cuda_device(packed)
    p = packed.to(device=dev, dtype=torch.uint8).contiguous()
    out = torch.empty(n, dtype=torch.uint8, device=dev)
    check(lib().lq_unpack_bits(ptr(p), n, ptr(out), stream_handle(dev)), "lq_unpack_bits")
    return _dev.back(out, packed.device)


# ============================================================
# Compressed chunk
# ============================================================
@dataclass
class OptimizedChunk:
    """One compressed (B, H, S, D) tensor (llm/compressed_kv_cache.py:70-93).

    Same fields as the reference.  The lanes live on the device in ``lanes``;
    ``streams`` / ``stream_meta`` / ``stream_word_offsets`` describe them in the
    reference's terms (one RANSStream per non-empty lane, meta (coset, coord, n))
    and are built on first access.
    """
    gpu_bitstream: torch.Tensor
    coset_packed: torch.Tensor
    scales: torch.Tensor
    orig_shape: tuple
    n_vectors: int
    n_heads: int
    blocks_per_head: int
    bits_per_dim: float
    orig_dtype: torch.dtype = torch.bfloat16
    lanes: Optional[codec.LaneChunk] = None
    _streams: Optional[List[RANSStream]] = field(default=None, repr=False)
    _meta: Optional[List[tuple]] = field(default=None, repr=False)
    _offsets: Optional[List[int]] = field(default=None, repr=False)
    _coset_counts: Optional[Tuple[int, int]] = field(default=None, repr=False)

    @property
    def coset_counts(self) -> Tuple[int, int]:
        if self._coset_counts is None:
            if self.lanes is None:
                self._coset_counts = (0, 0)
            else:
                n0 = int(self.lanes.tile_n0.sum().item())
                self._coset_counts = (n0, self.n_vectors - n0)
        return self._coset_counts

    def _materialise(self):
        if self._streams is not None:
            return
        self._streams, self._meta, self._offsets = [], [], []
        if self.lanes is None:
            return
        lc = self.lanes
        g = lc.geom
        words = lc.words[: lc.n_words].cpu().numpy().view(np.uint32)
        off = lc.lane_off.cpu().numpy().view(np.uint32)
        nbits = lc.lane_nbits.cpu().numpy().view(np.uint32)
        state = lc.lane_state.cpu().numpy().view(np.uint32)
        n0 = lc.tile_n0.cpu().numpy()
        lo = lc.tab_lo.cpu().numpy()
        ns = lc.tab_nsym.cpu().numpy()
        fr = lc.tab_freq.cpu().numpy().view(np.uint16).astype(np.int32)
        tables = {}
        for t in range(g.n_tiles):
            tb = min(g.tile_blocks, g.n_vectors - t * g.tile_blocks)
            for s in range(16):
                c, idx = s >> 3, s & 7
                n = int(n0[t]) if c == 0 else tb - int(n0[t])
                if n == 0:
                    continue
                if s not in tables:
                    f = fr[s, : ns[s]]
                    cum = np.concatenate([[0], np.cumsum(f)]).astype(np.int32)
                    tables[s] = RANSTable(lookup=np.repeat(np.arange(ns[s], dtype=np.int32), f).astype(np.int32),
                                          freqs=f.astype(np.int32), cumfreqs=cum,
                                          alphabet=list(range(int(lo[s]), int(lo[s]) + int(ns[s]))),
                                          n_symbols=int(ns[s]))
                l = t * 16 + s
                bs = np.concatenate([words[off[l]:off[l + 1]], np.zeros(1, np.uint32)])
                self._streams.append(RANSStream(bitstream=bs, n_bits=int(nbits[l]), initial_state=int(state[l]),
                                                n_symbols=n, table=tables[s]))
                self._meta.append((c, idx, n))
                self._offsets.append(int(off[l]))

    @property
    def streams(self) -> List[RANSStream]:
        self._materialise()
        return self._streams

    @property
    def stream_meta(self) -> List[tuple]:
        self._materialise()
        return self._meta

    @property
    def stream_word_offsets(self) -> List[int]:
        self._materialise()
        return self._offsets


def _tensor_bytes(t) -> int:
    return t.nelement() * t.element_size()


def _chunk_stored_bytes(c) -> int:
    """What one chunk costs under the reference's counting rule
    (llm/compressed_kv_cache.py:113-119): merged bitstream words, packed coset
    bits and fp16 scales -- tables, states and bit counts are not counted.
    Outlier records (no reference counterpart) are counted at 40 B each; chunk
    layouts without a merged bitstream report their own size."""
    if not hasattr(c, "gpu_bitstream"):
        return c.total_bytes
    n = _tensor_bytes(c.gpu_bitstream) + _tensor_bytes(c.coset_packed) + _tensor_bytes(c.scales)
    if c.lanes is not None and c.lanes.n_outliers:
        n += codec.OUTLIER_REC_BYTES * c.lanes.n_outliers
    return n


class CompressedKVLayer:
    """The chunks of one layer's K (or V), in append order; the attribute
    surface of the reference's class (llm/compressed_kv_cache.py:96-126)."""

    def __init__(self):
        self.chunks: List[OptimizedChunk] = []

    def append_chunk(self, chunk):
        self.chunks.append(chunk)

    @property
    def is_empty(self):
        return not self.chunks

    @property
    def total_seq(self):
        return sum(c.orig_shape[2] for c in self.chunks)

    @property
    def num_vectors(self):
        return sum(c.n_vectors for c in self.chunks)

    @property
    def total_bytes(self):
        return sum(_chunk_stored_bytes(c) for c in self.chunks)

    @property
    def fp16_equivalent_bytes(self):
        return 16 * self.num_vectors  # 8 fp16 values per E8 block


class UncompressibleKVLayer:
    """A layer kept raw because head_dim is not a multiple of 8
    (llm/compressed_kv_cache.py:129-143): it costs what it holds."""

    def __init__(self, tensor):
        self.data = tensor

    is_empty = property(lambda self: False)
    total_bytes = property(lambda self: _tensor_bytes(self.data))
    fp16_equivalent_bytes = total_bytes
    total_seq = property(lambda self: self.data.shape[2])


# One empty (1, 1, 0, 1) tensor per (device, dtype) stands in for a freed or
# not yet filled layer slot, as the reference keeps a shared placeholder.
_PLACEHOLDERS = {}


def _get_placeholder(device, dtype=torch.bfloat16):
    key = (torch.device(device), dtype)
    t = _PLACEHOLDERS.get(key)
    if t is None:
        t = _PLACEHOLDERS[key] = torch.zeros(1, 1, 0, 1, dtype=dtype, device=device)
    return t


def _host_numpy_tables(chunk_lanes: codec.LaneChunk, hist: torch.Tensor):
    """Tables normalised with numpy's argsort on the host (byte-identical to the reference)."""
    from ..core.gpu_ans import build_rans_table

    h = hist.view(16, -1).cpu().numpy().astype(np.int64)
    lo = np.zeros(16, np.int32)
    ns = np.zeros(16, np.int32)
    fr = np.zeros((16, 1024), np.int32)
    for s in range(16):
        nz = np.nonzero(h[s])[0]
        if nz.size == 0:
            continue
        a, b = int(nz.min()) - 2, int(nz.max()) + 2
        counts = np.array([h[s, i] if 0 <= i < h.shape[1] else 0 for i in range(a, b + 1)], np.int64)
        alphabet = list(range(a - 512, b - 512 + 1))
        t = build_rans_table(counts, alphabet)
        lo[s], ns[s] = alphabet[0], len(alphabet)
        fr[s, : len(alphabet)] = t.freqs
    return lo, ns, fr


# ============================================================
# CompressedKVCache
# ============================================================
class CompressedKVCache(DynamicCache):
    """llm/compressed_kv_cache.py:160-453 on the B200.

    Extra keyword arguments (defaults keep the reference's behaviour):
      tile_blocks  rANS lane tile in E8 blocks (None = one tile per chunk, i.e. the
                   reference's own 16-stream layout)
      table_mode   'device' (tables built on the GPU, ties by symbol index) or
                   'numpy' (histograms normalised with numpy's argsort on the host,
                   byte-identical bitstreams to the reference)
    """

    def __init__(self, bits_per_dim: int = 4, eval_only_no_entropy: bool = False,
                 tile_blocks: Optional[int] = codec.DEFAULT_TILE_BLOCKS, table_mode: str = "device"):
        super().__init__()
        assert bits_per_dim in (3, 4, 5)
        assert table_mode in ("device", "numpy")
        self.bits = bits_per_dim
        self.eval_only_no_entropy = eval_only_no_entropy
        self.tile_blocks = tile_blocks
        self.table_mode = table_mode
        if not hasattr(self, 'key_cache'):
            self.key_cache = []
        if not hasattr(self, 'value_cache'):
            self.value_cache = []
        self._comp_keys: List = []
        self._comp_values: List = []
        self.total_vectors = 0
        self._model_dtype = None

    def _compress_tensor(self, tensor: torch.Tensor,
                         scale_f32: Optional[torch.Tensor] = None) -> Tuple[Any, torch.Tensor]:
        """Quantise + entropy-code one (B, H, S, D) tensor (llm/compressed_kv_cache.py:176-287).

        scale_f32 (an addition, default off): fp32 per-head scales to use in
        place of the computed ones -- re-coding values that are already lattice
        points times these scales gives back exactly their lattice points."""
        device = tensor.device
        orig_dtype = tensor.dtype
        batch, heads, seq, hd = tensor.shape
        if hd % 8 != 0:
            return 'uncompressible', tensor
        n_heads = batch * heads
        bph = seq * (hd // 8)
        n_vectors = n_heads * bph
        x = tensor.to(_dev.cuda_device(tensor)).contiguous()
        if x.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            x = x.float()
        if n_vectors == 0:
            raise ValueError("cannot compress an empty tensor (the reference's scale would be NaN)")
        geom = codec.Geometry(1, n_heads, bph, codec.round_tile(self.tile_blocks, n_vectors))
        cd = codec.Codec(geom, x.device, keep_deq=True, deq_dtype=orig_dtype)
        if scale_f32 is None:
            cd.scales(x, self.bits)
        else:
            sf = scale_f32.to(device=x.device, dtype=torch.float32).reshape(-1)
            cd.scale_f32.copy_(sf)
            cd.scale_f16.copy_(sf.to(torch.float16))
        n_out = 0
        if self.eval_only_no_entropy or self.table_mode == "numpy":
            cd.quantize(x)
        else:  # device tables; chunks whose alphabet would exceed L get the outlier side channel
            n_out = cd.quantize_with_tables(x, None, codec.blocks_per_token(hd, geom.tile_blocks, bph))
        deq = cd.deq.view(tensor.shape)
        if self.eval_only_no_entropy:
            flags = cd.read_err()
            from .._lib import raise_flags

            raise_flags(flags & ~0x2, "_compress_tensor")  # symbol range only matters to the coder
            self.total_vectors += n_vectors
            chunk = OptimizedChunk(gpu_bitstream=torch.zeros(1, dtype=torch.int32, device=device),
                                   coset_packed=torch.zeros(1, dtype=torch.uint8, device=device),
                                   scales=cd.scale_f16.to(device), orig_shape=tensor.shape, n_vectors=n_vectors,
                                   n_heads=n_heads, blocks_per_head=bph, bits_per_dim=self.bits,
                                   orig_dtype=orig_dtype)
            chunk._streams, chunk._meta, chunk._offsets, chunk._coset_counts = [], [], [], (0, 0)
            return chunk, deq.to(device)
        if self.table_mode == "numpy":
            lo, ns, fr = _host_numpy_tables(None, cd.hist)
            cd.tab_lo.copy_(torch.from_numpy(lo))
            cd.tab_nsym.copy_(torch.from_numpy(ns))
            cd.tab_freq.copy_(torch.from_numpy(fr.astype(np.int16)))
        cd.expand_tables(enc=True, dec=False)
        cd.entropy_encode()
        from .._lib import raise_flags

        raise_flags(cd.read_err(), "_compress_tensor")
        nw = cd.n_words()
        lanes = codec.LaneChunk(geom=geom, bits=self.bits, orig_shape=tuple(tensor.shape), orig_dtype=orig_dtype,
                                scale_f32=cd.scale_f32, scale_f16=cd.scale_f16, coset_words=cd.coset_words,
                                tile_n0=cd.tile_n0, tab_lo=cd.tab_lo, tab_nsym=cd.tab_nsym, tab_freq=cd.tab_freq,
                                words=cd.words[:max(nw, 1)].clone(), lane_off=cd.lane_off,
                                lane_nbits=cd.lane_nbits, lane_state=cd.lane_state, n_words=nw,
                                outlier_rec=cd.out_rec[:n_out * 10].view(n_out, 10).clone() if n_out else None,
                                n_outliers=n_out)
        self.total_vectors += n_vectors
        coset_bytes = cd.coset_words.view(torch.uint8)[: (n_vectors + 7) // 8]
        chunk = OptimizedChunk(gpu_bitstream=lanes.words[:nw] if nw else torch.zeros(0, dtype=torch.int32,
                                                                                   device=x.device),
                               coset_packed=coset_bytes, scales=cd.scale_f16, orig_shape=tensor.shape,
                               n_vectors=n_vectors, n_heads=n_heads, blocks_per_head=bph, bits_per_dim=self.bits,
                               orig_dtype=orig_dtype, lanes=lanes)
        return chunk, deq.to(device)

    def _decompress_chunk(self, chunk: OptimizedChunk) -> torch.Tensor:
        """Full decompression with the fp16 scales (llm/compressed_kv_cache.py:289-332)."""
        if chunk.lanes is None:
            raise ValueError("chunk was stored without entropy coding (eval_only_no_entropy)")
        out = codec.decompress(chunk.lanes, out_dtype=chunk.orig_dtype)
        return out.view(chunk.orig_shape).to(chunk.gpu_bitstream.device)

    def _free_layer(self, layer_idx):
        """Free decompressed KV for a layer (llm/compressed_kv_cache.py:334-340)."""
        if layer_idx < len(self.key_cache):
            dev = self.key_cache[layer_idx].device if self.key_cache[layer_idx] is not None else 'cuda:0'
            dt = self._model_dtype or torch.bfloat16
            self.key_cache[layer_idx] = _get_placeholder(dev, dt)
            self.value_cache[layer_idx] = _get_placeholder(dev, dt)

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        """Compress new KV, append, return the full dequantised K/V (llm/compressed_kv_cache.py:342-395)."""
        device = key_states.device
        if self._model_dtype is None:
            self._model_dtype = key_states.dtype
        comp_k, k_dec_new = self._compress_tensor(key_states)
        comp_v, v_dec_new = self._compress_tensor(value_states)
        return self._store(layer_idx, device, key_states, value_states, comp_k, k_dec_new, comp_v, v_dec_new)

    def _store(self, layer_idx, device, key_states, value_states, comp_k, k_dec_new, comp_v, v_dec_new):
        """Bookkeeping of update() (llm/compressed_kv_cache.py:363-395): grow the
        per-layer lists to layer_idx, append the chunks, and extend the
        resident dequantised K/V along the sequence (what attention reads)."""
        missing = layer_idx + 1 - len(self._comp_keys)
        if missing > 0:
            self._comp_keys.extend([None] * missing)
            self._comp_values.extend([None] * missing)
        missing = layer_idx + 1 - len(self.key_cache)
        if missing > 0:
            ph = _get_placeholder(device, self._model_dtype)
            self.key_cache.extend([ph] * missing)
            self.value_cache.extend([ph] * missing)
        if comp_k == 'uncompressible':
            # stored raw; the returned tensors are this update's alone
            self._comp_keys[layer_idx] = UncompressibleKVLayer(key_states)
            self._comp_values[layer_idx] = UncompressibleKVLayer(value_states)
            self.key_cache[layer_idx], self.value_cache[layer_idx] = k_dec_new, v_dec_new
            return k_dec_new, v_dec_new
        for layers, chunk in ((self._comp_keys, comp_k), (self._comp_values, comp_v)):
            if layers[layer_idx] is None:
                layers[layer_idx] = CompressedKVLayer()
            layers[layer_idx].append_chunk(chunk)

        def grow(resident, new):
            return new if resident.shape[2] == 0 else torch.cat([resident, new], dim=2)

        self.key_cache[layer_idx] = grow(self.key_cache[layer_idx], k_dec_new)
        self.value_cache[layer_idx] = grow(self.value_cache[layer_idx], v_dec_new)
        return self.key_cache[layer_idx], self.value_cache[layer_idx]

    # ---- reporting (llm/compressed_kv_cache.py:399-453) ----
    def _layers(self):
        return [l for l in self._comp_keys + self._comp_values if l is not None]

    def compressed_bytes(self):
        return sum(l.total_bytes for l in self._layers())

    def fp16_equivalent_bytes(self):
        return sum(l.fp16_equivalent_bytes for l in self._layers())

    def decompressed_resident_bytes(self):
        return sum(_tensor_bytes(t) for t in self.key_cache + self.value_cache if t is not None)

    def actual_vram_bytes(self):
        return self.compressed_bytes() + self.decompressed_resident_bytes()

    def memory_report(self):
        """The reference's report text (same lines and number formats)."""
        comp, fp16 = self.compressed_bytes(), self.fp16_equivalent_bytes()
        decomp, actual = self.decompressed_resident_bytes(), self.actual_vram_bytes()
        eff_bits = 8 * comp / max(8 * self.total_vectors, 1)
        mb = lambda n: f"{n:,} B ({n / 1024 / 1024:.2f} MB)"  # noqa: E731
        return "\n".join([
            "CompressedKVCache Report (optimized side info)",
            f"  Bits/dim:     {self.bits} (target), {eff_bits:.3f} (effective)",
            f"  Layers:       {sum(x is not None for x in self._comp_keys)}",
            f"  Vectors:      {self.total_vectors:,}",
            "  OOR rate:     0.00%",
            "  ---",
            f"  Total compressed:  {mb(comp)}",
            f"  Decompressed now:  {mb(decomp)}",
            f"  Actual VRAM (KV):  {mb(actual)}",
            f"  FP16 baseline:     {mb(fp16)}",
            "  ---",
            f"  Theoretical ratio: {fp16 / max(comp, 1):.2f}x",
            f"  Actual ratio:      {fp16 / max(actual, 1):.2f}x",
        ])

    def get_seq_length(self, layer_idx=0):
        if layer_idx < len(self._comp_keys) and self._comp_keys[layer_idx] is not None:
            return self._comp_keys[layer_idx].total_seq
        return 0

    def get_mask_sizes(self, query_length, layer_idx=0):
        """(kv_length, kv_offset) for transformers' mask builders: the cached
        tokens plus the query's (the base class reads its own layer list,
        which this cache does not fill)."""
        q = int(query_length.shape[0]) if torch.is_tensor(query_length) else int(query_length)
        return self.get_seq_length(layer_idx) + q, 0
