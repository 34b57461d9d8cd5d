"""Device-side E8 + rANS codec: the host half of the C ABI.

``Codec`` owns the device buffers for one chunk geometry and launches the
kernels of liblq_b200.so in stream order without allocating or
synchronising, so a whole encode + decode can be captured in a CUDA graph.
``compress`` / ``decompress`` are the allocating, checking wrappers the
reference-facing API (``CompressedKVCache``, ``core.*``) is built on.

Geometry (reference llm/compressed_kv_cache.py:183-188): a chunk is a tensor
(B, H, S, D) read as n_heads = B*H rows of bph = S*D/8 E8 blocks.  A batch of
``n_chunks`` equal chunks is laid out back to back.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import L, NSTREAMS, HIST_BINS, check, lib, ptr, raise_flags, stream_handle

DEFAULT_TILE_BLOCKS = 1024


def vol_mult(bits: float) -> float:
    """fp32(4 ** -bits), the factor torch applies (llm/compressed_kv_cache.py:192)."""
    return float(torch.tensor(4.0 ** (-bits), dtype=torch.float32))


def _ceil_div(a: int, b: int) -> int:
    return -(-a // b)


def round_tile(tile_blocks: Optional[int], n_vectors: int) -> int:
    """Tile size in blocks (multiple of 32); None = one tile per chunk (reference stream layout)."""
    tb = n_vectors if tile_blocks is None else int(tile_blocks)
    tb = max(32, _ceil_div(max(tb, 1), 32) * 32)
    return tb


@dataclass
class Geometry:
    n_chunks: int
    n_heads: int
    bph: int
    tile_blocks: int

    @property
    def n_vectors(self) -> int:
        return self.n_heads * self.bph

    @property
    def n_tiles(self) -> int:
        return _ceil_div(self.n_vectors, self.tile_blocks)

    @property
    def n_lanes(self) -> int:
        return self.n_chunks * self.n_tiles * NSTREAMS

    @property
    def coset_words_per_chunk(self) -> int:
        return _ceil_div(self.n_vectors, 32)

    @property
    def words_capacity(self) -> int:
        # 10 bits per symbol is the most the coder emits (L = 1024, f >= 1)
        return self.n_chunks * (_ceil_div(8 * self.n_vectors * 10, 32) + NSTREAMS * self.n_tiles) + 1


@dataclass
class LaneChunk:
    """One compressed chunk (or a batch of equal chunks) resident on the device."""
    geom: Geometry
    bits: float
    orig_shape: tuple
    orig_dtype: torch.dtype
    scale_f32: torch.Tensor      # [n_chunks*n_heads] float32
    scale_f16: torch.Tensor      # [n_chunks*n_heads] float16
    coset_words: torch.Tensor    # [n_chunks*wpc] int32 (u32 bit words)
    tile_n0: torch.Tensor        # [n_chunks*n_tiles] int32
    tab_lo: torch.Tensor         # [n_chunks*16] int32
    tab_nsym: torch.Tensor       # [n_chunks*16] int32
    tab_freq: torch.Tensor       # [n_chunks*16, L] int16 (u16)
    words: torch.Tensor          # [n_words] int32 (u32)
    lane_off: torch.Tensor       # [n_lanes+1] int32 (u32)
    lane_nbits: torch.Tensor     # [n_lanes] int32 (u32)
    lane_state: torch.Tensor     # [n_lanes] int32 (u32)
    n_words: int = 0
    dec_tab: Optional[torch.Tensor] = field(default=None, repr=False)
    # outlier side channel: tokens with a symbol beyond OUTLIER_LIMIT, as records
    # (block index, coset, 8 symbols) -- only when the chunk would exceed L symbols
    outlier_rec: Optional[torch.Tensor] = field(default=None, repr=False)  # (n, 10) int32
    n_outliers: int = 0

    # ---- accounting -----------------------------------------------------
    def coset_bytes(self) -> int:
        return self.geom.n_chunks * _ceil_div(self.geom.n_vectors, 8)

    def compressed_bytes(self) -> int:
        """Bytes counted as CompressedKVCache.compressed_bytes counts them
        (llm/compressed_kv_cache.py:113-119): bitstream words + coset bits + fp16 scales
        (+ 40 bytes per outlier record)."""
        return 4 * self.n_words + self.coset_bytes() + 2 * self.scale_f16.numel() + OUTLIER_REC_BYTES * self.n_outliers

    def metadata_bytes(self) -> int:
        """Side information the reference does not count: lane offsets / bit counts / states
        (stored as u32 + u16 + u16 per lane) and the frequency tables (u16 per alphabet entry)."""
        n_lanes = self.geom.n_lanes
        tab = int(self.tab_nsym.clamp(min=0).sum().item()) * 2 + 8 * self.tab_nsym.numel()
        return 8 * n_lanes + tab + 4 * self.tile_n0.numel()


OUTLIER_LIMIT = 255     # symbols beyond +-255 go to the outlier records when a table would exceed L
OUTLIER_REC_BYTES = 40  # int32 block index, coset, 8 symbols


def blocks_per_token(head_dim: int, tile_blocks: int, bph: int) -> int:
    """Token granularity of the outlier records: head_dim/8 when it is a power
    of two <= 32 dividing the tile and the blocks per head, else 1."""
    b = head_dim // 8
    if 0 < b <= 32 and b & (b - 1) == 0 and tile_blocks % b == 0 and bph % b == 0:
        return b
    return 1


class Codec:
    """Persistent device buffers + kernel launches for one chunk geometry."""

    def __init__(self, geom: Geometry, device: torch.device | str = "cuda", keep_deq: bool = False,
                 deq_dtype: torch.dtype = torch.bfloat16):
        _lib.require_cuda()
        dev = torch.device(device)
        self.geom = geom
        self.device = dev
        g = geom
        nh = g.n_chunks * g.n_heads
        i32 = dict(dtype=torch.int32, device=dev)
        self.sigma2 = torch.empty(nh, dtype=torch.float32, device=dev)
        self.scale_f32 = torch.empty(nh, dtype=torch.float32, device=dev)
        self.scale_f16 = torch.empty(nh, dtype=torch.float16, device=dev)
        # int8 symbol columns + their int16 escape plane + per-tile flags (lq_sym_cols_bytes)
        self.sym_rows = torch.empty(int(lib().lq_sym_cols_bytes(g.n_chunks, g.n_vectors, g.tile_blocks)),
                                    dtype=torch.uint8, device=dev)
        self.coset_words = torch.empty(g.n_chunks * g.coset_words_per_chunk, **i32)
        self.tile_n0 = torch.empty(g.n_chunks * g.n_tiles, **i32)
        self.hist = torch.empty(g.n_chunks * NSTREAMS * HIST_BINS, **i32)
        self.tab_lo = torch.empty(g.n_chunks * NSTREAMS, **i32)
        self.tab_nsym = torch.empty(g.n_chunks * NSTREAMS, **i32)
        self.tab_freq = torch.empty(g.n_chunks * NSTREAMS, L, dtype=torch.int16, device=dev)
        self.enc_tab = torch.empty(g.n_chunks * NSTREAMS * L, **i32)
        self.dec_tab = torch.empty(g.n_chunks * NSTREAMS * L, **i32)
        self.words = torch.empty(g.words_capacity, **i32)
        self.lane_off = torch.empty(g.n_lanes + 1, **i32)
        self.lane_nbits = torch.empty(g.n_lanes, **i32)
        self.lane_state = torch.empty(g.n_lanes, **i32)
        self.err = torch.zeros(1, **i32)
        ws_s = lib().lq_head_scales_workspace(nh, g.bph * 8)
        ws_e = lib().lq_rans_encode_workspace(g.n_chunks, g.n_vectors, g.tile_blocks)
        ws_d = lib().lq_rans_decode_workspace(g.n_chunks, g.n_vectors, g.tile_blocks)
        self.ws = torch.empty(max(ws_s, ws_e, ws_d, 16), dtype=torch.uint8, device=dev)
        self.deq = (torch.empty(g.n_chunks * g.n_vectors * 8, dtype=deq_dtype, device=dev) if keep_deq else None)

    # ---- encode -------------------------------------------------------------
    def scales(self, x: torch.Tensor, bits: float):
        g = self.geom
        s = stream_handle(self.device)
        check(lib().lq_head_scales(ptr(x), _lib.dtype_code(x.dtype), g.n_chunks * g.n_heads, g.bph * 8,
                                   ctypes.c_float(vol_mult(bits)), ptr(self.sigma2), ptr(self.scale_f32),
                                   ptr(self.scale_f16), ptr(self.ws), self.ws.numel(), s), "lq_head_scales")

    def quantize(self, x: torch.Tensor, q_out: Optional[torch.Tensor] = None):
        g = self.geom
        s = stream_handle(self.device)
        deq = self.deq
        dq = _lib.dtype_code(deq.dtype) if deq is not None else 0
        check(lib().lq_e8_quantize(ptr(x), _lib.dtype_code(x.dtype), g.n_chunks, g.n_heads, g.bph,
                                   ptr(self.scale_f32), g.tile_blocks, ptr(self.sym_rows), ptr(self.coset_words),
                                   ptr(self.tile_n0), ptr(self.hist), ptr(deq), dq, ptr(q_out), ptr(self.err), s),
              "lq_e8_quantize")

    def quantize_outliers(self, x: torch.Tensor, q_out: Optional[torch.Tensor] = None, bpt: int = 1,
                          cap: Optional[int] = None):
        """quantize() with the outlier side channel (lq_e8_quantize_outliers)."""
        g = self.geom
        cap = int(cap or max(4096, g.n_vectors // 64))
        if getattr(self, "out_cap", 0) < cap:
            self.out_rec = torch.empty(g.n_chunks * cap * 10, dtype=torch.int32, device=self.device)
            self.out_count = torch.zeros(g.n_chunks, dtype=torch.int32, device=self.device)
            self.out_cap = cap
        s = stream_handle(self.device)
        deq = self.deq
        dq = _lib.dtype_code(deq.dtype) if deq is not None else 0
        check(lib().lq_e8_quantize_outliers(ptr(x), _lib.dtype_code(x.dtype), g.n_chunks, g.n_heads, g.bph,
                                            ptr(self.scale_f32), g.tile_blocks, ptr(self.sym_rows),
                                            ptr(self.coset_words), ptr(self.tile_n0), ptr(self.hist), ptr(deq), dq,
                                            ptr(q_out), OUTLIER_LIMIT, bpt, None, ptr(self.out_rec),
                                            ptr(self.out_count), self.out_cap, ptr(self.err), s),
              "lq_e8_quantize_outliers")

    def quantize_with_tables(self, x: torch.Tensor, q_out: Optional[torch.Tensor] = None, bpt: int = 1) -> int:
        """quantize + build_tables; when a table would exceed L symbols (or a
        symbol leaves the histogram range), quantise again with the outlier
        side channel.  Returns the number of outlier records (synchronises)."""
        self.quantize(x, q_out)
        self.build_tables()
        flags = self.read_err()
        if not flags & (_lib.EF_ALPHABET | _lib.EF_SYMRANGE | _lib.EF_NOCONVERGE):
            self.n_outliers = 0
            return 0
        self.err.zero_()
        self.quantize_outliers(x, q_out, bpt)
        self.build_tables()
        raise_flags(self.read_err(), "quantize (outlier pass)")
        self.n_outliers = int(self.out_count[:1].item())
        return self.n_outliers

    def build_tables(self):
        g = self.geom
        s = stream_handle(self.device)
        check(lib().lq_build_tables(ptr(self.hist), g.n_chunks * NSTREAMS, ptr(self.tab_lo), ptr(self.tab_nsym),
                                    ptr(self.tab_freq), ptr(self.err), s), "lq_build_tables")

    def expand_tables(self, enc: bool = True, dec: bool = True):
        g = self.geom
        s = stream_handle(self.device)
        check(lib().lq_expand_tables(ptr(self.tab_nsym), ptr(self.tab_freq), g.n_chunks * NSTREAMS,
                                     ptr(self.enc_tab) if enc else None, ptr(self.dec_tab) if dec else None,
                                     ptr(self.err), s), "lq_expand_tables")

    def entropy_encode(self):
        g = self.geom
        s = stream_handle(self.device)
        check(lib().lq_rans_encode(ptr(self.sym_rows), ptr(self.tile_n0), g.n_chunks, g.n_vectors, g.tile_blocks,
                                   ptr(self.tab_lo), ptr(self.tab_nsym), ptr(self.enc_tab), ptr(self.words),
                                   self.words.numel(), ptr(self.lane_off), ptr(self.lane_nbits),
                                   ptr(self.lane_state), ptr(self.ws), self.ws.numel(), ptr(self.err), s),
              "lq_rans_encode")

    def encode(self, x: torch.Tensor, bits: float, scale_f32: Optional[torch.Tensor] = None):
        """Whole encode in stream order: scales, E8 + symbols, tables, lanes."""
        if scale_f32 is None:
            self.scales(x, bits)
        else:
            self.scale_f32.copy_(scale_f32)
            self.scale_f16.copy_(scale_f32.to(torch.float16))
        self.quantize(x)
        self.build_tables()
        self.expand_tables(enc=True, dec=False)
        self.entropy_encode()

    # ---- decode -------------------------------------------------------------
    def decode(self, out: Optional[torch.Tensor], sym_out: Optional[torch.Tensor] = None,
               words: Optional[torch.Tensor] = None, n_words: Optional[int] = None):
        """Decode the lanes currently in the buffers (or `words`) to `out`."""
        g = self.geom
        s = stream_handle(self.device)
        w = self.words if words is None else words
        nw = w.numel() if n_words is None else n_words
        od = _lib.dtype_code(out.dtype) if out is not None else 0
        check(lib().lq_rans_decode(ptr(w), nw, ptr(self.lane_off), ptr(self.lane_nbits), ptr(self.lane_state),
                                   ptr(self.coset_words), ptr(self.tile_n0), g.n_chunks, g.n_heads, g.bph,
                                   g.tile_blocks, ptr(self.tab_lo), ptr(self.tab_nsym), ptr(self.tab_freq),
                                   ptr(self.dec_tab), ptr(self.scale_f16), ptr(out), od, ptr(sym_out),
                                   ptr(self.ws), self.ws.numel(), ptr(self.err), s), "lq_rans_decode")

    def read_err(self) -> int:
        return int(self.err.item()) & 0xFFFFFFFF

    def n_words(self) -> int:
        return int(self.lane_off[-1].item()) & 0xFFFFFFFF

    def chunks(self, bits: float, shape: tuple, dtype: torch.dtype, outliers: bool = False) -> list:
        """The batch now in the buffers as one LaneChunk per chunk (reads the
        lane offsets, so it synchronises).  Words, tables, scales and coset
        words are copied out, so the Codec can code the next batch.  shape /
        dtype: the (B, H, S, D) tensor and dtype of one chunk; outliers: the
        batch went through quantize_outliers (records are split per chunk)."""
        g = self.geom
        lpc, nh, wpc, nt = g.n_tiles * NSTREAMS, g.n_heads, g.coset_words_per_chunk, g.n_tiles
        off = self.lane_off.to(torch.int64) & 0xFFFFFFFF
        bounds = off[::lpc].tolist()  # first word of every chunk, then the total
        counts = self.out_count.tolist() if outliers else [0] * g.n_chunks
        geom1 = Geometry(1, g.n_heads, g.bph, g.tile_blocks)
        out = []
        for c in range(g.n_chunks):
            w0, w1 = int(bounds[c]), int(bounds[c + 1])
            lo = (off[c * lpc:(c + 1) * lpc + 1] - w0).to(torch.int32)
            n_out = int(counts[c])
            rec = None
            if n_out:
                base = c * self.out_cap * 10
                rec = self.out_rec[base:base + n_out * 10].view(n_out, 10).clone()
            sl = lambda t, n: t[c * n:(c + 1) * n].clone()  # noqa: E731
            out.append(LaneChunk(geom=geom1, bits=bits, orig_shape=tuple(shape), orig_dtype=dtype,
                                 scale_f32=sl(self.scale_f32, nh), scale_f16=sl(self.scale_f16, nh),
                                 coset_words=sl(self.coset_words, wpc), tile_n0=sl(self.tile_n0, nt),
                                 tab_lo=sl(self.tab_lo, NSTREAMS), tab_nsym=sl(self.tab_nsym, NSTREAMS),
                                 tab_freq=sl(self.tab_freq, NSTREAMS), words=self.words[w0:max(w1, w0 + 1)].clone(),
                                 lane_off=lo, lane_nbits=sl(self.lane_nbits, lpc),
                                 lane_state=sl(self.lane_state, lpc), n_words=w1 - w0, outlier_rec=rec,
                                 n_outliers=n_out))
        return out


# --------------------------------------------------------------------------
# allocating wrappers
# --------------------------------------------------------------------------
def _as_chunks(x: torch.Tensor, n_chunks: int) -> Tuple[int, int]:
    if x.dim() != 4:
        raise ValueError("expected a (batch, heads, seq, head_dim) tensor")
    b, h, s, d = x.shape
    if d % 8 != 0:
        raise ValueError("head_dim must be a multiple of 8")
    return (b * h) // n_chunks, s * d // 8


def compress(x: torch.Tensor, bits: float, tile_blocks: Optional[int] = DEFAULT_TILE_BLOCKS,
             scale_f32: Optional[torch.Tensor] = None, freqs: Optional[Tuple] = None, keep_deq: bool = False,
             q_out: Optional[torch.Tensor] = None):
    """Compress one (B, H, S, D) tensor as a chunk; returns (LaneChunk, deq or None).

    scale_f32: optional fp32 per-head scales to use instead of the computed ones.
    freqs: optional (tab_lo, tab_nsym, tab_freq) host/device tables replacing the
    device table build (e.g. tables normalised by numpy on the host).
    """
    _lib.require_cuda(x)
    x = x.contiguous()
    n_heads, bph = _as_chunks(x, 1)
    geom = Geometry(1, n_heads, bph, round_tile(tile_blocks, n_heads * bph))
    cd = Codec(geom, x.device, keep_deq=keep_deq, deq_dtype=x.dtype)
    if scale_f32 is None:
        cd.scales(x, bits)
    else:
        sf = scale_f32.to(device=x.device, dtype=torch.float32).reshape(-1)
        cd.scale_f32.copy_(sf)
        cd.scale_f16.copy_(sf.to(torch.float16))
    n_out = 0
    if freqs is None:
        n_out = cd.quantize_with_tables(x, q_out, blocks_per_token(x.shape[-1], geom.tile_blocks, bph))
    else:
        cd.quantize(x, q_out)
        lo, ns, fr = freqs
        cd.tab_lo.copy_(torch.as_tensor(lo, dtype=torch.int32).reshape(-1))
        cd.tab_nsym.copy_(torch.as_tensor(ns, dtype=torch.int32).reshape(-1))
        cd.tab_freq.copy_(torch.as_tensor(fr).to(torch.int32).to(torch.int16).reshape(NSTREAMS, L))
    cd.expand_tables(enc=True, dec=False)
    cd.entropy_encode()
    flags = cd.read_err()  # synchronises
    raise_flags(flags, "compress")
    nw = cd.n_words()
    chunk = LaneChunk(geom=geom, bits=bits, orig_shape=tuple(x.shape), orig_dtype=x.dtype,
                      scale_f32=cd.scale_f32, scale_f16=cd.scale_f16, coset_words=cd.coset_words,
                      tile_n0=cd.tile_n0, tab_lo=cd.tab_lo, tab_nsym=cd.tab_nsym, tab_freq=cd.tab_freq,
                      words=cd.words[:max(nw, 1)].clone(), lane_off=cd.lane_off, lane_nbits=cd.lane_nbits,
                      lane_state=cd.lane_state, n_words=nw,
                      outlier_rec=cd.out_rec[:n_out * 10].view(n_out, 10).clone() if n_out else None,
                      n_outliers=n_out)
    deq = cd.deq.view(x.shape) if keep_deq else None
    return chunk, deq


def expand_dec_tables(chunk: LaneChunk) -> torch.Tensor:
    if chunk.dec_tab is None:
        dev = chunk.words.device
        n_tab = chunk.tab_nsym.numel()
        dec = torch.empty(n_tab * L, dtype=torch.int32, device=dev)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        check(lib().lq_expand_tables(ptr(chunk.tab_nsym), ptr(chunk.tab_freq), n_tab, None, ptr(dec), ptr(err),
                                     stream_handle(dev)), "lq_expand_tables")
        chunk.dec_tab = dec
    return chunk.dec_tab


def staged_tables(chunk: LaneChunk) -> torch.Tensor:
    """The chunk's decode tables in the attention kernel's shared-memory form
    (lq_stage_tables, 64 KB per chunk), so each CTA fills its table region with
    one bulk copy.  Cached on the chunk."""
    st = getattr(chunk, "_staged_tab", None)
    if st is None:
        dec = expand_dec_tables(chunk)
        n_tab = chunk.tab_nsym.numel()
        st = torch.empty(n_tab * L, dtype=torch.int32, device=dec.device)
        check(lib().lq_stage_tables(ptr(dec), ptr(chunk.tab_lo), n_tab, ptr(st), stream_handle(dec.device)),
              "lq_stage_tables")
        chunk._staged_tab = st
    return st


def decompress(chunk: LaneChunk, out_dtype: Optional[torch.dtype] = None, want_symbols: bool = False):
    """Decode a LaneChunk to a tensor of its original shape (dtype out_dtype or the original)."""
    g = chunk.geom
    dev = chunk.words.device
    _lib.require_cuda()
    od = out_dtype or chunk.orig_dtype
    out = torch.empty(g.n_chunks * g.n_vectors * 8, dtype=od, device=dev)
    sym = torch.empty(g.n_chunks * g.n_vectors * 8, dtype=torch.int32, device=dev) if want_symbols else None
    dec = expand_dec_tables(chunk)
    ws = torch.empty(max(lib().lq_rans_decode_workspace(g.n_chunks, g.n_vectors, g.tile_blocks), 16),
                     dtype=torch.uint8, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    check(lib().lq_rans_decode(ptr(chunk.words), chunk.n_words, ptr(chunk.lane_off), ptr(chunk.lane_nbits),
                               ptr(chunk.lane_state), ptr(chunk.coset_words), ptr(chunk.tile_n0), g.n_chunks,
                               g.n_heads, g.bph, g.tile_blocks, ptr(chunk.tab_lo), ptr(chunk.tab_nsym),
                               ptr(chunk.tab_freq), ptr(dec), ptr(chunk.scale_f16), ptr(out),
                               _lib.dtype_code(od), ptr(sym), ptr(ws), ws.numel(), ptr(err), stream_handle(dev)),
          "lq_rans_decode")
    if chunk.n_outliers:
        patch_outliers(chunk, out, sym, err)
    raise_flags(int(err.item()) & 0xFFFFFFFF, "decompress")
    out = out.view(chunk.orig_shape)
    if want_symbols:
        return out, sym.view(-1, 8)
    return out


def lattice_points(chunk: LaneChunk) -> torch.Tensor:
    """The chunk's E8 points (n_blocks, 8) fp32, exactly: the decoded symbols
    (outlier records patched in) through symbols_to_e8 (core/entropy_coder.py:71-89)."""
    g = chunk.geom
    dev = chunk.words.device
    n = g.n_chunks * g.n_vectors
    _, sym = decompress(chunk, out_dtype=torch.float32, want_symbols=True)
    cos = torch.empty(n, dtype=torch.uint8, device=dev)
    s = stream_handle(dev)
    check(lib().lq_unpack_bits(ptr(chunk.coset_words), n, ptr(cos), s), "lq_unpack_bits")
    cos32 = cos.to(torch.int32)
    q = torch.empty(n, 8, dtype=torch.float32, device=dev)
    check(lib().lq_symbols_to_e8(ptr(cos32), ptr(sym.contiguous()), n, ptr(q), s), "lq_symbols_to_e8")
    return q


def patch_outliers(chunk: LaneChunk, out: Optional[torch.Tensor], sym: Optional[torch.Tensor],
                   err: torch.Tensor):
    """Write a chunk's outlier records back into its decoded output / symbols."""
    g = chunk.geom
    dev = chunk.words.device
    cnt = torch.tensor([chunk.n_outliers], dtype=torch.int32, device=dev)
    rec = chunk.outlier_rec.contiguous()
    check(lib().lq_patch_outliers(ptr(rec), ptr(cnt), 1, chunk.n_outliers, g.n_heads, g.bph, ptr(chunk.scale_f16),
                                  ptr(out), _lib.dtype_code(out.dtype) if out is not None else 0, ptr(sym), ptr(err),
                                  stream_handle(dev)), "lq_patch_outliers")
