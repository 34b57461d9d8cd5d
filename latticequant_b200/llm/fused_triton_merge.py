"""Compact fixed-rate chunks merged with an fp16 fallback -- the API of
llm/fused_triton_merge.py (and of llm/triton_kv_integration.py's decompress)
on the B200.

A ``CompressedChunk`` stores a (B, H, S, D) tensor as its E8 blocks: blocks
whose lattice coordinates fit b bits (check_representable,
core/compact_storage.py:235-249) as b-byte codes (pack_e8, :87-154), the
others as fp16 rows of their dequantised values, plus the representable mask
and the fp32 head scales.  ``fused_decompress_chunk`` is one CUDA pass over
all blocks (lq_compact_merge): decode a code times its head scale, or copy
the fallback row.  The reference's merge kernel takes coord7's parity with a
signed remainder and decodes blocks whose partial sum is odd and negative
wrongly; this one uses the non-negative remainder, as unpack_e8 does.
(The reference's own module imports a chunk class its cache no longer
defines; the chunk here carries the fields its kernel reads.)
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from .. import _lib, codec
from .._lib import check, lib, ptr, raise_flags, stream_handle
from ..core.compact_storage import check_representable, pack_e8
from .compressed_kv_cache import CompressedKVCache


@dataclass
class CompressedChunk:
    """Compact chunk: codes of the representable blocks + fp16 fallback rows."""
    packed: torch.Tensor        # (n_repr, b) uint8
    fallback: torch.Tensor      # (n_oor, 8) float16
    repr_mask: torch.Tensor     # (n_blocks,) bool
    scales: torch.Tensor        # (n_heads,) float32
    orig_shape: tuple
    blocks_per_head: int
    bits_per_dim: int
    orig_dtype: torch.dtype = torch.float16

    @property
    def n_vectors(self) -> int:
        return self.repr_mask.numel()

    @property
    def total_bytes(self) -> int:
        return (self.packed.numel() + self.fallback.numel() * 2 + (self.repr_mask.numel() + 7) // 8
                + self.scales.numel() * 4)

    @property
    def oor_rate(self) -> float:
        return self.fallback.shape[0] / max(self.n_vectors, 1)


def compress_compact(tensor: torch.Tensor, bits_per_dim: int = 4):
    """(B, H, S, D) -> (CompressedChunk, dequantised tensor): per-head scales and
    E8 points as _compress_tensor computes them (llm/compressed_kv_cache.py:176-204)."""
    _lib.require_cuda(tensor)
    x = tensor.contiguous()
    B, H, S, D = x.shape
    if D % 8:
        raise ValueError("head_dim must be a multiple of 8")
    n_heads, bph = B * H, S * D // 8
    # tiles of the codec's default size: a tile is one warp's work (no
    # bitstream is made here, so the tiling does not change any output)
    geom = codec.Geometry(1, n_heads, bph, codec.round_tile(codec.DEFAULT_TILE_BLOCKS, n_heads * bph))
    cd = codec.Codec(geom, x.device, keep_deq=True, deq_dtype=x.dtype)
    cd.scales(x, bits_per_dim)
    q = torch.empty(n_heads * bph, 8, dtype=torch.float32, device=x.device)
    cd.quantize(x, q)
    raise_flags(cd.read_err() & ~0x2, "compress_compact")  # symbol range is the coder's limit, not this layout's
    mask = check_representable(q, bits_per_dim)
    packed = pack_e8(q[mask], bits_per_dim) if bool(mask.any()) else torch.zeros(0, bits_per_dim, dtype=torch.uint8,
                                                                                  device=x.device)
    head = torch.arange(n_heads * bph, device=x.device) // bph
    fb = (q[~mask] * cd.scale_f32[head[~mask]].unsqueeze(1)).to(torch.float16).contiguous()
    chunk = CompressedChunk(packed=packed, fallback=fb, repr_mask=mask, scales=cd.scale_f32.clone(),
                            orig_shape=tuple(x.shape), blocks_per_head=bph, bits_per_dim=bits_per_dim,
                            orig_dtype=x.dtype)
    return chunk, cd.deq.view(x.shape).clone()


def fused_decompress_chunk(chunk: CompressedChunk) -> torch.Tensor:
    """One pass: decode representable blocks, copy fallback rows -> fp16 (B, H, S, D)
    (llm/fused_triton_merge.py:137-177)."""
    dev = chunk.repr_mask.device
    _lib.require_cuda(chunk.repr_mask)
    batch, heads, seq, hd = chunk.orig_shape
    bph = chunk.blocks_per_head
    n = batch * heads * bph
    assert n * 8 == batch * heads * seq * hd and chunk.repr_mask.numel() == n
    m = chunk.repr_mask.to(torch.int32)
    repr_rank = (torch.cumsum(m, 0) - m).to(torch.int32)
    fb_rank = (torch.arange(n, device=dev, dtype=torch.int32) - repr_rank).to(torch.int32)
    out = torch.empty(n, 8, dtype=torch.float16, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    mask8 = chunk.repr_mask.to(torch.uint8).contiguous()
    check(lib().lq_compact_merge(ptr(chunk.packed.contiguous()), chunk.packed.shape[0], chunk.bits_per_dim, ptr(mask8),
                                 ptr(repr_rank), ptr(fb_rank), ptr(chunk.fallback.contiguous()),
                                 chunk.fallback.shape[0], ptr(chunk.scales), batch * heads, bph, ptr(out), ptr(err),
                                 stream_handle(dev)), "lq_compact_merge")
    raise_flags(int(err.item()) & 0xFFFFFFFF, "fused_decompress_chunk")
    return out.reshape(batch, heads, seq, hd)


class FusedTritonKVCache(CompressedKVCache):
    """CompressedKVCache storing compact fixed-rate chunks (fp16 fallback for
    out-of-range blocks) and decompressing them with the fused merge."""

    def _compress_tensor(self, tensor: torch.Tensor):
        if tensor.shape[-1] % 8:
            return "uncompressible", tensor
        chunk, deq = compress_compact(tensor, self.bits)
        self.total_vectors += chunk.n_vectors
        return chunk, deq

    def _decompress_chunk(self, chunk) -> torch.Tensor:
        if isinstance(chunk, CompressedChunk):
            return fused_decompress_chunk(chunk)
        return super()._decompress_chunk(chunk)
