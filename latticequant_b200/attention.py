"""Fused dequant + decode attention over compressed K/V chunks (CUDA, sm_100a).

The reference serves decode attention from the dequantised buffer that
CompressedKVCache.update() returns (llm/compressed_kv_cache.py:342-395),
which transformers' SDPA reads after repeat_kv.  ``decode_attention`` reads
the compressed K and V chunks instead: lq_attn_decode rebuilds every E8
block in registers (symbols_to_e8, core/entropy_coder.py:71-89, times the
fp16 head scale, llm/compressed_kv_cache.py:330) and folds it into the
softmax of the query heads that share its KV head.  ``merge_attention``
combines results over disjoint key sets (the chunks of one layer, or the
sequence shards of several GPUs) from their log-sum-exp.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional, Sequence, Tuple

import torch

from . import _lib
from ._lib import ChunkView, check, lib, ptr, raise_flags, stream_handle
from .codec import LaneChunk, decompress, expand_dec_tables, staged_tables


def chunk_view(chunk: LaneChunk) -> ChunkView:
    """The C view (struct lq_chunk_view) of a single-chunk LaneChunk."""
    g = chunk.geom
    if g.n_chunks != 1:
        raise ValueError("attention reads one chunk per K/V tensor")
    dec = expand_dec_tables(chunk)
    v = ChunkView()
    v.words = chunk.words.data_ptr()
    v.n_words = chunk.n_words
    v.lane_off = chunk.lane_off.data_ptr()
    v.lane_nbits = chunk.lane_nbits.data_ptr()
    v.lane_state = chunk.lane_state.data_ptr()
    v.coset_words = chunk.coset_words.data_ptr()
    v.tile_n0 = chunk.tile_n0.data_ptr()
    v.tab_lo = chunk.tab_lo.data_ptr()
    v.tab_nsym = chunk.tab_nsym.data_ptr()
    v.tab_freq = chunk.tab_freq.data_ptr()
    v.dec_tab = dec.data_ptr()
    v.scale_f16 = chunk.scale_f16.data_ptr()
    v.n_heads = g.n_heads
    v.bph = g.bph
    v.tile_blocks = g.tile_blocks
    v.staged_tab = staged_tables(chunk).data_ptr()
    return v


def attention_workspace_bytes(k_chunk: LaneChunk, group: int) -> int:
    g = k_chunk.geom
    d = k_chunk.orig_shape[-1]
    return int(lib().lq_attn_decode_workspace(g.n_heads, g.bph, g.tile_blocks, group, d))


def supports(k_chunk: LaneChunk, group: int) -> bool:
    """Whether the fused kernel takes this chunk geometry (head_dim 64/128,
    group 1..8, tiles that do not straddle heads)."""
    return attention_workspace_bytes(k_chunk, group) > 0


def _q3(q: torch.Tensor, kshape) -> torch.Tensor:
    B, Hkv, S, D = kshape
    if q.dim() == 4:
        if q.shape[2] != 1:
            raise ValueError("decode attention takes one query position")
        q3 = q.reshape(q.shape[0], q.shape[1], q.shape[3])
    elif q.dim() == 3:
        q3 = q
    else:
        raise ValueError("q must be (B, Hq, D) or (B, Hq, 1, D)")
    if q3.shape[0] != B or q3.shape[2] != D or q3.shape[1] % Hkv != 0:
        raise ValueError(f"q {tuple(q.shape)} does not match K/V {tuple(kshape)}")
    return q3


class DecodeAttention:
    """A prepared fused attention over one (K chunk, V chunk) pair: device
    workspace and error word allocated once, launches without host syncs (so
    a decode step can be captured in a CUDA graph); flags() reads the error word."""

    def __init__(self, k_chunk: LaneChunk, v_chunk: LaneChunk, group: int, shape: Optional[Tuple[int, ...]] = None,
                 scale_per_token: bool = False):
        """shape: the attention geometry (B, Hkv, S, D); by default the chunks'
        tensor shape.  scale_per_token: the chunks were compressed from the
        (B, Hkv*S, 1, D) view, i.e. with one scale per token (decode appends)."""
        kshape, vshape = tuple(k_chunk.orig_shape), tuple(v_chunk.orig_shape)
        if len(kshape) != 4 or kshape != vshape:
            raise ValueError("K and V chunks must hold tensors of one 4-d shape")
        if shape is None:
            if scale_per_token:
                raise ValueError("per-token chunks need the attention shape")
            shape = kshape
        shape = tuple(int(d) for d in shape)
        B, Hkv, S, D = shape
        if scale_per_token and kshape != (B, Hkv * S, 1, D):
            raise ValueError(f"per-token chunk shape {kshape} does not match {shape}")
        if not scale_per_token and kshape != shape:
            raise ValueError(f"chunk shape {kshape} does not match {shape}")
        self.shape = shape
        self.scale_per_token = bool(scale_per_token)
        self.group = int(group)
        self.k, self.v = k_chunk, v_chunk
        self.kv, self.vv = chunk_view(k_chunk), chunk_view(v_chunk)
        need = int(lib().lq_attn_decode_workspace(B * Hkv, S * D // 8, k_chunk.geom.tile_blocks, self.group, D))
        if need == 0:
            raise ValueError(f"fused attention does not take head_dim={D}, group={group}, "
                             f"tile_blocks={k_chunk.geom.tile_blocks} with {S * D // 8} blocks per head")
        dev = k_chunk.words.device
        self.workspace = torch.empty(need, dtype=torch.uint8, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.mask = None
        if k_chunk.n_outliers or v_chunk.n_outliers:
            self._prepare_outliers()

    def _prepare_outliers(self):
        """Tokens with outlier records in K or V are left out of the fused kernel
        (tok_mask) and attended exactly from their decoded rows."""
        B, Hkv, S, D = self.shape
        bpt = D // 8
        dev = self.k.words.device
        toks = []
        for ch in (self.k, self.v):
            if ch.n_outliers:
                toks.append(ch.outlier_rec[:, 0].long() // bpt)  # token index over all heads (head-major)
        tg = torch.unique(torch.cat(toks))
        words = (S + 31) // 32
        mask = torch.zeros(B * Hkv * words, dtype=torch.int64, device=dev)
        lh, tok = tg // S, tg % S
        mask.index_add_(0, lh * words + tok // 32, torch.ones_like(tok) << (tok % 32))
        self.mask = mask.to(torch.int32)  # bit patterns fit: each bit is added once
        kd = decompress(self.k, out_dtype=torch.float32).reshape(B * Hkv, S, D)
        vd = decompress(self.v, out_dtype=torch.float32).reshape(B * Hkv, S, D)
        self.ex_head = lh
        self.ex_k = kd[lh, tok].contiguous()
        self.ex_v = vd[lh, tok].contiguous()

    def _launch(self, q3, out, lse, sm_scale):
        B, Hkv, S, D = self.shape
        check(lib().lq_attn_decode(ctypes.byref(self.kv), ctypes.byref(self.vv), ptr(q3), _lib.dtype_code(q3.dtype),
                                   B, Hkv, S, int(self.scale_per_token), self.group, D, float(sm_scale), ptr(out),
                                   _lib.dtype_code(out.dtype), ptr(lse), ptr(self.mask), ptr(self.workspace),
                                   self.workspace.numel(), ptr(self.err), stream_handle(q3.device)), "lq_attn_decode")

    def __call__(self, q3: torch.Tensor, out: torch.Tensor, lse: Optional[torch.Tensor] = None,
                 sm_scale: Optional[float] = None):
        B, Hkv, S, D = self.shape
        if sm_scale is None:
            sm_scale = 1.0 / math.sqrt(D)
        if self.mask is None:
            self._launch(q3, out, lse, sm_scale)
            return
        # fused part without the outlier tokens, exact part over them, merged by lse
        rows = q3.shape[0] * q3.shape[1]
        o1 = torch.empty(q3.shape, dtype=torch.float32, device=q3.device)
        l1 = torch.empty(q3.shape[:2], dtype=torch.float32, device=q3.device)
        self._launch(q3, o1, l1, sm_scale)
        qf = q3.float().reshape(rows, D)
        row_head = (torch.arange(rows, device=q3.device) // q3.shape[1]) * Hkv + \
                   (torch.arange(rows, device=q3.device) % q3.shape[1]) // self.group
        s = (qf @ self.ex_k.T) * sm_scale
        s = s.masked_fill(row_head[:, None] != self.ex_head[None, :], float("-inf"))
        l2 = torch.logsumexp(s, -1)
        w = torch.exp(s - torch.where(torch.isfinite(l2), l2, torch.zeros_like(l2))[:, None])
        o2 = (w @ self.ex_v)
        merge_attention(torch.stack([o1.reshape(rows, D), o2]), torch.stack([l1.reshape(rows), l2]),
                        out=out.view(rows, D), lse=lse.view(rows) if lse is not None else None)

    def flags(self) -> int:
        return int(self.err.item()) & 0xFFFFFFFF


def decode_attention(q: torch.Tensor, k_chunk: LaneChunk, v_chunk: LaneChunk, sm_scale: Optional[float] = None,
                     out_dtype: Optional[torch.dtype] = None, return_lse: bool = False,
                     out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None):
    """softmax(q K^T * sm_scale) V for one decode step, K/V read compressed.

    q: (B, Hq, D) or (B, Hq, 1, D) on the device; K/V chunks of a (B, Hkv, S, D)
    tensor each with Hq a multiple of Hkv (GQA as repeat_kv).  Returns o with
    q's shape (and the fp32 (B, Hq) log-sum-exp of the scores if return_lse).
    """
    _lib.require_cuda(q)
    q3 = _q3(q, tuple(k_chunk.orig_shape)).contiguous()
    Hkv, D = k_chunk.orig_shape[1], k_chunk.orig_shape[3]
    op = DecodeAttention(k_chunk, v_chunk, q3.shape[1] // Hkv)
    dev = q.device
    if out is None:
        out = torch.empty(q3.shape, dtype=out_dtype or q.dtype, device=dev)
    if return_lse and lse is None:
        lse = torch.empty(q3.shape[:2], dtype=torch.float32, device=dev)
    op(q3, out, lse if return_lse else None, sm_scale)
    raise_flags(op.flags(), "decode_attention")
    o = out.view(tuple(q.shape[:-1]) + (D,)) if q.dim() == 4 else out
    return (o, lse) if return_lse else o


def compact_index(chunk) -> Tuple[torch.Tensor, torch.Tensor]:
    """(mask_words, word_rank) of a compact chunk (llm.fused_triton_merge.
    CompressedChunk): bit i of word w marks block 32w+i representable; the
    rank is the representable blocks before word w.  Cached on the chunk."""
    cached = getattr(chunk, "_lq_index", None)
    if cached is not None:
        return cached
    m = chunk.repr_mask.reshape(-1)
    n = m.numel()
    nw = (n + 31) // 32
    bits = torch.zeros(nw * 32, dtype=torch.int64, device=m.device)
    bits[:n] = m.to(torch.int64)
    bits = bits.view(nw, 32)
    words = (bits << torch.arange(32, device=m.device, dtype=torch.int64)).sum(1)
    words = torch.where(words >= 2 ** 31, words - 2 ** 32, words).to(torch.int32).contiguous()
    cnt = bits.sum(1)
    rank = (torch.cumsum(cnt, 0) - cnt).to(torch.int32).contiguous()
    chunk._lq_index = (words, rank)
    return chunk._lq_index


def compact_view(chunk) -> "_lib.CompactView":
    words, rank = compact_index(chunk)
    B, H, S, D = chunk.orig_shape
    packed = chunk.packed.contiguous()
    fb = chunk.fallback.contiguous()
    return _lib.CompactView(packed.data_ptr() if packed.numel() else None, packed.shape[0],
                            fb.data_ptr() if fb.numel() else None, fb.shape[0], words.data_ptr(), rank.data_ptr(),
                            chunk.scales.data_ptr(), B * H, S * D // 8, int(chunk.bits_per_dim))


class CompactDecodeAttention:
    """decode_attention_compact prepared once for a (K chunk, V chunk) pair
    (llm.fused_triton_merge.CompressedChunk each): workspace, error word and
    chunk views allocated up front, launches without host syncs; flags()
    reads the error word."""

    def __init__(self, k_chunk, v_chunk, group: int):
        kshape = tuple(k_chunk.orig_shape)
        if tuple(v_chunk.orig_shape) != kshape:
            raise ValueError("K and V chunks differ in shape")
        self.k, self.v, self.group, self.shape = k_chunk, v_chunk, int(group), kshape
        B, Hkv, S, D = kshape
        dev = k_chunk.repr_mask.device
        _lib.require_cuda(k_chunk.repr_mask)
        need = int(lib().lq_attn_compact_workspace(B * Hkv, S, self.group, D))
        if need == 0:
            raise ValueError(f"compact attention does not take shape {kshape} with group {group} "
                             "(head_dim 64/128, seq*head_dim/8 a multiple of 32, group 1..8)")
        self.workspace = torch.empty(need, dtype=torch.uint8, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.kv, self.vv = compact_view(k_chunk), compact_view(v_chunk)

    def __call__(self, q3: torch.Tensor, out: torch.Tensor, lse: Optional[torch.Tensor] = None,
                 sm_scale: Optional[float] = None):
        """q3 (B, Hq, D) contiguous -> out (B, Hq, D); lse (B, Hq) fp32 if given."""
        B, Hkv, S, D = self.shape
        if q3.shape != (B, Hkv * self.group, D) or not q3.is_contiguous():
            raise ValueError(f"q must be a contiguous ({B}, {Hkv * self.group}, {D}) tensor")
        scale = (1.0 / math.sqrt(D)) if sm_scale is None else float(sm_scale)
        check(lib().lq_attn_decode_compact(ctypes.byref(self.kv), ctypes.byref(self.vv), ptr(q3),
                                           _lib.dtype_code(q3.dtype), B, Hkv, S, self.group, D, scale, ptr(out),
                                           _lib.dtype_code(out.dtype), ptr(lse) if lse is not None else None,
                                           ptr(self.workspace), self.workspace.numel(), ptr(self.err),
                                           stream_handle(q3.device)), "lq_attn_decode_compact")
        return out

    def flags(self) -> int:
        return int(self.err.item()) & 0xFFFFFFFF


def decode_attention_compact(q: torch.Tensor, k_chunk, v_chunk, sm_scale: Optional[float] = None,
                             out_dtype: Optional[torch.dtype] = None, return_lse: bool = False,
                             out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None):
    """decode_attention over compact-layout chunks (llm.fused_triton_merge.
    CompressedChunk of a (B, Hkv, S, D) tensor each): the reference merges
    them into fp16 K/V for SDPA (llm/fused_triton_merge.py:137-177); here one
    kernel reads the codes and fallback rows and attends.  Same arguments and
    results as decode_attention."""
    _lib.require_cuda(q)
    kshape = tuple(k_chunk.orig_shape)
    if tuple(v_chunk.orig_shape) != kshape:
        raise ValueError("K and V chunks differ in shape")
    q3 = _q3(q, kshape).contiguous()
    B, Hkv, S, D = kshape
    op = CompactDecodeAttention(k_chunk, v_chunk, q3.shape[1] // Hkv)
    dev = q.device
    if out is None:
        out = torch.empty(q3.shape, dtype=out_dtype or q.dtype, device=dev)
    if return_lse and lse is None:
        lse = torch.empty(q3.shape[:2], dtype=torch.float32, device=dev)
    op(q3, out, lse if return_lse else None, sm_scale)
    raise_flags(op.flags(), "decode_attention_compact")
    o = out.view(tuple(q.shape[:-1]) + (D,)) if q.dim() == 4 else out
    return (o, lse) if return_lse else o


def merge_attention(o_parts: Sequence[torch.Tensor] | torch.Tensor, lse_parts: Sequence[torch.Tensor] | torch.Tensor,
                    out_dtype: Optional[torch.dtype] = None, out: Optional[torch.Tensor] = None,
                    lse: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Combine attention over disjoint key sets: o = sum_i o_i exp(lse_i - lse).

    o_parts: n tensors (or one stacked tensor) of shape (..., D); lse_parts the
    matching (...) log-sum-exps.  Returns (o, lse); out / lse may be given."""
    o = torch.stack(list(o_parts)) if not torch.is_tensor(o_parts) else o_parts
    ls = torch.stack(list(lse_parts)) if not torch.is_tensor(lse_parts) else lse_parts
    _lib.require_cuda(o)
    n, D = o.shape[0], o.shape[-1]
    rows = o[0].numel() // D
    if ls.numel() != n * rows:
        raise ValueError("lse parts do not match the o parts")
    of = o.reshape(n, rows, D)
    of = of if (of.dtype == torch.float32 and of.is_contiguous()) else of.to(torch.float32).contiguous()
    lf = ls.reshape(n, rows)
    lf = lf if (lf.dtype == torch.float32 and lf.is_contiguous()) else lf.to(torch.float32).contiguous()
    if out is None:
        out = torch.empty((rows, D), dtype=out_dtype or o.dtype, device=o.device)
    if lse is None:
        lse = torch.empty(rows, dtype=torch.float32, device=o.device)
    if out.numel() != rows * D or lse.numel() != rows or not out.is_contiguous():
        raise ValueError("merge outputs have the wrong size")
    check(lib().lq_attn_merge(ptr(of), ptr(lf), n, rows, D, ptr(out), _lib.dtype_code(out.dtype), ptr(lse),
                              stream_handle(o.device)), "lq_attn_merge")
    return out.view(o.shape[1:]), lse.view(ls.shape[1:])


def merge_attention_packed(parts: torch.Tensor, rows: int, head_dim: int, out_dtype: torch.dtype = torch.float32,
                           out: Optional[torch.Tensor] = None,
                           lse: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """merge_attention over parts packed as one fp32 tensor (n_parts, rows *
    head_dim + rows): each part's o rows, then its lse values -- what one
    all-gather of every rank's packed (o, lse) gives.  Returns (o (rows, D), lse (rows,))."""
    _lib.require_cuda(parts)
    if parts.dtype != torch.float32 or not parts.is_contiguous() or parts.dim() != 2 or \
            parts.shape[1] != rows * (head_dim + 1):
        raise ValueError("parts must be a contiguous fp32 (n_parts, rows * (head_dim + 1)) tensor")
    if out is None:
        out = torch.empty((rows, head_dim), dtype=out_dtype, device=parts.device)
    if lse is None:
        lse = torch.empty(rows, dtype=torch.float32, device=parts.device)
    check(lib().lq_attn_merge_packed(ptr(parts), parts.shape[0], rows, head_dim, ptr(out), _lib.dtype_code(out.dtype),
                                     ptr(lse), stream_handle(parts.device)), "lq_attn_merge_packed")
    return out, lse


def dense_merge_attention(q: torch.Tensor, segments: Sequence[tuple], o_parts: Optional[torch.Tensor],
                          lse_parts: Optional[torch.Tensor], n_kv_heads: int, sm_scale: Optional[float] = None,
                          out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Attention of one decode position over dense K/V segments, merged with the
    finished attention of compressed parts, in one launch (lq_attn_dense_merge).

    q: (B, Hq, D) or (B, Hq, 1, D); segments: (k, v, n) with k, v contiguous
    (B, n_kv_heads, cap, D) buffers of which the first n tokens count -- n an
    int, or a (1,) int64 device tensor holding the last valid slot (n = value +
    1, read on the device: CUDA-graph replays); o_parts / lse_parts: stacked
    (n_parts, B, Hq, D) fp32 and (n_parts, B, Hq) fp32 (natural log) or None.
    Returns (B, Hq, D) in q's dtype (written to `out` if given); `lse`
    (B, Hq) fp32 optional."""
    _lib.require_cuda(q)
    B, Hq, D = q.shape[0], q.shape[1], q.shape[-1]
    if Hq % n_kv_heads != 0:
        raise ValueError("query heads must be a multiple of the kv heads")
    if len(segments) > _lib.DENSE_MAX_SEGMENTS:
        raise ValueError(f"at most {_lib.DENSE_MAX_SEGMENTS} dense segments")
    q3 = q.reshape(B, Hq, D)
    q3 = q3 if q3.is_contiguous() else q3.contiguous()
    scale = (1.0 / math.sqrt(D)) if sm_scale is None else float(sm_scale)
    n = len(segments)
    kp = (ctypes.c_void_p * max(n, 1))()
    vp = (ctypes.c_void_p * max(n, 1))()
    cap = (ctypes.c_int64 * max(n, 1))()
    ln = (ctypes.c_int64 * max(n, 1))()
    last = (ctypes.c_void_p * max(n, 1))()
    kv_dtype = None
    for i, (k, v, cnt) in enumerate(segments):
        if k.shape != v.shape or k.dim() != 4 or k.shape[0] != B or k.shape[1] != n_kv_heads or k.shape[3] != D \
                or not (k.is_contiguous() and v.is_contiguous()) or k.dtype != v.dtype:
            raise ValueError("dense segments must be contiguous (B, n_kv_heads, cap, D) K/V pairs of one dtype")
        if kv_dtype is not None and k.dtype != kv_dtype:
            raise ValueError("dense segments must share one dtype")
        kv_dtype = k.dtype
        kp[i], vp[i], cap[i] = k.data_ptr(), v.data_ptr(), k.shape[2]
        if torch.is_tensor(cnt):
            if cnt.dtype != torch.int64 or cnt.device != q.device:
                raise ValueError("a device segment length is a (1,) int64 tensor on the query's device")
            ln[i], last[i] = 0, cnt.data_ptr()
        else:
            if not 0 <= int(cnt) <= k.shape[2]:
                raise ValueError("a dense segment's length exceeds its buffer")
            ln[i], last[i] = int(cnt), None
    n_parts = 0
    if o_parts is not None:
        n_parts = o_parts.shape[0]
        if o_parts.dtype != torch.float32 or lse_parts is None or lse_parts.dtype != torch.float32 or \
                not (o_parts.is_contiguous() and lse_parts.is_contiguous()) or \
                o_parts.numel() != n_parts * B * Hq * D or lse_parts.numel() != n_parts * B * Hq:
            raise ValueError("parts must be contiguous fp32 (n_parts, B, Hq, D) and (n_parts, B, Hq) tensors")
    if out is None:
        out = torch.empty(B, Hq, D, dtype=q.dtype, device=q.device)
    if out.dtype != q.dtype or out.numel() != B * Hq * D or not out.is_contiguous():
        raise ValueError("out must be a contiguous (B, Hq, D) tensor of the query's dtype")
    if lse is not None and (lse.dtype != torch.float32 or lse.numel() != B * Hq or not lse.is_contiguous()):
        raise ValueError("lse must be a contiguous fp32 (B, Hq) tensor")
    check(lib().lq_attn_dense_merge(
        ptr(q3), _lib.dtype_code(q.dtype), n, *(ctypes.cast(a, ctypes.c_void_p) for a in (kp, vp, cap, ln, last)),
        _lib.dtype_code(kv_dtype) if kv_dtype is not None else _lib.dtype_code(q.dtype),
        ptr(o_parts) if n_parts else None, ptr(lse_parts) if n_parts else None, n_parts, B, n_kv_heads, Hq // n_kv_heads,
        D, scale, ptr(out), ptr(lse), stream_handle(q.device)), "lq_attn_dense_merge")
    return out
