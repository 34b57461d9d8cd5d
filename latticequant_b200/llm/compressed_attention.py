"""A CompressedKVCache whose decode steps attend over the compressed cache.

The reference keeps a resident dequantised copy of every layer's K/V next to
its compressed chunks (update() concatenates the new dequantised tokens and
returns the whole buffer, llm/compressed_kv_cache.py:377-395), so its actual
memory ratio is below 1.  ``CompressedAttentionKVCache`` keeps per layer:

* the compressed chunks: a prefill chunk with one scale per (batch, KV head)
  exactly as the reference's ``_compress_tensor`` makes it, and chunks of
  ``tail_tokens`` decode tokens encoded together ("lazy per-tile encoding"),
  each token keeping the scale the reference gives its own one-token chunk
  (the tail is compressed through its (B, Hkv*T, 1, D) view, so every token
  is a head of the chunk);
* the tail of decode tokens not yet encoded: raw (to encode them later) and
  dequantised with the fp32 scale, as update() returns them.

A decode step (one query position) runs the fused kernel (lq_attn_decode)
over every chunk and exact attention over the tail, then merges the parts by
log-sum-exp (lq_attn_merge).  ``lq_compressed_attention`` is the
transformers attention function that does this inside a model: register it
with ``register_attention()`` and attach the cache with ``cache.bind(model)``.
Prefill (several query positions) keeps the reference's semantics: attention
over the dequantised K/V that update() returns.
"""
from __future__ import annotations

import math
from typing import List, Optional, Tuple

import torch

from .. import attention as A
from .. import codec
from ..codec import LaneChunk
from .compressed_kv_cache import CompressedKVCache, CompressedKVLayer, OptimizedChunk

ATTN_NAME = "lq_compressed"
# rANS layout: flushed tails are attended from their dequantised tokens up to
# this many per layer, and beyond it from per-token-scale parts of at most
# this many tokens each (recoded together as tails arrive)
TAIL_MERGE_MAX = 1024


def _attn_tile(bph: int, limit: int) -> Optional[int]:
    """Largest tile (multiple of 32, at most `limit`) dividing the blocks per head."""
    t = (min(limit, bph) // 32) * 32
    while t >= 32:
        if bph % t == 0:
            return t
        t -= 32
    return None


class _Part:
    """One compressed (K, V) chunk pair of a layer and its prepared attention:
    LaneChunks (rANS lanes) or, for layout "compact", CompressedChunks.
    opt_k / opt_v: the layer's stored chunk objects the part reads (rANS)."""

    def __init__(self, k, v, shape, per_token: bool, layout: str = "rans", opt_k=None, opt_v=None):
        self.k, self.v, self.shape, self.per_token, self.layout = k, v, tuple(shape), per_token, layout
        self.opt_k, self.opt_v = opt_k, opt_v
        self.ops = {}

    def op(self, group: int):
        if group not in self.ops:
            if self.layout == "compact":
                self.ops[group] = A.CompactDecodeAttention(self.k, self.v, group)
            else:
                self.ops[group] = A.DecodeAttention(self.k, self.v, group, shape=self.shape,
                                                    scale_per_token=self.per_token)
        return self.ops[group]


class _LayerState:
    def __init__(self):
        self.parts: List[_Part] = []
        self.dense_k: List[torch.Tensor] = []  # chunks the fused kernel cannot take, kept dequantised
        self.dense_v: List[torch.Tensor] = []
        self.tail_raw_k = self.tail_raw_v = None
        self.tail_deq_k = self.tail_deq_v = None
        self.n_tail = 0
        self.seq = 0
        # flushed tails kept dequantised, appended to one buffer that grows by
        # doubling; its token count is also on the device (as the last valid
        # index), where the attention reads it, so a captured decode step stays
        # valid across flushes until the buffer has to grow
        self.tail_dense_k = self.tail_dense_v = None
        self.n_tail_dense = 0
        self.tail_dense_last: Optional[torch.Tensor] = None

    # dense segments a decode step attends besides the open tail: at most
    # this many (consolidated into one tensor when the list reaches it)
    MAX_DENSE = 4

    def push_dense(self, k: torch.Tensor, v: torch.Tensor):
        """Keep a (B, H, n, D) K/V pair dequantised (attended by lq_attn_dense_merge)."""
        self.dense_k.append(k.contiguous())
        self.dense_v.append(v.contiguous())
        self.consolidate()

    def consolidate(self):
        if len(self.dense_k) >= self.MAX_DENSE:
            self.dense_k = [torch.cat(self.dense_k, 2)]
            self.dense_v = [torch.cat(self.dense_v, 2)]

    def reserve_tail_dense(self, like: torch.Tensor, tokens: int):
        """Make the dense tail buffer hold at least `tokens` tokens shaped like
        `like` (B, H, *, D) (a new, doubled buffer when it must grow)."""
        old = self.tail_dense_k
        if old is not None and old.shape[2] >= tokens:
            return
        B, H, _, D = like.shape
        cap = max(tokens, 2 * old.shape[2] if old is not None else 0)
        k = torch.empty(B, H, cap, D, dtype=like.dtype, device=like.device)
        v = torch.empty_like(k)
        if self.n_tail_dense:
            k[:, :, :self.n_tail_dense].copy_(old[:, :, :self.n_tail_dense])
            v[:, :, :self.n_tail_dense].copy_(self.tail_dense_v[:, :, :self.n_tail_dense])
        self.tail_dense_k, self.tail_dense_v = k, v
        if self.tail_dense_last is None:
            self.tail_dense_last = torch.full((1,), self.n_tail_dense - 1, dtype=torch.int64, device=like.device)

    def push_tail_dense(self, k: torch.Tensor, v: torch.Tensor):
        """Append flushed tail tokens (B, H, n, D), kept dequantised."""
        n = k.shape[2]
        self.reserve_tail_dense(k, self.n_tail_dense + n)
        self.tail_dense_k[:, :, self.n_tail_dense:self.n_tail_dense + n].copy_(k)
        self.tail_dense_v[:, :, self.n_tail_dense:self.n_tail_dense + n].copy_(v)
        self.n_tail_dense += n
        self.tail_dense_last.fill_(self.n_tail_dense - 1)

    def dense_tail_tokens(self):
        """(K, V) of the flushed tails kept dequantised, or None."""
        if not self.n_tail_dense:
            return None
        return self.tail_dense_k[:, :, :self.n_tail_dense], self.tail_dense_v[:, :, :self.n_tail_dense]


class CompressedAttentionKVCache(CompressedKVCache):
    """CompressedKVCache without the resident dequantised buffer; see the module text.

      tail_tokens  decode tokens encoded together (a multiple of 2; 64 makes
                   one 1024-block tile per (batch, KV head) at head_dim 128)
      layout       "rans" (entropy-coded lanes, llm/compressed_kv_cache.py's
                   format) or "compact" (the fixed-rate codes + fp16 fallback
                   rows of llm/fused_triton_merge.py, bits 3..5): prefill
                   chunks in that layout are attended with
                   lq_attn_decode_compact; encoded tails stay dequantised
    """

    def __init__(self, bits_per_dim: int = 4, tail_tokens: int = 64,
                 tile_blocks: Optional[int] = codec.DEFAULT_TILE_BLOCKS, table_mode: str = "device",
                 head_range: Optional[Tuple[int, int]] = None, group=None, layout: str = "rans"):
        super().__init__(bits_per_dim=bits_per_dim, eval_only_no_entropy=False, tile_blocks=tile_blocks,
                         table_mode=table_mode)
        if layout not in ("rans", "compact"):
            raise ValueError("layout must be 'rans' or 'compact'")
        if layout == "compact" and bits_per_dim not in (3, 4, 5):
            raise ValueError("the compact layout takes 3, 4 or 5 bits per dimension")
        self.layout = layout
        if tail_tokens < 2 or tail_tokens % 2:
            raise ValueError("tail_tokens must be an even number >= 2")
        self.tail_tokens = int(tail_tokens)
        self._state: List[_LayerState] = []
        # KV-head sharding: keep only KV heads [h0, h1) of every layer; the
        # attention function attends with their query heads and all-gathers
        # the heads' outputs over `group` (torch.distributed; None = default)
        self.head_range = None if head_range is None else (int(head_range[0]), int(head_range[1]))
        self.group = group
        self.n_kv_heads_total = None
        self._qcodecs = {}  # decode-step quantisers, one per token shape (buffers reused every step)
        self._graph_idx: Optional[torch.Tensor] = None  # graph mode: the tail slot of the step, on the device
        self._tail_ar: Optional[torch.Tensor] = None

    # ---- storage -----------------------------------------------------------
    def _layer(self, i: int) -> _LayerState:
        while len(self._state) <= i:
            self._state.append(_LayerState())
        while len(self._comp_keys) <= i:
            self._comp_keys.append(None)
            self._comp_values.append(None)
        if self._comp_keys[i] is None:
            self._comp_keys[i] = CompressedKVLayer()
            self._comp_values[i] = CompressedKVLayer()
        return self._state[i]

    def _compress_with_tile(self, x: torch.Tensor, tile: int, scale_f32: Optional[torch.Tensor] = None):
        saved = self.tile_blocks
        self.tile_blocks = tile
        try:
            return self._compress_tensor(x, scale_f32=scale_f32)
        finally:
            self.tile_blocks = saved

    def _quantise_only(self, x: torch.Tensor) -> torch.Tensor:
        """update()'s dequantised output for x (q * fp32 scale in x's dtype), no coding."""
        b, h, s, d = x.shape
        key = (b, h, s, d, x.dtype, x.device)
        cd = self._qcodecs.get(key)
        if cd is None:
            # 32-block tiles: a tile is one warp's work, and a decode step's
            # tokens are few blocks (the values do not depend on the tiling)
            geom = codec.Geometry(1, b * h, s * d // 8, codec.round_tile(32, b * h * s * d // 8))
            cd = self._qcodecs[key] = codec.Codec(geom, x.device, keep_deq=True, deq_dtype=x.dtype)
        cd.scales(x.contiguous(), self.bits)
        cd.quantize(x.contiguous())
        return cd.deq.view(x.shape).clone()

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        if self._model_dtype is None:
            self._model_dtype = key_states.dtype
        if self.head_range is not None:
            self.n_kv_heads_total = key_states.shape[1]
            h0, h1 = self.head_range
            key_states = key_states[:, h0:h1].contiguous()
            value_states = value_states[:, h0:h1].contiguous()
        st = self._layer(layer_idx)
        B, H, S, D = key_states.shape
        if D % 8 != 0 or D not in (64, 128):
            raise ValueError("CompressedAttentionKVCache needs head_dim 64 or 128")
        if S > 1 or st.seq == 0:
            return self._update_chunk(st, layer_idx, key_states, value_states)
        return self._update_token(st, layer_idx, key_states, value_states)

    def _update_chunk(self, st, layer_idx, k, v):
        """A multi-token update: one chunk, as the reference compresses it."""
        B, H, S, D = k.shape
        history = self._materialise(st) if st.seq > 0 else None
        self._flush_tail(st, layer_idx, force=True)
        if self.layout == "compact":
            from .fused_triton_merge import compress_compact, fused_decompress_chunk

            ck, kd = compress_compact(k, int(self.bits))
            cv, vd = compress_compact(v, int(self.bits))
            self.total_vectors += ck.n_vectors + cv.n_vectors
            self._comp_keys[layer_idx].append_chunk(ck)
            self._comp_values[layer_idx].append_chunk(cv)
            if (S * D // 8) % 32 == 0:
                st.parts.append(_Part(ck, cv, (B, H, S, D), per_token=False, layout="compact"))
            else:  # heads not 32-block aligned: keep this chunk merged (fp16 values)
                st.push_dense(fused_decompress_chunk(ck), fused_decompress_chunk(cv))
            st.seq += S
            if history is not None:
                return torch.cat([history[0], kd], 2), torch.cat([history[1], vd], 2)
            return kd, vd
        tile = _attn_tile(S * D // 8, self.tile_blocks or codec.DEFAULT_TILE_BLOCKS)
        ck, kd = self._compress_with_tile(k, tile or 32)
        cv, vd = self._compress_with_tile(v, tile or 32)
        self._comp_keys[layer_idx].append_chunk(ck)
        self._comp_values[layer_idx].append_chunk(cv)
        if tile is not None:
            st.parts.append(_Part(ck.lanes, cv.lanes, (B, H, S, D), per_token=False))
        else:  # no tile divides the blocks per head: keep this chunk dequantised (fp16 scale)
            st.push_dense(self._decompress_chunk(ck), self._decompress_chunk(cv))
        st.seq += S
        if history is not None:
            return torch.cat([history[0], kd], 2), torch.cat([history[1], vd], 2)
        return kd, vd

    def _update_token(self, st, layer_idx, k, v):
        """A one-token update: quantise now (update()'s output), encode with the tail later."""
        B, H, S, D = k.shape
        T = self.tail_tokens
        if self._graph_idx is not None:
            # graph mode: the slot is a device index, the host bookkeeping is
            # graph_advance()'s (a replayed step runs none of this Python)
            kvd = self._quantise_only(torch.cat([k, v], 1))
            idx = self._graph_idx
            st.tail_raw_k.index_copy_(2, idx, k)
            st.tail_raw_v.index_copy_(2, idx, v)
            st.tail_deq_k.index_copy_(2, idx, kvd[:, :H].contiguous())
            st.tail_deq_v.index_copy_(2, idx, kvd[:, H:].contiguous())
            return kvd[:, :H], kvd[:, H:]
        if st.tail_raw_k is None or st.tail_raw_k.shape[:2] != (B, H):
            # zeroed: a graph-mode step attends over every slot, and its mask
            # gives the unwritten ones weight 0, which must not meet a NaN
            st.tail_raw_k = torch.zeros(B, H, T, D, dtype=k.dtype, device=k.device)
            st.tail_raw_v = torch.zeros_like(st.tail_raw_k)
            st.tail_deq_k = torch.zeros_like(st.tail_raw_k)
            st.tail_deq_v = torch.zeros_like(st.tail_raw_k)
            # flushed tails are attended dequantised (the first TAIL_MERGE_MAX
            # tokens in the rANS layout, all in the compact one): room for up
            # to four tails, at most a sixteenth of the context so far
            st.reserve_tail_dense(st.tail_deq_k, T * min(4, max(1, st.seq // (16 * T))))
        # K and V of the token in one call: each (batch, head) row has its own
        # scale, so stacking them along the heads changes no value
        kvd = self._quantise_only(torch.cat([k, v], 1))
        kd, vd = kvd[:, :H], kvd[:, H:]
        i = st.n_tail
        st.tail_raw_k[:, :, i] = k[:, :, 0]
        st.tail_raw_v[:, :, i] = v[:, :, 0]
        st.tail_deq_k[:, :, i] = kd[:, :, 0]
        st.tail_deq_v[:, :, i] = vd[:, :, 0]
        st.n_tail += 1
        st.seq += 1
        self.total_vectors += 2 * B * H * D // 8
        if st.n_tail == T:
            self._flush_tail(st, layer_idx)
        return kd, vd

    def _flush_tail(self, st, layer_idx, force=False):
        """Encode the tail as one chunk with a scale per token (every token a head)."""
        n = st.n_tail
        if n == 0:
            return
        B, H, T, D = st.tail_raw_k.shape
        kk = st.tail_raw_k[:, :, :n].reshape(B, H * n, 1, D)
        vv = st.tail_raw_v[:, :, :n].reshape(B, H * n, 1, D)
        tile = _attn_tile(n * D // 8, self.tile_blocks or codec.DEFAULT_TILE_BLOCKS)
        saved = self.total_vectors
        if self.layout == "compact":
            # stored compact (one scale per token); attended from the dequantised
            # tail, since a token's 16 blocks are not a 32-block-aligned head
            from .fused_triton_merge import compress_compact

            ck, _ = compress_compact(kk, int(self.bits))
            cv, _ = compress_compact(vv, int(self.bits))
            tile = None
        else:
            ck, _ = self._compress_with_tile(kk, tile or 32)
            cv, _ = self._compress_with_tile(vv, tile or 32)
        self.total_vectors = saved  # counted when the tokens arrived
        self._comp_keys[layer_idx].append_chunk(ck)
        self._comp_values[layer_idx].append_chunk(cv)
        if tile is not None and not force and st.n_tail_dense + n <= TAIL_MERGE_MAX:
            # stored encoded; attended from its dequantised tokens (update()'s
            # values), which join the layer's dense tail buffer
            st.push_tail_dense(st.tail_deq_k[:, :, :n], st.tail_deq_v[:, :, :n])
        elif tile is not None and not force:
            prev = st.parts[-1] if st.parts and st.parts[-1].per_token and st.parts[-1].opt_k is not None else None
            # merged tails grow up to TAIL_MERGE_MAX tokens, then a new part starts
            # (a recode costs time in proportion to the part's tokens)
            if prev is not None and prev.shape[2] + n <= TAIL_MERGE_MAX:
                self._merge_tail_parts(st, layer_idx, prev, ck, cv, n)
            else:
                st.parts.append(_Part(ck.lanes, cv.lanes, (B, H, n, D), per_token=True, opt_k=ck, opt_v=cv))
        else:
            st.push_tail_dense(st.tail_deq_k[:, :, :n], st.tail_deq_v[:, :, :n])
        st.n_tail = 0

    def _merge_tail_parts(self, st, layer_idx, prev: "_Part", ck, cv, n_new: int):
        """Recode the layer's encoded tail part and the chunk just flushed as ONE
        per-token-scale chunk, so a decode step attends over one tail part
        however many tails have been flushed.  Each token keeps its lattice
        points and its scale: the chunks' points times their fp32 scales are
        coded again with those scales (x / s rounds back to the same points),
        only the rANS tables and lanes change."""
        B, H, n_old, D = prev.shape
        n = n_old + n_new

        def joined(old_lanes, new_lanes):
            q = torch.cat([codec.lattice_points(old_lanes).view(B, H, n_old, D),
                           codec.lattice_points(new_lanes).view(B, H, n_new, D)], 2)
            s = torch.cat([old_lanes.scale_f32.view(B, H, n_old), new_lanes.scale_f32.view(B, H, n_new)], 2)
            return (q * s.unsqueeze(-1)).reshape(B, H * n, 1, D), s.reshape(-1)

        tile = _attn_tile(n * D // 8, self.tile_blocks or codec.DEFAULT_TILE_BLOCKS)
        xk, sk = joined(prev.k, ck.lanes)
        xv, sv = joined(prev.v, cv.lanes)
        saved = self.total_vectors
        mk, _ = self._compress_with_tile(xk, tile or 32, scale_f32=sk)
        mv, _ = self._compress_with_tile(xv, tile or 32, scale_f32=sv)
        self.total_vectors = saved  # counted when the tokens arrived
        # the stored chunks: the two tails' entries become the merged one
        for layers, gone, merged in ((self._comp_keys, (prev.opt_k, ck), mk), (self._comp_values, (prev.opt_v, cv), mv)):
            chunks = layers[layer_idx].chunks
            chunks[:] = [c for c in chunks if all(c is not g for g in gone)]
            chunks.append(merged)
        if tile is not None:
            st.parts[-1] = _Part(mk.lanes, mv.lanes, (B, H, n, D), per_token=True, opt_k=mk, opt_v=mv)
        else:  # no tile divides the merged tail: keep it dequantised (fp16 scale), as a chunk would be
            st.parts.pop()
            st.push_dense(self._decompress_chunk(mk).view(B, H, n, D), self._decompress_chunk(mv).view(B, H, n, D))

    def _materialise(self, st, dtype: Optional[torch.dtype] = None):
        """Every token of a layer, dequantised (fp16 scale for chunks, fp32 for the
        tail), in `dtype` (default: the model's)."""
        dt = dtype or self._model_dtype
        ks, vs = [], []
        for p in st.parts:
            if p.layout == "compact":
                from .fused_triton_merge import fused_decompress_chunk

                ks.append(fused_decompress_chunk(p.k).to(dt))
                vs.append(fused_decompress_chunk(p.v).to(dt))
                continue
            ks.append(codec.decompress(p.k, out_dtype=dt).view(p.shape))
            vs.append(codec.decompress(p.v, out_dtype=dt).view(p.shape))
        ks += [t.to(dt) for t in st.dense_k]
        vs += [t.to(dt) for t in st.dense_v]
        td = st.dense_tail_tokens()
        if td is not None:
            ks.append(td[0].to(dt))
            vs.append(td[1].to(dt))
        if st.n_tail:
            ks.append(st.tail_deq_k[:, :, :st.n_tail].to(dt))
            vs.append(st.tail_deq_v[:, :, :st.n_tail].to(dt))
        return torch.cat(ks, 2), torch.cat(vs, 2)

    # ---- attention -----------------------------------------------------------
    def decode_attention(self, layer_idx: int, query: torch.Tensor, scaling: Optional[float] = None) -> torch.Tensor:
        """Attention of one query position over the layer's whole cache.

        query (B, Hq, 1, D) -> (B, Hq, 1, D) in the query's dtype."""
        st = self._state[layer_idx]
        B, Hq, Q, D = query.shape
        if Q != 1:
            raise ValueError("decode_attention takes one query position")
        scaling = (1.0 / math.sqrt(D)) if scaling is None else float(scaling)
        q3 = query.reshape(B, Hq, D).contiguous()
        # the compressed parts (fused kernels) write their (o, lse) into one
        # stacked buffer; one launch attends the dense tokens and merges all
        P = len(st.parts)
        po = pl = None
        if P:
            po = torch.empty(P, B, Hq, D, dtype=torch.float32, device=query.device)
            pl = torch.empty(P, B, Hq, dtype=torch.float32, device=query.device)
            for i, p in enumerate(st.parts):
                p.op(Hq // p.shape[1])(q3, po[i], pl[i], scaling)
        segs = [(k, v, k.shape[2]) for k, v in zip(st.dense_k, st.dense_v)]
        if st.tail_dense_k is not None:  # length read on the device: valid across flushes in a captured step
            segs.append((st.tail_dense_k, st.tail_dense_v, st.tail_dense_last))
        if self._graph_idx is not None:  # the whole tail; slots past the step's are not counted
            segs.append((st.tail_deq_k, st.tail_deq_v, self._graph_idx))
        elif st.n_tail:
            segs.append((st.tail_deq_k, st.tail_deq_v, st.n_tail))
        if not P and not segs:
            raise ValueError(f"layer {layer_idx} holds no tokens to attend over")
        H = st.parts[0].shape[1] if P else segs[0][0].shape[1]
        out = A.dense_merge_attention(q3, segs, po, pl, H, scaling)
        return out.view(B, Hq, 1, D)

    # ---- CUDA-graph decode steps (llm.graph_decode) --------------------------
    def enter_graph(self, idx: torch.Tensor):
        """Decode-step updates write the token into tail slot `idx` (a (1,)
        int64 device tensor the captured step advances) and attend over the
        whole tail with a mask past that slot, with no host bookkeeping, so a
        step can be captured in a CUDA graph and replayed; graph_advance() is
        the bookkeeping of each replay.  Needs the tail buffers (one eager
        decode step) and a tail that is not full."""
        for st in self._state:
            if st.tail_raw_k is None:
                raise RuntimeError("graph mode needs one eager decode step first")
            if st.n_tail >= self.tail_tokens:
                raise RuntimeError("flush the full tails before entering graph mode")
        self._graph_idx = idx
        self._tail_ar = torch.arange(self.tail_tokens, device=idx.device)

    def exit_graph(self):
        self._graph_idx = None

    def graph_advance(self, n: int = 1):
        """Host bookkeeping of n replayed decode steps."""
        for st in self._state:
            B, H, _, D = st.tail_raw_k.shape
            st.n_tail += n
            st.seq += n
            self.total_vectors += n * 2 * B * H * D // 8

    def tail_full(self) -> bool:
        return any(st.n_tail >= self.tail_tokens for st in self._state)

    def graph_signature(self):
        """The device buffers a captured decode step reads (parts, dense
        segments, tails): a flush that leaves it unchanged leaves the captured
        step valid (the tail slot restarts at 0)."""
        def ptr(t):
            return None if t is None else t.data_ptr()

        return tuple((tuple(id(p) for p in st.parts), tuple(ptr(t) for t in st.dense_k + st.dense_v),
                      ptr(st.tail_dense_k), ptr(st.tail_dense_v), ptr(st.tail_raw_k), ptr(st.tail_deq_k))
                     for st in self._state)

    def flush_tails(self):
        """Encode every full tail (what an eager update does at the 64th token)."""
        for li, st in enumerate(self._state):
            if st.n_tail >= self.tail_tokens:
                self._flush_tail(st, li)

    def flags(self) -> int:
        """OR of the fused attention kernels' error words (synchronises)."""
        f = 0
        for st in self._state:
            for p in st.parts:
                for op in p.ops.values():
                    f |= op.flags()
        return f

    # ---- transformers glue ---------------------------------------------------
    def bind(self, model) -> "CompressedAttentionKVCache":
        """Point every attention module of `model` (modules with a layer_idx) at
        this cache and switch the model to the compressed attention function."""
        register_attention()
        for m in model.modules():
            if hasattr(m, "layer_idx") and hasattr(m, "num_key_value_groups"):
                m._lq_cache = self
        cfg = getattr(model, "config", None)
        if cfg is not None:
            if hasattr(model, "set_attn_implementation"):
                model.set_attn_implementation(ATTN_NAME)
            else:
                cfg._attn_implementation = ATTN_NAME
        return self

    def get_seq_length(self, layer_idx=0):
        if layer_idx < len(self._state):
            return self._state[layer_idx].seq
        return 0

    def get_mask_sizes(self, query_length, layer_idx=0):
        q = int(query_length.shape[0]) if torch.is_tensor(query_length) else int(query_length)
        return self.get_seq_length(layer_idx) + q, 0

    def decompressed_resident_bytes(self):
        total = 0
        for st in self._state:
            for t in st.dense_k + st.dense_v + [st.tail_raw_k, st.tail_raw_v, st.tail_deq_k, st.tail_deq_v,
                                                st.tail_dense_k, st.tail_dense_v]:
                if t is not None:
                    total += t.nelement() * t.element_size()
        return total


def lq_compressed_attention(module, query, key, value, attention_mask, scaling=None, dropout=0.0, **kwargs):
    """transformers attention function.  A decode step (one query position) of a
    module bound to a CompressedAttentionKVCache reads the compressed cache;
    every other call runs SDPA over the K/V it is given (what update()
    returned: the dequantised tokens).  With a KV-head-sharded cache the
    module's K/V are this rank's heads: it attends with their query heads and
    all-gathers every rank's heads (sharding.gather_heads)."""
    cache = getattr(module, "_lq_cache", None)
    if cache is not None and cache.head_range is not None:
        h0, h1 = cache.head_range
        g = query.shape[1] // cache.n_kv_heads_total
        o = _attend(module, cache, query[:, h0 * g:h1 * g], key, value, attention_mask, scaling)
        from ..sharding import gather_heads

        return gather_heads(o, cache.group), None
    return _attend(module, cache, query, key, value, attention_mask, scaling), None


def _attend(module, cache, query, key, value, attention_mask, scaling):
    """(B, Q, Hq, D) attention output of one module call (see lq_compressed_attention)."""
    st = None
    if cache is not None and query.shape[2] == 1 and module.layer_idx < len(cache._state):
        st = cache._state[module.layer_idx]
        if st.seq == 0:
            st = None
    if st is not None:
        masked = attention_mask is not None and bool((attention_mask < 0).any())
        if not masked:
            o = cache.decode_attention(module.layer_idx, query.contiguous(), scaling)
            return o.transpose(1, 2).contiguous()
        key, value = cache._materialise(st)  # padding masks: attend over the dequantised cache
    # grouped query heads read their KV head in place (no repeat_kv copies)
    o = torch.nn.functional.scaled_dot_product_attention(
        query, key, value, attn_mask=attention_mask, is_causal=attention_mask is None and query.shape[2] > 1,
        scale=scaling, enable_gqa=query.shape[1] != key.shape[1])
    return o.transpose(1, 2).contiguous()


def register_attention():
    from transformers import AttentionInterface

    AttentionInterface.register(ATTN_NAME, lq_compressed_attention)
