"""Checkpointing of compressed chunks and caches.

The reference keeps results in memory and writes only JSON metrics
(llm/e2e_eval.py:488-507); it has no way to persist a compressed cache.
Here a LaneChunk is saved as its device arrays (lane words, lane offsets /
bit counts / states, coset words, per-tile coset-0 counts, tables, scales)
plus its geometry, and a cache as its chunks per layer plus the state that is
not derivable from them.  Files are plain ``torch.save`` dictionaries of CPU
tensors, strings and integers (loadable with ``weights_only=True``), tagged
with a format version.  Loading places everything on the given device; the
decode tables are rebuilt on first use.
"""
from __future__ import annotations

from typing import Any, Dict, Optional

import torch

from . import codec
from .codec import Geometry, LaneChunk

FORMAT = "latticequant_b200.chunk/1"
CACHE_FORMAT = "latticequant_b200.cache/1"
_DT = {torch.float32: "float32", torch.float16: "float16", torch.bfloat16: "bfloat16"}
_DT_INV = {v: k for k, v in _DT.items()}
_ARRAYS = ("scale_f32", "scale_f16", "coset_words", "tile_n0", "tab_lo", "tab_nsym", "tab_freq", "lane_off",
           "lane_nbits", "lane_state")


def chunk_state(ch: LaneChunk) -> Dict[str, Any]:
    """A LaneChunk as a dictionary of CPU tensors and plain values."""
    g = ch.geom
    d = {"format": FORMAT, "geom": [g.n_chunks, g.n_heads, g.bph, g.tile_blocks], "bits": float(ch.bits),
         "orig_shape": [int(s) for s in ch.orig_shape], "orig_dtype": _DT[ch.orig_dtype], "n_words": int(ch.n_words),
         "words": ch.words[:max(ch.n_words, 1)].detach().cpu().clone()}
    for k in _ARRAYS:
        d[k] = getattr(ch, k).detach().cpu().clone()
    d["n_outliers"] = int(ch.n_outliers)
    d["outlier_rec"] = ch.outlier_rec.detach().cpu().clone() if ch.n_outliers else None
    return d


def chunk_from_state(d: Dict[str, Any], device="cuda") -> LaneChunk:
    if d.get("format") != FORMAT:
        raise ValueError(f"not a {FORMAT} record: {d.get('format')!r}")
    g = Geometry(*[int(v) for v in d["geom"]])
    arrs = {k: d[k].to(device) for k in _ARRAYS}
    if arrs["lane_off"].numel() != g.n_lanes + 1 or arrs["tile_n0"].numel() != g.n_chunks * g.n_tiles:
        raise ValueError("chunk record does not match its geometry")
    if int(d["n_words"]) > d["words"].numel() or int(arrs["lane_off"][-1].item()) > max(int(d["n_words"]), 1):
        raise ValueError("chunk record: lane offsets run past the words")
    n_out = int(d.get("n_outliers", 0))
    rec = d.get("outlier_rec")
    if n_out and (rec is None or tuple(rec.shape) != (n_out, 10)):
        raise ValueError("chunk record: outlier records do not match their count")
    return LaneChunk(geom=g, bits=float(d["bits"]), orig_shape=tuple(d["orig_shape"]),
                     orig_dtype=_DT_INV[d["orig_dtype"]], words=d["words"].to(device), n_words=int(d["n_words"]),
                     outlier_rec=rec.to(device) if n_out else None, n_outliers=n_out, **arrs)


def save_chunk(ch: LaneChunk, path: str):
    torch.save(chunk_state(ch), path)


def load_chunk(path: str, device="cuda") -> LaneChunk:
    return chunk_from_state(torch.load(path, map_location="cpu", weights_only=True), device)


# ---- caches -------------------------------------------------------------------
def _tensor_or_none(t: Optional[torch.Tensor]):
    return None if t is None else t.detach().cpu().clone()


def cache_state(cache) -> Dict[str, Any]:
    """CompressedKVCache / VariableRateKVCache / CompressedAttentionKVCache state."""
    from .llm.compressed_attention import CompressedAttentionKVCache
    from .llm.compressed_kv_cache import CompressedKVLayer, UncompressibleKVLayer

    if getattr(cache, "layout", "rans") != "rans":
        raise ValueError("caches in the compact layout cannot be saved (only rANS-lane chunks)")
    layers = []
    for lk, lv in zip(cache._comp_keys, cache._comp_values):
        if lk is None:
            layers.append(None)
        elif isinstance(lk, UncompressibleKVLayer):
            layers.append({"raw_k": _tensor_or_none(lk.data), "raw_v": _tensor_or_none(lv.data)})
        else:
            assert isinstance(lk, CompressedKVLayer)
            if any(c.lanes is None for c in lk.chunks + lv.chunks):
                raise ValueError("chunks stored without entropy coding cannot be saved")
            layers.append({"k": [chunk_state(c.lanes) for c in lk.chunks],
                           "v": [chunk_state(c.lanes) for c in lv.chunks]})
    d = {"format": CACHE_FORMAT, "class": type(cache).__name__, "bits": cache.bits,
         "tile_blocks": cache.tile_blocks, "table_mode": cache.table_mode, "total_vectors": cache.total_vectors,
         "model_dtype": _DT.get(cache._model_dtype), "layers": layers,
         "bits_schedule": [dict(x) for x in getattr(cache, "bits_schedule", [])],
         "eval_only_no_entropy": bool(getattr(cache, "eval_only_no_entropy", False))}
    if isinstance(cache, CompressedAttentionKVCache):
        d["tail_tokens"] = cache.tail_tokens
        d["attn"] = [{"parts": [[i, list(p.shape), p.per_token] for i, p in enumerate(st.parts)],
                      "dense_k": [_tensor_or_none(t) for t in st.dense_k + _tail_dense(st, 0)],
                      "dense_v": [_tensor_or_none(t) for t in st.dense_v + _tail_dense(st, 1)],
                      "tail": [_tensor_or_none(t) for t in (st.tail_raw_k, st.tail_raw_v, st.tail_deq_k,
                                                            st.tail_deq_v)],
                      "n_tail": st.n_tail, "seq": st.seq, "part_chunks": _part_chunk_index(cache, li)}
                     for li, st in enumerate(cache._state)]
    else:
        d["resident"] = [None if t is None or t.numel() == 0 else "rebuild" for t in cache.key_cache]
    return d


def _tail_dense(st, i: int) -> list:
    """The layer's flushed tails kept dequantised (saved as one more dense segment)."""
    td = st.dense_tail_tokens()
    return [] if td is None else [td[i]]


def _part_chunk_index(cache, li):
    """Which of the layer's chunks each attention part reads (by identity of the lanes)."""
    lk = cache._comp_keys[li]
    ids = {id(c.lanes): j for j, c in enumerate(lk.chunks)} if lk is not None else {}
    return [ids[id(p.k)] for p in cache._state[li].parts]


def save_cache(cache, path: str):
    torch.save(cache_state(cache), path)


def _rebuild_resident(lanes: LaneChunk, dtype):
    """update()'s dequantised tokens (q * fp32 scale) from a chunk: the decoded
    E8 points times the fp32 head scales, in the model dtype."""
    q = codec.decompress(lanes, out_dtype=torch.float32, want_symbols=True)[1]
    from .core.entropy_coder import symbols_to_e8

    n = q.shape[0]
    cos = torch.zeros(n, dtype=torch.int32, device=q.device)
    cw = lanes.coset_words.view(torch.int32)
    bits = (cw.view(-1, 1) >> torch.arange(32, device=q.device, dtype=torch.int32)) & 1
    cos[:] = bits.reshape(-1)[:n]
    if lanes.n_outliers:  # extracted blocks keep their coset in the records
        cos[lanes.outlier_rec[:, 0].long()] = lanes.outlier_rec[:, 1]
    pts = symbols_to_e8(cos, q[:, :7], q[:, 7])
    g = lanes.geom
    sc = lanes.scale_f32.view(g.n_heads, 1, 1)
    out = (pts.view(g.n_heads, g.bph, 8) * sc).to(dtype)
    return out.view(lanes.orig_shape)


def load_cache(path: str, device="cuda"):
    d = torch.load(path, map_location="cpu", weights_only=True)
    if d.get("format") != CACHE_FORMAT:
        raise ValueError(f"not a {CACHE_FORMAT} record: {d.get('format')!r}")
    from .allocation.eval_alloc import VariableRateKVCache
    from .llm.compressed_attention import CompressedAttentionKVCache, _LayerState, _Part
    from .llm.compressed_kv_cache import (CompressedKVCache, CompressedKVLayer, OptimizedChunk,
                                          UncompressibleKVLayer, _get_placeholder)

    cls = {"CompressedKVCache": CompressedKVCache, "VariableRateKVCache": VariableRateKVCache,
           "CompressedAttentionKVCache": CompressedAttentionKVCache}.get(d["class"])
    if cls is None:
        raise ValueError(f"unknown cache class {d['class']}")
    if cls is CompressedAttentionKVCache:
        cache = cls(bits_per_dim=d["bits"], tail_tokens=d["tail_tokens"], tile_blocks=d["tile_blocks"],
                    table_mode=d["table_mode"])
    elif cls is VariableRateKVCache:
        cache = cls(d["bits_schedule"], eval_only_no_entropy=d["eval_only_no_entropy"], tile_blocks=d["tile_blocks"],
                    table_mode=d["table_mode"])
        cache.bits = d["bits"]
    else:
        cache = cls(bits_per_dim=d["bits"], tile_blocks=d["tile_blocks"], table_mode=d["table_mode"])
    cache.total_vectors = d["total_vectors"]
    cache._model_dtype = _DT_INV.get(d["model_dtype"])
    dt = cache._model_dtype or torch.bfloat16

    def opt(st):
        lc = chunk_from_state(st, device)
        g = lc.geom
        return OptimizedChunk(gpu_bitstream=lc.words[:lc.n_words], coset_packed=lc.coset_words.view(torch.uint8)[
            :(g.n_vectors + 7) // 8], scales=lc.scale_f16, orig_shape=torch.Size(lc.orig_shape),
            n_vectors=g.n_vectors, n_heads=g.n_heads, blocks_per_head=g.bph, bits_per_dim=lc.bits,
            orig_dtype=lc.orig_dtype, lanes=lc)

    for li, layer in enumerate(d["layers"]):
        cache._comp_keys.append(None)
        cache._comp_values.append(None)
        cache.key_cache.append(_get_placeholder(device, dt))
        cache.value_cache.append(_get_placeholder(device, dt))
        if layer is None:
            continue
        if "raw_k" in layer:
            cache._comp_keys[li] = UncompressibleKVLayer(layer["raw_k"].to(device))
            cache._comp_values[li] = UncompressibleKVLayer(layer["raw_v"].to(device))
            cache.key_cache[li] = layer["raw_k"].to(device)
            cache.value_cache[li] = layer["raw_v"].to(device)
            continue
        lk, lv = CompressedKVLayer(), CompressedKVLayer()
        for st in layer["k"]:
            lk.append_chunk(opt(st))
        for st in layer["v"]:
            lv.append_chunk(opt(st))
        cache._comp_keys[li], cache._comp_values[li] = lk, lv
        if not isinstance(cache, CompressedAttentionKVCache) and d["resident"][li] == "rebuild":
            cache.key_cache[li] = torch.cat([_rebuild_resident(c.lanes, dt) for c in lk.chunks], 2)
            cache.value_cache[li] = torch.cat([_rebuild_resident(c.lanes, dt) for c in lv.chunks], 2)
    if isinstance(cache, CompressedAttentionKVCache):
        for li, a in enumerate(d["attn"]):
            st = _LayerState()
            lk, lv = cache._comp_keys[li], cache._comp_values[li]
            for (i, shape, per_token), j in zip(a["parts"], a["part_chunks"]):
                st.parts.append(_Part(lk.chunks[j].lanes, lv.chunks[j].lanes, tuple(shape), bool(per_token),
                                      opt_k=lk.chunks[j], opt_v=lv.chunks[j]))
            st.dense_k = [t.to(device) for t in a["dense_k"]]
            st.dense_v = [t.to(device) for t in a["dense_v"]]
            st.consolidate()
            tr = [None if t is None else t.to(device) for t in a["tail"]]
            st.tail_raw_k, st.tail_raw_v, st.tail_deq_k, st.tail_deq_v = tr
            st.n_tail, st.seq = int(a["n_tail"]), int(a["seq"])
            cache._state.append(st)
    return cache
