"""Multi-GPU placement of the compressed KV cache and sequence-sharded decode.

The reference runs on one device (README.md:251; llm/e2e_eval.py:60) and has
no collective.  Here the codec shards with no data-path traffic: a unit is a
(layer, KV head) pair, placed round-robin over the ranks, and every chunk,
scale and table lives with its unit.  Decode attention over a long context
may instead shard the sequence: each rank attends over its context slice,
producing (o, lse) per query row, and one all-gather of those partials (a few
hundred KB) plus the log-sum-exp merge (lq_attn_merge) gives the full result.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Tuple

import torch
import torch.distributed as dist


def shard_units(n_layers: int, n_kv_heads: int, world: int, rank: int) -> List[Tuple[int, int]]:
    """(layer, kv_head) units of this rank, round-robin in layer-major order."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world / rank")
    units = [(l, h) for l in range(n_layers) for h in range(n_kv_heads)]
    return units[rank::world]


def sequence_slice(seq_len: int, world: int, rank: int, align: int = 1) -> Tuple[int, int]:
    """Contiguous context slice [lo, hi) of this rank; slice starts are multiples
    of `align` tokens (a compressed tile's tokens) and the slices cover the context."""
    if world <= 0 or not 0 <= rank < world or align <= 0:
        raise ValueError("bad world / rank / align")
    units = -(-seq_len // align)
    lo_u = units * rank // world
    hi_u = units * (rank + 1) // world
    return min(lo_u * align, seq_len), min(hi_u * align, seq_len)


def head_slice(n_kv_heads: int, world: int, rank: int) -> Tuple[int, int]:
    """KV heads [h0, h1) of this rank when a cache is sharded by KV head (equal
    slices: the KV head count must be a multiple of the world size)."""
    if world <= 0 or not 0 <= rank < world or n_kv_heads % world:
        raise ValueError(f"{n_kv_heads} KV heads cannot be split evenly over {world} ranks")
    per = n_kv_heads // world
    return rank * per, (rank + 1) * per


def gather_heads(o_local: torch.Tensor, group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """(B, Q, H_local, D) attention outputs of every rank's head slice ->
    (B, Q, world * H_local, D), rank r's heads at [r * H_local, (r+1) * H_local)."""
    world = dist.get_world_size(group)
    o = o_local.contiguous()
    buf = torch.empty((world,) + tuple(o.shape), dtype=o.dtype, device=o.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(buf, o, group=group)
    else:
        dist.all_gather(list(buf.unbind(0)), o, group=group)
    B, Q, H, D = o.shape
    return buf.permute(1, 2, 0, 3, 4).reshape(B, Q, world * H, D)


def gather_partials(o_local: torch.Tensor, lse_local: torch.Tensor,
                    group: Optional[dist.ProcessGroup] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """All-gather the per-rank attention partials: (world, *o.shape), (world, *lse.shape)."""
    world = dist.get_world_size(group)
    o = o_local.contiguous()
    ls = lse_local.contiguous()
    o_all = torch.empty((world,) + tuple(o.shape), dtype=o.dtype, device=o.device)
    l_all = torch.empty((world,) + tuple(ls.shape), dtype=ls.dtype, device=ls.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(o_all, o, group=group)
        dist.all_gather_into_tensor(l_all, ls, group=group)
    else:
        dist.all_gather(list(o_all.unbind(0)), o, group=group)
        dist.all_gather(list(l_all.unbind(0)), ls, group=group)
    return o_all, l_all


def sequence_sharded_merge(o_local: torch.Tensor, lse_local: torch.Tensor,
                           group: Optional[dist.ProcessGroup] = None,
                           merge: Optional[Callable] = None,
                           out_dtype: Optional[torch.dtype] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Attention over the whole context from each rank's slice result.

    o_local: (..., D) fp32 attention over this rank's keys; lse_local: (...)
    their log-sum-exp.  Every rank returns the merged (o, lse).  `merge`
    defaults to the CUDA merge (attention.merge_attention)."""
    o_all, l_all = gather_partials(o_local, lse_local, group)
    if merge is None:
        from .attention import merge_attention

        merge = merge_attention
    return merge(o_all, l_all, out_dtype=out_dtype)
