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


def _pack_partials(o_local: torch.Tensor, lse_local: torch.Tensor) -> torch.Tensor:
    """One flat buffer: the o rows (..., D) followed by the lse values (...)."""
    o = o_local.reshape(-1)
    ls = lse_local.reshape(-1).to(o.dtype)
    return torch.cat([o, ls])


def _all_gather_flat(buf: torch.Tensor, group: Optional[dist.ProcessGroup]) -> torch.Tensor:
    world = dist.get_world_size(group)
    out = torch.empty((world, buf.numel()), dtype=buf.dtype, device=buf.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, buf, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), buf, group=group)
    return out


def gather_partials(o_local: torch.Tensor, lse_local: torch.Tensor,
                    group: Optional[dist.ProcessGroup] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """All-gather the per-rank attention partials with ONE collective (o and
    lse packed in one buffer): returns (world, *o.shape), (world, *lse.shape)
    views of the gathered buffer."""
    n_o = o_local.numel()
    packed = _all_gather_flat(_pack_partials(o_local, lse_local), group)
    world = packed.shape[0]
    o_all = packed[:, :n_o].reshape((world,) + tuple(o_local.shape))
    l_all = packed[:, n_o:].reshape((world,) + tuple(lse_local.shape))
    return o_all, l_all


def sequence_sharded_merge(o_local: torch.Tensor, lse_local: torch.Tensor,
                           group: Optional[dist.ProcessGroup] = None,
                           merge: Optional[Callable] = None,
                           out_dtype: Optional[torch.dtype] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Attention over the whole context from each rank's slice result.

    o_local: (..., D) fp32 attention over this rank's keys; lse_local: (...)
    their log-sum-exp.  Every rank returns the merged (o, lse).  One
    all-gather moves every rank's (o, lse) as one packed buffer; `merge`
    defaults to the CUDA merge of that packed layout
    (attention.merge_attention_packed, no copies)."""
    if merge is not None:
        o_all, l_all = gather_partials(o_local, lse_local, group)
        return merge(o_all, l_all, out_dtype=out_dtype)
    from .attention import merge_attention_packed

    D = o_local.shape[-1]
    rows = o_local.numel() // D
    packed = _all_gather_flat(_pack_partials(o_local.float(), lse_local.float()), group)
    o, lse = merge_attention_packed(packed, rows, D, out_dtype=out_dtype or o_local.dtype)
    return o.view(o_local.shape), lse.view(lse_local.shape)
