"""Host logic of the multi-GPU paths on CPU (gloo, world size 2): unit
placement, context slicing, and the sequence-sharded all-gather + LSE merge
(with a float64 torch merge standing in for the CUDA merge kernel)."""
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from latticequant_b200 import sharding


def test_shard_units_cover_each_unit_once():
    for world in (1, 2, 3, 8):
        seen = []
        for r in range(world):
            seen += sharding.shard_units(32, 8, world, r)
        assert sorted(seen) == [(l, h) for l in range(32) for h in range(8)]
    # round-robin balance: 256 units over 8 ranks -> 32 each
    assert all(len(sharding.shard_units(32, 8, 8, r)) == 32 for r in range(8))


def test_sequence_slices_tile_and_cover():
    for S, world, align in ((32768, 8, 64), (1000, 3, 64), (64, 4, 64), (131072, 8, 64)):
        spans = [sharding.sequence_slice(S, world, r, align) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == S
        for (a, b), (c, d) in zip(spans, spans[1:]):
            assert b == c and a <= b
        assert all(lo % align == 0 for lo, _ in spans)
    with pytest.raises(ValueError):
        sharding.sequence_slice(10, 2, 2)


def _attn(q, k, v):
    """q (R, D), k/v (R, S, D) -> o (R, D), lse (R,) in float64."""
    s = torch.einsum("rd,rsd->rs", q, k) / math.sqrt(q.shape[-1])
    lse = torch.logsumexp(s, -1)
    return torch.einsum("rs,rsd->rd", torch.exp(s - lse[:, None]), v), lse


def _torch_merge(o_all, l_all, out_dtype=None):
    lse = torch.logsumexp(l_all, 0)
    w = torch.exp(l_all - lse)
    return (w[..., None] * o_all).sum(0), lse


def _worker(rank, world, port, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(5)
        R, S, D = 6, 200, 16
        q = torch.randn(R, D, generator=g, dtype=torch.float64)
        k = torch.randn(R, S, D, generator=g, dtype=torch.float64)
        v = torch.randn(R, S, D, generator=g, dtype=torch.float64)
        lo, hi = sharding.sequence_slice(S, world, rank, 8)
        o_loc, l_loc = _attn(q, k[:, lo:hi], v[:, lo:hi])
        o, lse = sharding.sequence_sharded_merge(o_loc, l_loc, merge=_torch_merge)
        o_ref, l_ref = _attn(q, k, v)
        result[rank] = float(max((o - o_ref).abs().max(), (lse - l_ref).abs().max()))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_sequence_sharded_merge_gloo_world2():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        result = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, 2, port, result)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        assert all(p.exitcode == 0 for p in procs)
        assert len(result) == 2 and max(result.values()) < 1e-12


class _Stub:
    """An attention module bound to a head-sharded cache with no compressed
    state yet, so lq_compressed_attention takes its SDPA path."""

    def __init__(self, head_range, n_kv):
        self.layer_idx = 0
        self._lq_cache = type("C", (), {})()
        self._lq_cache.head_range = head_range
        self._lq_cache.n_kv_heads_total = n_kv
        self._lq_cache.group = None
        self._lq_cache._state = []


def _head_worker(rank, world, port, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from latticequant_b200.llm.compressed_attention import lq_compressed_attention

        g = torch.Generator().manual_seed(9)
        B, Hkv, G, Q, S, D = 2, 4, 3, 5, 5, 16
        q = torch.randn(B, Hkv * G, Q, D, generator=g, dtype=torch.float64)
        k = torch.randn(B, Hkv, S, D, generator=g, dtype=torch.float64)
        v = torch.randn(B, Hkv, S, D, generator=g, dtype=torch.float64)
        h0, h1 = sharding.head_slice(Hkv, world, rank)
        # what update() hands the module on this rank: its KV heads only
        o, _ = lq_compressed_attention(_Stub((h0, h1), Hkv), q, k[:, h0:h1], v[:, h0:h1], None, scaling=0.25)
        ref = torch.nn.functional.scaled_dot_product_attention(
            q, k.repeat_interleave(G, 1), v.repeat_interleave(G, 1), is_causal=True, scale=0.25).transpose(1, 2)
        result[rank] = float((o - ref).abs().max()) if o.shape == ref.shape else float("inf")
    finally:
        dist.destroy_process_group()


def test_head_slices_cover():
    assert [sharding.head_slice(8, 4, r) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        sharding.head_slice(8, 3, 0)


def test_kv_head_sharded_attention_gloo_world2():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        result = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_head_worker, args=(r, 2, port, result)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        assert all(p.exitcode == 0 for p in procs)
        assert len(result) == 2 and max(result.values()) < 1e-12
