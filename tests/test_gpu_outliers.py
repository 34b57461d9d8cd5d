"""Chunks whose alphabet would exceed L = 1024 symbols (the reference's
build_rans_table never ends there) or whose lattice coordinates leave the
symbol range: the outlier side channel takes the offending tokens whole into
records, the streams code them as zero blocks, and decode / attention put
them back exactly."""
import math
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _heavy(seed, shape=(2, 2, 256, 128), plant=((0, 0, 5, 3, 66.0), (0, 0, 9, 7, -66.0), (1, 1, 100, 0, 4000.0))):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(shape, generator=g)
    for b, h, s, d, v in plant:
        x[b, h, s, d] = v
    return x.to(torch.bfloat16).cuda()


def _exact_deq(x, chunk):
    """q * fp16 head scale from the quantiser's own lattice points."""
    from latticequant_b200 import codec

    B, H, S, D = x.shape
    geom = codec.Geometry(1, B * H, S * D // 8, chunk.geom.tile_blocks)
    cd = codec.Codec(geom, x.device)
    cd.scale_f32.copy_(chunk.scale_f32)
    q = torch.empty(B * H * S * D // 8, 8, dtype=torch.float32, device=x.device)
    cd.quantize_outliers(x.contiguous(), q, 16)
    sc = chunk.scale_f16.float().view(B * H, 1, 1)
    return (q.view(B * H, S * D // 8, 8) * sc).view(x.shape)


def test_outlier_chunk_round_trips_exactly():
    from latticequant_b200 import codec

    x = _heavy(0)
    ch, _ = codec.compress(x, 5, tile_blocks=1024)
    assert ch.n_outliers > 0 and ch.n_outliers % 16 == 0  # whole tokens (head_dim 128 = 16 blocks)
    assert ch.compressed_bytes() > 4 * ch.n_words
    out = codec.decompress(ch, out_dtype=torch.float32)
    ref = _exact_deq(x, ch)
    assert torch.equal(out + 0.0, ref + 0.0)
    # the extracted tokens' symbols come back through sym_out too
    _, sym = codec.decompress(ch, out_dtype=torch.float32, want_symbols=True)
    r = ch.outlier_rec.long()
    assert torch.equal(sym[r[:, 0]], ch.outlier_rec[:, 2:])
    # ordinary data takes no outlier path
    y = torch.randn(2, 2, 256, 128, device="cuda", dtype=torch.bfloat16)
    cy, _ = codec.compress(y, 5, tile_blocks=1024)
    assert cy.n_outliers == 0


def test_attention_over_outlier_chunks():
    from oracle import lq_oracle as O

    from latticequant_b200 import attention, codec

    k = _heavy(1)
    v = _heavy(2, plant=((1, 0, 17, 9, -5000.0),))
    kc, _ = codec.compress(k, 5, tile_blocks=1024)
    vc, _ = codec.compress(v, 5, tile_blocks=1024)
    assert kc.n_outliers and vc.n_outliers
    q = torch.randn(2, 8, 128, device="cuda", dtype=torch.float32) / math.sqrt(128)
    o, lse = attention.decode_attention(q, kc, vc, out_dtype=torch.float32, return_lse=True)
    kd = codec.decompress(kc, out_dtype=torch.float32).cpu().numpy()
    vd = codec.decompress(vc, out_dtype=torch.float32).cpu().numpy()
    ref = O.decode_attention_f64(q.cpu().numpy(), kd, vd, 1 / math.sqrt(128))
    err = np.abs(o.cpu().numpy() - ref).max(-1) / np.abs(ref).max(-1)
    assert err.max() <= 1e-3, err.max()
    assert torch.isfinite(lse).all()


def test_cache_accepts_chunks_the_reference_cannot_code(tmp_path):
    from latticequant_b200 import serialize
    from latticequant_b200.llm.compressed_kv_cache import CompressedKVCache

    cache = CompressedKVCache(5)
    k = _heavy(3)
    v = _heavy(4)
    kf, vf = cache.update(k, v, 0)
    ch = cache._comp_keys[0].chunks[0]
    assert ch.lanes.n_outliers > 0
    dec = cache._decompress_chunk(ch)
    assert torch.equal((dec.float() + 0.0), (_exact_deq(k, ch.lanes).to(torch.bfloat16).float() + 0.0))
    p = os.path.join(tmp_path, "c.pt")
    serialize.save_chunk(ch.lanes, p)
    back = serialize.load_chunk(p)
    from latticequant_b200 import codec

    assert torch.equal(codec.decompress(back, out_dtype=torch.float32), codec.decompress(ch.lanes, out_dtype=torch.float32))
