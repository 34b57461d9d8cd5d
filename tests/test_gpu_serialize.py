"""Save / load of compressed chunks and caches (new: the reference cannot
persist a compressed cache).  A loaded chunk decodes to the same bytes; a
loaded cache continues with the same values as the original (the resident
buffer is rebuilt from the symbols, which do not carry the sign of a zero
coordinate: -0.0 comes back as +0.0, as in the reference's own
_decompress_chunk)."""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_chunk_round_trip(tmp_path):
    from latticequant_b200 import codec, serialize

    torch.manual_seed(0)
    x = torch.randn(2, 4, 256, 128, device="cuda", dtype=torch.bfloat16)
    ch, _ = codec.compress(x, 4, tile_blocks=512)
    p = os.path.join(tmp_path, "c.pt")
    serialize.save_chunk(ch, p)
    ch2 = serialize.load_chunk(p)
    a = codec.decompress(ch)
    b = codec.decompress(ch2)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    assert ch2.compressed_bytes() == ch.compressed_bytes() and ch2.orig_shape == ch.orig_shape
    d = torch.load(p, weights_only=True)
    d["lane_off"][-1] = d["n_words"] + 5
    with pytest.raises(ValueError):
        serialize.chunk_from_state(d)


@pytest.mark.parametrize("kind", ["plain", "attention"])
def test_cache_round_trip_continues_identically(tmp_path, kind):
    from latticequant_b200 import serialize
    from latticequant_b200.llm.compressed_attention import CompressedAttentionKVCache
    from latticequant_b200.llm.compressed_kv_cache import CompressedKVCache

    make = (lambda: CompressedKVCache(4)) if kind == "plain" else (lambda: CompressedAttentionKVCache(4, 64))
    torch.manual_seed(1)
    c1 = make()
    steps = [torch.randn(1, 2, 128, 128, device="cuda", dtype=torch.float16)] + \
            [torch.randn(1, 2, 1, 128, device="cuda", dtype=torch.float16) for _ in range(70)]
    for t in steps[:40]:
        for layer in (0, 1):
            c1.update(t, t * 0.5, layer)
    p = os.path.join(tmp_path, "cache.pt")
    serialize.save_cache(c1, p)
    c2 = serialize.load_cache(p)
    assert c2.compressed_bytes() == c1.compressed_bytes() and c2.get_seq_length(1) == c1.get_seq_length(1)
    q = torch.randn(1, 8, 1, 128, device="cuda", dtype=torch.float32)
    for t in steps[40:]:
        for layer in (0, 1):
            k1, v1 = c1.update(t, t * 0.5, layer)
            k2, v2 = c2.update(t, t * 0.5, layer)
            assert torch.equal(k1, k2) and torch.equal(v1, v2)
        if kind == "attention":
            assert torch.equal(c1.decode_attention(0, q), c2.decode_attention(0, q))
    assert c2.compressed_bytes() == c1.compressed_bytes()
