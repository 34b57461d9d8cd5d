"""Compact layout + fp16 fallback, merged by lq_compact_merge: equal to the
dequantised E8 points (q * fp32 head scale, fp16) block for block, including
blocks whose coord0..6 sum is odd and negative (the case the reference's merge
kernel decodes wrongly), and to the oracle's unpack for the coded blocks."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits", [3, 4, 5])
def test_fused_merge_equals_dequantised_points(bits):
    from oracle import lq_oracle as O

    from latticequant_b200.llm.fused_triton_merge import compress_compact, fused_decompress_chunk

    torch.manual_seed(bits)
    x = torch.randn(2, 4, 96, 128, device="cuda", dtype=torch.float16)
    chunk, deq = compress_compact(x, bits)
    out = fused_decompress_chunk(chunk)
    assert 0.05 < chunk.oor_rate < 0.6  # both paths exercised
    # the fp16 of (q * fp32 scale) for every block; deq is the same product in x's dtype
    # (bit for bit once zeros are made +0: a code does not carry the sign of a zero coordinate)
    assert torch.equal((out + 0.0).view(torch.int16), (deq + 0.0).view(torch.int16))
    # coded blocks against the oracle's unpack (the 4-bit fp16 path of core/triton_dequant.py)
    if bits == 4:
        m = chunk.repr_mask.cpu().numpy()
        bph = chunk.blocks_per_head
        head = (np.arange(m.size) // bph)[m].astype(np.int32)
        ref = O.unpack_e8_4bit_f16(chunk.packed.cpu().numpy(), chunk.scales.cpu().numpy(), head)
        got = out.reshape(-1, 8)[torch.from_numpy(m).cuda()].cpu().numpy().view(np.uint16)
        assert np.array_equal(got, np.asarray(ref).view(np.uint16).reshape(got.shape))
    # some coded blocks have odd negative partial sums
    from latticequant_b200.core.compact_storage import unpack_e8

    pts = unpack_e8(chunk.packed, bits)
    ints = (pts - 0.5 * (pts[:, :1] - pts[:, :1].floor() > 0.25).float()).round().long()
    ps = ints[:, :7].sum(1)
    assert bool(((ps < 0) & (ps % 2 != 0)).any())


def test_fused_cache_update_and_decompress():
    from latticequant_b200.llm.fused_triton_merge import FusedTritonKVCache

    torch.manual_seed(0)
    cache = FusedTritonKVCache(4)
    k = torch.randn(1, 8, 64, 128, device="cuda", dtype=torch.float16)
    v = torch.randn(1, 8, 64, 128, device="cuda", dtype=torch.float16)
    kf, vf = cache.update(k, v, 0)
    ch = cache._comp_keys[0].chunks[0]
    assert torch.equal(cache._decompress_chunk(ch), kf)
    assert cache.compressed_bytes() > 0
