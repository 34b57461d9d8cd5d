"""lq_attn_dense_merge: attention over dense K/V segments merged with finished
attention parts, against float64 attention over the same keys.  This is the
decode-step attention over the uncompressed end of a layer's cache (the
reference's SDPA over the buffer update() returns, llm/compressed_kv_cache.py:
342-395, restricted to those tokens) joined with the compressed parts by
log-sum-exp.

Tolerance: max |o - o_ref| <= 1e-3 * max |o_ref| per query row for fp32
outputs; a bf16 / fp16 output may add one unit in its last place (2^-7 /
2^-10 of the row's max) for its own rounding.  lse within 1e-4 (relative to
max(1, |lse|)).
"""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

RTOL = 1e-3


def _ref(q, segs, o_parts, lse_parts, G, scale):
    """float64 attention of q (B, Hq, D) over the segments' tokens, merged with parts."""
    B, Hq, D = q.shape
    ks = [k[:, :, :n].double() for k, _, n in segs]
    vs = [v[:, :, :n].double() for _, v, n in segs]
    qd = q.double().cpu().numpy()
    los, lss = [], []
    if ks and sum(k.shape[2] for k in ks) > 0:
        K = torch.cat(ks, 2).cpu().numpy()
        V = torch.cat(vs, 2).cpu().numpy()
        Kr = np.repeat(K, G, axis=1)
        Vr = np.repeat(V, G, axis=1)
        s = np.einsum("bhd,bhsd->bhs", qd, Kr) * scale
        mx = s.max(-1, keepdims=True)
        e = np.exp(s - mx)
        los.append(np.einsum("bhs,bhsd->bhd", e, Vr) / e.sum(-1, keepdims=True))
        lss.append(mx[..., 0] + np.log(e.sum(-1)))
    if o_parts is not None:
        for i in range(o_parts.shape[0]):
            los.append(o_parts[i].double().cpu().numpy())
            lss.append(lse_parts[i].double().cpu().numpy())
    L = np.stack(lss)
    M = L.max(0)
    w = np.exp(L - M)
    o = (np.stack(los) * w[..., None]).sum(0) / w.sum(0)[..., None]
    return o, M + np.log(w.sum(0))


def _row_err(o, ref):
    return float((np.abs(o - ref).max(-1) / np.abs(ref).max(-1)).max())


CASES = [
    # B, Hkv, G, D, segment (cap, len) list, n_parts, q dtype, kv dtype
    (2, 8, 4, 128, [(64, 64), (64, 64), (64, 37)], 1, torch.bfloat16, torch.bfloat16),
    (1, 4, 1, 64, [(100, 100)], 2, torch.float16, torch.float16),
    (3, 2, 8, 128, [(5, 5), (64, 1)], 0, torch.float32, torch.bfloat16),
    (2, 2, 3, 64, [], 3, torch.bfloat16, torch.bfloat16),
    (1, 8, 4, 128, [(300, 300), (64, 64), (64, 0)], 1, torch.float32, torch.float32),
]


@pytest.mark.parametrize("case", CASES, ids=[f"B{c[0]}H{c[1]}G{c[2]}D{c[3]}s{len(c[4])}p{c[5]}" for c in CASES])
def test_dense_merge_matches_float64(case):
    from latticequant_b200 import attention as A

    B, H, G, D, seglist, P, qdt, kdt = case
    g = torch.Generator().manual_seed(7)
    q = (torch.randn(B, H * G, D, generator=g) / math.sqrt(D)).to(qdt).cuda()
    segs = []
    for cap, n in seglist:
        k = (torch.randn(B, H, cap, D, generator=g) * 2).to(kdt).cuda()
        v = torch.randn(B, H, cap, D, generator=g).to(kdt).cuda()
        segs.append((k, v, n))
    po = pl = None
    if P:
        po = torch.randn(P, B, H * G, D, generator=g).cuda()
        pl = (torch.randn(P, B, H * G, generator=g) * 3).cuda()
    lse = torch.empty(B, H * G, dtype=torch.float32, device="cuda")
    scale = 1 / math.sqrt(D)
    o = A.dense_merge_attention(q, segs, po, pl, H, scale, lse=lse)
    assert o.dtype == qdt and o.shape == (B, H * G, D)
    ref, lref = _ref(q.float(), segs, po, pl, G, scale)
    ulp = {torch.float32: 0.0, torch.bfloat16: 2.0 ** -7, torch.float16: 2.0 ** -10}[qdt]
    assert _row_err(o.float().cpu().numpy(), ref) <= RTOL + ulp
    assert np.abs(lse.cpu().numpy() - lref).max() < 1e-4 * max(1.0, np.abs(lref).max())


def test_dense_merge_device_length_follows_slot_index():
    """A segment length read on the device (the last valid slot + 1): the
    result equals the host-length call, and changing the slot on the device
    changes it without a new call's arguments (CUDA-graph replays)."""
    from latticequant_b200 import attention as A

    B, H, G, D, T = 2, 4, 4, 128, 64
    g = torch.Generator().manual_seed(9)
    q = (torch.randn(B, H * G, D, generator=g) / math.sqrt(D)).to(torch.bfloat16).cuda()
    k = torch.randn(B, H, T, D, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(B, H, T, D, generator=g).to(torch.bfloat16).cuda()
    po = torch.randn(1, B, H * G, D, generator=g).cuda()
    pl = torch.randn(1, B, H * G, generator=g).cuda()
    idx = torch.tensor([10], dtype=torch.int64, device="cuda")
    out = torch.empty(B, H * G, D, dtype=torch.bfloat16, device="cuda")
    graph = torch.cuda.CUDAGraph()
    A.dense_merge_attention(q, [(k, v, idx)], po, pl, H, out=out)  # warm-up outside the capture
    torch.cuda.synchronize()
    with torch.cuda.graph(graph):
        A.dense_merge_attention(q, [(k, v, idx)], po, pl, H, out=out)
    for slot in (10, 0, 63, 31):
        idx.fill_(slot)
        graph.replay()
        torch.cuda.synchronize()
        host = A.dense_merge_attention(q, [(k, v, slot + 1)], po, pl, H)
        assert torch.equal(out, host)
    del graph


def test_dense_merge_rejects_bad_arguments():
    from latticequant_b200 import attention as A

    q = torch.randn(1, 4, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(1, 2, 8, 128, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        A.dense_merge_attention(q, [(k, k, 8)] * 9, None, None, 2)  # too many segments
    with pytest.raises(ValueError):
        A.dense_merge_attention(q, [(k, k[:, :, :4], 4)], None, None, 2)  # K/V shapes differ
    with pytest.raises(ValueError):
        A.dense_merge_attention(q, [(k, k, 9)], None, None, 2)  # more tokens than the buffer holds
    # the C entry point refuses it as well
    import ctypes

    from latticequant_b200._lib import LQ_OK, dtype_code, lib

    arr = lambda t, *v: (t * 1)(*v)  # noqa: E731
    rc = lib().lq_attn_dense_merge(
        ctypes.c_void_p(q.data_ptr()), dtype_code(q.dtype), 1,
        ctypes.cast(arr(ctypes.c_void_p, k.data_ptr()), ctypes.c_void_p),
        ctypes.cast(arr(ctypes.c_void_p, k.data_ptr()), ctypes.c_void_p),
        ctypes.cast(arr(ctypes.c_int64, 8), ctypes.c_void_p), ctypes.cast(arr(ctypes.c_int64, 9), ctypes.c_void_p),
        None, dtype_code(k.dtype), None, None, 0, 1, 2, 2, 128, 0.1, ctypes.c_void_p(q.data_ptr()), None, None)
    assert rc != LQ_OK
