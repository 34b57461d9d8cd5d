"""The allocation-free scale entry point, lq_head_scales_static.

Some callers of this library cannot allocate device memory: a host process
that owns all GPU memory and offers no allocator (a serving engine with a
pre-reserved pool, a plugin loaded from another language without torch), or a
decode step that must not pay the device-wide synchronisation that a
cudaMalloc/cudaFree can bring.  lq_head_scales_static gives them the per-head
variance/scale computation with its scratch inside the library's own static
device array (4 MiB).  This file checks it through the C ABI against the
regular lq_head_scales (caller workspace), bit for bit, on two calls in a row,
and that a problem too big for the array is refused before any launch.  It is
collected last so a failure here leaves every other test already run.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

LQ_OK, LQ_ERR_CAPACITY, LQ_BF16 = 0, -3, 2
STATIC_FLOATS = 1 << 20


def _bind(lib):
    f = lib.lq_head_scales_static
    f.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p,
                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return f


def _outs(n):
    return (torch.empty(n, dtype=torch.float32, device="cuda"), torch.empty(n, dtype=torch.float32, device="cuda"),
            torch.empty(n, dtype=torch.float16, device="cuda"))


def test_static_scratch_matches_workspace_entry_point():
    from latticequant_b200 import _lib

    lib = _lib.lib()
    static = _bind(lib)
    P, stream = _lib.ptr, _lib.stream_handle()
    n_heads, elems = 16, 1 << 20  # config-2 heads: 8192 tokens x 128 channels; needs level-1 scratch
    need = lib.lq_head_scales_workspace(n_heads, elems)
    assert 0 < need <= 4 * STATIC_FLOATS
    vol = ctypes.c_float(float(torch.tensor(4.0 ** -4, dtype=torch.float32)))
    for call, seed in enumerate((11, 12)):  # two calls in a row share (and reuse) the static array
        g = torch.Generator(device="cuda")
        g.manual_seed(seed)
        x = (torch.randn(n_heads, elems, device="cuda", generator=g) *
             torch.exp(torch.randn(n_heads, 1, device="cuda", generator=g))).to(torch.bfloat16)
        ref_s2, ref_s32, ref_s16 = _outs(n_heads)
        ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        _lib.check(lib.lq_head_scales(P(x), LQ_BF16, n_heads, elems, vol, P(ref_s2), P(ref_s32), P(ref_s16), P(ws),
                                      need, stream), "lq_head_scales")
        s2, s32, s16 = _outs(n_heads)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        alloc_before, reserved_before = torch.cuda.memory_allocated(), torch.cuda.memory_reserved()
        rc = static(P(x), LQ_BF16, n_heads, elems, vol, P(s2), P(s32), P(s16), stream)
        torch.cuda.synchronize()
        assert rc == LQ_OK
        # nothing goes through torch's allocator, and the device's free memory
        # does not drop by anything near the scratch size (a cudaMalloc of the
        # 4 MiB scratch would); the slack allows for unrelated driver activity
        assert torch.cuda.memory_allocated() == alloc_before
        assert torch.cuda.memory_reserved() == reserved_before
        if call == 1:  # after the first call's set-up
            assert free_before - torch.cuda.mem_get_info()[0] < 2 * STATIC_FLOATS
        assert torch.equal(s2.view(torch.int32), ref_s2.view(torch.int32)), call
        assert torch.equal(s32.view(torch.int32), ref_s32.view(torch.int32)), call
        assert torch.equal(s16.view(torch.int16), ref_s16.view(torch.int16)), call


def test_static_scratch_refuses_oversized_problem():
    from latticequant_b200 import _lib

    lib = _lib.lib()
    static = _bind(lib)
    n_heads, elems = 256, 1 << 20  # 256 heads of 2^20: needs more than the 4 MiB array
    assert lib.lq_head_scales_workspace(n_heads, elems) > 4 * STATIC_FLOATS
    x = torch.zeros(n_heads, elems, dtype=torch.bfloat16, device="cuda")
    s2, s32, s16 = _outs(n_heads)
    s32.fill_(-1.0)
    rc = static(_lib.ptr(x), LQ_BF16, n_heads, elems, ctypes.c_float(1.0), _lib.ptr(s2), _lib.ptr(s32),
                _lib.ptr(s16), _lib.stream_handle())
    torch.cuda.synchronize()
    assert rc == LQ_ERR_CAPACITY
    assert lib.lq_strerror(rc).decode()
    assert bool((s32 == -1.0).all())  # nothing was launched
