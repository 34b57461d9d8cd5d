"""Host-side logic of the reference-facing API and the C ABI surface (no GPU).

The library is loaded and its exports are checked against the header; no
compute entry point is called here.
"""
import ctypes
import torch
import os
import re

import numpy as np
import pytest

from conftest import ROOT, golden

LIB = os.path.join(ROOT, "latticequant_b200", "liblq_b200.so")
HDR = os.path.join(ROOT, "include", "latticequant_b200.h")


def _declared():
    text = open(HDR).read()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char \*)\s*\*?\s*(lq_\w+)\s*\(", text, re.M)))


@pytest.fixture(scope="module")
def cabi():
    if not os.path.exists(LIB):
        from latticequant_b200 import _build

        _build.build()
    return ctypes.CDLL(LIB)


def test_library_exports_every_declared_symbol(cabi):
    names = _declared()
    assert len(names) >= 20
    for n in names:
        assert hasattr(cabi, n), n


def test_library_exports_only_the_declared_abi(cabi):
    """The export map keeps internal C++ helpers and the static CUDA runtime
    local: the dynamic symbol table holds exactly the header's lq_* names."""
    import shutil
    import subprocess

    if shutil.which("nm") is None:
        pytest.skip("nm not available")
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if len(ln.split()) == 3}
    assert exported == set(_declared()), sorted(exported ^ set(_declared()))


def test_host_only_entry_points(cabi):
    cabi.lq_version.restype = ctypes.c_int
    cabi.lq_strerror.restype = ctypes.c_char_p
    cabi.lq_strerror.argtypes = [ctypes.c_int]
    assert cabi.lq_version() >= 100
    for code in (0, -1, -2, -3, -4, -5):
        assert cabi.lq_strerror(code)
    cabi.lq_rans_encode_workspace.restype = ctypes.c_size_t
    cabi.lq_rans_encode_workspace.argtypes = [ctypes.c_int64] * 3
    cabi.lq_head_scales_workspace.restype = ctypes.c_size_t
    cabi.lq_head_scales_workspace.argtypes = [ctypes.c_int64] * 2
    assert cabi.lq_rans_encode_workspace(64, 8 * 131072, 1024) > 0
    assert cabi.lq_head_scales_workspace(16, 128) == 0          # small heads fold in one pass
    assert cabi.lq_head_scales_workspace(16, 1 << 20) > 0


def test_static_scales_refuse_oversized_counts_before_any_device_call(cabi):
    """lq_head_scales_static checks its scratch capacity on the host, before it
    asks for a device: head counts whose scratch size would overflow a 64-bit
    product are refused with LQ_ERR_CAPACITY (x is never dereferenced)."""
    f = cabi.lq_head_scales_static
    f.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_float] + \
        [ctypes.c_void_p] * 4
    f.restype = ctypes.c_int
    dummy = ctypes.c_void_p(256)
    for n_heads in (255, 1 << 40, 1 << 57, (1 << 63) - 1):
        assert f(dummy, 2, n_heads, 1 << 20, ctypes.c_float(1.0), None, None, None, None) == -3, n_heads


def test_build_rans_table_matches_reference_fixtures():
    from latticequant_b200.core.gpu_ans import L, build_rans_table

    g = golden("rans.npz")
    for i in range(int(g["n_cases"])):
        t = build_rans_table(g[f"c{i}_counts"], list(g[f"c{i}_alphabet"]))
        assert np.array_equal(t.freqs, g[f"c{i}_freqs"]), i
        assert np.array_equal(t.cumfreqs, g[f"c{i}_cumfreqs"]), i
        assert np.array_equal(t.lookup, g[f"c{i}_lookup"]), i
        assert t.cumfreqs[-1] == L


def test_build_rans_table_rejects_alphabet_over_L():
    from latticequant_b200.core.gpu_ans import build_rans_table

    with pytest.raises(ValueError):
        build_rans_table(np.ones(1025, np.int64), list(range(1025)))


def test_host_formulas_match_reference():
    from latticequant_b200.core import compact_storage as cs
    from latticequant_b200.core import e8_quantizer as e8

    assert e8.G_E8 == 0.0717
    for b in (3, 4, 5):
        assert e8.compute_scale(1.0, b) == np.sqrt(2 * np.pi * np.e * 4.0 ** (-b))
        assert cs.representable_range(b) == (-(2 ** (b - 1)), 2 ** (b - 1) - 1)


def test_compact_tensor_accounting():
    import torch

    from latticequant_b200.core.compact_storage import CompactE8Tensor

    ct = CompactE8Tensor(packed=torch.zeros(1000, 4, dtype=torch.uint8), scales=torch.zeros(3, dtype=torch.float32),
                         bits_per_dim=4, orig_shape=(1, 3, 1000, 8), group_size=1000, num_vectors=1000)
    assert ct.total_bytes == 4000 + 12
    assert ct.fp16_bytes == 16000
    assert abs(ct.effective_bits_per_dim - (4012 * 8) / 8000) < 1e-12
    assert "CompactE8Tensor" in ct.summary()


def test_geometry_and_capacity():
    from latticequant_b200 import codec

    g = codec.Geometry(3, 8, 8192 * 16, 1024)
    assert g.n_tiles == 1024 and g.n_lanes == 3 * 1024 * 16
    assert g.words_capacity >= 3 * (8 * g.n_vectors * 10) // 32
    assert codec.round_tile(None, 1000) == 1024 and codec.round_tile(33, 1) == 64
    assert codec.vol_mult(4) == 4.0 ** -4


def test_rht_signs_match_reference():
    from latticequant_b200.core.pipeline import RHT, hadamard_matrix, to_blocks, from_blocks

    g = golden("rht.npz")
    for d in (8, 64, 128):
        for seed in (0, 7):
            assert np.array_equal(RHT(d, seed=seed).signs.numpy(), g[f"signs_d{d}_s{seed}"])
    H = hadamard_matrix(8)
    assert torch.equal(H @ H.T, 8 * torch.eye(8))
    w = torch.arange(32.0).reshape(2, 16)
    assert torch.equal(from_blocks(to_blocks(w)), w)


def test_compact_index_words_and_ranks():
    """attention.compact_index: bit i of word w = block 32w+i representable
    (bit 31 included, as a negative int32), rank = representable blocks before
    word w; a ragged last word."""
    import types

    import numpy as np
    import torch

    from latticequant_b200 import attention

    rng = np.random.default_rng(3)
    for n in (32, 70, 1000):
        m = rng.random(n) < 0.7
        m[31] = True
        ch = types.SimpleNamespace(repr_mask=torch.from_numpy(m))
        words, rank = attention.compact_index(ch)
        nw = (n + 31) // 32
        pad = np.zeros(nw * 32, bool)
        pad[:n] = m
        bits = pad.reshape(nw, 32)
        ref_w = (bits.astype(np.uint64) << np.arange(32, dtype=np.uint64)).sum(1).astype(np.uint32)
        assert np.array_equal(words.numpy().view(np.uint32), ref_w)
        cnt = bits.sum(1)
        assert np.array_equal(rank.numpy(), np.concatenate([[0], np.cumsum(cnt)[:-1]]).astype(np.int32))
        assert attention.compact_index(ch) is ch._lq_index  # cached
