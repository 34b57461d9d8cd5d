"""ctypes binding of liblq_b200.so (the C ABI declared in include/latticequant_b200.h).

The library is the only compute path: there is no CPU fallback.  Loading
fails loudly when the shared object is missing or when no CUDA device is
visible at the first call that needs one.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblq_b200.so")

# status codes / flags / dtypes (include/latticequant_b200.h)
LQ_OK = 0
LQ_ERR_INVALID, LQ_ERR_ALPHABET, LQ_ERR_CAPACITY, LQ_ERR_CUDA, LQ_ERR_STREAM = -1, -2, -3, -4, -5
EF_ALPHABET, EF_SYMRANGE, EF_CAPACITY, EF_BITSTREAM, EF_NONFINITE, EF_NOCONVERGE = 0x1, 0x2, 0x4, 0x8, 0x10, 0x20
EF_TIMEOUT = 0x40
LQ_F32, LQ_F16, LQ_BF16 = 0, 1, 2
L = 1024
SYM_LIMIT = 512
HIST_BINS = 1024
NSTREAMS = 16
DENSE_MAX_SEGMENTS = 8  # lq_attn_dense_merge segments per call

_FLAG_TEXT = {
    EF_ALPHABET: "a stream alphabet exceeds L=1024 symbols (the reference's build_rans_table loops forever here)",
    EF_SYMRANGE: f"a lattice coordinate lies outside [-{SYM_LIMIT}, {SYM_LIMIT})",
    EF_CAPACITY: "compressed output larger than the buffer capacity",
    EF_BITSTREAM: "corrupt bitstream or lane metadata",
    EF_NONFINITE: "non-finite value in the input or in input/scale",
    EF_NOCONVERGE: "rANS frequency normalisation did not converge",
    EF_TIMEOUT: "a bulk copy into shared memory did not complete within a second",
}

_lib = None
_lock = threading.Lock()


class LatticeQuantError(RuntimeError):
    """Raised for device-side data errors reported through the error word."""


class ChunkView(ctypes.Structure):
    """struct lq_chunk_view: device pointers + geometry of one compressed chunk."""

    _fields_ = [("words", ctypes.c_void_p), ("n_words", ctypes.c_int64),
                ("lane_off", ctypes.c_void_p), ("lane_nbits", ctypes.c_void_p), ("lane_state", ctypes.c_void_p),
                ("coset_words", ctypes.c_void_p), ("tile_n0", ctypes.c_void_p),
                ("tab_lo", ctypes.c_void_p), ("tab_nsym", ctypes.c_void_p), ("tab_freq", ctypes.c_void_p),
                ("dec_tab", ctypes.c_void_p), ("scale_f16", ctypes.c_void_p),
                ("n_heads", ctypes.c_int64), ("bph", ctypes.c_int64), ("tile_blocks", ctypes.c_int64),
                ("staged_tab", ctypes.c_void_p)]


class CompactView(ctypes.Structure):
    """struct lq_compact_view: a compact-layout chunk (packed codes, fp16
    fallback rows, mask words with per-word ranks, head scales)."""

    _fields_ = [("packed", ctypes.c_void_p), ("n_repr", ctypes.c_int64),
                ("fallback", ctypes.c_void_p), ("n_fallback", ctypes.c_int64),
                ("mask_words", ctypes.c_void_p), ("word_rank", ctypes.c_void_p), ("scales", ctypes.c_void_p),
                ("n_heads", ctypes.c_int64), ("bph", ctypes.c_int64), ("bits", ctypes.c_int)]


def _declare(lib):
    vp, i64, i32, f32, sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
    sig = {
        "lq_version": ([], i32),
        "lq_strerror": ([i32], ctypes.c_char_p),
        "lq_head_scales_workspace": ([i64, i64], sz),
        "lq_head_scales": ([vp, i32, i64, i64, f32, vp, vp, vp, vp, sz, vp], i32),
        "lq_sym_cols_bytes": ([i64, i64, i64], sz),
        "lq_e8_quantize": ([vp, i32, i64, i64, i64, vp, i64, vp, vp, vp, vp, vp, i32, vp, vp, vp], i32),
        "lq_encode_e8": ([vp, i64, vp, i32, vp], i32),
        "lq_build_tables": ([vp, i64, vp, vp, vp, vp, vp], i32),
        "lq_expand_tables": ([vp, vp, i64, vp, vp, vp, vp], i32),
        "lq_rans_encode_workspace": ([i64, i64, i64], sz),
        "lq_rans_encode": ([vp, vp, i64, i64, i64, vp, vp, vp, vp, i64, vp, vp, vp, vp, sz, vp, vp], i32),
        "lq_rans_decode_workspace": ([i64, i64, i64], sz),
        "lq_rans_decode": ([vp, i64, vp, vp, vp, vp, vp, i64, i64, i64, i64, vp, vp, vp, vp, vp, vp, i32, vp, vp,
                            sz, vp, vp], i32),
        "lq_rans_decode_streams": ([vp, i64, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp, vp, vp, vp], i32),
        "lq_pack_e8": ([vp, i64, i32, vp, vp, vp], i32),
        "lq_unpack_e8": ([vp, i64, i32, vp, vp, vp, vp, vp], i32),
        "lq_head_scales_static": ([vp, i32, i64, i64, f32, vp, vp, vp, vp], i32),
        "lq_selftest": ([i32, vp, vp, i64, ctypes.c_uint32, vp, vp], i32),
        "lq_attn_decode_workspace": ([i64, i64, i64, i32, i32], sz),
        "lq_attn_decode": ([ctypes.POINTER(ChunkView), ctypes.POINTER(ChunkView), vp, i32, i64, i64, i64, i32, i32,
                            i32, f32, vp, i32, vp, vp, vp, sz, vp, vp], i32),
        "lq_attn_merge": ([vp, vp, i64, i64, i32, vp, i32, vp, vp], i32),
        "lq_attn_merge_packed": ([vp, i64, i64, i32, vp, i32, vp, vp], i32),
        "lq_stage_tables": ([vp, vp, i64, vp, vp], i32),
        "lq_attn_dense_merge": ([vp, i32, i32, vp, vp, vp, vp, vp, i32, vp, vp, i64, i64, i64, i32, i32, f32, vp, vp,
                                 vp], i32),
        "lq_attn_compact_workspace": ([i64, i64, i32, i32], sz),
        "lq_attn_decode_compact": ([ctypes.POINTER(CompactView), ctypes.POINTER(CompactView), vp, i32, i64, i64, i64,
                                    i32, i32, f32, vp, i32, vp, vp, sz, vp, vp], i32),
        "lq_fwht": ([vp, i64, i32, vp, vp, vp, vp], i32),
        "lq_compact_merge": ([vp, i64, i32, vp, vp, vp, vp, i64, vp, i64, i64, vp, vp, vp], i32),
        "lq_e8_quantize_outliers": ([vp, i32, i64, i64, i64, vp, i64, vp, vp, vp, vp, vp, i32, vp, i32, i32, vp, vp,
                                     vp, i64, vp, vp], i32),
        "lq_patch_outliers": ([vp, vp, i64, i64, i64, i64, vp, vp, i32, vp, vp, vp], i32),
        "lq_quantize_e8": ([vp, i64, f32, vp, vp, vp], i32),
        "lq_e8_to_symbols": ([vp, i64, vp, vp, vp], i32),
        "lq_symbols_to_e8": ([vp, vp, i64, vp, vp], i32),
        "lq_check_e8": ([vp, i64, f32, i32, vp, vp, vp, vp], i32),
        "lq_pack_bits": ([vp, i64, vp, vp], i32),
        "lq_unpack_bits": ([vp, i64, vp, vp], i32),
        "lq_map_symbols": ([vp, i64, vp, ctypes.c_int32, i32, vp, vp], i32),
        "lq_rans_encode_streams": ([vp, vp, vp, vp, vp, vp, i64, vp, vp, vp, vp, vp, vp], i32),
        "lq_rans_finish_streams": ([vp, vp, vp, i64, vp, vp, vp], i32),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    return lib


def exported_symbols():
    """Names the library must export (every function of the C ABI header)."""
    import re

    hdr = os.path.join(HERE, "..", "include", "latticequant_b200.h")
    text = open(hdr).read()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char \*)\s*\*?\s*(lq_\w+)\s*\(", text, re.M)))


def lib():
    """Load (building first if the sources are newer) the CUDA library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                from . import _build

                _build.build()
            if not os.path.exists(LIB_PATH):
                raise ImportError(f"latticequant_b200: CUDA library {LIB_PATH} is missing; run "
                                  f"`python -m latticequant_b200._build`")
            _lib = _declare(ctypes.CDLL(LIB_PATH))
    return _lib


def require_cuda(t: torch.Tensor | None = None):
    if not torch.cuda.is_available():
        raise RuntimeError("latticequant_b200 needs a CUDA device (B200, sm_100a); there is no CPU fallback")
    if t is not None and not t.is_cuda:
        raise ValueError("latticequant_b200: tensor must live on a CUDA device")


def ptr(t: torch.Tensor | None):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def stream_handle(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def check(status: int, what: str):
    if status != LQ_OK:
        msg = lib().lq_strerror(status).decode()
        if status == LQ_ERR_CAPACITY:
            raise LatticeQuantError(f"{what}: {msg}")
        raise RuntimeError(f"{what}: {msg} (status {status})")


def raise_flags(flags: int, what: str):
    if flags:
        texts = [t for f, t in _FLAG_TEXT.items() if flags & f]
        if flags & EF_ALPHABET:
            raise ValueError(f"{what}: " + "; ".join(texts))
        raise LatticeQuantError(f"{what}: " + "; ".join(texts))


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return LQ_F32
    if dt == torch.float16:
        return LQ_F16
    if dt == torch.bfloat16:
        return LQ_BF16
    raise ValueError(f"latticequant_b200: unsupported dtype {dt} (float32, float16, bfloat16)")
