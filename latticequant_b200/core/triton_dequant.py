"""4-bit compact unpack + per-head scale -> float16 (the API of core/triton_dequant.py).

The reference implements this as a Triton kernel; here it is the CUDA
library's lq_unpack_e8 (same signature and output, no Triton).
"""
from __future__ import annotations

import torch

from .. import _dev
from .._lib import check, lib, ptr, stream_handle


def triton_unpack_e8_4bit(packed: torch.Tensor, scales: torch.Tensor, head_indices: torch.Tensor) -> torch.Tensor:
    """(N, 4) uint8 packed E8 + scales[head_indices] -> (N, 8) float16 (core/triton_dequant.py:139-177)."""
    assert packed.dtype == torch.uint8
    assert packed.shape[1] == 4
    assert packed.is_cuda
    dev = packed.device
    p = packed.contiguous()
    n = p.shape[0]
    sc = scales.to(device=dev, dtype=torch.float32).contiguous()
    hi = head_indices.to(device=dev, dtype=torch.int32).contiguous()
    out = torch.empty(n, 8, dtype=torch.float16, device=dev)
    check(lib().lq_unpack_e8(ptr(p), n, 4, ptr(sc), ptr(hi), None, ptr(out), stream_handle(dev)), "lq_unpack_e8")
    return out
