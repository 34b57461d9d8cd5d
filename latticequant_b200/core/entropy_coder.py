"""Parity-aware symbolisation -- the API of core/entropy_coder.py on the B200.

coset bit + 7 free coordinates + coord8_half = floor(coord8 / 2); the 8th
coordinate's parity follows from the even-sum constraint of D8.
"""
from __future__ import annotations

import torch

from .. import _dev
from .._lib import check, lib, ptr, stream_handle


def e8_to_symbols(q: torch.Tensor):
    """E8 point -> (coset, free_coords (N,7), coord8_half), int64 (core/entropy_coder.py:46-68)."""
    qb, dev, _, _ = _dev.as_blocks_f32(q)
    n = qb.shape[0]
    cos = torch.empty(n, dtype=torch.int32, device=qb.device)
    sym = torch.empty(n, 8, dtype=torch.int32, device=qb.device)
    check(lib().lq_e8_to_symbols(ptr(qb), n, ptr(cos), ptr(sym), stream_handle(qb.device)), "e8_to_symbols")
    coset = _dev.back(cos.long(), dev)
    free = _dev.back(sym[:, :7].long(), dev)
    c8h = _dev.back(sym[:, 7].long(), dev)
    return coset, free, c8h


def symbols_to_e8(coset: torch.Tensor, free_coords: torch.Tensor, coord8_half: torch.Tensor) -> torch.Tensor:
    """Inverse of e8_to_symbols, float32 (N, 8) (core/entropy_coder.py:71-89)."""
    dev_out = coset.device
    dev = _dev.cuda_device(coset)
    n = coset.shape[0]
    cos = coset.to(device=dev, dtype=torch.int32).contiguous()
    sym = torch.cat([free_coords.to(device=dev, dtype=torch.int32), coord8_half.to(device=dev, dtype=torch.int32)
                     .reshape(-1, 1)], dim=1).contiguous()
    q = torch.empty(n, 8, dtype=torch.float32, device=dev)
    check(lib().lq_symbols_to_e8(ptr(cos), ptr(sym), n, ptr(q), stream_handle(dev)), "symbols_to_e8")
    return _dev.back(q, dev_out)
