"""Quantization pipeline -- the API of core/pipeline.py on the B200.

d-dim vector -> RHT -> 8-dim blocks -> E8 quantise -> parity-aware symbols,
and back.  The Walsh-Hadamard butterflies run in lq_fwht (bit-exact with the
reference's torch arithmetic); the E8 quantiser, scale and symbolisation are
this package's CUDA mirrors.  RHT's sign vector comes from torch's CPU
generator exactly as the reference draws it (core/pipeline.py:94-100), so
encoder and decoder built with one seed agree with the reference's.
"""
from __future__ import annotations

import numpy as np
import torch

from .. import _dev
from .._lib import check, lib, ptr, stream_handle
from .e8_quantizer import compute_scale, encode_e8, quantize_e8, theoretical_mse, G_E8  # noqa: F401
from .entropy_coder import (FrequencyModel, e8_to_symbols, measure_ideal_code_length, measure_real_ans,  # noqa: F401
                            symbols_to_e8)


def hadamard_matrix(n: int) -> torch.Tensor:
    """Sylvester construction, entries +-1, unnormalised (core/pipeline.py:33-46)."""
    assert n > 0 and (n & (n - 1)) == 0, f"n must be power of 2, got {n}"
    H = torch.tensor([[1.0]])
    while H.shape[0] < n:
        H = torch.cat([torch.cat([H, H], dim=1), torch.cat([H, -H], dim=1)], dim=0)
    return H


def _fwht(x: torch.Tensor, pre=None, post=None) -> torch.Tensor:
    d = x.shape[-1]
    assert d > 0 and (d & (d - 1)) == 0, f"d must be power of 2, got {d}"
    dev = x.device
    xc = x.to(device=_dev.cuda_device(x), dtype=torch.float32).contiguous()
    out = torch.empty_like(xc)
    n = xc.numel() // d
    sg = lambda s: None if s is None else s.to(device=xc.device, dtype=torch.float32).contiguous()
    pre, post = sg(pre), sg(post)
    check(lib().lq_fwht(ptr(xc), n, d, ptr(pre), ptr(post), ptr(out), stream_handle(xc.device)), "lq_fwht")
    return _dev.back(out, dev)


def fast_hadamard_transform(x: torch.Tensor) -> torch.Tensor:
    """H x / sqrt(d) over the last dimension (core/pipeline.py:49-69)."""
    return _fwht(x)


def inverse_fast_hadamard_transform(x: torch.Tensor) -> torch.Tensor:
    """The same transform (H is symmetric, H^-1 = H/d) (core/pipeline.py:72-78)."""
    return _fwht(x)


class RHT:
    """w = (1/sqrt(d)) H D_eps v with random signs eps (core/pipeline.py:81-122)."""

    def __init__(self, d: int, seed: int = 0):
        assert d % 8 == 0, f"d must be divisible by 8, got {d}"
        self.d = d
        gen = torch.Generator()
        gen.manual_seed(seed)
        self.signs = torch.where(torch.rand(d, generator=gen) < 0.5, torch.ones(d), -torch.ones(d))

    def forward(self, v: torch.Tensor) -> torch.Tensor:
        return _fwht(v, pre=self.signs)

    def inverse(self, w: torch.Tensor) -> torch.Tensor:
        return _fwht(w, post=self.signs)


def to_blocks(w: torch.Tensor) -> torch.Tensor:
    """(..., d) -> (..., d/8, 8) (core/pipeline.py:125-133)."""
    *batch, d = w.shape
    assert d % 8 == 0
    return w.reshape(*batch, d // 8, 8)


def from_blocks(blocks: torch.Tensor) -> torch.Tensor:
    """(..., K, 8) -> (..., 8K) (core/pipeline.py:136-144)."""
    *batch, K, eight = blocks.shape
    assert eight == 8
    return blocks.reshape(*batch, K * 8)


def _mean_square(w: torch.Tensor) -> float:
    """(w ** 2).mean().item() in torch's CPU summation order (lq_head_scales
    over one head of every element)."""
    x = w.to(device=_dev.cuda_device(w), dtype=torch.float32).contiguous()
    s2 = torch.empty(1, dtype=torch.float32, device=x.device)
    n = x.numel()
    ws_bytes = int(lib().lq_head_scales_workspace(1, n))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=x.device)
    check(lib().lq_head_scales(ptr(x), 0, 1, n, 1.0, ptr(s2), None, None, ptr(ws) if ws_bytes else None, ws_bytes,
                               stream_handle(x.device)), "lq_head_scales")
    return float(s2.item())


class LatticeQuantEncoder:
    """RHT -> sigma^2 -> scale -> E8 -> symbols (core/pipeline.py:151-239)."""

    def __init__(self, d: int, bits_per_dim: float, rht_seed: int = 0):
        self.d = d
        self.bits = bits_per_dim
        self.rht = RHT(d, seed=rht_seed)
        self.model = None

    def encode(self, v: torch.Tensor) -> dict:
        N = v.shape[0]
        w = self.rht.forward(v)
        sigma2 = _mean_square(w)
        scale = compute_scale(sigma2, self.bits)
        blocks = to_blocks(w)
        K = blocks.shape[1]
        blocks_flat = blocks.reshape(N * K, 8)
        q_flat = quantize_e8(blocks_flat, scale)
        w_hat = from_blocks(q_flat.reshape(N, K, 8))
        v_hat = self.rht.inverse(w_hat)
        lattice_points = q_flat / scale
        coset, free_coords, coord8_half = e8_to_symbols(lattice_points)
        return {"v_hat": v_hat, "w": w, "w_hat": w_hat, "scale": scale, "sigma2": sigma2, "coset": coset,
                "free_coords": free_coords, "coord8_half": coord8_half, "N": N, "K": K}

    def measure_rate(self, enc: dict, train_ratio: float = 0.5) -> dict:
        """Ideal and real (this package's rANS) rates on a train/test split
        (core/pipeline.py:207-239)."""
        coset = enc["coset"].cpu().numpy()
        free = enc["free_coords"].cpu().numpy()
        c8h = enc["coord8_half"].cpu().numpy()
        split = int(len(coset) * train_ratio)
        model = FrequencyModel()
        model.fit(coset[:split], free[:split], c8h[:split])
        self.model = model
        ideal = measure_ideal_code_length(model, coset[split:], free[split:], c8h[split:])
        real = measure_real_ans(model, coset[split:], free[split:], c8h[split:])
        return {"ideal_test_bpd": ideal["bits_per_dim"], "ans_test_bpd": real.get("bits_per_dim")}
