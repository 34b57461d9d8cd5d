"""E8 lattice quantiser -- the API of core/e8_quantizer.py, computed on the B200.

encode_d8 / encode_e8 / quantize_e8 run the CUDA kernels of liblq_b200.so
(bit-exact with the reference's torch arithmetic on the CPU for float32
input; other dtypes are computed in float32).  compute_scale and
theoretical_mse are the reference's closed-form host formulas.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from .. import _dev
from .._lib import check, lib, ptr, stream_handle

G_E8 = 0.0717      # normalized second moment (core/e8_quantizer.py:131)
VOL_E8_UNIT = 1.0  # core/e8_quantizer.py:132


def _encode(x: torch.Tensor, d8_only: int) -> torch.Tensor:
    xb, dev, shape, dtype = _dev.as_blocks_f32(x)
    out = torch.empty_like(xb)
    check(lib().lq_encode_e8(ptr(xb), xb.shape[0], ptr(out), d8_only, stream_handle(xb.device)), "encode_e8")
    out = out.reshape(shape)
    return _dev.back(out if dtype == torch.float32 or not dtype.is_floating_point else out.to(dtype), dev)


def encode_d8(x: torch.Tensor) -> torch.Tensor:
    """Nearest point of D8 = {z in Z^8 : sum(z) even} (core/e8_quantizer.py:20-58)."""
    return _encode(x, 1)


def encode_e8(x: torch.Tensor) -> torch.Tensor:
    """Nearest point of E8 = D8 u (D8 + 1/2); ties keep D8 (core/e8_quantizer.py:61-83)."""
    return _encode(x, 0)


def quantize_e8(x: torch.Tensor, scale: float) -> torch.Tensor:
    """Q(x / scale) * scale on 8-dim blocks (core/e8_quantizer.py:90-110)."""
    xb, dev, shape, dtype = _dev.as_blocks_f32(x)
    out = torch.empty_like(xb)
    sc = float(np.float32(scale))
    check(lib().lq_quantize_e8(ptr(xb), xb.shape[0], ctypes.c_float(sc), None, ptr(out), stream_handle(xb.device)),
          "quantize_e8")
    out = out.reshape(shape)
    return _dev.back(out if dtype == torch.float32 else out.to(dtype), dev)


def dequantize_error(x: torch.Tensor, x_hat: torch.Tensor) -> dict:
    """Per-dimension MSE and max error (core/e8_quantizer.py:113-124)."""
    err = x - x_hat
    mse_total = (err ** 2).mean().item()
    mse_per_dim = (err ** 2).reshape(-1, 8).mean().item()
    return {"mse_per_dim": mse_per_dim, "mse_total": mse_total, "max_abs_err": err.abs().max().item()}


def compute_scale(sigma2: float, bits_per_dim: float) -> float:
    """a = sqrt(2*pi*e*sigma2*4^-b) (core/e8_quantizer.py:137-148)."""
    target_vol_2n = 2 * np.pi * np.e * sigma2 * (4 ** (-bits_per_dim))
    return np.sqrt(target_vol_2n)


def theoretical_mse(sigma2: float, bits_per_dim: float) -> float:
    """G(E8) * 2*pi*e * sigma2 * 4^-b (core/e8_quantizer.py:151-156)."""
    return G_E8 * 2 * np.pi * np.e * sigma2 * (4 ** (-bits_per_dim))
