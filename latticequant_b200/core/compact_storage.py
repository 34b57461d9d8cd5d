"""Compact fixed-rate E8 storage -- the API of core/compact_storage.py on the B200.

b bytes per block, big-endian: [coset | u0..u6 (b bits) | u7 >> 1 (b-1 bits)],
u = int + 2^(b-1); coord7's low bit follows from the even sum.  pack_e8 is
strict and raises the reference's ValueError messages.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Tuple

import torch

from .. import _dev
from .._lib import check, lib, ptr, stream_handle


def _check(q: torch.Tensor, atol: float, bits: int):
    qb, dev, _, _ = _dev.as_blocks_f32(q)
    n = qb.shape[0]
    valid = torch.empty(n, dtype=torch.uint8, device=qb.device)
    coset = torch.empty(n, dtype=torch.uint8, device=qb.device)
    in_range = torch.empty(n, dtype=torch.uint8, device=qb.device) if bits > 0 else None
    check(lib().lq_check_e8(ptr(qb), n, ctypes.c_float(atol), bits, ptr(valid), ptr(coset), ptr(in_range),
                            stream_handle(qb.device)), "lq_check_e8")
    return qb, dev, valid.bool(), coset, in_range


def validate_e8(q: torch.Tensor, atol: float = 1e-5) -> Tuple[torch.Tensor, torch.Tensor]:
    """(is_valid (N,) bool, coset (N,) long) (core/compact_storage.py:39-80)."""
    _, dev, valid, coset, _ = _check(q, atol, 0)
    return _dev.back(valid, dev), _dev.back(coset.long(), dev)


def representable_range(bits_per_dim: int) -> Tuple[int, int]:
    R = 2 ** (bits_per_dim - 1)
    return -R, R - 1


def check_representable(q: torch.Tensor, bits_per_dim: int) -> torch.Tensor:
    """Valid E8 points whose integer coordinates fit b bits (core/compact_storage.py:235-249)."""
    _, dev, _, _, in_range = _check(q, 1e-5, bits_per_dim)
    return _dev.back(in_range.bool(), dev)


def pack_e8(q: torch.Tensor, bits_per_dim: int) -> torch.Tensor:
    """Strict pack of valid in-range E8 points into (N, b) bytes (core/compact_storage.py:87-154)."""
    assert bits_per_dim in (3, 4, 5), f"Only integer bit rates 3,4,5 supported, got {bits_per_dim}"
    assert q.shape[-1] == 8, f"Expected 8-dim vectors, got {q.shape[-1]}"
    qb, dev, valid, coset, in_range = _check(q, 1e-5, bits_per_dim)
    N = qb.shape[0]
    n_invalid = int((~valid).sum().item())
    if n_invalid > 0:
        raise ValueError(
            f"{n_invalid}/{N} inputs are not valid E₈ points. "
            f"All coordinates must be consistently integer or half-integer "
            f"with even sum on the integer representation."
        )
    R = 2 ** (bits_per_dim - 1)
    n_oor = int((~in_range.bool()).sum().item())
    if n_oor > 0:
        ints = (qb - 0.5 * coset.float().unsqueeze(-1)).round().long()
        max_abs = ints.abs().max().item()
        raise ValueError(
            f"{n_oor}/{N} vectors have coordinates outside [{-R}, {R-1}]. "
            f"Max |coord| = {max_abs}. "
            f"At {bits_per_dim} bits/dim, lattice coordinates must fit in "
            f"{bits_per_dim}-bit signed range. "
            f"Use check_representable() to filter, use more bits, "
            f"or handle non-representable vectors in a separate path."
        )
    out = torch.empty(N, bits_per_dim, dtype=torch.uint8, device=qb.device)
    bad = torch.zeros(2, dtype=torch.int32, device=qb.device)
    check(lib().lq_pack_e8(ptr(qb), N, bits_per_dim, ptr(out), ptr(bad), stream_handle(qb.device)), "lq_pack_e8")
    return _dev.back(out, dev)


def unpack_e8(packed_bytes: torch.Tensor, bits_per_dim: int) -> torch.Tensor:
    """(N, b) bytes -> (N, 8) float32 E8 points (core/compact_storage.py:157-222)."""
    assert bits_per_dim in (3, 4, 5)
    assert packed_bytes.dtype == torch.uint8
    assert packed_bytes.ndim == 2
    assert packed_bytes.shape[1] == bits_per_dim, \
        f"Expected {bits_per_dim} bytes per vector, got {packed_bytes.shape[1]}"
    dev = _dev.cuda_device(packed_bytes)
    p = packed_bytes.to(dev).contiguous()
    n = p.shape[0]
    q = torch.empty(n, 8, dtype=torch.float32, device=dev)
    check(lib().lq_unpack_e8(ptr(p), n, bits_per_dim, None, None, ptr(q), None, stream_handle(dev)), "lq_unpack_e8")
    return _dev.back(q, packed_bytes.device)


@dataclass
class CompactE8Tensor:
    """Packed data + scales with theoretical storage accounting (core/compact_storage.py:279-331)."""
    packed: torch.Tensor
    scales: torch.Tensor
    bits_per_dim: int
    orig_shape: tuple
    group_size: int
    num_vectors: int

    @property
    def packed_bytes(self) -> int:
        return self.packed.nelement() * self.packed.element_size()

    @property
    def scale_bytes(self) -> int:
        return self.scales.nelement() * self.scales.element_size()

    @property
    def total_bytes(self) -> int:
        return self.packed_bytes + self.scale_bytes

    @property
    def fp16_bytes(self) -> int:
        return self.num_vectors * 8 * 2

    @property
    def effective_bits_per_dim(self) -> float:
        return (self.total_bytes * 8) / (self.num_vectors * 8)

    @property
    def compression_ratio(self) -> float:
        return self.fp16_bytes / self.total_bytes

    def summary(self) -> str:
        return "\n".join([
            "CompactE8Tensor (theoretical storage)",
            f"  Vectors: {self.num_vectors:,} x 8-dim",
            f"  Nominal rate: {self.bits_per_dim} bits/dim",
            f"  Effective rate: {self.effective_bits_per_dim:.3f} bits/dim (incl. scales)",
            f"  Packed: {self.packed_bytes:,} B | Scales: {self.scale_bytes:,} B | Total: {self.total_bytes:,} B",
            f"  FP16 equiv: {self.fp16_bytes:,} B | Compression: {self.compression_ratio:.2f}x",
        ])


def quantize_and_pack(x: torch.Tensor, bits_per_dim: int, scale: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """encode_e8(x / scale) -> (packed representable rows, in_range mask) (core/compact_storage.py:338-360)."""
    from .e8_quantizer import quantize_e8  # noqa: F401 (same division semantics)

    xb, dev, _, _ = _dev.as_blocks_f32(x)
    n = xb.shape[0]
    q = torch.empty_like(xb)
    sc = float(torch.tensor(scale, dtype=torch.float32))
    check(lib().lq_quantize_e8(ptr(xb), n, ctypes.c_float(sc), ptr(q), None, stream_handle(xb.device)), "quantize")
    in_range = check_representable(q, bits_per_dim)
    if int(in_range.sum().item()) == 0:
        return _dev.back(torch.zeros(0, bits_per_dim, dtype=torch.uint8, device=xb.device), dev), \
            _dev.back(in_range, dev)
    packed = pack_e8(q[in_range], bits_per_dim)
    return _dev.back(packed, dev), _dev.back(in_range, dev)


def unpack_and_dequantize(packed: torch.Tensor, bits_per_dim: int, scale: float) -> torch.Tensor:
    """unpack_e8(packed) * scale (core/compact_storage.py:363-370)."""
    dev = _dev.cuda_device(packed)
    q = unpack_e8(packed.to(dev), bits_per_dim)
    return _dev.back(q * scale, packed.device)
