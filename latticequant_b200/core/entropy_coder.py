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


# ============================================================
# Frequency model and code-length measurement (core/entropy_coder.py:112-251)
# ============================================================
import numpy as np  # noqa: E402


class FrequencyModel:
    """Per-(coset, coordinate) symbol counts (core/entropy_coder.py:112-139);
    host bookkeeping over numpy arrays, as the reference does it."""

    def __init__(self):
        self.tables = {}
        self.totals = {}
        self.coset_prob = [0.5, 0.5]

    def fit(self, coset: np.ndarray, free_coords: np.ndarray, coord8_half: np.ndarray):
        p_half = (coset == 1).mean()
        self.coset_prob = [max(1 - p_half, 1e-30), max(p_half, 1e-30)]
        all_symbols = np.concatenate([free_coords, coord8_half[:, None]], axis=1)
        for c in [0, 1]:
            mask = coset == c
            if mask.sum() == 0:
                continue
            syms_c = all_symbols[mask]
            for idx in range(8):
                unique, counts = np.unique(syms_c[:, idx], return_counts=True)
                self.tables[(c, idx)] = dict(zip(unique.tolist(), counts.tolist()))
                self.totals[(c, idx)] = int(mask.sum())


def measure_ideal_code_length(model: FrequencyModel, coset: np.ndarray, free_coords: np.ndarray,
                              coord8_half: np.ndarray) -> dict:
    """Laplace-smoothed ideal code length (core/entropy_coder.py:147-185)."""
    N = len(coset)
    total_bits = 0.0
    n0 = (coset == 0).sum()
    total_bits += n0 * (-np.log2(model.coset_prob[0]))
    total_bits += (N - n0) * (-np.log2(model.coset_prob[1]))
    all_symbols = np.concatenate([free_coords, coord8_half[:, None]], axis=1)
    for c_val in [0, 1]:
        mask = coset == c_val
        if mask.sum() == 0:
            continue
        syms_c = all_symbols[mask]
        total_c = model.totals.get((c_val, 0), syms_c.shape[0])
        for idx in range(8):
            table = model.tables.get((c_val, idx), {})
            alphabet_size = len(table) + 1
            unique_vals, counts = np.unique(syms_c[:, idx], return_counts=True)
            for val, cnt in zip(unique_vals, counts):
                prob = (table.get(int(val), 0) + 1) / (total_c + alphabet_size)
                total_bits += cnt * (-np.log2(prob))
    return {"total_bits": total_bits, "bits_per_dim": total_bits / (N * 8)}


def measure_real_ans(model: FrequencyModel, coset: np.ndarray, free_coords: np.ndarray,
                     coord8_half: np.ndarray) -> dict:
    """Real coded size with this package's rANS on Laplace-smoothed tables (the
    reference measures constriction's coder here, core/entropy_coder.py:191-251)."""
    from .entropy_storage import compress_symbols

    streams, _ = compress_symbols(model, np.asarray(coset), np.asarray(free_coords), np.asarray(coord8_half))
    total_bits = 32 * sum(len(s.bitstream) for s in streams if s is not None)
    return {"total_bits": total_bits, "bits_per_dim": total_bits / (len(coset) * 8), "status": "ok"}
