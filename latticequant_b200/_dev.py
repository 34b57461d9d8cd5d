"""Device plumbing shared by the reference-facing modules: move inputs to the
GPU, return results on the caller's device.  No arithmetic happens here."""
from __future__ import annotations

import numpy as np
import torch

from . import _lib


def cuda_device(t: torch.Tensor | None = None) -> torch.device:
    _lib.require_cuda()
    if t is not None and t.is_cuda:
        return t.device
    return torch.device("cuda", torch.cuda.current_device())


def as_blocks_f32(x: torch.Tensor):
    """(..., 8) tensor -> contiguous float32 (N, 8) on a CUDA device, plus the caller's device/shape/dtype."""
    if not isinstance(x, torch.Tensor):
        x = torch.as_tensor(x)
    if x.shape[-1] != 8:
        raise ValueError(f"Expected 8-dim vectors, got {x.shape[-1]}")
    dev = cuda_device(x)
    xb = x.reshape(-1, 8).to(device=dev, dtype=torch.float32).contiguous()
    return xb, x.device, x.shape, x.dtype


def back(t: torch.Tensor, device) -> torch.Tensor:
    return t if t.device == torch.device(device) else t.to(device)


def np_to_dev(a, dtype, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(np.asarray(a), dtype=dtype)).to(device)
