"""The E8 quantiser's Gaussian check, after the reference's
sanity_check_gaussian (core/e8_quantizer.py:163-248): 1,000,000 i.i.d.
N(0, 1) 8-vectors (torch seed 42), quantize_e8 at the scale of
compute_scale(1, b), MSE against the theory G(E8) * 2*pi*e * 4^-b and the gap
MSE / 4^-b against 2*pi*e*G(E8) = 1.2246.

The reference prints these and asserts nothing.  Here the lattice points are
checked bit for bit against the oracle's encode_e8 on the same inputs, and
the gap must stay within 1% of 1.2246 (the oracle measures 1.2241-1.2244 at
b = 2..5, a ratio of 0.9996-0.9998 to the theory MSE).
"""
import numpy as np
import pytest
import torch

from oracle import lq_oracle as O

pytestmark = pytest.mark.gpu

N = 1_000_000


@pytest.mark.parametrize("bits", [2.0, 3.0, 4.0, 5.0])
def test_gaussian_mse_gap(bits):
    from latticequant_b200.core.e8_quantizer import G_E8, compute_scale, quantize_e8, theoretical_mse

    x = torch.randn(N, 8, generator=torch.Generator().manual_seed(42))
    scale = compute_scale(1.0, bits)
    xhat = quantize_e8(x.cuda(), scale).cpu()
    s32 = np.float32(scale)
    want = O.encode_e8((x.numpy() / s32).astype(np.float32)) * s32
    assert np.array_equal(xhat.numpy().view(np.uint32), want.view(np.uint32))
    mse = float(((x.double() - xhat.double()) ** 2).mean())
    gap = mse / 4.0 ** -bits
    theory_gap = 2 * np.pi * np.e * G_E8
    assert abs(gap / theory_gap - 1.0) < 0.01, (gap, theory_gap)
    assert abs(mse / theoretical_mse(1.0, bits) - 1.0) < 0.01
