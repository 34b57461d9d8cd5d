"""Device helpers that stand in for library routines must agree with them bit for bit.

* the quantiser divides x by the head scale with a reciprocal and one FMA
  correction (Markstein); it must equal IEEE division (torch's CUDA `/`)
* block -> head / tile indices use a multiply-shift division by invariant
  integers; it must equal integer division
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LQ_SELFTEST_DIV, LQ_SELFTEST_FASTDIV = 1, 2


def _div(a, b):
    from latticequant_b200 import _lib

    out = torch.empty_like(a)
    _lib.check(_lib.lib().lq_selftest(LQ_SELFTEST_DIV, _lib.ptr(a), _lib.ptr(b), a.numel(), 0, _lib.ptr(out),
                                      _lib.stream_handle()), "selftest div")
    return out


def test_scale_division_equals_ieee():
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    n = 1 << 25
    for trial in range(6):
        if trial == 0:    # bf16 K/V values over a wide dynamic range
            a = (torch.randn(n, device="cuda", generator=g) * torch.exp(2 * torch.randn(n, device="cuda", generator=g)))
            a = a.to(torch.bfloat16).float()
        elif trial == 1:  # arbitrary fp32 mantissas, exponents in [-60, 60]
            m = torch.rand(n, device="cuda", generator=g) + 1.0
            e = torch.randint(-60, 61, (n,), device="cuda", generator=g).float()
            a = m * torch.exp2(e) * torch.where(torch.rand(n, device="cuda", generator=g) < 0.5, -1.0, 1.0)
        elif trial == 2:  # exact multiples of the scale
            b0 = torch.rand(n, device="cuda", generator=g) + 0.1
            a = torch.randint(-600, 600, (n,), device="cuda", generator=g).float() * b0
        elif trial == 3:  # signed zeros, tiny and huge values
            a = torch.tensor([0.0, -0.0, 1e-30, -1e-30, 1e30, -1e30, 1e-45, 3e38] * (n // 8), device="cuda")
        elif trial == 4:  # fp16 values
            a = torch.randn(n, device="cuda", generator=g).half().float() * 30
        else:             # values near rounding boundaries of x / scale
            a = (torch.randint(-50, 50, (n,), device="cuda", generator=g).float() + 0.5)
        if trial == 2:
            b = b0
        elif trial == 5:
            b = torch.exp2(torch.randint(-8, 8, (n,), device="cuda", generator=g).float())  # powers of two
        else:
            b = torch.exp(torch.randn(n, device="cuda", generator=g) * 3)
        want = a / b
        got = _div(a.contiguous(), b.contiguous())
        bad = (got.view(torch.int32) != want.view(torch.int32)) & ~(torch.isnan(got) & torch.isnan(want))
        assert int(bad.sum().item()) == 0, (trial, a[bad][:4].tolist(), b[bad][:4].tolist())


@pytest.mark.parametrize("d", [1, 2, 3, 7, 16, 17, 1000, 131072, 1048575, 1 << 30, (1 << 31) - 1])
def test_fast_integer_division(d):
    from latticequant_b200 import _lib

    g = torch.Generator(device="cuda")
    g.manual_seed(d)
    num = torch.randint(0, 1 << 31, (1 << 22,), device="cuda", generator=g, dtype=torch.int64)
    num[:8] = torch.tensor([0, 1, d - 1, d, d + 1, (1 << 31) - 1, 2 * d - 1, 2 * d], device="cuda").clamp(0, (1 << 31) - 1)
    n32 = num.to(torch.int32)
    out = torch.empty_like(n32)
    _lib.check(_lib.lib().lq_selftest(LQ_SELFTEST_FASTDIV, _lib.ptr(n32), None, n32.numel(), d, _lib.ptr(out),
                                      _lib.stream_handle()), "selftest fastdiv")
    assert torch.equal(out.to(torch.int64), num // d)
