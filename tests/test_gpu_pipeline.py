"""core/pipeline.py (RHT, fast Hadamard, LatticeQuantEncoder) against
fixtures made by running the reference (tests/golden/rht.npz), and the
entropy_storage API round trips on this package's rANS."""
import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu


def _eq(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def test_fast_hadamard_bit_exact():
    from latticequant_b200.core import pipeline as P

    g = golden("rht.npz")
    for d in (8, 64, 128, 256):
        y = P.fast_hadamard_transform(torch.from_numpy(g[f"fwht_x_d{d}"]).cuda())
        assert _eq(y.cpu().numpy(), g[f"fwht_y_d{d}"]), d


def test_rht_forward_inverse_bit_exact():
    from latticequant_b200.core import pipeline as P

    g = golden("rht.npz")
    r = P.RHT(128, seed=0)
    v = torch.from_numpy(g["rht_v"]).cuda()
    w = r.forward(v)
    assert _eq(w.cpu().numpy(), g["rht_w"])
    assert _eq(r.inverse(w).cpu().numpy(), g["rht_inv"])


@pytest.mark.parametrize("bits", [3, 4, 5])
def test_lattice_quant_encoder_matches_reference(bits):
    from latticequant_b200.core import pipeline as P

    g = golden("rht.npz")
    enc = P.LatticeQuantEncoder(128, bits, rht_seed=0)
    e = enc.encode(torch.from_numpy(g[f"enc{bits}_v"]).cuda())
    assert np.float32(e["sigma2"]) == np.float32(g[f"enc{bits}_sigma2"])
    assert e["scale"] == g[f"enc{bits}_scale"]
    for key in ("w", "w_hat", "v_hat"):
        assert _eq(e[key].cpu().numpy(), g[f"enc{bits}_{key}"]), key
    for key in ("coset", "free_coords", "coord8_half"):
        assert np.array_equal(e[key].cpu().numpy(), g[f"enc{bits}_{key}"]), key
    r = enc.measure_rate(e)
    assert abs(r["ans_test_bpd"] - r["ideal_test_bpd"]) < 0.1 * r["ideal_test_bpd"]


def test_entropy_storage_round_trip_and_rate():
    from latticequant_b200.core import entropy_storage as ES
    from latticequant_b200.core.e8_quantizer import compute_scale, encode_e8
    from latticequant_b200.core.entropy_coder import (FrequencyModel, e8_to_symbols,
                                                      measure_ideal_code_length)

    torch.manual_seed(0)
    for bits in (3, 4, 5):
        x = torch.randn(20000, 8, device="cuda")
        scale = compute_scale(1.0, bits)
        q = encode_e8(x / scale)
        c = ES.compress_e8(q, bits, scale)
        q2 = ES.decompress_e8(c, "cuda")
        assert torch.equal(q, q2)  # lossless (core/entropy_storage.py:369-405)
        xr = ES.decompress_dequantize(c, "cuda")
        assert torch.equal(xr, q2 * scale)
        # rate against the ideal Laplace-smoothed code length (core/entropy_storage.py:448-477)
        cos, free, c8h = [t.cpu().numpy() for t in e8_to_symbols(q)]
        m = FrequencyModel()
        m.fit(cos, free, c8h)
        ideal = measure_ideal_code_length(m, cos, free, c8h)["bits_per_dim"]
        real = c.compressed_bits / (8 * q.shape[0])
        assert real < ideal * 1.05 + 0.02, (bits, real, ideal)
        assert c.total_bytes > c.compressed_bytes and "CompressedE8Tensor" in c.summary()
    # no out-of-range: large lattice points still round-trip (core/entropy_storage.py:408-445)
    big = encode_e8(torch.randn(4000, 8, device="cuda") * 40)
    cb = ES.compress_e8(big, 5, 1.0)
    assert torch.equal(ES.decompress_e8(cb, "cuda"), big)
    # quantize_compress / decompress_dequantize (core/entropy_storage.py:330-362)
    x = torch.randn(5000, 8, device="cuda")
    cq = ES.quantize_compress(x, 4, 1.0)
    xr = ES.decompress_dequantize(cq, "cuda")
    assert torch.equal(xr, encode_e8(x / compute_scale(1.0, 4)) * cq.scales[0].item())
