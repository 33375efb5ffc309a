"""Quantize-on-append kernel vs the oracle rule: codes, scales, biases bit-exact.

Covers both cache dtypes, 4- and 8-bit codes, group sizes 32/64/128 and the
edge cases the affine rule has (constant groups, zero groups, |min| == |max|
ties, key-outlier channels, values near the rounding midpoints).
"""
import numpy as np
import pytest

from helpers import BF16, F16, from_torch, gen, to_torch_bits
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def edge_rows(rng, D):
    rows = [gen(rng, (64, D)), gen(rng, (16, D), outlier_channels=4)]
    rows.append(np.full((2, D), 0.3, np.float32))           # constant groups
    rows.append(np.zeros((2, D), np.float32))               # zero groups
    t = rng.standard_normal((4, D)).astype(np.float32)
    t[:, 0], t[:, 1] = 2.0, -2.0                             # |min| == |max| ties
    rows.append(t)
    rows.append((rng.integers(-64, 64, (8, D)) / 8.0).astype(np.float32))  # exact grid values
    rows.append(gen(rng, (8, D)) * 1e-3)
    rows.append(gen(rng, (8, D)) * 300.0)
    return np.concatenate(rows)


@pytest.mark.parametrize("dt", [F16, BF16])
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
def test_quantize_bit_exact(dt, bits, gs):
    import kvq
    rng = np.random.default_rng(7 + bits + gs)
    D = 256
    x = O.to_dtype_bits(edge_rows(rng, D), dt)
    want = O.quantize(x, gs, bits, dt)
    p, s, b = kvq.quantize(to_torch_bits(x, dt), gs, bits)
    np.testing.assert_array_equal(p.cpu().numpy().view(np.uint32), want[0])
    np.testing.assert_array_equal(from_torch(s, dt), want[1])
    np.testing.assert_array_equal(from_torch(b, dt), want[2])


def test_quantize_empty_and_unaligned():
    import kvq
    import torch
    rng = np.random.default_rng(3)
    x = O.to_dtype_bits(gen(rng, (5, 65 * 64)), F16)[:, 64:]  # rows 64 elements into a buffer
    t = to_torch_bits(np.ascontiguousarray(x), F16)
    p, s, b = kvq.quantize(t, 64, 4)
    want = O.quantize(np.ascontiguousarray(x), 64, 4, F16)
    np.testing.assert_array_equal(p.cpu().numpy().view(np.uint32), want[0])
    e = torch.empty(0, 128, dtype=torch.float16, device="cuda")
    p, s, b = kvq.quantize(e, 64, 8)
    assert p.shape == (0, 32)
