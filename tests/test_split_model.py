"""CPU model of the fp32-class l2sq dot: each cloud scaled by one power of two so its
largest |x| lies in [2^14, 2^15), hi = fp16(x 2^e), lo = fp16(x 2^e - hi), and the dot
accumulated from hi*hi + hi*lo + lo*hi (exact products) rescaled by 2^-(e_x + e_y).

Checks the per-product bound the GPU parity tests use (3 2^-22 |x_k y_k|, inside their
2^-19), that a power-of-two rescaling of a cloud leaves the split unchanged, and where
the model stops holding (fp16 subnormals for tiny clouds)."""
import numpy as np
import pytest


def cloud_exponent(x):
    m = float(np.max(np.abs(x))) if x.size else 0.0
    if m == 0.0:
        return 0
    _, ex = np.frexp(np.float32(m))
    return int(max(-60, min(60, 15 - int(ex))))


def halves(x):
    e = cloud_exponent(x)
    s = np.ldexp(x.astype(np.float32), e).astype(np.float32)
    hi = s.astype(np.float16)
    lo = (s - hi.astype(np.float32)).astype(np.float16)
    return hi.astype(np.float64), lo.astype(np.float64), e


def split_products(x, y):
    """Per-element products of the model (exact in fp64: 11-bit x 11-bit mantissas)."""
    hx, lx, ex = halves(x)
    hy, ly, ey = halves(y)
    return (hx * hy + hx * ly + lx * hy) * 2.0 ** -(ex + ey)


@pytest.mark.parametrize("scale", [1.0, 2.0 ** -30, 2.0 ** 40, 1e-3, 7e5])
def test_product_error_within_bound(scale):
    rng = np.random.default_rng(5)
    x = (rng.normal(size=(200, 64)) * scale).astype(np.float32)
    y = (rng.standard_cauchy(size=(200, 64)) * scale).astype(np.float32)  # heavy tails: wide exponent range
    exact = x.astype(np.float64) * y.astype(np.float64)
    err = np.abs(split_products(x, y) - exact)
    bound = 3 * 2.0 ** -22 * np.abs(exact)
    # elements far below the cloud's largest one lose low bits to fp16 subnormals: an
    # absolute floor of 2^-38 max|x| per operand element
    floor = 2.0 ** -38 * (np.abs(x).max() * np.abs(y.astype(np.float64)) + np.abs(y).max() * np.abs(x.astype(np.float64)))
    assert np.all(err <= bound + floor)
    assert np.all(bound + floor <= 2.0 ** -19 * np.abs(exact) + floor)


def test_power_of_two_rescale_keeps_the_split():
    rng = np.random.default_rng(6)
    x = rng.normal(size=(50, 33)).astype(np.float32)
    hx, lx, ex = halves(x)
    for k in (-20, -3, 5, 30):
        h2, l2, e2 = halves(np.ldexp(x, k).astype(np.float32))
        assert e2 == ex - k
        assert np.array_equal(h2, hx) and np.array_equal(l2, lx)


def test_scaled_cloud_max_fits_fp16():
    rng = np.random.default_rng(7)
    for scale in (1e-12, 1e-3, 1.0, 3e4, 1e15):
        x = (rng.normal(size=(64, 16)) * scale).astype(np.float32)
        e = cloud_exponent(x)
        top = np.abs(np.ldexp(x, e)).max()
        assert 2.0 ** 14 <= top < 2.0 ** 15
