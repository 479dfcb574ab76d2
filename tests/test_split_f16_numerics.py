"""The split-f16 operand scheme, restated in numpy and checked without a
GPU: the accuracy argument behind ET_B200_PRECISION_F16X3.

An operand tensor x gets one power-of-two exponent e from its max |x| (the
rule scale_from_amax_kernel applies: max = f 2^k, f in [0.5, 1), e = 10 - k),
and is stored as binary16 hi = rn16(x 2^e), lo = rn16(x 2^e - hi).  The GEMM
accumulates hi.hi + hi.lo + lo.hi and scales by 2^-(e_A + e_B).  These tests
pin (1) the representation error of the pair, (2) the normwise error of the
three-product contraction against float64, at the same 1e-5 bar the GPU
linear tests use, and (3) that an operand far outside binary16's range is
brought into it by its exponent.
"""
import numpy as np
import pytest

TARGET = 10  # the library's default scale target


def exponent(x: np.ndarray) -> int:
    amax = float(np.abs(x).max())
    if not np.isfinite(amax) or amax == 0.0:
        return 0
    _, k = np.frexp(np.float32(amax))
    return int(np.clip(TARGET - k, -60, 60))


def split16(x: np.ndarray, e: int):
    xs = (x.astype(np.float32) * np.float32(2.0 ** e)).astype(np.float32)
    hi = xs.astype(np.float16)
    lo = (xs - hi.astype(np.float32)).astype(np.float16)
    return hi, lo


def contract(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """C = A B^T through split-f16 pairs: exact products, float64 sums."""
    ea, eb = exponent(a), exponent(b)
    ah, al = (t.astype(np.float64) for t in split16(a, ea))
    bh, bl = (t.astype(np.float64) for t in split16(b, eb))
    c = ah @ bh.T + ah @ bl.T + al @ bh.T
    return c * 2.0 ** (-(ea + eb))


@pytest.mark.parametrize("scale", [1e-7, 1e-3, 1.0, 3e2, 1e4])
def test_pair_keeps_22_bits_in_the_window(scale):
    rng = np.random.default_rng(7)
    x = (rng.standard_normal(1 << 16) * scale).astype(np.float32)
    e = exponent(x)
    hi, lo = split16(x, e)
    assert np.isfinite(hi).all() and np.isfinite(lo).all()
    back = (hi.astype(np.float64) + lo.astype(np.float64)) * 2.0 ** (-e)
    err = np.abs(back - x.astype(np.float64))
    # elements whose lo stays a normal binary16 (|x 2^e| >= 2^-3): 22 bits
    window = np.abs(x.astype(np.float64) * 2.0 ** e) >= 2.0 ** -3
    assert window.mean() > 0.99
    assert (err[window] <= 2.0 ** -21 * np.abs(x[window])).all()
    # below the window the error is absolute: half a binary16 subnormal step
    assert (err <= 2.0 ** -21 * np.abs(x) + 2.0 ** -25 * 2.0 ** (-e)).all()


@pytest.mark.parametrize("sa,sb", [(1.0, 0.05), (1e4, 1e-3), (1e-5, 30.0), (2e-7, 1e3)])
def test_three_product_contraction_meets_the_linear_bar(sa, sb):
    rng = np.random.default_rng(11)
    a = (rng.standard_normal((96, 512)) * sa).astype(np.float32)
    b = (rng.standard_normal((64, 512)) * sb).astype(np.float32)
    ref = a.astype(np.float64) @ b.astype(np.float64).T
    got = contract(a, b)
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err <= 1e-5, err
    # and well inside it: the scheme's own error is ~2^-21 relative per product
    assert err <= 1e-6, err


def test_exponent_puts_the_max_below_the_overflow():
    # (exponents are clamped to [-60, 60], which covers maxima from ~1e-15 to
    # ~1e21; the 2^-(e_A + e_B) rescale then stays a normal f32 power of two)
    for amax in (1e-14, 3.1e-8, 0.5, 1.0, 65504.0 * 7, 1e15):
        x = np.array([amax, -amax / 3], np.float32)
        e = exponent(x)
        top = abs(float(x[0]) * 2.0 ** e)
        assert 2.0 ** (TARGET - 1) <= top < 2.0 ** TARGET
        assert top * 64 <= 65504 * 1.01  # 64x headroom to binary16's largest finite
