"""The two-term fp16 operand scheme of the tensor-core prefill (projection
GEMMs and causal attention), restated in numpy with IEEE fp16 rounding, and
checked against the bounds the kernels rely on.

* A row (an activation row, a weight row, a Q row, a K row, or a V column
  within one tile) is scaled by 2^-e so that its maximum lies in
  [2^14, 2^15), with e read from the maximum's exponent and clamped to
  [-120, 120]. It is split into hi = fp16(x) and lo = fp16(x - hi). Every
  element then comes back to within 2^-22 of the row maximum.
* Probabilities p in [0, 1] (the attention's P operand) are split unscaled.
  Each comes back to within 2^-22 p + 2^-25 (the fp16 subnormal step).
* The MMAs sum hi.hi + hi.lo + lo.hi, each product exact in fp32, and drop
  lo.lo. A dot product of n such terms is then within 3 * 2^-22 * n * max|a| * max|b|
  of the exact one.

These are properties of the arithmetic, restated here. The kernels' own
results are compared with the reference on the GPU (tests/test_prefill_gpu.py,
tests/test_gemm_gpu.py).
"""
import numpy as np
import pytest


def pow2_ex(mx):
    """e with mx 2^-e in [2^14, 2^15); 0 for mx == 0; clamped to [-120, 120]."""
    if mx <= 0.0:
        return 0
    _, fe = np.frexp(np.float32(mx))  # mx in [2^(fe-1), 2^fe)
    return int(min(max(int(fe) - 15, -120), 120))


def split(x):
    """x (float32) -> fp16 hi, lo with x = hi + lo + r."""
    x = np.asarray(x, dtype=np.float32)
    hi = x.astype(np.float16)
    lo = (x - hi.astype(np.float32)).astype(np.float16)
    return hi, lo


def split_row(row):
    e = pow2_ex(float(np.abs(row).max()))
    scaled = (row.astype(np.float32) * np.float32(2.0 ** -e)).astype(np.float32)
    hi, lo = split(scaled)
    return hi, lo, e


def rows(rng):
    """Rows over wide magnitudes, a zero row and wide dynamic ranges within a row."""
    out = [rng.standard_normal(64).astype(np.float32) * np.float32(10.0 ** k)
           for k in range(-8, 9)]
    out.append(np.zeros(64, np.float32))
    r = rng.standard_normal(64).astype(np.float32) * np.float32(1e-6)
    r[5] = 3.0e2
    out.append(r)
    r = rng.standard_normal(4864).astype(np.float32)
    r[::97] *= np.float32(1e5)
    out.append(r)
    return out


def test_scaled_rows_reconstruct_within_2e_minus_22_of_the_maximum():
    rng = np.random.default_rng(7)
    for row in rows(rng):
        hi, lo, e = split_row(row)
        mx = float(np.abs(row).max())
        if mx > 0:
            scaled_max = mx * 2.0 ** -e
            assert 2.0 ** 14 <= scaled_max < 2.0 ** 15
        back = (hi.astype(np.float64) + lo.astype(np.float64)) * 2.0 ** e
        err = float(np.abs(back - row.astype(np.float64)).max())
        assert err <= 2.0 ** -22 * mx, (err, mx)


def test_unscaled_probabilities_reconstruct():
    rng = np.random.default_rng(11)
    # the softmax's exp2 of non-positive arguments: [0, 1], down to underflow
    p = np.exp2(-rng.uniform(0.0, 40.0, 200000)).astype(np.float32)
    p = np.concatenate([p, np.float32([0.0, 1.0, 2.0 ** -14, 2.0 ** -24, 3.0e-8])])
    hi, lo = split(p)
    back = hi.astype(np.float64) + lo.astype(np.float64)
    err = np.abs(back - p.astype(np.float64))
    assert np.all(err <= 2.0 ** -22 * p.astype(np.float64) + 2.0 ** -25)


@pytest.mark.parametrize("n", [64, 896, 4864])
def test_three_product_dot_within_bound(n):
    rng = np.random.default_rng(n)
    for trial in range(50):
        a = rng.standard_normal(n).astype(np.float32) * np.float32(10.0 ** rng.uniform(-4, 4))
        b = rng.standard_normal(n).astype(np.float32) * np.float32(10.0 ** rng.uniform(-4, 4))
        if trial % 5 == 0:  # a few large entries, as in real activations
            a[rng.integers(0, n, 3)] *= np.float32(300.0)
        ahi, alo, ea = split_row(a)
        bhi, blo, eb = split_row(b)
        f = lambda v: v.astype(np.float64)
        # every fp16 x fp16 product is exact in fp32 (22 significant bits)
        prods = f(ahi) * f(bhi) + f(ahi) * f(blo) + f(alo) * f(bhi)
        got = float(prods.sum()) * 2.0 ** (ea + eb)
        exact = float(np.dot(f(a), f(b)))
        bound = 3 * 2.0 ** -22 * n * float(np.abs(a).max()) * float(np.abs(b).max())
        assert abs(got - exact) <= bound, (n, trial, got, exact, bound)


def test_fp16_products_are_exact_in_fp32():
    rng = np.random.default_rng(3)
    x = rng.standard_normal(100000).astype(np.float16)
    y = rng.standard_normal(100000).astype(np.float16)
    p32 = x.astype(np.float32) * y.astype(np.float32)
    p64 = x.astype(np.float64) * y.astype(np.float64)
    assert np.array_equal(p32.astype(np.float64), p64)
