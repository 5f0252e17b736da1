"""The exact hash-bin sums of the float64 pipeline, restated on the CPU.

exact_bins_add / exact_bins_value in cresso_b200/csrc/spectral64.cu split a
value v (|v| < 2^66) into three integer limbs of round(|v| 2^60) (42 bits
each, negated for negative v) and add them with 64-bit integer atomics.  This
restates those IEEE operations with numpy float64 / int64 and checks the
properties the kernels rely on: the split is exact apart from the one
rounding of |v| 2^60, integer limb sums do not depend on the order of the
additions, and the result is within that rounding of the exact sum.  (The
kernels themselves are checked on the GPU: test_run_to_run_deterministic
and the float64 golden cases.)
"""

from fractions import Fraction

import numpy as np


def to_limbs(v: float):
    a = abs(v)
    sc = np.float64(a) * np.float64(2.0 ** 60)
    h = np.floor(sc * np.float64(2.0 ** -84))
    r1 = sc - h * np.float64(2.0 ** 84)
    m = np.floor(r1 * np.float64(2.0 ** -42))
    r0 = r1 - m * np.float64(2.0 ** 42)
    hi, mid, lo = int(h), int(m), int(np.rint(r0))
    if v < 0:
        hi, mid, lo = -hi, -mid, -lo
    return hi, mid, lo


def from_limbs(hi: int, mid: int, lo: int) -> float:
    return float(np.float64(hi) * 2.0 ** 24 + np.float64(mid) * 2.0 ** -18 + np.float64(lo) * 2.0 ** -60)


def sample(rng, n):
    mag = 10.0 ** rng.uniform(-12, 19, n)  # up to 1e19 < 2^66
    return mag * rng.choice([-1.0, 1.0], n)


def test_split_is_exact_up_to_the_grid_rounding():
    rng = np.random.default_rng(0)
    for v in sample(rng, 4000):
        hi, mid, lo = to_limbs(float(v))
        assert 0 <= abs(mid) < 2 ** 42 and 0 <= abs(lo) <= 2 ** 42 and abs(hi) < 2 ** 42
        s = Fraction(hi) * 2 ** 84 + Fraction(mid) * 2 ** 42 + Fraction(lo)  # the integer round(|v| 2^60), signed
        exact = Fraction(float(v)) * 2 ** 60
        assert abs(s - exact) <= Fraction(1, 2)


def test_limb_sums_do_not_depend_on_the_order():
    rng = np.random.default_rng(1)
    v = sample(rng, 3000)
    v[::97] = rng.uniform(-2.0, 2.0, v[::97].size)  # mixed magnitudes and signs in one bin
    totals = set()
    for perm in range(5):
        order = rng.permutation(v.size) if perm else np.arange(v.size)
        acc = [0, 0, 0]
        for x in v[order]:
            for k, limb in enumerate(to_limbs(float(x))):
                acc[k] += limb  # the kernels' int64 atomics wrap like this sum (no overflow here)
        totals.add(from_limbs(*acc))
    assert len(totals) == 1


def test_sum_within_the_grid_rounding_of_the_exact_sum():
    rng = np.random.default_rng(2)
    v = rng.uniform(0.0, 3.0, 5000)  # the density rel^p of one bin
    acc = [0, 0, 0]
    for x in v:
        for k, limb in enumerate(to_limbs(float(x))):
            acc[k] += limb
    got = Fraction(from_limbs(*acc))
    exact = sum(Fraction(float(x)) for x in v)
    # n roundings of 2^-61 each, and one rounding of the float64 result
    assert abs(got - exact) <= Fraction(v.size, 2 ** 61) + abs(exact) * Fraction(1, 2 ** 52)
