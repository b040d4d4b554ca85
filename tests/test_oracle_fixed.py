"""The oracle's fixed-point float64 sum against the known answers of eagle's own
fixed-point tests (tests/test_CanonicalReduce.cu:172-211): exact on the cancellation
ladder and on the kappa fixture, IEEE on specials, and the rule that picks it
(canonical.h:304-313, test_CanonicalReduce.cu:213-217)."""

import numpy as np
import pytest


def same(a, b) -> bool:
    return np.float64(a).tobytes() == np.float64(b).tobytes()


@pytest.mark.parametrize("n", (163840, 655360 + 3))
def test_exact_on_the_base_ladder(orc, n):
    x, units = orc.ladder(n, 30, 0)
    assert same(orc.reduce_fixed(x)[0], np.ldexp(float(units), -10))


@pytest.mark.parametrize("g", (0, 10, 20, 30, 40))
def test_exact_on_the_kappa_ladder(orc, g):
    x, units = orc.ladder(655360, 0, g)
    assert same(orc.reduce_fixed(x)[0], np.ldexp(float(units), -10))


@pytest.mark.parametrize("n", (257, 2048 * 3 + 1, 1000000))
@pytest.mark.parametrize("kappa", (1.0, 1024.0, 1048576.0))
def test_exact_on_the_fixture(orc, n, kappa):
    x, exact, _ = orc.fixture(n, kappa)
    assert same(orc.reduce_fixed(x)[0], exact)


def test_ieee_specials(orc):
    inf = np.inf
    x = orc.corpus(9001, 5)
    x[1000] = inf
    assert orc.reduce_fixed(x)[0] == inf
    x[7000] = -inf
    assert np.isnan(orc.reduce_fixed(x)[0])
    x[7000] = 1.0
    x[3] = np.nan
    assert np.isnan(orc.reduce_fixed(x)[0])
    # signed zero is not kept; subnormals round once; overflow is +inf
    assert same(orc.reduce_fixed(np.array([-0.0, -0.0]))[0], 0.0)
    tiny = np.finfo(np.float64).smallest_subnormal
    assert same(orc.reduce_fixed(np.array([tiny, 3 * tiny, -tiny]))[0], 3 * tiny)
    big = np.finfo(np.float64).max
    assert orc.reduce_fixed(np.array([big, big]))[0] == inf
    assert same(orc.reduce_fixed(np.array([big, big, -big]))[0], big)


def test_the_unit_truncates_below_2_to_the_106(orc):
    """A term more than 2^106 below the largest is cut at the unit: the
    fixed-point sum of (2^200, 1, -2^200) is 0, where the (hi, comp) tree keeps 1.
    The device tests use it to tell the two leaves apart."""
    x = np.array([2.0 ** 200, 1.0, -(2.0 ** 200)])
    assert same(orc.reduce_fixed(x)[0], 0.0)
    assert orc.reduce(x)[0] == 1.0


def test_columns_and_companion(orc):
    rows, cols = 10007, 3
    x = orc.corpus(rows * cols, 11)
    c = orc.corpus(rows * cols, 12) * 1e-17
    got = orc.reduce_fixed(x, columns=cols, comp=c)
    for j in range(cols):
        assert same(got[j], orc.reduce_fixed(x.reshape(rows, cols)[:, j].copy(), comp=c.reshape(rows, cols)[:, j].copy())[0])


def test_rule_from_ratio(orc):
    assert orc.fixed_leaf(32) and orc.fixed_leaf(64) and orc.fixed_leaf(8)
    assert not orc.fixed_leaf(2) and not orc.fixed_leaf(1)


def test_oracle_value_is_the_correctly_rounded_exact_sum(orc):
    """The oracle's fixed-point sum rounds an exactly held sum as math.fsum does
    (ties to even, a sticky bit past a tie, subnormal results, overflow to inf)."""
    import math
    from fractions import Fraction

    from test_gpu_reduce_fixed import _exact_cases

    for x in _exact_cases():
        a = np.array(x, dtype=np.float64)
        try:
            want = np.float64(math.fsum(a))
        except OverflowError:
            want = np.float64(np.inf if sum(Fraction(v) for v in a) > 0 else -np.inf)
        assert orc.reduce_fixed(a).tobytes() == want.tobytes(), x[:4]
