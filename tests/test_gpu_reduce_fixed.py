"""The fixed-point float64 leaf on the device (``eagle_backend_x_b200_reduce_fixed``)
against the oracle's restatement of eagle's FixedPartial, bit for bit: the sizes of
eagle's reduction tests, the cancellation ladder and the kappa fixture (exact sums),
IEEE specials, columns with a companion plane, repeated launches
(tests/test_CanonicalReduce.cu:121-211)."""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SIZES = (1, 2, 3, 255, 256, 257, 4095, 4096, 4097, 8193, 12345, 65536, 65537, 100003, (1 << 20) + 37)


def fixed(eb, x, **kw):
    return eb.reduce(torch.from_numpy(np.ascontiguousarray(x)).cuda(), fixed=True, **kw).cpu().numpy()


@pytest.mark.parametrize("n", SIZES)
def test_device_equals_oracle_on_the_corpus(eb, orc, n):
    x = orc.corpus(n, 4242 + n)
    assert fixed(eb, x).tobytes() == orc.reduce_fixed(x).tobytes(), n


def test_exact_on_the_ladders_and_the_fixture(eb, orc):
    for n, er, g in ((163840, 30, 0), (655363, 30, 0), (655360, 0, 0), (655360, 0, 20), (655360, 0, 40)):
        x, units = orc.ladder(n, er, g)
        assert fixed(eb, x)[0] == np.ldexp(float(units), -10), (n, er, g)
    for n in (257, 2048 * 3 + 1, 1000000):
        for kappa in (1.0, 1024.0, 1048576.0):
            x, exact, _ = orc.fixture(n, kappa)
            got = fixed(eb, x)
            assert got.tobytes() == np.float64(exact).tobytes(), (n, kappa)


def test_ieee_specials(eb, orc):
    x = orc.corpus(9001, 5)
    x[1000] = np.inf
    assert fixed(eb, x)[0] == np.inf
    x[7000] = -np.inf
    assert np.isnan(fixed(eb, x)[0])
    x[7000] = 1.0
    x[3] = np.nan
    assert np.isnan(fixed(eb, x)[0])
    assert fixed(eb, np.array([-0.0, -0.0])).tobytes() == np.float64(0.0).tobytes()
    tiny = np.finfo(np.float64).smallest_subnormal
    assert fixed(eb, np.array([tiny, 3 * tiny, -tiny]))[0] == 3 * tiny
    big = np.finfo(np.float64).max
    assert fixed(eb, np.array([big, big]))[0] == np.inf
    assert fixed(eb, np.array([big, big, -big]))[0] == big


def test_the_two_leaves_differ_where_they_should(eb, orc):
    """(2^200, 1, -2^200): the fixed-point unit cuts the 1 (sum 0); the (hi, comp)
    leaf keeps it -- and a B200 (FP32:FP64 = 2) takes the (hi, comp) leaf by itself."""
    x = np.array([2.0 ** 200, 1.0, -(2.0 ** 200)])
    assert fixed(eb, x).tobytes() == orc.reduce_fixed(x).tobytes() == np.float64(0.0).tobytes()
    plain = eb.reduce(torch.from_numpy(x).cuda()).cpu().numpy()
    assert plain.tobytes() == orc.reduce(x).tobytes() and plain[0] == 1.0


@pytest.mark.parametrize("rows,cols", ((4097, 3), (100003, 2), (17, 65)))
def test_columns_with_a_companion(eb, orc, rows, cols):
    x = orc.corpus(rows * cols, 31).reshape(rows, cols)
    c = orc.corpus(rows * cols, 32).reshape(rows, cols) * 1e-17
    got = eb.reduce(torch.from_numpy(x).cuda(), fixed=True, comp=torch.from_numpy(c).cuda()).cpu().numpy()
    assert got.tobytes() == orc.reduce_fixed(x, columns=cols, comp=c).tobytes()


def test_repeated_launches_agree(eb, orc):
    x = orc.corpus(1 << 20, 77)
    r = eb.Reducer(torch.from_numpy(x).cuda(), fixed=True)
    first = r().cpu().numpy().copy()
    for _ in range(3):
        assert r().cpu().numpy().tobytes() == first.tobytes()
    assert first.tobytes() == orc.reduce_fixed(x).tobytes()


def test_refusals(eb):
    from eagle_b200 import _abi

    with pytest.raises(ValueError):
        eb.reduce(torch.ones(10, dtype=torch.float32, device="cuda"), fixed=True)
    with pytest.raises(ValueError):
        eb.reduce(torch.ones(10, dtype=torch.float64, device="cuda"), fixed=True, pair_out=True)
    d = _abi.new(_abi.ReduceDesc, dtype=_abi.REDUCE_F64, op=_abi.REDUCE_OP_SUM, device=0, n=10, columns=1,
                 flags=_abi.REDUCE_PAIR_OUT)
    with pytest.raises(eb.BackendUnsupported):
        _abi.check(_abi.lib().eagle_backend_x_b200_reduce_fixed(ctypes.byref(d)))
    d.flags = 0
    d.op = _abi.REDUCE_OP_MAX
    with pytest.raises(ValueError):
        _abi.check(_abi.lib().eagle_backend_x_b200_reduce_fixed(ctypes.byref(d)))


def _exact_cases():
    """Sums the fixed-point partial holds exactly (terms within 2^40 of each other,
    at most 4096 of them, so no unit lift or halving drops a bit): its rounded value
    must then be the correctly rounded exact sum, which math.fsum gives. Ties to even,
    a sticky bit past a tie, cancellation down to subnormals."""
    e = np.ldexp
    cases = [
        [1.0, e(1.0, -53)],                       # exactly half an ulp above 1: ties to 1
        [1.0, e(3.0, -53)],                       # 1.5 ulp: ties up to the even 1 + 2 ulp
        [1.0 + e(1.0, -52), e(1.0, -53)],         # odd significand: the tie goes up
        [1.0, e(1.0, -53), e(1.0, -100)],         # a sticky bit past the tie: up
        [1.0, -e(1.0, -53), -e(1.0, -100)],       # below 1: the other side
        [e(1.0, -1022), -e(1.0, -1074)],          # a subnormal result
        [e(3.0, -1074), e(5.0, -1074), -e(1.0, -1073)],
        [-e(1.0, 600), e(1.0, 600), e(1.0, 550)],
        [np.finfo(np.float64).max, e(1.0, 970)],  # exactly half an ulp above max: ties to even (max is odd)
    ]
    rng = np.random.default_rng(99)
    for n in (3, 100, 4096):
        for scale in (0, 300, -900):
            x = rng.uniform(-1, 1, n) * np.ldexp(1.0, rng.integers(-20, 21, n) + scale)
            cases.append(list(x))
    return cases


def test_value_is_the_correctly_rounded_exact_sum(eb, orc):
    import math

    from fractions import Fraction

    for x in _exact_cases():
        a = np.array(x, dtype=np.float64)
        try:
            want = np.float64(math.fsum(a))
        except OverflowError:  # rounds past the largest double
            want = np.float64(np.inf if sum(Fraction(v) for v in a) > 0 else -np.inf)
        got = fixed(eb, a)
        assert got.tobytes() == want.tobytes(), (x[:4], got, want)
        assert orc.reduce_fixed(a).tobytes() == want.tobytes()
