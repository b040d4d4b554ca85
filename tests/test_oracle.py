"""The oracle (the CPU restatement the GPU engine is checked against), pinned
against the reference's own known answers and independent restatements of its
test oracles. No GPU needed.

Pins (paths relative to the eagle source tree):
* README.md:99-106: the oscillator at n = 1e6 finishes in 1000 steps with
  x[:3] = [0.54057281 0.54057112 0.54056944];
* tests/CanonicalReduceCases.h:73-110: the independent tree oracle (restated
  below in plain Python, without sharing code with oracle.cpp), over the sizes
  of :186-190 on the adversarial corpus of :49-60; thread-count invariance
  (:194-240); chunked == unchunked (:242-263); the exact-sum contract (:283-315);
  min / max with infinities (:317-343); columns (:345-359);
* python/tests/test_active_set.py:49-56: the map is flatnonzero(~mask) over the
  sizes (0, 1, 7, 256, 257, 4096, 100_003);
* python/tests/test_until_done_auto.py:160-184: bandK and the policy sequence,
  restated independently;
* benchmarks/perf_card/perf_card.py:255-317: one RKF7(8) attempt (tableau, stage
  sums, error ratio) against the card's own functions run with Lorenz's right-hand
  side (tests/golden/rkf78_lorenz.json).
"""

import json
import math
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
SIZES = (1, 2, 3, 255, 256, 257, 4095, 4096, 4097, 8193, 12345, 65536, 65537, 100003, (1 << 20) + 37)


# ------------------------------------------------------------- independent tree

def _join(a, b):
    s = a[0] + b[0]
    bb = s - a[0]
    e = (a[0] - (s - bb)) + (b[0] - bb)
    return (s, (a[1] + b[1]) + e if math.isfinite(s) else 0.0)


def _py_tree(x):
    """tests/CanonicalReduceCases.h:80-110 in plain Python floats (IEEE binary64)."""
    n = len(x)
    parts = []
    for b in range(0, n, 4096):
        cnt = min(4096, n - b)
        s = []
        for t in range(min(cnt, 256)):
            p = (float(x[b + t]), 0.0)
            for k in range(t + 256, cnt, 256):
                p = _join(p, (float(x[b + k]), 0.0))
            s.append(p)
        off = 128
        while off >= 1:
            for t in range(off):
                if t + off < len(s):
                    s[t] = _join(s[t], s[t + off])
            off //= 2
        parts.append(s[0])
    while len(parts) > 1:
        parts = [_join(parts[i], parts[i + 1]) if i + 1 < len(parts) else parts[i] for i in range(0, len(parts), 2)]
    h, c = parts[0]
    return h + c if math.isfinite(h) else h


def _bits(v):
    return np.float64(v).view(np.uint64)


@pytest.mark.parametrize("n", [s for s in SIZES if s <= 100003])
def test_tree_equals_independent_oracle(orc, n):
    x = orc.corpus(n, 1000 + n)
    assert _bits(orc.reduce(x)[0]) == _bits(_py_tree(x))


def test_thread_count_invariance(orc):
    saved = orc.threads()
    try:
        for n in SIZES:
            x = orc.corpus(n, 1000 + n)
            got = set()
            for th in (1, 2, 4, 8):
                orc.threads(th)
                got.add(int(_bits(orc.reduce(x)[0])))
            assert len(got) == 1, n
    finally:
        orc.threads(saved)


def test_chunked_equals_unchunked(orc):
    for n in SIZES:
        if n > 200000:
            continue
        x = orc.corpus(n, 31 + n)
        full = orc.reduce(x)[0]
        for q in range(4):
            chunk = 4096 << q
            roots = [orc.pairwise(orc.leaf_partials(x[b:b + chunk])) for b in range(0, n, chunk)]
            r = orc.pairwise(np.array(roots))
            assert _bits(orc.partial_value(r[0], r[1])) == _bits(full), (n, chunk)


def _ulps(got, exact, dtype):
    e = dtype(exact)
    return abs(float(got) - exact) / float(np.nextafter(e, dtype(np.inf)) - e)


@pytest.mark.parametrize("dtype,u,one_ulp_upto", [(np.float32, 2.0 ** -24, 2.0 ** 20),
                                                 (np.float64, 2.0 ** -53, 2.0 ** 48)])
def test_exact_fixture_contract(orc, dtype, u, one_ulp_upto):
    for n in (257, 2048 * 3 + 1, 1000000):
        for kappa in (1.0, 1024.0, 1048576.0):
            x, exact, k = orc.fixture(n, kappa, dtype)
            err = _ulps(orc.reduce(x)[0], exact, dtype)
            assert err <= 1.0 + n * k * u, (n, kappa)
            if n * k <= one_ulp_upto:
                assert err <= 1.0, (n, kappa)


def _plain_tree_f32(x):
    """tests/CanonicalReduceCases.h:118-139: plain adds, leaves of 256 halved by
    stride, then pairwise (the pre-compensation tree), in float32."""
    n = x.size
    full = n // 256 * 256
    blocks = x[:full].reshape(-1, 256).copy()
    off = 128
    while off >= 1:
        blocks[:, :off] = blocks[:, :off] + blocks[:, off:2 * off]
        off //= 2
    parts = list(blocks[:, 0])
    if full < n:
        s = list(x[full:])
        off = 128
        while off >= 1:
            for t in range(off):
                if t + off < len(s):
                    s[t] = np.float32(s[t] + s[t + off])
            off //= 2
        parts.append(s[0])
    parts = np.array(parts, dtype=np.float32)
    while parts.size > 1:
        m = parts.size
        nxt = parts[0:m - 1:2] + parts[1:m:2]
        parts = np.concatenate([nxt, parts[m - 1:]]) if m % 2 else nxt
    return parts[0]


def test_plain_tree_misses_the_contract(orc):
    """Non-vacuity (CanonicalReduceCases.h:265-281): on the kappa = 2^10 float32
    fixture the plain tree misses 1 ULP; the canonical tree meets it."""
    x, exact, _ = orc.fixture(1000000, 1024.0, np.float32)
    assert _ulps(_plain_tree_f32(x), exact, np.float32) > 1.0
    assert _ulps(orc.reduce(x)[0], exact, np.float32) <= 1.0


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_non_finite_follows_ieee(orc, dtype):
    x = orc.corpus(9001, 5, dtype)
    x[1000] = np.inf
    assert orc.reduce(x)[0] == np.inf
    x[7000] = -np.inf
    assert np.isnan(orc.reduce(x)[0])


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_min_max_exact(orc, dtype):
    for n in (1, 257, 9001):
        x = orc.corpus(n, 31 + n, dtype)
        assert orc.reduce(x, "min")[0] == x.min()
        assert orc.reduce(x, "max")[0] == x.max()
    x = orc.corpus(9001, 5, dtype)
    x[1000], x[7000] = np.inf, -np.inf
    assert orc.reduce(x, "min")[0] == -np.inf
    assert orc.reduce(x, "max")[0] == np.inf


def test_columns_equal_flat(orc):
    rows, cols = 9001, 7
    x = orc.corpus(rows * cols, 21)
    got = orc.reduce(x, columns=cols)
    for j in range(cols):
        assert _bits(got[j]) == _bits(_py_tree(x.reshape(rows, cols)[:, j]))


def test_integer_sums_exact(orc):
    rng = np.random.default_rng(3)
    x = rng.integers(-2 ** 40, 2 ** 40, size=100003, dtype=np.int64)
    assert orc.reduce(x)[0] == x.sum()
    y = rng.integers(-1000, 1000, size=100003, dtype=np.int32)
    assert orc.reduce(y)[0] == y.sum()


# ------------------------------------------------------------------- compaction

@pytest.mark.parametrize("n", (0, 1, 7, 256, 257, 4096, 100_003))
def test_compaction_is_flatnonzero(orc, n):
    mask = np.random.default_rng([7, n]).random(n) < 0.6
    m, c = orc.compact(mask)
    assert c == int((~mask).sum())
    assert np.array_equal(m, np.flatnonzero(~mask))
    k, ck = orc.compact(mask, drop=False)
    assert np.array_equal(k, np.flatnonzero(mask)) and ck == int(mask.sum())


def test_compaction_trigger_rule(orc):
    n = 100_003
    mask = np.random.default_rng([9, n]).random(n) < 0.9
    m, c, live32, fire = orc.compact(mask, span=n, theta=0.5, trigger=True)
    keep = ~mask
    groups = int(sum(keep[g:g + 32].any() for g in range(0, n, 32)))
    assert live32 == groups
    assert fire == int(c < 0.5 * 32 * groups and c < n and n >= 4096)


# ------------------------------------------------------------------------ policy

def _band_k_restated(rate, newly, live, k, k_max=64, k_min=8):
    """python/tests/test_until_done_auto.py:160-171, restated."""
    if newly <= 0:
        return k_max
    e = (2.0 * rate * live * k / newly) ** 0.5
    p = 1
    while p * 2 ** 0.5 <= e:
        p *= 2
    return min(max(p, k_min), k_max)


def test_band_k_matches_restatement(orc):
    rng = np.random.default_rng(11)
    for _ in range(3000):
        live = int(rng.integers(0, 1 << 24))
        newly = int(rng.integers(-2, 1 << 20))
        k = int(2 ** rng.integers(0, 12))
        rate = float(rng.choice([0.5, 8.0, 100.0, 3.3]))
        kmax = int(2 ** rng.integers(3, 14))
        assert orc.band_k(rate, newly, live, k, kmax, 8) == _band_k_restated(rate, newly, live, k, kmax, 8)


def test_policy_sequence(orc):
    """The device POLICY op's cells walked on the host equal the documented sequence."""
    n, max_steps, kmax = 1000, 500, 64
    stops = np.random.default_rng(5).integers(1, 700, size=n)

    def finished_after(total_steps):
        return int((stops <= total_steps).sum())

    seq, k, fin_at, done = [], 16, 0, 0
    word = min(k, max_steps)
    while fin_at != n and done < max_steps:
        seq.append(word)
        fin = finished_after(done + word)
        live, newly = n - fin, fin - fin_at
        done += word
        fin_at = fin
        k = _band_k_restated(8.0, newly, live, k, kmax)
        word = min(k, max_steps - done)
    cells = np.array([16, 0, 0, max_steps, 8000, 0], dtype=np.int64)
    wordc = np.array([min(16, max_steps)], dtype=np.int64)
    go = np.array([1], dtype=np.uint32)
    hist = np.zeros(kmax + 1, dtype=np.int64)
    got = []
    while go[0]:
        got.append(int(wordc[0]))
        orc.policy_step(finished_after(int(cells[2]) + int(wordc[0])), n, cells, wordc, go, hist, 8, kmax)
    assert got == seq


# -------------------------------------------------------------------- oscillator

def test_readme_known_answer(orc):
    """README.md:99-106: finished, 1000 steps, x[:3] to the printed digits."""
    n = 1_000_000
    om = np.linspace(1.0, 3.0, n)
    x, v, t = np.ones(n), np.zeros(n), np.zeros(n)
    m = np.zeros(n, np.uint8)
    steps, fin, longest, total = orc.oscillator_run(om, x, v, t, m, t_end=1.0, dt=1e-3, max_steps=10_000)
    assert fin == n and longest == 1000 and total == 1000 * n
    assert np.array_equal(np.round(x[:3], 8), [0.54057281, 0.54057112, 0.54056944])


def test_oscillator_cap_and_continue(orc):
    rng = np.random.default_rng(2)
    n = 5000
    om = rng.uniform(1, 3, n)
    te = 10.0 ** rng.uniform(-2, 1, n)
    te[0] = 10.0  # t after 10_000 additions of 1e-3 is 9.999999999999897 < 10: never finishes
    a = [np.ones(n), np.zeros(n), np.zeros(n), np.zeros(n, np.uint8)]
    _, fin, longest, _ = orc.oscillator_run(om, *a, t_end=te, dt=1e-3, max_steps=10_000)
    assert a[3][0] == 0 and fin < n and longest == 10_000
    # two runs of 3000 then 7000 steps leave the bits of one run of 10_000
    b = [np.ones(n), np.zeros(n), np.zeros(n), np.zeros(n, np.uint8)]
    orc.oscillator_run(om, *b, t_end=te, dt=1e-3, max_steps=3000)
    orc.oscillator_run(om, *b, t_end=te, dt=1e-3, max_steps=7000)
    for p, q in zip(a, b):
        assert np.array_equal(p, q)


def test_fma_variant_within_tolerance(orc):
    """The contracted variant differs from the exact one by rounding only: within
    1e-12 of the state's scale (sqrt(x^2 + v^2/omega^2)), steps and mask identical."""
    rng = np.random.default_rng(4)
    n = 20000
    om = rng.uniform(1, 3, n)
    te = 10.0 ** rng.uniform(-2, 1, n)
    runs = []
    for fused in (False, True):
        st = [np.ones(n), np.zeros(n), np.zeros(n), np.zeros(n, np.uint8)]
        steps, *_ = orc.oscillator_run(om, *st, t_end=te, dt=1e-3, max_steps=10_000, fused=fused)
        runs.append((st, steps))
    (a, sa), (b, sb) = runs
    assert np.array_equal(sa, sb) and np.array_equal(a[2], b[2]) and np.array_equal(a[3], b[3])
    scale = np.sqrt(a[0] ** 2 + (a[1] / om) ** 2)
    assert np.max(np.abs(a[0] - b[0]) / scale) < 1e-12
    assert np.max(np.abs(a[1] - b[1]) / (scale * om)) < 1e-12


# ----------------------------------------------------------------- golden files

def test_golden_fixtures(orc):
    """The committed fixtures (tests/golden/make_golden.py) still come out bit for bit."""
    with open(os.path.join(GOLDEN, "golden.json")) as f:
        g = json.load(f)
    for case in g["reduce"]:
        x = orc.corpus(case["n"], case["seed"])
        assert int(_bits(orc.reduce(x)[0])) == int(case["bits"], 16), case
    for case in g["oscillator"]:
        rng = np.random.default_rng(case["seed"])
        n = case["n"]
        om = rng.uniform(1, 3, n)
        te = 10.0 ** rng.uniform(-2, 1, n)
        st = [np.ones(n), np.zeros(n), np.zeros(n), np.zeros(n, np.uint8)]
        steps, fin, longest, total = orc.oscillator_run(om, *st, t_end=te, dt=1e-3, max_steps=case["max_steps"],
                                                        fused=case["fma"])
        assert (fin, longest, total) == (case["finished"], case["longest"], case["total"])
        xs = orc.reduce(st[0])[0]
        assert int(_bits(xs)) == int(case["sum_x_bits"], 16)


# --------------------------------------------------------------- Philox / walk

def test_philox_statistics(orc):
    """Philox-4x32-10 as restated (Salmon et al., SC'11): distinct counters and keys give
    distinct words, bits are balanced, and one flipped counter bit changes about half
    of the 128 output bits."""
    outs = np.stack([orc.philox4x32_10([k, 0, 7, 0], 99) for k in range(4096)])
    assert len({tuple(o) for o in outs}) == 4096
    bits = np.unpackbits(outs.view(np.uint8))
    assert abs(bits.mean() - 0.5) < 0.01
    flips = []
    for k in range(256):
        a = orc.philox4x32_10([k, 1, 2, 3], 5)
        b = orc.philox4x32_10([k ^ 1, 1, 2, 3], 5)
        flips.append(int(np.unpackbits((a ^ b).view(np.uint8)).sum()))
    assert 60 < np.mean(flips) < 68
    assert not np.array_equal(orc.philox4x32_10([1, 2, 3, 4], 5), orc.philox4x32_10([1, 2, 3, 4], 6))


def test_gambler_mean_absorption_time(orc):
    """E[T] = s (100 - s) for a fair walk from s; averaged over s ~ U{1..99} it is 1683.3."""
    n = 1 << 18
    pos = np.random.default_rng(3).integers(1, 100, n).astype(np.int32)
    want = float(np.mean(pos.astype(np.float64) * (100 - pos)))
    time, term = np.zeros(n, np.int64), np.zeros(n, np.uint8)
    fin, longest, total = orc.gambler_run(pos, time, term, seed=1, max_steps=1_000_000)
    assert fin == n and total == int(time.sum())
    assert abs(time.mean() - want) < 0.02 * want
    assert set(np.unique(pos)) <= {0, 100}


def test_det_pow_tracks_pow(orc):
    """The controller's deterministic power stays within 5e-14 relative of libm's pow
    over r in [1e-300, 1e300], e = -1/8, -1/9 (the k * ln 2 terms of the reductions
    round in double). What the controller needs is the same bits on host and device,
    which the GPU tests check; its accuracy only keeps the step sizes sensible."""
    import math
    g = np.random.default_rng(1)
    for r in np.concatenate([10.0 ** g.uniform(-300, 300, 4000), g.uniform(0.5, 2.0, 1000), [1.0, 2.0, 0.5]]):
        for e in (-1.0 / 8.0, -1.0 / 9.0):
            want = math.pow(r, e)
            got = orc.det_pow(r, e)
            assert abs(got / want - 1.0) <= 5e-14, (r, e, got, want)
    assert orc.det_pow(0.0, -0.125) == math.inf and orc.det_pow(math.inf, -0.125) == 0.0
    assert math.isnan(orc.det_pow(math.nan, -0.125))


def test_lorenz_reaches_t_final_and_counts(orc):
    """Every sample of the Lorenz configuration reaches t_final well inside the cap;
    accepted + rejected attempts equal the per-sample attempt count the run reports."""
    n = 512
    g = np.random.default_rng(2)
    rho = g.uniform(20.0, 40.0, n)
    x, y, z = (g.normal(1.0, 0.1, n) for _ in range(3))
    t, h = np.zeros(n), np.full(n, 1e-3)
    na, nr = np.zeros(n, np.uint32), np.zeros(n, np.uint32)
    term = np.zeros(n, np.uint8)
    fin, longest, total = orc.lorenz_run(rho, x, y, z, t, h, na, nr, term, max_steps=200_000)
    assert fin == n and np.all(t == 10.0) and np.all(term == 1)
    att = na.astype(np.int64) + nr
    assert int(att.sum()) == total and int(att.max()) == longest
    assert 100 < att.mean() < 2000 and np.all(np.isfinite(z))


def test_rkf78_attempt_matches_the_perf_cards_code():
    """The oracle's RKF7(8) attempt of Lorenz-63 (the scheme the Lorenz configuration
    runs: Fehlberg's tableau, left-to-right term sums skipping zero coefficients, the
    mixed max-norm error ratio) bit for bit against the same attempt computed by eagle's
    own perf-card functions (tests/golden/rkf78_lorenz.json, written by
    tests/golden/make_rkf78_golden.py from benchmarks/perf_card/perf_card.py), on 96
    states, steps and rho values, accepted and rejected."""
    import json
    import os

    import oracle

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "rkf78_lorenz.json")
    with open(path) as f:
        g = json.load(f)

    def f64(h):
        return np.array([int(h, 16)], dtype=np.uint64).view(np.float64)[0]

    rejected = 0
    for c in g["cases"]:
        s8, err, ratio = oracle.lorenz_stages([f64(v) for v in c["s0"]], f64(c["step"]), rho=f64(c["rho"]),
                                              sigma=g["sigma"], beta=g["beta"], rtol=g["rtol"], atol=g["atol"])
        assert [int(np.float64(v).view(np.uint64)) for v in s8] == [int(v, 16) for v in c["s8"]], c
        assert [int(np.float64(v).view(np.uint64)) for v in err] == [int(v, 16) for v in c["err"]], c
        assert int(np.float64(ratio).view(np.uint64)) == int(c["ratio"], 16), c
        rejected += ratio >= 1.0
    assert 0 < rejected < len(g["cases"])
