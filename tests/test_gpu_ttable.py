"""The persistent oscillator's known-stop path: a sample that starts at t = +0 finds
the step it stops at from the launch's shared t sequence (T[0] = +0, T[k+1] = T[k] +
dt) instead of adding dt and testing at every step. Its x, v, t, mask and the run
counters must stay those of the step-by-step model (the oracle) bit for bit -- at
t_end values on, just below and just above the sequence's terms, at and below +0, NaN
and infinite; for dt = 0; for samples starting at -0 or elsewhere (the step-by-step
path) mixed with +0 ones in one warp; and for budgets past the table's reach."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _t_seq(dt, k):
    t = np.zeros(k + 1)
    for i in range(k):
        t[i + 1] = t[i] + dt
    return t


def _run_both(eb, orc, om, te, t0, dt, max_steps, fma=True, mode="persist"):
    n = om.size
    planes = dict(omega=torch.from_numpy(om).cuda(), t_end=torch.from_numpy(te).cuda(), dt=dt,
                  x=torch.ones(n, dtype=torch.float64, device="cuda"),
                  v=torch.zeros(n, dtype=torch.float64, device="cuda"),
                  t=torch.from_numpy(t0.copy()).cuda())
    term = torch.zeros(n, dtype=torch.uint8, device="cuda")
    runner = eb.until_done(eb.oscillator, max_steps=max_steps, mode=mode, fma=fma, terminated=term, **planes)
    rep = runner.run()
    dev = [planes[k].cpu().numpy() for k in ("x", "v", "t")] + [term.cpu().numpy()]
    st = [np.ones(n), np.zeros(n), t0.copy(), np.zeros(n, np.uint8)]
    _, fin, longest, total = orc.oscillator_run(om, *st, t_end=te, dt=dt, max_steps=max_steps, fused=fma)
    for a, b, name in zip(dev, st, ("x", "v", "t", "terminated")):
        assert a.tobytes() == b.tobytes(), name
    assert (rep.finished, rep.steps, rep.step_sum) == (fin, longest, total)
    return rep


@pytest.mark.parametrize("fma", (False, True))
def test_t_end_on_and_around_the_sequence(eb, orc, fma):
    dt, cap = 1e-3, 3000
    t = _t_seq(dt, cap)
    picks = [1, 2, 15, 16, 17, 63, 64, 65, 1000, 1023, 1024, 1025, 2047, 2048, 2999, 3000]
    te = []
    for k in picks:
        te += [t[k], np.nextafter(t[k], -np.inf), np.nextafter(t[k], np.inf)]
    te += [0.0, -0.0, -1.0, np.nan, np.inf, -np.inf, t[cap] + 1.0, 5e-324]
    te = np.array(te * 9)[: 32 * 13]  # several warps' worth, mixed
    n = te.size
    om = np.random.default_rng(3).uniform(1, 3, n)
    _run_both(eb, orc, om, te, np.zeros(n), dt, cap, fma)


def test_mixed_starts_in_one_warp(eb, orc):
    """+0 starts take the known-stop path; -0 and other starts the step-by-step one."""
    n = 4096
    rng = np.random.default_rng(11)
    om = rng.uniform(1, 3, n)
    te = 10.0 ** rng.uniform(-2, 0.5, n)
    t0 = np.zeros(n)
    t0[1::3] = -0.0
    t0[2::5] = rng.uniform(0, 0.5, t0[2::5].size)
    _run_both(eb, orc, om, te, t0, 1e-3, 5000)


def test_dt_zero_and_long_budgets(eb, orc):
    n = 1000
    rng = np.random.default_rng(12)
    om = rng.uniform(1, 3, n)
    te = rng.uniform(-0.5, 0.5, n)  # dt = 0: only t_end <= 0 stops (after one step)
    _run_both(eb, orc, om, te, np.zeros(n), 0.0, 700)
    te = rng.uniform(0, 80.0, n)  # a budget past the table's reach: step by step
    _run_both(eb, orc, om, te, np.zeros(n), 1e-3, 70_000)


@pytest.mark.parametrize("cap", (1, 7, 16, 1025, 16384, 16385, 65536))
def test_budgets_at_the_table_edges(eb, orc, cap):
    n = 777
    rng = np.random.default_rng(cap)
    om = rng.uniform(1, 3, n)
    t = _t_seq(1e-3, cap)
    te = np.where(rng.random(n) < 0.5, rng.uniform(0, t[cap] * 1.2 + 1e-3, n), t[rng.integers(0, cap + 1, n)])
    _run_both(eb, orc, om, te, np.zeros(n), 1e-3, cap)
