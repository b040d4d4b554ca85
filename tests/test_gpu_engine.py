"""The until-done engine on the GPU against the oracle: every plane (x, v, t, mask)
bit for bit, and the run report (finished, done, the longest sample's steps, the
executed steps) exactly, for each schedule (band: the WHILE graph with fused
compaction; persist; fused) and both arithmetic profiles (exact, contracted).

Rows follow python/tests/test_until_done.py:1-30 and test_until_done_steps.py of the
eagle source tree: a finishing kernel equals the explicit run of each sample to its
stop; the cap leaves samples unfinished and the status ``max_steps``; a second run
continues from the current state; samples already finished are not stepped."""

import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

MODES = ("band", "band_eager", "persist", "fused")
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.json")


def _spread_inputs(n, seed):
    rng = np.random.default_rng(seed)
    om = rng.uniform(1, 3, n)
    te = 10.0 ** rng.uniform(-2, 1, n)
    return om, te


def _device_run(eb, om, te, n, max_steps, mode, fma, x0=None, mask0=None, runs=1, **kw):
    planes = dict(omega=torch.from_numpy(om).cuda(), t_end=te if np.ndim(te) == 0 else torch.from_numpy(te).cuda(),
                  dt=1e-3, x=torch.ones(n, dtype=torch.float64, device="cuda") if x0 is None
                  else torch.from_numpy(x0.copy()).cuda(),
                  v=torch.zeros(n, dtype=torch.float64, device="cuda"),
                  t=torch.zeros(n, dtype=torch.float64, device="cuda"))
    term = torch.zeros(n, dtype=torch.uint8, device="cuda") if mask0 is None else torch.from_numpy(mask0.copy()).cuda()
    runner = eb.until_done(eb.oscillator, max_steps=max_steps, mode=mode, fma=fma, terminated=term, **planes, **kw)
    reps = [runner.run() for _ in range(runs)]
    return [planes[k].cpu().numpy() for k in ("x", "v", "t")] + [term.cpu().numpy()], reps


def _oracle_run(orc, om, te, n, max_steps, fma, x0=None, mask0=None, runs=1):
    st = [np.ones(n) if x0 is None else x0.copy(), np.zeros(n), np.zeros(n),
          np.zeros(n, np.uint8) if mask0 is None else mask0.copy()]
    outs = [orc.oscillator_run(om, *st, t_end=te, dt=1e-3, max_steps=max_steps, fused=fma) for _ in range(runs)]
    return st, outs


def _assert_same(dev, ref):
    for a, b, name in zip(dev, ref, ("x", "v", "t", "terminated")):
        assert a.tobytes() == b.tobytes(), name


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("fma", (False, True))
def test_uniform_stop_readme_batch(eb, orc, mode, fma):
    """The README batch at n = 100_000 (the CPU config): every sample finishes at 1000 steps."""
    n = 100_000
    om = np.linspace(1.0, 3.0, n)
    dev, (rep,) = _device_run(eb, om, 1.0, n, 10_000, mode, fma)
    ref, ((_, fin, longest, total),) = _oracle_run(orc, om, 1.0, n, 10_000, fma)
    _assert_same(dev, ref)
    assert rep.done and rep.finished == n and rep.steps == 1000 == longest and rep.step_sum == total
    # sample 0 (omega = 1 exactly) does not depend on n: README.md:105's x[0]
    assert round(float(dev[0][0]), 8) == 0.54057281


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("fma", (False, True))
@pytest.mark.parametrize("n", (1, 31, 257, 100_003))
def test_spread_stops(eb, orc, mode, fma, n):
    om, te = _spread_inputs(n, 7 + n)
    dev, (rep,) = _device_run(eb, om, te, n, 10_000, mode, fma)
    ref, ((_, fin, longest, total),) = _oracle_run(orc, om, te, n, 10_000, fma)
    _assert_same(dev, ref)
    assert (rep.finished, rep.steps, rep.step_sum, rep.done) == (fin, longest, total, fin == n)


@pytest.mark.parametrize("mode", MODES)
def test_spread_stops_large(eb, orc, mode):
    n = 1 << 21
    om, te = _spread_inputs(n, 5)
    dev, (rep,) = _device_run(eb, om, te, n, 10_000, mode, True)
    ref, ((_, fin, longest, total),) = _oracle_run(orc, om, te, n, 10_000, True)
    _assert_same(dev, ref)
    assert (rep.finished, rep.steps, rep.step_sum) == (fin, longest, total)


@pytest.mark.parametrize("mode", MODES)
def test_cap_leaves_samples_running(eb, orc, mode):
    n = 4096
    om, te = _spread_inputs(n, 9)
    te[::7] = 10.0  # t after 10_000 steps is 9.999999999999897: these never finish
    dev, (rep,) = _device_run(eb, om, te, n, 10_000, mode, False)
    ref, ((_, fin, longest, total),) = _oracle_run(orc, om, te, n, 10_000, False)
    _assert_same(dev, ref)
    assert not rep.done and rep.finished == fin < n and rep.steps == 10_000 == longest


@pytest.mark.parametrize("mode", MODES)
def test_second_run_continues(eb, orc, mode):
    n = 20_000
    om, te = _spread_inputs(n, 10)
    dev, reps = _device_run(eb, om, te, n, 1500, mode, False, runs=3)
    ref, outs = _oracle_run(orc, om, te, n, 1500, False, runs=3)
    _assert_same(dev, ref)
    for rep, (_, fin, longest, total) in zip(reps, outs):
        assert (rep.finished, rep.steps, rep.step_sum) == (fin, longest, total)


@pytest.mark.parametrize("mode", MODES)
def test_finished_samples_are_not_stepped(eb, orc, mode):
    n = 10_000
    om, te = _spread_inputs(n, 12)
    mask0 = (np.random.default_rng(1).random(n) < 0.3).astype(np.uint8)
    x0 = np.random.default_rng(2).normal(1, 0.1, n)
    dev, (rep,) = _device_run(eb, om, te, n, 10_000, mode, True, x0=x0, mask0=mask0)
    ref, ((_, fin, longest, total),) = _oracle_run(orc, om, te, n, 10_000, True, x0=x0, mask0=mask0)
    _assert_same(dev, ref)
    assert (rep.finished, rep.steps, rep.step_sum) == (fin, longest, total)


@pytest.mark.parametrize("mode", MODES)
def test_zero_budget_and_empty_batch(eb, orc, mode):
    n = 1000
    om, te = _spread_inputs(n, 13)
    mask0 = (np.arange(n) % 3 == 0).astype(np.uint8)
    dev, (rep,) = _device_run(eb, om, te, n, 0, mode, False, mask0=mask0)
    assert rep.finished == int(mask0.sum()) and rep.steps == 0 and rep.step_sum == 0
    assert np.array_equal(dev[0], np.ones(n)) and np.array_equal(dev[3], mask0)
    runner = eb.until_done(eb.oscillator, max_steps=100, mode=mode, omega=torch.zeros(0, dtype=torch.float64,
                           device="cuda"), t_end=1.0, dt=1e-3, x=torch.zeros(0, dtype=torch.float64, device="cuda"),
                           v=torch.zeros(0, dtype=torch.float64, device="cuda"),
                           t=torch.zeros(0, dtype=torch.float64, device="cuda"))
    rep = runner.run()
    assert rep.done and rep.finished == 0 and rep.steps == 0


def test_band_small_k_range(eb, orc):
    """The band schedule with its K pinned small (many passes, many compactions)."""
    n = 50_000
    om, te = _spread_inputs(n, 14)
    dev, (rep,) = _device_run(eb, om, te, n, 3000, "band", False, k_first=8, k_min=8, k_max=8)
    ref, ((_, fin, longest, total),) = _oracle_run(orc, om, te, n, 3000, False)
    _assert_same(dev, ref)
    assert (rep.finished, rep.steps, rep.step_sum) == (fin, longest, total)
    assert rep.launches == 3000 // 8 + (1 if 3000 % 8 else 0) or rep.launches < 3000 // 8


def test_engine_matches_golden(eb):
    with open(GOLDEN) as f:
        cases = json.load(f)["oscillator"]
    for c in cases:
        om, te = _spread_inputs(c["n"], c["seed"])
        x = torch.ones(c["n"], dtype=torch.float64, device="cuda")
        res = eb.simulate(eb.oscillator, max_steps=c["max_steps"], fma=c["fma"], omega=torch.from_numpy(om).cuda(),
                          t_end=torch.from_numpy(te).cuda(), dt=1e-3, x=x,
                          v=torch.zeros_like(x), t=torch.zeros_like(x))
        assert (res.report.finished, res.steps, res.report.step_sum) == (c["finished"], c["longest"], c["total"])
        assert res.status == ("finished" if c["finished"] == c["n"] else "max_steps")
        assert int(eb.reduce(res.x).cpu().numpy().view(np.uint64)[0]) == int(c["sum_x_bits"], 16)


def test_simulate_with_host_arrays(eb, orc):
    """Host (numpy) planes are staged through the device and written back in place."""
    n = 100_000
    om = np.linspace(1.0, 3.0, n)
    x, v, t = np.ones(n), np.zeros(n), np.zeros(n)
    res = eb.simulate(eb.oscillator, max_steps=10_000, omega=om, t_end=1.0, dt=1e-3, x=x, v=v, t=t)
    assert res.status == "finished" and res.steps == 1000
    ref, _ = _oracle_run(orc, om, 1.0, n, 10_000, False)
    assert x.tobytes() == ref[0].tobytes() and res.x is x
