"""The persist oscillator's longest-first claims: the engine sorts the samples by
their estimated stop steps ((t_end - t) / dt, longest first) and the lanes claim them
in that order. Only the schedule changes, so x, v, t, the mask and the run report
must be the oracle's bits, as with claims in index order -- for uniform and
per-sample t_end, samples already terminated, starts away from t = +0, NaN and
infinite t_end, dt = 0, batches that end inside a sort tile, continued runs and
budgets whose buckets are wider than one step."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _run(eb, om, te, t0, x0, mask0, dt, max_steps, fma, index_order, runs=1):
    n = om.size
    planes = dict(omega=torch.from_numpy(om).cuda(),
                  t_end=te if np.ndim(te) == 0 else torch.from_numpy(te).cuda(), dt=dt,
                  x=torch.from_numpy(x0.copy()).cuda(), v=torch.zeros(n, dtype=torch.float64, device="cuda"),
                  t=torch.from_numpy(t0.copy()).cuda())
    term = torch.from_numpy(mask0.copy()).cuda()
    runner = eb.until_done(eb.oscillator, max_steps=max_steps, mode="persist", fma=fma, terminated=term,
                           index_order=index_order, **planes)
    reps = [runner.run() for _ in range(runs)]
    return [planes[k].cpu().numpy() for k in ("x", "v", "t")] + [term.cpu().numpy()], reps


def _check(eb, orc, om, te, t0=None, x0=None, mask0=None, dt=1e-3, max_steps=10_000, fma=True, runs=1):
    n = om.size
    t0 = np.zeros(n) if t0 is None else t0
    x0 = np.ones(n) if x0 is None else x0
    mask0 = np.zeros(n, np.uint8) if mask0 is None else mask0
    st = [x0.copy(), np.zeros(n), t0.copy(), mask0.copy()]
    outs = [orc.oscillator_run(om, *st, t_end=te, dt=dt, max_steps=max_steps, fused=fma) for _ in range(runs)]
    for index_order in (False, True):
        dev, reps = _run(eb, om, te, t0, x0, mask0, dt, max_steps, fma, index_order, runs)
        for a, b, name in zip(dev, st, ("x", "v", "t", "terminated")):
            assert a.tobytes() == b.tobytes(), (name, index_order)
        for rep, (_, fin, longest, total) in zip(reps, outs):
            assert (rep.finished, rep.steps, rep.step_sum) == (fin, longest, total), index_order


@pytest.mark.parametrize("n", (1, 31, 32_769, 100_003))
@pytest.mark.parametrize("fma", (False, True))
def test_spread_stops(eb, orc, n, fma):
    rng = np.random.default_rng(n)
    _check(eb, orc, rng.uniform(1, 3, n), 10.0 ** rng.uniform(-2, 1, n), fma=fma)


def test_uniform_stop_and_mixed_starts(eb, orc):
    n = 50_000
    rng = np.random.default_rng(5)
    t0 = np.zeros(n)
    t0[1::3] = -0.0
    t0[2::5] = rng.uniform(0, 0.9, t0[2::5].size)
    _check(eb, orc, rng.uniform(1, 3, n), 1.0, t0=t0)


def test_terminated_specials_and_dt_zero(eb, orc):
    n = 70_001
    rng = np.random.default_rng(6)
    om = rng.uniform(1, 3, n)
    te = 10.0 ** rng.uniform(-2, 1, n)
    te[::97] = np.nan
    te[1::89] = np.inf
    te[2::83] = -np.inf
    te[3::79] = 0.0
    mask0 = (rng.random(n) < 0.25).astype(np.uint8)
    x0 = rng.normal(1, 0.1, n)
    _check(eb, orc, om, te, x0=x0, mask0=mask0)
    _check(eb, orc, om, rng.uniform(-0.5, 0.5, n), dt=0.0, max_steps=300)  # only t_end <= 0 stops


def test_continued_runs_and_wide_buckets(eb, orc):
    n = 40_000
    rng = np.random.default_rng(7)
    om, te = rng.uniform(1, 3, n), 10.0 ** rng.uniform(-2, 1, n)
    _check(eb, orc, om, te, max_steps=1500, runs=3)  # later runs start away from t = +0
    _check(eb, orc, om, rng.uniform(0, 60.0, n), max_steps=70_000)  # 35 steps per bucket


def test_ordered_launch_replays_in_a_cuda_graph(eb, orc):
    """The persist launch only enqueues (mask count, the claim order, the run), so it
    captures into a CUDA graph; each replay is a fresh run with the oracle's bits."""
    n = 60_000
    rng = np.random.default_rng(8)
    om, te = rng.uniform(1, 3, n), 10.0 ** rng.uniform(-2, 1, n)
    x0 = rng.normal(1, 0.1, n)
    d_x0 = torch.from_numpy(x0).cuda()
    planes = dict(omega=torch.from_numpy(om).cuda(), t_end=torch.from_numpy(te).cuda(), dt=1e-3,
                  x=d_x0.clone(), v=torch.zeros(n, dtype=torch.float64, device="cuda"),
                  t=torch.zeros(n, dtype=torch.float64, device="cuda"))
    term = torch.zeros(n, dtype=torch.uint8, device="cuda")
    runner = eb.until_done(eb.oscillator, max_steps=10_000, mode="persist", fma=True, terminated=term, **planes)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        runner.launch(s)  # the first launch builds the device's t sequence outside the capture
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        runner.launch(s)
    st = [x0.copy(), np.zeros(n), np.zeros(n), np.zeros(n, np.uint8)]
    _, fin, longest, total = orc.oscillator_run(om, *st, t_end=te, dt=1e-3, max_steps=10_000, fused=True)
    for _ in range(2):
        planes["x"].copy_(d_x0)
        planes["v"].zero_()
        planes["t"].zero_()
        term.zero_()
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        dev = [planes[k].cpu().numpy() for k in ("x", "v", "t")] + [term.cpu().numpy()]
        for a, b, name in zip(dev, st, ("x", "v", "t", "terminated")):
            assert a.tobytes() == b.tobytes(), name
        rep = runner.report(s)
        assert (rep.finished, rep.steps, rep.step_sum) == (fin, longest, total)
    del g


def test_large_ordered_launch_eager_and_captured(eb, orc):
    """A batch of 2^22 + 12345 samples (128 full runs of 32768 and a ragged one, some
    samples terminated before the run): the oracle's bits for every plane, the mask and
    the report, called eagerly and replayed twice from a CUDA graph."""
    n = (1 << 22) + 12345
    rng = np.random.default_rng(12)
    om, te = rng.uniform(1, 3, n), 10.0 ** rng.uniform(-2, 0.3, n)
    x0 = rng.normal(1, 0.1, n)
    mask0 = (rng.random(n) < 0.02).astype(np.uint8)
    d_x0 = torch.from_numpy(x0).cuda()
    d_m0 = torch.from_numpy(mask0).cuda()
    planes = dict(omega=torch.from_numpy(om).cuda(), t_end=torch.from_numpy(te).cuda(), dt=1e-3,
                  x=d_x0.clone(), v=torch.zeros(n, dtype=torch.float64, device="cuda"),
                  t=torch.zeros(n, dtype=torch.float64, device="cuda"))
    term = d_m0.clone()
    runner = eb.until_done(eb.oscillator, max_steps=2500, mode="persist", fma=True, terminated=term, **planes)
    st = [x0.copy(), np.zeros(n), np.zeros(n), mask0.copy()]
    _, fin, longest, total = orc.oscillator_run(om, *st, t_end=te, dt=1e-3, max_steps=2500, fused=True)

    def reset():
        planes["x"].copy_(d_x0)
        planes["v"].zero_()
        planes["t"].zero_()
        term.copy_(d_m0)

    def check(rep):
        dev = [planes[k].cpu().numpy() for k in ("x", "v", "t")] + [term.cpu().numpy()]
        for a, b, name in zip(dev, st, ("x", "v", "t", "terminated")):
            assert a.tobytes() == b.tobytes(), name
        assert (rep.finished, rep.steps, rep.step_sum) == (fin, longest, total)

    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        reset()
        runner.launch(s)
    s.synchronize()
    check(runner.report(s))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        runner.launch(s)
    for _ in range(2):
        reset()
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        check(runner.report(s))
    del g
