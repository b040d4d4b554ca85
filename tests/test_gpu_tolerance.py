"""The 1e-12 state tolerance at the headline batch's own size.

The engine's contracted profile (``fma=True``: fma(dt, v0, x0) and fma(-c, x0, v0),
as a device compiler contracts the hawk body of README.md:89-97 by default) and its
exact profile (every operation rounded once as written: eagle's exact host profile)
are each bit-exact against the oracle's twin of the same profile (tests/
test_gpu_engine.py, the bench's parity check). This test bounds the distance
between the two profiles on the 2^24-sample heterogeneous-stop batch itself:

* the step counts, t and the mask are identical (t never contracts);
* per sample, max(|x_f - x_e|, |v_f - v_e| / omega) <= 1e-12 * A, A the sample's
  amplitude sqrt(x_e^2 + (v_e / omega)^2): the tolerance is read relative to the
  state's scale, since x and v themselves pass through zero twice a period, where
  no relative bound on one component can hold;
* the fraction of samples within 1e-12 of each component itself is reported.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _c2(n):
    omega = np.random.default_rng(1).uniform(1.0, 3.0, n)
    x0 = np.random.default_rng(2).normal(1.0, 0.1, n)
    t_end = 10.0 ** np.random.default_rng(3).uniform(-2.0, 1.0, n)
    return omega, x0, t_end


def _run(eb, omega, x0, t_end, fma):
    dev = "cuda"
    planes = dict(omega=torch.from_numpy(omega).to(dev), t_end=torch.from_numpy(t_end).to(dev),
                  x=torch.from_numpy(x0).to(dev), v=torch.zeros(omega.size, dtype=torch.float64, device=dev),
                  t=torch.zeros(omega.size, dtype=torch.float64, device=dev))
    res = eb.simulate(eb.oscillator, max_steps=10_000, mode="persist", fma=fma, dt=1e-3, **planes)
    return res


def test_contracted_within_1e12_of_the_written_order_at_full_size(eb):
    n = 1 << 24
    omega, x0, t_end = _c2(n)
    f = _run(eb, omega, x0, t_end, True)
    e = _run(eb, omega, x0, t_end, False)
    assert (f.report.finished, f.steps, f.report.step_sum) == (e.report.finished, e.steps, e.report.step_sum)
    assert torch.equal(f.t, e.t) and torch.equal(f.finished, e.finished)
    om = torch.from_numpy(omega).cuda()
    amp = torch.sqrt(e.x * e.x + (e.v / om) ** 2)
    dev = torch.maximum((f.x - e.x).abs(), (f.v - e.v).abs() / om)
    worst = float((dev / amp).max())
    assert worst <= 1e-12, worst
    comp = torch.maximum((f.x - e.x).abs() / e.x.abs(), (f.v - e.v).abs() / e.v.abs().clamp_min(1e-300))
    within = float((comp <= 1e-12).double().mean())
    print(f"max state-scale deviation {worst:.3e}; samples within 1e-12 of each component: {within:.6f}")
