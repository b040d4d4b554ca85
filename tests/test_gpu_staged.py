"""The host-staged until-done run (chunked host-to-device copies overlapping the
chunks' runs) leaves the bits of one device-resident run: state, mask and the
report against the oracle, over ragged chunk splits and two runs in a row with
new host inputs."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _host(seed, n):
    rng = np.random.default_rng(seed)
    return dict(omega=rng.uniform(1, 3, n), t_end=10.0 ** rng.uniform(-2, 0.5, n), x=rng.normal(1.0, 0.1, n),
                v=np.zeros(n), t=np.zeros(n))


@pytest.mark.parametrize("chunks", (1, 7, 16))
@pytest.mark.parametrize("mode", ("persist", "fused", "band"))
def test_staged_run_matches_the_oracle(eb, orc, chunks, mode):
    n = 200_003
    dev = {k: torch.zeros(n, dtype=torch.float64, device="cuda") for k in ("omega", "t_end", "x", "v", "t")}
    mask = torch.zeros(n, dtype=torch.uint8, device="cuda")
    mask.fill_(1)  # launch zeroes it
    r = eb.StagedRunner(eb.oscillator, max_steps=5000, chunks=chunks, mode=mode, fma=True, terminated=mask, dt=1e-3,
                        **dev)
    for seed in (1, 2):
        h = _host(seed, n)
        pinned = {k: torch.from_numpy(v).pin_memory() for k, v in h.items()}
        r.launch(pinned)
        rep = r.report()
        st = [h["x"].copy(), h["v"].copy(), h["t"].copy(), np.zeros(n, np.uint8)]
        _, fin, longest, total = orc.oscillator_run(h["omega"], *st, t_end=h["t_end"], dt=1e-3, max_steps=5000,
                                                    fused=True)
        for k, want in zip(("x", "v", "t"), st[:3]):
            assert dev[k].cpu().numpy().tobytes() == want.tobytes(), k
        assert mask.cpu().numpy().tobytes() == st[3].tobytes()
        assert (rep.finished, rep.steps, rep.step_sum, rep.done) == (fin, longest, total, fin == n)
        assert eb.reduce(dev["x"]).item() == orc.reduce(st[0])[0]


def test_staged_refuses_mismatched_host_planes(eb):
    n = 1000
    dev = {k: torch.zeros(n, dtype=torch.float64, device="cuda") for k in ("omega", "x", "v", "t")}
    r = eb.StagedRunner(eb.oscillator, max_steps=10, chunks=2, mode="persist", t_end=1.0, dt=1e-3, **dev)
    with pytest.raises(ValueError, match="host plane"):
        r.launch({"x": torch.zeros(n - 1, dtype=torch.float64)})
