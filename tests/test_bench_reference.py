"""The bench's reference arm on the CPU (no GPU needed): it runs the oracle -- the
CPU restatement of eagle's host path -- over the same seeded batch as the engine arm,
on every host core, and prints one JSON line in the driver's contract with the same
metric, unit and config as the engine's line; on a batch it runs whole, it also
carries the canonical sum's bits, which must be those of the oracle's own run."""

import json
import os
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_line(orc):
    n = 1 << 16
    env = dict(os.environ, OMP_NUM_THREADS="1")  # as torchrun sets it: the arm must still use every core
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--n", str(n),
                        "--steps", "2", "--warmup", "1"], capture_output=True, text=True, env=env, cwd=ROOT,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0 and line["scaling"] == "strong"
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    cores = len(os.sched_getaffinity(0))
    assert line["cpu_baseline"]["cores"] == cores
    # the whole batch ran: its sum is the oracle's canonical sum of the same run
    omega = np.random.default_rng(1).uniform(1.0, 3.0, n)
    x0 = np.random.default_rng(2).normal(1.0, 0.1, n)
    t_end = 10.0 ** np.random.default_rng(3).uniform(-2.0, 1.0, n)
    st = [x0.copy(), np.zeros(n), np.zeros(n), np.zeros(n, np.uint8)]
    orc.oscillator_run(omega, *st, t_end=t_end, dt=1e-3, max_steps=10_000, fused=True, steps_out=False)
    want = orc.reduce(st[0])[0]
    assert line["result"]["sum_x_bits"] == "0x%016x" % int(np.float64(want).view(np.uint64))
