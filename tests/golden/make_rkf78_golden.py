"""Write tests/golden/rkf78_lorenz.json: RKF7(8) attempts of Lorenz-63 computed by the
reference's own code -- ``rkf78_stages`` and ``error_ratio`` of eagle's perf card
(benchmarks/perf_card/perf_card.py:281-309, its Fehlberg tableau :255-278 and
``sum_terms`` :313-317), imported from the eagle source tree -- with Lorenz's
right-hand side in place of the card's Kepler one and the tolerances of the Lorenz
configuration. The card's functions loop over six state components, so the Lorenz
state rides in the first three and three components with zero derivative follow;
they add nothing to the error ratio. The oracle's restatement of the same attempt is
checked against these bits in tests/test_oracle.py (no GPU).

Needs the eagle source tree, so it runs in the development container only; the JSON it
writes is what travels. Run from the repository root:
``python tests/golden/make_rkf78_golden.py /path/to/eagle``.
"""

import json
import os
import sys

import numpy as np

SIGMA, BETA, RTOL, ATOL = 10.0, 8.0 / 3.0, 1e-9, 1e-12


def _bits(v):
    return "%016x" % int(np.float64(v).view(np.uint64))


def main(eagle_root):
    sys.path.insert(0, os.path.join(eagle_root, "benchmarks", "perf_card"))
    sys.path.insert(0, os.path.join(eagle_root, "benchmarks"))
    import perf_card as pc

    rho_now = {"rho": 28.0}

    def lorenz_rhs(s, sqrt):  # the card's rhs slot: six components, the last three fixed
        x, y, z = s[0], s[1], s[2]
        return [SIGMA * (y - x), x * (rho_now["rho"] - z) - y, x * y - BETA * z, 0.0, 0.0, 0.0]

    pc.kepler_rhs = lorenz_rhs  # rkf78_stages looks the rhs up by this name at call time
    pc.RTOL, pc.ATOL = RTOL, ATOL  # error_ratio reads the tolerances as module globals
    g = np.random.default_rng(2026)
    cases = []
    for i in range(96):
        rho = float(g.uniform(20.0, 40.0))
        s0 = [float(v) for v in g.normal(0.0, [8.0, 9.0, 9.0]) + [0.0, 0.0, 25.0]]
        step = float(10.0 ** g.uniform(-5.0, -1.0)) if i % 8 else float(g.uniform(0.1, 0.5))  # some rejected
        rho_now["rho"] = rho
        s8, err = pc.rkf78_stages(s0 + [0.0, 0.0, 0.0], step, lambda v: v ** 0.5)
        ratio = pc.error_ratio(s0 + [0.0, 0.0, 0.0], s8, err, abs, max)
        cases.append({"s0": [_bits(v) for v in s0], "step": _bits(step), "rho": _bits(rho),
                      "s8": [_bits(v) for v in s8[:3]], "err": [_bits(v) for v in err[:3]], "ratio": _bits(ratio)})
    out = {"sigma": SIGMA, "beta": BETA, "rtol": RTOL, "atol": ATOL,
           "source": "eagle benchmarks/perf_card/perf_card.py rkf78_stages + error_ratio, Lorenz rhs",
           "cases": cases}
    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "rkf78_lorenz.json"), "w") as f:
        json.dump(out, f, indent=1)
    print(f"{len(cases)} cases")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
