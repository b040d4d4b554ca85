"""Lorenz-63 under the adaptive RKF7(8) attempt (the 2^22-sample stiff-tail
configuration: sigma 10, beta 8/3, rho ~ U[20, 40], start ~ N(1, 0.1), t_final 10,
rtol 1e-9, atol 1e-12, h0 1e-3) on the GPU against the oracle: x, y, z, t, h, the
accept / reject counts and the mask bit for bit, the report exactly, the canonical
sum of the final z bit for bit; both schedules; the cap and a continued run; the
hawk-ABI persist entry through launch_raw."""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from eagle_b200 import _abi  # noqa: E402

PLANES = ("rho", "x", "y", "z", "t", "h", "n_acc", "n_rej")


def _start(n, seed=3):
    g = np.random.default_rng(seed)
    p = {"rho": g.uniform(20.0, 40.0, n)}
    for name in ("x", "y", "z"):
        p[name] = g.normal(1.0, 0.1, n)
    p["t"] = np.zeros(n)
    p["h"] = np.full(n, 1e-3)
    p["n_acc"] = np.zeros(n, np.uint32)
    p["n_rej"] = np.zeros(n, np.uint32)
    return p


def _device(eb, p0, max_steps, mode, runs=1, params=None, **kw):
    n = p0["x"].size
    planes = {k: torch.from_numpy(v.view(np.int32) if v.dtype == np.uint32 else v.copy()).cuda()
              for k, v in p0.items()}
    term = torch.zeros(n, dtype=torch.uint8, device="cuda")
    prm = dict(sigma=10.0, beta=8.0 / 3.0, t_final=10.0, rtol=1e-9, atol=1e-12)
    prm.update(params or {})
    r = eb.until_done(eb.lorenz, max_steps=max_steps, mode=mode, terminated=term, **planes, **prm, **kw)
    reps = [r.run() for _ in range(runs)]
    out = {k: v.cpu().numpy() for k, v in planes.items()}
    out["n_acc"] = out["n_acc"].view(np.uint32)
    out["n_rej"] = out["n_rej"].view(np.uint32)
    return out, term.cpu().numpy(), reps, planes


def _oracle(orc, p0, max_steps, runs=1, params=None):
    p = {k: v.copy() for k, v in p0.items()}
    term = np.zeros(p["x"].size, np.uint8)
    prm = params or {}
    outs = [orc.lorenz_run(*(p[k] for k in PLANES), term, max_steps=max_steps, **prm) for _ in range(runs)]
    return p, term, outs


def _same(a, b):
    for k in PLANES[1:]:
        assert a[k].tobytes() == b[k].tobytes(), k


@pytest.mark.parametrize("mode", ("persist", "fused"))
@pytest.mark.parametrize("n", (1, 1000, 20_011))
def test_attempts_bitwise(eb, orc, mode, n):
    p0 = _start(n)
    d, m, (rep,), planes = _device(eb, p0, 200_000, mode)
    r, rm, ((fin, longest, total),) = _oracle(orc, p0, 200_000)
    _same(d, r)
    assert m.tobytes() == rm.tobytes()
    assert (rep.finished, rep.steps, rep.step_sum, rep.done) == (fin, longest, total, fin == n)
    assert fin == n and np.all(r["t"] == 10.0)
    assert eb.reduce(planes["z"]).item() == orc.reduce(r["z"])[0]


@pytest.mark.parametrize("mode", ("persist", "fused"))
def test_cap_and_continue(eb, orc, mode):
    p0 = _start(5000, 4)
    d, m, reps, _ = _device(eb, p0, 120, mode, runs=4)
    r, rm, outs = _oracle(orc, p0, 120, runs=4)
    _same(d, r)
    assert m.tobytes() == rm.tobytes()
    for rep, (fin, longest, total) in zip(reps, outs):
        assert (rep.finished, rep.steps, rep.step_sum) == (fin, longest, total)
    assert not reps[0].done and reps[0].finished == 0


def test_params_reach_the_attempt(eb, orc):
    p0 = _start(3000, 5)
    prm = dict(sigma=9.5, beta=2.5, t_final=4.0, rtol=1e-7, atol=1e-10)
    d, m, (rep,), _ = _device(eb, p0, 200_000, "persist", params=prm)
    r, rm, ((fin, longest, total),) = _oracle(orc, p0, 200_000, params=prm)
    _same(d, r)
    assert (rep.finished, rep.steps, rep.step_sum) == (fin, longest, total)


def test_hawk_abi_persist_entry(eb, orc):
    n = 4099
    p0 = _start(n, 6)
    planes = {k: torch.from_numpy(v.view(np.int32) if v.dtype == np.uint32 else v.copy()).cuda()
              for k, v in p0.items()}
    term = torch.zeros(n, dtype=torch.uint8, device="cuda")
    fin = torch.zeros(1, dtype=torch.int32, device="cuda")
    budget = torch.tensor([200_000], dtype=torch.int64, device="cuda")
    words = torch.zeros(4, dtype=torch.int64, device="cuda")

    def h(tn, k, _width=None):
        return _abi.ScalarHandle(tn.data_ptr(), k, 1, 2, 0)

    args = [h(planes["rho"], n, 8), ctypes.c_double(10.0), ctypes.c_double(8.0 / 3.0), ctypes.c_double(10.0),
            ctypes.c_double(1e-9), ctypes.c_double(1e-12), h(term, n, 1)]
    args += [h(planes[k], n, 4 if k.startswith("n_") else 8) for k in PLANES[1:]]
    args += [h(fin, 1, 4), h(budget, 1, 8), ctypes.c_int64(0), ctypes.c_int64(n), ctypes.c_int64(n),
             ctypes.c_uint64(words.data_ptr()), ctypes.c_uint64(0), ctypes.c_uint64(words.data_ptr() + 4),
             ctypes.c_uint64(words.data_ptr() + 8), ctypes.c_uint32(16)]
    ptrs = (ctypes.c_void_p * len(args))(*[ctypes.addressof(a) for a in args])
    d = _abi.new(_abi.LaunchRawDesc, device=-1, function=eb.entry("lorenz_persist"),
                 stream=torch.cuda.current_stream().cuda_stream, args=ctypes.addressof(ptrs), arg_count=len(args))
    d.grid[:] = (148, 1, 1)
    d.block[:] = (128, 1, 1)
    _abi.check(_abi.lib().eagle_backend_launch_raw(ctypes.byref(d)))
    torch.cuda.synchronize()
    r, rm, ((f, longest, total),) = _oracle(orc, p0, 200_000)
    assert planes["z"].cpu().numpy().tobytes() == r["z"].tobytes()
    assert planes["n_rej"].cpu().numpy().view(np.uint32).tobytes() == r["n_rej"].tobytes()
    assert int(fin.item()) == f == n and int(words.cpu().numpy()[1]) == total


def test_band_modes_refused(eb):
    p0 = _start(16)
    with pytest.raises(Exception, match="persist"):
        _device(eb, p0, 10, "band")
