"""The built-in step entries through eagle's own launch seams: the role-packed
hawk kernel ABI (plugin/plugin_registry/registry.h:605-710 of the eagle source
tree) launched by ``eagle_backend_run_device`` (partition triple appended by the
seam, eagle/exec/DeviceKernel.h:47-84) and by ``eagle_backend_launch_raw`` with the
range / persist tails (python/eagle/_plan_binding.py:455-460, :582-591), against
the oracle; a multi-partition launch covers the same samples as one."""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from eagle_b200 import _abi  # noqa: E402


def _h(t, n):
    return _abi.ScalarHandle(t.data_ptr(), n, 1, 2, t.device.index)


def _setup(n, seed):
    rng = np.random.default_rng(seed)
    om = rng.uniform(1, 3, n)
    te = 10.0 ** rng.uniform(-2, 1, n)
    dev = dict(om=torch.from_numpy(om).cuda(), te=torch.from_numpy(te).cuda(),
               x=torch.ones(n, dtype=torch.float64, device="cuda"), v=torch.zeros(n, dtype=torch.float64, device="cuda"),
               t=torch.zeros(n, dtype=torch.float64, device="cuda"), m=torch.zeros(n, dtype=torch.uint8, device="cuda"),
               fin=torch.zeros(1, dtype=torch.int32, device="cuda"))
    return om, te, dev


def _role_args(dev, n, budget_cell):
    """The spread entries' role arguments in arg_spec order."""
    return [_h(dev["om"], n), _h(dev["te"], n), ctypes.c_double(1e-3), _h(dev["m"], n), _h(dev["x"], n),
            _h(dev["v"], n), _h(dev["t"], n), _h(dev["fin"], 1), _h(budget_cell, 1)]


def _oracle(orc, om, te, n, budget, fma):
    st = [np.ones(n), np.zeros(n), np.zeros(n), np.zeros(n, np.uint8)]
    _, fin, longest, total = orc.oscillator_run(om, *st, t_end=te, dt=1e-3, max_steps=budget, fused=fma)
    return st, fin, longest, total


def _check(dev, ref):
    for k, r in zip(("x", "v", "t", "m"), ref):
        assert dev[k].cpu().numpy().tobytes() == r.tobytes(), k


@pytest.mark.parametrize("fma", (False, True))
@pytest.mark.parametrize("parts", (1, 3))
def test_run_device_plain_entry(eb, orc, fma, parts):
    n = 30_001
    om, te, dev = _setup(n, 1)
    budget = torch.tensor([10_000], dtype=torch.int64, device="cuda")
    fn = eb.entry("oscillator_spread" + ("_fma" if fma else ""))
    args = _role_args(dev, n, budget)
    addrs = (ctypes.c_uint64 * len(args))(*[ctypes.addressof(a) for a in args])
    stream = torch.cuda.current_stream().cuda_stream
    bounds = np.linspace(0, n, parts + 1).astype(int)
    for b0, b1 in zip(bounds[:-1], bounds[1:]):
        d = _abi.new(_abi.LaunchDesc, device=-1, block=128, function=fn, nparams=len(args), base=int(b0),
                     count=int(b1 - b0), n_samples=n, stream=stream)
        d.params = ctypes.cast(addrs, ctypes.POINTER(ctypes.c_uint64))
        launched = ctypes.c_int32()
        _abi.check(_abi.lib().eagle_backend_run_device(ctypes.byref(d), ctypes.byref(launched)))
        assert launched.value == 1
    torch.cuda.synchronize()
    ref, fin, _, _ = _oracle(orc, om, te, n, 10_000, fma)
    _check(dev, ref)
    assert int(dev["fin"].item()) == fin


def test_run_device_refuses_bad_partition(eb):
    d = _abi.new(_abi.LaunchDesc, function=eb.entry("oscillator"), base=5, count=10, n_samples=12)
    launched = ctypes.c_int32()
    assert _abi.lib().eagle_backend_run_device(ctypes.byref(d), ctypes.byref(launched)) == _abi.INDEX
    d = _abi.new(_abi.LaunchDesc, function=eb.entry("oscillator"), base=0, count=0, n_samples=12)
    assert _abi.lib().eagle_backend_run_device(ctypes.byref(d), ctypes.byref(launched)) == _abi.OK
    assert launched.value == 0


@pytest.mark.parametrize("entry", ("range", "persist"))
def test_launch_raw_fast_entries(eb, orc, entry):
    n = 100_003
    om, te, dev = _setup(n, 2)
    budget = torch.tensor([10_000], dtype=torch.int64, device="cuda")
    words = torch.zeros(4, dtype=torch.int64, device="cuda")  # next|steps (u32 each), stepsum (u64), util
    util = torch.zeros(2, dtype=torch.int64, device="cuda")
    args = _role_args(dev, n, budget) + [ctypes.c_int64(0), ctypes.c_int64(n), ctypes.c_int64(n)]
    next_p, steps_p, sum_p = words.data_ptr(), words.data_ptr() + 4, words.data_ptr() + 8
    if entry == "range":
        args += [ctypes.c_uint64(steps_p), ctypes.c_uint64(sum_p)]
        grid = ((n + 255) // 256, 1, 1)
    else:
        args += [ctypes.c_uint64(next_p), ctypes.c_uint64(util.data_ptr()), ctypes.c_uint64(steps_p),
                 ctypes.c_uint64(sum_p), ctypes.c_uint32(64)]
        grid = (148 * 4, 1, 1)
    ptrs = (ctypes.c_void_p * len(args))(*[ctypes.addressof(a) for a in args])
    d = _abi.new(_abi.LaunchRawDesc, device=-1, function=eb.entry(f"oscillator_spread_{entry}"),
                 stream=torch.cuda.current_stream().cuda_stream, args=ctypes.addressof(ptrs), arg_count=len(args))
    d.grid[:] = grid
    d.block[:] = (256, 1, 1)
    _abi.check(_abi.lib().eagle_backend_launch_raw(ctypes.byref(d)))
    torch.cuda.synchronize()
    ref, fin, longest, total = _oracle(orc, om, te, n, 10_000, False)
    _check(dev, ref)
    w = words.cpu().numpy().view(np.uint32)
    assert int(dev["fin"].item()) == fin and int(w[1]) == longest
    assert int(words.cpu().numpy()[1]) == total
    if entry == "persist":
        u = util.cpu().numpy()
        assert u[0] == total and u[1] >= total


def test_function_attribute(eb):
    v = ctypes.c_int32()
    _abi.check(_abi.lib().eagle_backend_function_attribute(eb.entry("oscillator_spread_persist"), 4, ctypes.byref(v)))
    assert 0 < v.value <= 255
