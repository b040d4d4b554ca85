"""The eagle-shaped Python face of the B200 engine.

Mirrors the until-done surface of eagle (paths relative to the eagle source tree):

* :func:`simulate` / :class:`SimResult` -- python/eagle/_simulate.py:451-483, :777
  (bind the model's planes like a call, allocate the ``terminated`` mask, run until
  every sample finishes or ``max_steps``; ``status`` is ``"finished"`` or ``"max_steps"``);
* :func:`until_done` / :class:`Runner` / :class:`RunReport` -- python/eagle/_until_done.py:120-171,
  :528, :1775 (``run()`` continues from the current mask and state, ``reset()`` clears
  the mask);
* :func:`reduce` -- python/eagle/_graph_reduce.py:98 (the canonical reduction);
* :func:`compact` / :func:`mask_count` -- python/eagle/_active_set.py:482-525 and
  _until_done.py:374-387.

Planes are torch CUDA tensors (the engine works on them in place) or host arrays
(numpy / CPU tensors), which are staged through the device and written back. Every
computation runs in ``libeagle_b200.so`` on the GPU; there is no CPU path.
"""

from __future__ import annotations

import ctypes
import time
from dataclasses import dataclass

import numpy as np

from . import _abi

_torch = None


def _t():
    global _torch
    if _torch is None:
        import torch

        _torch = torch
    return _torch


def _stream_handle(stream=None) -> int:
    torch = _t()
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def _ptr(x) -> int:
    return int(x.data_ptr())


# ------------------------------------------------------------------------- models

@dataclass(frozen=True)
class Model:
    """A built-in step body: its plane and Param names in the engine's order."""

    name: str
    planes: tuple      # per-sample planes, read-only first then mutable
    mutable: tuple
    params: tuple


class _Oscillator(Model):
    """The Euler oscillator of eagle's README (README.md:89-97)::

        x = x0 + dt * v0; v = v0 - dt * omega * omega * x0; t += dt; terminated = t >= t_end

    ``t_end`` may be a number (a Param) or a per-sample plane."""


oscillator = _Oscillator(name="oscillator", planes=("omega", "t_end", "x", "v", "t"), mutable=("x", "v", "t"),
                         params=("t_end", "dt"))


class _Gambler(Model):
    """The gambler's-ruin walk: ``pos`` (int32) moves +1 or -1 per step and the sample
    stops at 0 or 100; ``time`` (int64) counts its steps. Step s of sample i moves +1
    when bit (s mod 128) of Philox-4x32-10(counter = (s // 128, id_base + i), key =
    seed) is set. Params: ``seed`` and ``id_base`` (default 0)."""


gambler = _Gambler(name="gambler", planes=("pos", "time"), mutable=("pos", "time"), params=("seed", "id_base"))


class _Lorenz(Model):
    """Lorenz-63 under eagle's perf-card adaptive RKF7(8) attempt: per-sample ``rho``;
    state ``x, y, z, t, h`` (float64) and ``n_acc, n_rej`` (uint32 counts); Params
    ``sigma, beta, t_final, rtol, atol``. One until-done step is one attempt."""


lorenz = _Lorenz(name="lorenz", planes=("rho", "x", "y", "z", "t", "h", "n_acc", "n_rej"),
                 mutable=("x", "y", "z", "t", "h", "n_acc", "n_rej"),
                 params=("sigma", "beta", "t_final", "rtol", "atol"))

_MODES = {"band": _abi.MODE_BAND, "persist": _abi.MODE_PERSIST, "fused": _abi.MODE_FUSED,
          "band_eager": _abi.MODE_BAND_EAGER}


# ------------------------------------------------------------------------- reports

@dataclass(frozen=True)
class RunReport:
    """What one :meth:`Runner.run` did (python/eagle/_until_done.py:120-171).

    ``finished`` counts set mask bytes at the end, ``done`` is ``finished == n``,
    ``steps`` the longest sample's steps in this run (exact), ``launches`` the loop
    passes, ``compactions`` the compactions run, ``step_sum`` the steps executed."""

    n: int
    finished: int
    done: bool
    steps: int
    launches: int
    compactions: int
    step_sum: int
    mode: str
    exact_steps: bool = True
    report_bytes: int = 0


class SimResult:
    """What one :meth:`Simulation.run` produced (python/eagle/_simulate.py:451-483):
    ``state`` maps each mutable plane to its array; each is also an attribute and an
    item. ``finished`` is the mask, ``done``/``status``/``steps``/``report``/``wall_s``."""

    __slots__ = ("state", "finished", "done", "steps", "status", "report", "n", "wall_s")

    def __init__(self, *, state, finished, report, wall_s):
        put = object.__setattr__
        put(self, "state", dict(state))
        put(self, "finished", finished)
        put(self, "report", report)
        put(self, "done", bool(report.done))
        put(self, "steps", int(report.steps))
        put(self, "status", "finished" if report.done else "max_steps")
        put(self, "n", int(report.n))
        put(self, "wall_s", float(wall_s))

    def __setattr__(self, name, value):
        raise AttributeError("a SimResult is read-only")

    def __getattr__(self, name):
        state = object.__getattribute__(self, "state")
        if name in state:
            return state[name]
        raise AttributeError(f"the result has no field or state plane {name!r} (state: {sorted(state)})")

    def __getitem__(self, name):
        return self.state[name]

    def __repr__(self) -> str:
        return f"SimResult(status={self.status!r}, n={self.n}, steps={self.steps}, state={list(self.state)})"


# ------------------------------------------------------------------------- runner

def _as_device_plane(name, value, n, device, *, staged, dtype=None):
    """A contiguous CUDA tensor (float64 unless ``dtype``) for ``value``; host arrays
    are staged (copied in, and remembered in ``staged`` for the copy back)."""
    torch = _t()
    dtype = dtype or torch.float64
    if isinstance(value, torch.Tensor) and value.is_cuda:
        if value.dtype != dtype or not value.is_contiguous() or value.numel() != n:
            raise ValueError(f"plane {name!r} must be a contiguous {dtype} tensor of {n} samples")
        return value
    host = torch.as_tensor(np.asarray(value) if not isinstance(value, torch.Tensor) else value)
    if host.dtype != dtype or host.numel() != n:
        raise ValueError(f"plane {name!r} must hold {n} {dtype} samples")
    dev = host.reshape(-1).to(device, non_blocking=True)
    staged.append((name, value, dev))
    return dev


class Runner:
    """The until-done loop of one model over one batch (python/eagle/_until_done.py:528).

    ``run()`` runs every live sample until it terminates or has taken ``max_steps``
    steps in this run and returns a :class:`RunReport`; a second ``run()`` continues
    from the current mask and state; ``reset()`` clears the mask. ``mode`` picks the
    schedule: ``"band"`` (one CUDA graph: WHILE over the fused step + compaction
    kernel), ``"persist"`` (one persistent launch) or ``"fused"`` (one lane per sample,
    one launch); ``"auto"`` takes ``"band"``. All modes leave identical bits. ``fma``
    contracts the model's multiply-adds as a device compiler does by default. The
    persist oscillator claims its samples longest first (their stop steps estimated
    from ``t_end``, ``t`` and ``dt``); ``index_order=True`` claims them in index order
    instead -- the same bits, a slower schedule."""

    def __init__(self, model: Model, *, max_steps: int, mode: str = "auto", fma: bool = False, terminated=None,
                 device=None, k_first: int = 0, k_min: int = 0, k_max: int = 0, chunk: int = 0,
                 overhead_steps: float = 0.0, interval_steps: float = 0.0, ctas_per_sm: int = 0,
                 index_order: bool = False, **planes):
        torch = _t()
        self._ctas_per_sm = int(ctas_per_sm)
        if model not in (oscillator, gambler, lorenz):
            raise ValueError(f"eagle_b200: unknown model {model!r}")
        if max_steps is None or int(max_steps) < 0:
            raise ValueError("max_steps must be >= 0")
        if model is lorenz:
            mode = "persist" if mode == "auto" else mode
            self._init_lorenz(max_steps=max_steps, mode=mode, terminated=terminated, device=device, chunk=chunk,
                              **planes)
            return
        if model is gambler:
            mode = "persist" if mode == "auto" else mode
            self._init_gambler(max_steps=max_steps, mode=mode, terminated=terminated, device=device, chunk=chunk,
                               **planes)
            return
        mode = "band" if mode == "auto" else mode
        if mode not in _MODES:
            raise ValueError(f"mode must be one of {sorted(_MODES)} or 'auto'")
        missing = {"omega", "t_end", "dt", "x", "v", "t"} - set(planes)
        if missing:
            raise TypeError(f"oscillator needs {sorted(missing)}")
        extra = set(planes) - {"omega", "t_end", "dt", "x", "v", "t"}
        if extra:
            raise TypeError(f"oscillator takes no plane(s) {sorted(extra)}")
        n = int(np.asarray(planes["omega"]).size) if not isinstance(planes["omega"], torch.Tensor) \
            else planes["omega"].numel()
        self.device = torch.device(device) if device is not None else (
            planes["x"].device if isinstance(planes["x"], torch.Tensor) and planes["x"].is_cuda
            else torch.device("cuda", torch.cuda.current_device()))
        self._staged = []
        self.n = n
        self.mode = mode
        self.max_steps = int(max_steps)
        self.fma = bool(fma)
        spread = not np.isscalar(planes["t_end"]) and not (isinstance(planes["t_end"], torch.Tensor)
                                                           and planes["t_end"].dim() == 0)
        self.spread = spread
        dev_planes = {}
        for name in ("omega", "x", "v", "t") + (("t_end",) if spread else ()):
            dev_planes[name] = _as_device_plane(name, planes[name], n, self.device, staged=self._staged)
        self.planes = dev_planes
        if terminated is None:
            terminated = torch.zeros(n, dtype=torch.bool, device=self.device)
        elif not (isinstance(terminated, torch.Tensor) and terminated.is_cuda):
            raise ValueError("terminated must be a CUDA tensor (bool or uint8)")
        if terminated.dtype not in (torch.bool, torch.uint8) or not terminated.is_contiguous():
            raise ValueError("terminated must be a contiguous bool/uint8 CUDA tensor")
        self.terminated = terminated
        d = _abi.new(_abi.EngineDesc)
        d.flags = (_abi.FLAG_FMA if self.fma else 0) | (_abi.FLAG_INDEX_ORDER if index_order else 0)
        d.device = self.device.index if self.device.index is not None else -1
        d.model = _abi.MODEL_OSCILLATOR_SPREAD if spread else _abi.MODEL_OSCILLATOR
        d.mode = _MODES[mode]
        d.n = n
        d.max_steps = self.max_steps
        order = ("omega", "t_end", "x", "v", "t") if spread else ("omega", "x", "v", "t")
        for i, name in enumerate(order):
            d.planes[i] = _ptr(dev_planes[name])
        if spread:
            d.uniforms[0] = float(planes["dt"])
        else:
            d.uniforms[0] = float(planes["t_end"])
            d.uniforms[1] = float(planes["dt"])
        d.terminated = _ptr(terminated)
        d.k_first, d.k_min, d.k_max, d.chunk = int(k_first), int(k_min), int(k_max), int(chunk)
        d.overhead_steps, d.interval_steps = float(overhead_steps), float(interval_steps)
        d.ctas_per_sm = self._ctas_per_sm
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _abi.check(_abi.lib().eagle_backend_x_b200_engine_create(ctypes.byref(d), ctypes.byref(h)))
        self._h = h

    def _init_gambler(self, *, max_steps, mode, terminated, device, chunk, **planes):
        torch = _t()
        if mode not in ("persist", "fused"):
            raise ValueError("the gambler model runs under mode 'persist' or 'fused'")
        missing = {"pos", "time", "seed"} - set(planes)
        if missing:
            raise TypeError(f"gambler needs {sorted(missing)}")
        extra = set(planes) - {"pos", "time", "seed", "id_base"}
        if extra:
            raise TypeError(f"gambler takes no plane(s) {sorted(extra)}")
        pos = planes["pos"]
        n = pos.numel() if isinstance(pos, torch.Tensor) else int(np.asarray(pos).size)
        self.device = torch.device(device) if device is not None else (
            pos.device if isinstance(pos, torch.Tensor) and pos.is_cuda
            else torch.device("cuda", torch.cuda.current_device()))
        self._staged = []
        self.n, self.mode, self.max_steps, self.fma, self.spread = n, mode, int(max_steps), False, False
        self.planes = {"pos": _as_device_plane("pos", pos, n, self.device, staged=self._staged, dtype=torch.int32),
                       "time": _as_device_plane("time", planes["time"], n, self.device, staged=self._staged,
                                                dtype=torch.int64)}
        if terminated is None:
            terminated = torch.zeros(n, dtype=torch.bool, device=self.device)
        elif not (isinstance(terminated, torch.Tensor) and terminated.is_cuda
                  and terminated.dtype in (torch.bool, torch.uint8) and terminated.is_contiguous()):
            raise ValueError("terminated must be a contiguous bool/uint8 CUDA tensor")
        self.terminated = terminated
        d = _abi.new(_abi.EngineDesc)
        d.device = self.device.index if self.device.index is not None else -1
        d.model = _abi.MODEL_GAMBLER
        d.mode = _MODES[mode]
        d.n = n
        d.max_steps = self.max_steps
        d.planes[0] = _ptr(self.planes["pos"])
        d.planes[1] = _ptr(self.planes["time"])
        seed = int(planes["seed"]) & ((1 << 64) - 1)
        d.iuniforms[0] = seed - (1 << 64) if seed >= (1 << 63) else seed
        d.iuniforms[1] = int(planes.get("id_base", 0))
        d.terminated = _ptr(terminated)
        d.chunk = int(chunk)
        d.ctas_per_sm = self._ctas_per_sm
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _abi.check(_abi.lib().eagle_backend_x_b200_engine_create(ctypes.byref(d), ctypes.byref(h)))
        self._h = h

    def _init_lorenz(self, *, max_steps, mode, terminated, device, chunk, **planes):
        torch = _t()
        if mode not in ("persist", "fused"):
            raise ValueError("the lorenz model runs under mode 'persist' or 'fused'")
        names = ("rho", "x", "y", "z", "t", "h", "n_acc", "n_rej")
        params = ("sigma", "beta", "t_final", "rtol", "atol")
        missing = (set(names) | set(params)) - set(planes)
        if missing:
            raise TypeError(f"lorenz needs {sorted(missing)}")
        extra = set(planes) - set(names) - set(params)
        if extra:
            raise TypeError(f"lorenz takes no plane(s) {sorted(extra)}")
        x = planes["x"]
        n = x.numel() if isinstance(x, torch.Tensor) else int(np.asarray(x).size)
        self.device = torch.device(device) if device is not None else (
            x.device if isinstance(x, torch.Tensor) and x.is_cuda else torch.device("cuda", torch.cuda.current_device()))
        self._staged = []
        self.n, self.mode, self.max_steps, self.fma, self.spread = n, mode, int(max_steps), False, False
        self.planes = {}
        for name in names:
            dt = torch.int32 if name in ("n_acc", "n_rej") else torch.float64
            self.planes[name] = _as_device_plane(name, planes[name], n, self.device, staged=self._staged, dtype=dt)
        if terminated is None:
            terminated = torch.zeros(n, dtype=torch.bool, device=self.device)
        elif not (isinstance(terminated, torch.Tensor) and terminated.is_cuda
                  and terminated.dtype in (torch.bool, torch.uint8) and terminated.is_contiguous()):
            raise ValueError("terminated must be a contiguous bool/uint8 CUDA tensor")
        self.terminated = terminated
        d = _abi.new(_abi.EngineDesc)
        d.device = self.device.index if self.device.index is not None else -1
        d.model = _abi.MODEL_LORENZ
        d.mode = _MODES[mode]
        d.n = n
        d.max_steps = self.max_steps
        for k, name in enumerate(names):
            d.planes[k] = _ptr(self.planes[name])
        for k, name in enumerate(params[:4]):
            d.uniforms[k] = float(planes[name])
        d.uniforms_ext[0] = float(planes["atol"])
        d.terminated = _ptr(terminated)
        d.chunk = int(chunk)
        d.ctas_per_sm = self._ctas_per_sm
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _abi.check(_abi.lib().eagle_backend_x_b200_engine_create(ctypes.byref(d), ctypes.byref(h)))
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                _abi.lib().eagle_backend_x_b200_engine_release(h)
            except Exception:
                pass
            self._h = None

    def launch(self, stream=None) -> None:
        """Enqueue one run on ``stream`` (default: torch's current stream); no sync."""
        torch = _t()
        with torch.cuda.device(self.device):
            _abi.check(_abi.lib().eagle_backend_x_b200_engine_launch(self._h, _stream_handle(stream)))

    def report(self, stream=None) -> RunReport:
        """Wait for ``stream`` and read the last run's report (one small copy)."""
        torch = _t()
        r = _abi.new(_abi.Report)
        with torch.cuda.device(self.device):
            _abi.check(_abi.lib().eagle_backend_x_b200_engine_report(self._h, _stream_handle(stream),
                                                                     ctypes.byref(r)))
        return RunReport(n=int(r.n), finished=int(r.finished), done=bool(r.done), steps=int(r.steps),
                         launches=int(r.launches), compactions=int(r.compactions), step_sum=int(r.step_sum),
                         mode=self.mode, report_bytes=int(r.report_bytes))

    def run(self, stream=None) -> RunReport:
        self.launch(stream)
        rep = self.report(stream)
        self._copy_back(stream)
        return rep

    def time_kernel(self, launches: int) -> None:
        """Time the main kernel (the persistent or fused step entry; the band graph as
        a whole) of each of the next ``launches`` launches with CUDA events on the
        launch stream; 0 disarms. Read the times with :meth:`kernel_ms`."""
        torch = _t()
        with torch.cuda.device(self.device):
            _abi.check(_abi.lib().eagle_backend_x_b200_engine_time_kernel(self._h, int(launches)))

    def kernel_ms(self, cap: int = 65536) -> list:
        """Milliseconds of each launch timed since :meth:`time_kernel` (waits for them)."""
        torch = _t()
        buf = (ctypes.c_float * max(1, cap))()
        count = ctypes.c_int32()
        with torch.cuda.device(self.device):
            _abi.check(_abi.lib().eagle_backend_x_b200_engine_kernel_ms(self._h, buf, int(cap), ctypes.byref(count)))
        return [float(buf[i]) for i in range(min(int(count.value), cap))]

    def reset(self) -> None:
        """Clear the mask: every sample is live again (its state is kept)."""
        self.terminated.zero_()

    def _copy_back(self, stream=None) -> None:
        torch = _t()
        for name, host, dev in self._staged:
            if name in ("x", "v", "t", "pos", "time", "y", "z", "h", "n_acc", "n_rej"):
                if isinstance(host, torch.Tensor):
                    host.copy_(dev.reshape(host.shape))
                else:
                    np.copyto(host, dev.cpu().numpy().reshape(np.shape(host)))


def until_done(model: Model, *, max_steps: int, **kwargs) -> Runner:
    """The :class:`Runner` of ``model`` over the given planes (python/eagle/_until_done.py:1775)."""
    return Runner(model, max_steps=max_steps, **kwargs)


class StagedRunner:
    """The until-done loop fed from host memory in chunks: chunk k's host-to-device
    copies run on a copy stream while chunk k-1 steps on the compute stream, so the
    transfer of a run overlaps its work instead of preceding it. Samples are
    independent, so the chunked runs leave the bits of one run over all samples.

    ``planes`` are the device planes and Params as for :class:`Runner` (CUDA
    tensors of ``n`` samples); :meth:`launch` takes the per-sample inputs to copy
    in, as pinned host tensors keyed by plane name, and zeroes the mask. The chunk
    runs rotate over ``streams`` compute streams, each persistent run holding
    ``ctas_per_sm`` CTAs per SM: a run lasts at least as long as its longest sample
    whatever its size, and its resident CTAs wait out that tail, so narrower runs
    side by side keep the tails of one chunk under the work of the others."""

    def __init__(self, model: Model, *, max_steps: int, chunks: int = 8, streams: int = 4, ctas_per_sm: int = 1,
                 full_tail: int = 2, terminated=None, device=None, **kwargs):
        torch = _t()
        per_sample = {k: v for k, v in kwargs.items() if isinstance(v, torch.Tensor) and v.is_cuda and v.dim() == 1}
        if not per_sample:
            raise ValueError("StagedRunner needs the device planes")
        n = next(iter(per_sample.values())).numel()
        if any(v.numel() != n or not v.is_contiguous() for v in per_sample.values()):
            raise ValueError("every device plane must be a contiguous tensor of the same length")
        chunks = max(1, min(int(chunks), n))
        self.n, self.device = n, next(iter(per_sample.values())).device
        if terminated is None:
            terminated = torch.zeros(n, dtype=torch.uint8, device=self.device)
        self.terminated = terminated
        self.planes = per_sample
        bounds = [n * k // chunks for k in range(chunks + 1)]
        self.bounds = list(zip(bounds[:-1], bounds[1:]))
        self.runners = []
        for k, (lo, hi) in enumerate(self.bounds):
            sub = {key: (v[lo:hi] if key in per_sample else v) for key, v in kwargs.items()}
            # the last ``full_tail`` chunks run alone at the end: let them fill the GPU
            cps = 0 if k >= len(self.bounds) - int(full_tail) else ctas_per_sm
            self.runners.append(Runner(model, max_steps=max_steps, terminated=terminated[lo:hi], device=self.device,
                                       ctas_per_sm=cps, **sub))
        self.mode = self.runners[0].mode
        self.copy_stream = torch.cuda.Stream(self.device)
        self.streams = [torch.cuda.Stream(self.device) for _ in range(max(1, int(streams)))]
        self._start = torch.cuda.Event()
        self._ready = [torch.cuda.Event() for _ in self.bounds]
        self._done = [torch.cuda.Event() for _ in self.streams]

    def launch(self, host: dict, stream=None) -> None:
        """Enqueue one run whose inputs come from the pinned host tensors ``host``."""
        torch = _t()
        lib = _abi.lib()
        stream = stream or torch.cuda.current_stream(self.device)
        for name, h in host.items():
            dev = self.planes[name]
            if h.numel() != self.n or h.element_size() != dev.element_size() or h.is_cuda:
                raise ValueError(f"host plane {name!r} must be {self.n} host samples of {dev.dtype}")
        self._start.record(stream)  # the previous run is done with the buffers
        self.copy_stream.wait_event(self._start)
        for cs in self.streams:
            cs.wait_event(self._start)
        cs = self.copy_stream.cuda_stream
        msize = self.terminated.element_size()
        for k, (lo, hi) in enumerate(self.bounds):
            for name, h in host.items():
                dev = self.planes[name]
                es = dev.element_size()
                _abi.check(lib.eagle_backend_memcpy(dev.data_ptr() + lo * es, h.data_ptr() + lo * es,
                                                    (hi - lo) * es, _abi.COPY_H2D, cs))
            _abi.check(lib.eagle_backend_memset_device(self.terminated.data_ptr() + lo * msize, (hi - lo) * msize, cs))
            self._ready[k].record(self.copy_stream)
            run_on = self.streams[k % len(self.streams)]
            run_on.wait_event(self._ready[k])
            self.runners[k].launch(run_on)
        for ev, cs_ in zip(self._done, self.streams):
            ev.record(cs_)
            stream.wait_event(ev)

    def report(self, stream=None) -> RunReport:
        """The run's report over all chunks: every chunk's counters copied on
        ``stream``, one host wait, then read."""
        torch = _t()
        self.report_enqueue(stream)
        (stream if stream is not None else torch.cuda.current_stream(self.device)).synchronize()
        return self.report_read()

    def report_enqueue(self, stream=None) -> None:
        """Put the device-to-host copies of every chunk's counters on ``stream`` (no
        wait): :meth:`report_read` reads them once a wait covers the copies, so the
        host can enqueue the next run meanwhile."""
        torch = _t()
        lib = _abi.lib()
        s = _stream_handle(stream)
        with torch.cuda.device(self.device):
            for r in self.runners:
                _abi.check(lib.eagle_backend_x_b200_engine_report_enqueue(r._h, s))

    def report_read(self) -> RunReport:
        """The report from the copies :meth:`report_enqueue` made (after a wait for them)."""
        torch = _t()
        lib = _abi.lib()
        with torch.cuda.device(self.device):
            reps = []
            for r in self.runners:
                rep = _abi.new(_abi.Report)
                _abi.check(lib.eagle_backend_x_b200_engine_report_read(r._h, ctypes.byref(rep)))
                reps.append(RunReport(n=int(rep.n), finished=int(rep.finished), done=bool(rep.done),
                                      steps=int(rep.steps), launches=int(rep.launches),
                                      compactions=int(rep.compactions), step_sum=int(rep.step_sum), mode=self.mode,
                                      report_bytes=int(rep.report_bytes)))
        fin = sum(r.finished for r in reps)
        return RunReport(n=self.n, finished=fin, done=fin == self.n, steps=max(r.steps for r in reps),
                         launches=sum(r.launches for r in reps), compactions=sum(r.compactions for r in reps),
                         step_sum=sum(r.step_sum for r in reps), mode=self.mode,
                         report_bytes=sum(r.report_bytes for r in reps))


def simulate(model: Model, *, max_steps: int, mode: str = "auto", fma: bool = False, **planes) -> SimResult:
    """Run ``model`` on every sample until each finishes or ``max_steps`` (python/eagle/_simulate.py:777).

    ``planes`` bind the model's arguments by name (numbers for Params, arrays for
    per-sample planes); the mutable planes are updated in place and returned in the
    :class:`SimResult` together with the ``finished`` mask."""
    t0 = time.perf_counter()
    runner = Runner(model, max_steps=max_steps, mode=mode, fma=fma, **planes)
    report = runner.run()
    wall = time.perf_counter() - t0
    state = {}
    for name in model.mutable:
        host = planes[name]
        state[name] = host if not (hasattr(host, "is_cuda") and host.is_cuda) else runner.planes[name]
    return SimResult(state=state, finished=runner.terminated, report=report, wall_s=wall)


# ------------------------------------------------------------------------- reduction

_REDUCE_DTYPES = None


def _reduce_dtype(x):
    torch = _t()
    global _REDUCE_DTYPES
    if _REDUCE_DTYPES is None:
        _REDUCE_DTYPES = {torch.float32: _abi.REDUCE_F32, torch.float64: _abi.REDUCE_F64,
                          torch.int32: _abi.REDUCE_I32, torch.int64: _abi.REDUCE_I64, torch.uint8: _abi.REDUCE_U8,
                          torch.bool: _abi.REDUCE_U8}
    if x.dtype not in _REDUCE_DTYPES:
        raise TypeError(f"eagle_b200.reduce: dtype {x.dtype} is not reducible")
    return _REDUCE_DTYPES[x.dtype]


_OPS = {"sum": _abi.REDUCE_OP_SUM, "max": _abi.REDUCE_OP_MAX, "all": _abi.REDUCE_OP_ALL, "min": _abi.REDUCE_OP_MIN}
_POLICIES = {"compensated": _abi.REDUCE_COMPENSATED, "ordered": _abi.REDUCE_ORDERED, "auto": _abi.REDUCE_AUTO}


class Reducer:
    """A prepared canonical reduction of one (n, columns) CUDA plane: work buffers
    allocated once (the seam's query), so :meth:`__call__` only enqueues (and can be
    captured in a CUDA graph). ``fixed=True`` sums float64 on eagle's 128-bit
    fixed-point leaf (``eagle_backend_x_b200_reduce_fixed``), the path eagle takes on
    devices whose FP32:FP64 ratio is 8 or worse; on such a device the plain call
    takes it by itself."""

    def __init__(self, x, op: str = "sum", *, policy: str = "ordered", comp=None, pair_out: bool = False,
                 out=None, fixed: bool = False):
        torch = _t()
        if not (isinstance(x, torch.Tensor) and x.is_cuda and x.is_contiguous()):
            raise ValueError("eagle_b200.reduce takes a contiguous CUDA tensor")
        self.x = x
        n = x.shape[0] if x.dim() > 0 else 1
        cols = x.numel() // n if n else 1
        d = _abi.new(_abi.ReduceDesc)
        d.dtype = _reduce_dtype(x)
        d.op = _OPS[op]
        d.device = x.device.index
        d.n = n
        d.policy = _POLICIES[policy]
        d.flags = _abi.REDUCE_PAIR_OUT if pair_out else 0
        d.columns = cols
        self.comp = comp
        if comp is not None:
            d.comp_in = _ptr(comp)
        if fixed and (d.dtype != _abi.REDUCE_F64 or d.op != _abi.REDUCE_OP_SUM or pair_out):
            raise ValueError("the fixed-point leaf sums float64 and writes one value per column")
        self._entry = _abi.lib().eagle_backend_x_b200_reduce_fixed if fixed else \
            _abi.lib().eagle_backend_x_reduce_canonical
        _abi.check(self._entry(ctypes.byref(d)))  # query
        elem = x.element_size()
        self.work_a = torch.empty(int(d.work_elems) * elem, dtype=torch.uint8, device=x.device)
        self.work_b = torch.empty(int(d.work_elems) * elem, dtype=torch.uint8, device=x.device)
        self.out = out if out is not None else torch.empty(cols * (2 if pair_out else 1), dtype=x.dtype,
                                                           device=x.device)
        d.in_ = _ptr(x)
        d.out = _ptr(self.out)
        d.work_a = _ptr(self.work_a)
        d.work_b = _ptr(self.work_b)
        self.desc = d

    def __call__(self, stream=None):
        self.desc.stream = _stream_handle(stream)
        _abi.check(self._entry(ctypes.byref(self.desc)))
        return self.out


def reduce(x, op: str = "sum", *, policy: str = "ordered", comp=None, pair_out: bool = False, fixed: bool = False,
           stream=None):
    """The canonical reduction of each column of the CUDA plane ``x`` (python/eagle/_graph_reduce.py:98):
    a tensor of ``columns`` results (``2 * columns`` with ``pair_out``: hi then comp); ``fixed``
    takes the 128-bit fixed-point float64 leaf (eagle/reduce/canonical.h:153-313)."""
    return Reducer(x, op, policy=policy, comp=comp, pair_out=pair_out, fixed=fixed)(stream)


# ------------------------------------------------------------------------- filtering

class Compactor:
    """A prepared active-set compaction of an ``n``-sample mask (scratch from the
    seam's query, allocated once): :meth:`__call__` only enqueues."""

    def __init__(self, mask, *, drop: bool = True, trigger: bool = False, theta: float = 0.5, span=None):
        torch = _t()
        if not (isinstance(mask, torch.Tensor) and mask.is_cuda and mask.dtype in (torch.bool, torch.uint8)):
            raise ValueError("compact takes a bool/uint8 CUDA mask")
        n = mask.numel()
        dev = mask.device
        self.mask = mask
        self.index_map = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
        self.count = torch.zeros(1, dtype=torch.int32, device=dev)
        d = _abi.new(_abi.CompactDesc)
        d.flags = _abi.COMPACT_MASK_IS_DROP if drop else 0
        d.device = dev.index
        d.n = n
        _abi.check(_abi.lib().eagle_backend_compact_device(ctypes.byref(d)))  # query
        self.scratch = torch.empty(max(int(d.scratch_bytes), 1), dtype=torch.uint8, device=dev)
        d.mask = _ptr(mask)
        d.index_map = _ptr(self.index_map)
        d.count = _ptr(self.count)
        d.scratch = _ptr(self.scratch)
        self.trigger = trigger
        if trigger:
            self.live32 = torch.zeros(1, dtype=torch.int32, device=dev)
            self.fire = torch.zeros(1, dtype=torch.int32, device=dev)
            self.span = span if span is not None else torch.full((1,), n, dtype=torch.int32, device=dev)
            d.live32, d.fire, d.span = _ptr(self.live32), _ptr(self.fire), _ptr(self.span)
            d.theta = float(theta)
        self.desc = d

    def __call__(self, stream=None):
        self.desc.stream = _stream_handle(stream)
        _abi.check(_abi.lib().eagle_backend_compact_device(ctypes.byref(self.desc)))
        return self.index_map, self.count


def compact(mask, *, drop: bool = True, stream=None):
    """``(index_map, count)``: the ascending indices of the samples ``mask`` keeps
    (``drop=True``: the unset bytes, a ``terminated`` mask). ``index_map[:count]`` is
    valid; ``count`` is a one-element device tensor."""
    return Compactor(mask, drop=drop)(stream)


def mask_count(mask, cell=None, stream=None):
    """``cell[0] = number of set bytes of mask`` (memset, then the MASK_COUNT cell op)."""
    torch = _t()
    if cell is None:
        cell = torch.zeros(1, dtype=torch.int32, device=mask.device)
    s = _stream_handle(stream)
    _abi.check(_abi.lib().eagle_backend_memset_device(_ptr(cell), 4, s))
    d = _abi.new(_abi.CellOpDesc)
    d.op = _abi.CELL_MASK_COUNT
    d.device = mask.device.index
    d.stream = s
    d.n = mask.numel()
    d.p[0] = _ptr(mask)
    d.p[1] = _ptr(cell)
    _abi.check(_abi.lib().eagle_backend_cell_op(ctypes.byref(d)))
    return cell


def cell_op(op: int, n: int, pointers, ints=(), device: int = -1, stream=None) -> None:
    """Enqueue one of the seam's built-in cell ops (BUMP, MASK_COUNT, POLICY, ...)."""
    d = _abi.new(_abi.CellOpDesc)
    d.op = int(op)
    d.device = int(device)
    d.stream = _stream_handle(stream)
    d.n = int(n)
    for k, p in enumerate(pointers):
        d.p[k] = int(p)
    for k, v in enumerate(ints):
        d.i[k] = int(v)
    _abi.check(_abi.lib().eagle_backend_cell_op(ctypes.byref(d)))


def entry(name: str, device: int = -1) -> int:
    """The raw CUfunction handle of a built-in step entry (for run_device / launch_raw)."""
    f = ctypes.c_uint64()
    _abi.check(_abi.lib().eagle_backend_x_b200_entry(name.encode(), int(device), ctypes.byref(f)))
    return int(f.value)


class CompactSum:
    """The canonical ordered sum of the float64 ``values`` that ``mask`` keeps, in
    sample order (eagle: ActiveSet.compact, python/eagle/_active_set.py:482-525, then
    the ``ordered`` reduction of python/eagle/_graph_reduce.py:98-173 over the
    compacted plane). :meth:`__call__` is one call of
    ``eagle_backend_x_b200_compact_sum``: a keep bitmap and the leaf starts, then each
    4096-survivor leaf summed straight from ``values``; the kept values are never
    written. :meth:`gather` writes them instead (``eagle_backend_x_b200_compact_gather``
    into ``kept``), for callers that need the compacted plane itself. Buffers are
    allocated once; calls only enqueue. ``drop=True`` treats set bytes as dropped (a
    ``terminated`` mask), ``drop=False`` as kept."""

    def __init__(self, mask, values, *, drop: bool = False, pair_out: bool = False):
        torch = _t()
        if not (isinstance(mask, torch.Tensor) and mask.is_cuda and mask.dtype in (torch.bool, torch.uint8)):
            raise ValueError("CompactSum takes a bool/uint8 CUDA mask")
        if not (isinstance(values, torch.Tensor) and values.is_cuda and values.dtype == torch.float64
                and values.is_contiguous() and values.numel() == mask.numel()):
            raise ValueError("CompactSum takes contiguous float64 CUDA values, one per mask byte")
        n = mask.numel()
        dev = mask.device
        self.mask, self.values, self.n, self.drop = mask, values, n, drop
        self.count = torch.zeros(1, dtype=torch.int32, device=dev)
        self.out = torch.empty(2 if pair_out else 1, dtype=torch.float64, device=dev)
        self.flags = _abi.REDUCE_PAIR_OUT if pair_out else 0
        flags = _abi.COMPACT_MASK_IS_DROP if drop else 0
        d = _abi.new(_abi.CompactDesc, flags=flags, device=dev.index, n=n)
        with torch.cuda.device(dev):
            _abi.check(_abi.lib().eagle_backend_x_b200_compact_sum(ctypes.byref(d), 0, 0, self.flags))  # query
        self.scratch = torch.empty(max(int(d.scratch_bytes), 1), dtype=torch.uint8, device=dev)
        d.mask, d.count, d.scratch = _ptr(mask), _ptr(self.count), _ptr(self.scratch)
        self.sdesc = d
        self.kept = None
        self._gdesc = None

    def gather(self, stream=None):
        """Enqueue the compaction that writes the kept values in sample order into
        ``kept`` and their number into ``count`` (no sum)."""
        torch = _t()
        if self._gdesc is None:
            dev = self.mask.device
            # at least one leaf's worth, so that a rank can always share its first 4095 survivors
            self.kept = torch.empty(max(self.n, 4096), dtype=torch.float64, device=dev)
            d = _abi.new(_abi.CompactDesc, flags=_abi.COMPACT_MASK_IS_DROP if self.drop else 0, device=dev.index,
                         n=self.n)
            _abi.check(_abi.lib().eagle_backend_x_b200_compact_gather(ctypes.byref(d), 0, 0, 8))  # query
            self._gscratch = torch.empty(max(int(d.scratch_bytes), 1), dtype=torch.uint8, device=dev)
            d.mask, d.count, d.scratch = _ptr(self.mask), _ptr(self.count), _ptr(self._gscratch)
            self._gdesc = d
        self._gdesc.stream = _stream_handle(stream)
        _abi.check(_abi.lib().eagle_backend_x_b200_compact_gather(ctypes.byref(self._gdesc), _ptr(self.values),
                                                                   _ptr(self.kept), 8))

    def __call__(self, stream=None):
        self.sdesc.stream = _stream_handle(stream)
        _abi.check(_abi.lib().eagle_backend_x_b200_compact_sum(ctypes.byref(self.sdesc), _ptr(self.values),
                                                               _ptr(self.out), self.flags))
        return self.out


# ------------------------------------------------------------------------- physical reorder

def _plane_table(planes):
    torch = _t()
    tab = (_abi.ReorderPlane * max(1, len(planes)))()
    for k, p in enumerate(planes):
        if not (isinstance(p, torch.Tensor) and p.is_cuda and p.is_contiguous()):
            raise ValueError("reorder planes must be contiguous CUDA tensors")
        tab[k].data = _ptr(p)
        tab[k].elem_bytes = p.element_size()
    return tab


def reorder(planes, mask, perm, inv, index_map, count, span, *, fire=None, drop: bool = True, stream=None):
    """Physically reorder ``planes`` (the ``mask`` among them) in place over
    ``[0, span)``: the kept samples first in ascending order, the dropped ones after
    (eagle/filtering/Reorder.h; ``eagle_backend_reorder_device``). ``perm`` / ``inv``
    (int32) follow the moves, ``index_map`` becomes the identity over ``[0, count)``;
    ``count``, ``span`` (and ``fire``, which gates the whole call on the device) are
    one-element uint32/int32 CUDA cells. Enqueue only; the scratch is allocated here."""
    torch = _t()
    n = perm.numel()
    tab = _plane_table(planes)
    d = _abi.new(_abi.ReorderDesc, flags=_abi.COMPACT_MASK_IS_DROP if drop else 0, device=perm.device.index,
                 n_planes=len(planes), planes=ctypes.addressof(tab), mask=_ptr(mask), perm=_ptr(perm), inv=_ptr(inv),
                 index_map=_ptr(index_map), count=_ptr(count), span=_ptr(span),
                 fire=_ptr(fire) if fire is not None else 0, n=n)
    _abi.check(_abi.lib().eagle_backend_reorder_device(ctypes.byref(d)))  # query
    scratch = torch.empty(max(1, int(d.scratch_bytes)), dtype=torch.uint8, device=perm.device)
    d.scratch = _ptr(scratch)
    d.stream = _stream_handle(stream)
    _abi.check(_abi.lib().eagle_backend_reorder_device(ctypes.byref(d)))
    return scratch  # keep alive until the stream is past the call


def restore(planes, perm, inv, *, stream=None):
    """Undo every reorder since the last restore (``eagle_backend_x_restore_device``):
    each plane back in sample order, ``perm`` and ``inv`` the identity."""
    torch = _t()
    n = perm.numel()
    tab = _plane_table(planes)
    d = _abi.new(_abi.ReorderDesc, device=perm.device.index, n_planes=len(planes), planes=ctypes.addressof(tab),
                 perm=_ptr(perm), inv=_ptr(inv), n=n)
    _abi.check(_abi.lib().eagle_backend_x_restore_device(ctypes.byref(d)))  # query
    scratch = torch.empty(max(1, int(d.scratch_bytes)), dtype=torch.uint8, device=perm.device)
    d.scratch = _ptr(scratch)
    d.stream = _stream_handle(stream)
    _abi.check(_abi.lib().eagle_backend_x_restore_device(ctypes.byref(d)))
    return scratch


def reorder_classes(planes, mask, class_plane, perm, inv, index_map, count, span, offsets, class_sorts, classes: int,
                    *, fire=None, drop: bool = True, within: bool = False, stream=None):
    """Stable counting sort of ``planes`` in place by ``(live, class)`` over
    ``[0, span)`` (dead last), or by class over ``[0, count)`` with ``within``
    (eagle/filtering/ReorderClasses.h; ``eagle_backend_reorder_classes_device``).
    ``offsets`` (uint32[classes + 1]) receives each key's first slot; ``class_sorts``
    counts the sorts that ran. Enqueue only; returns the scratch to keep alive."""
    torch = _t()
    tab = _plane_table(planes)
    flags = (_abi.COMPACT_MASK_IS_DROP if drop else 0) | (_abi.CLASSES_WITHIN_LIVE if within else 0)
    d = _abi.new(_abi.ReorderClassesDesc, flags=flags, device=perm.device.index, n_planes=len(planes),
                 planes=ctypes.addressof(tab), mask=_ptr(mask), perm=_ptr(perm), inv=_ptr(inv),
                 index_map=_ptr(index_map), count=_ptr(count), span=_ptr(span),
                 fire=_ptr(fire) if fire is not None else 0, n=perm.numel(), class_plane=_ptr(class_plane),
                 classes=int(classes), offsets=_ptr(offsets), class_sorts=_ptr(class_sorts))
    _abi.check(_abi.lib().eagle_backend_reorder_classes_device(ctypes.byref(d)))  # query
    scratch = torch.empty(max(1, int(d.scratch_bytes)), dtype=torch.uint8, device=perm.device)
    d.scratch = _ptr(scratch)
    d.stream = _stream_handle(stream)
    _abi.check(_abi.lib().eagle_backend_reorder_classes_device(ctypes.byref(d)))
    return scratch
