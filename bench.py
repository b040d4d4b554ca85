"""Benchmark: sample-steps/s of eagle's until-done loop on the 16M-sample
heterogeneous-stop Euler oscillator, per GPU shard, with the HBM roofline figures.

Workload (one "step" = one until-done run of the whole batch, from its initial
state, then the canonical sum of the final x): n = 16,777,216 fp64 samples per GPU,
omega ~ U[1, 3], x ~ N(1, 0.1), v = t = 0, dt = 1e-3, t_end log-uniform in
[0.01, 10] per sample, max_steps = 10,000 (about 1446 steps per sample on average,
2.4e10 sample-steps per run). Synthetic, seeded (numpy default_rng: seed 1 omega,
2 x, 3 t_end; rank r > 0 uses [seed, r]). Under torchrun every rank runs its own
contiguous shard of N x 16M samples (weak scaling); the rank partials of the
canonical sum are all-gathered over NCCL and folded in rank order on the device.

``--impl reference`` times the CPU restatement of eagle's host path (the oracle,
OpenMP over all host cores) on a bounded prefix of the same workload.
"""

from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "sample-steps/s, 16M heterogeneous-stop oscillator; HBM GB/s vs roofline"
UNIT = "sample-steps/s"
N_PER_GPU = 1 << 24
MAX_STEPS = 10_000
DT = 1e-3
B_STEP = 66  # bytes one sample-step of eagle's unfused kernel reads and writes (omega, t_end, x, v, t, mask)
WORKLOAD = "euler-oscillator-heterogeneous-stop"


def _args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="engine", choices=("engine", "reference"))
    p.add_argument("--mode", default="auto", choices=("auto", "band", "band_eager", "persist", "fused"))
    p.add_argument("--n", type=int, default=None, help="samples per GPU (default: the workload's)")
    p.add_argument("--workload", default="oscillator",
                   choices=("oscillator", "lorenz", "gambler", "compact_sum", "compact", "reorder"),
                   help="oscillator: the headline 16M heterogeneous-stop run; the others time the other "
                        "configurations' kernels (Lorenz RKF7(8) 2^22, gambler's ruin 2^26, compact-then-sum "
                        "2^28, the active-set compaction alone 2^28, the physical reorder and the K-class "
                        "sort of 2^24) for their own lines")
    p.add_argument("--no-fma", action="store_true", help="exact (uncontracted) arithmetic profile")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--e2e-chunks", type=int, default=8)
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=15.0)
    return p.parse_args()


def _inputs(rank: int, n: int):
    def rng(seed):
        return np.random.default_rng(seed if rank == 0 else [seed, rank])

    omega = rng(1).uniform(1.0, 3.0, n)
    x0 = rng(2).normal(1.0, 0.1, n)
    t_end = 10.0 ** rng(3).uniform(-2.0, 1.0, n)
    return omega, x0, t_end


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            pk = json.load(f)
        return float(pk["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _fp64_peak():
    """FP64 lane-instructions per second of this GPU, in T/s: 64 FP64 lanes per SM per
    cycle x SMs x the measured max SM clock (no FP64 figure is measured on this pool)."""
    import torch

    props = torch.cuda.get_device_properties(0)
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            mhz = float(json.load(f)["sm_max_mhz"])
    except Exception:
        mhz = 1965.0
    return 64 * props.multi_processor_count * mhz * 1e6 / 1e12


class _Clocks:
    """SM clock and clock-event reasons sampled through NVML every 10 ms during the
    timed region (reading only; nothing is set)."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, cuda_index: int):
        self.cuda_index = cuda_index
        self.samples = []
        self.smax = None
        self._stop = threading.Event()
        self._thread = None

    def __enter__(self):
        try:
            import pynvml
            import torch

            p = torch.cuda.get_device_properties(self.cuda_index)
            ids = (p.pci_domain_id, p.pci_bus_id, p.pci_device_id)
            if not all(isinstance(v, int) and v >= 0 for v in ids):
                return self
            bus = "%08X:%02X:%02X.0" % ids  # NVML's PCI bus id string (torch gives the three numbers)
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            self.smax = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)

            def poll():
                while not self._stop.is_set():
                    try:
                        clk = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        reasons = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.samples.append((clk, reasons))
                    except Exception:
                        pass
                    self._stop.wait(0.01)

            self._thread = threading.Thread(target=poll, daemon=True)
            self._thread.start()
        except Exception:
            self._thread = None
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.smax, "reasons": [], "samples": 0}
        reasons = sorted(name for name, bit in self.REASONS.items() if any(r & bit for _, r in self.samples))
        return {"sm_mhz": statistics.median(c for c, _ in self.samples), "sm_max_mhz": self.smax,
                "reasons": reasons, "samples": len(self.samples)}


def _cpu_baseline(omega, x0, t_end, budget_s: float):
    """The oracle (CPU restatement of eagle's host path, OpenMP, all host threads)
    on a contiguous prefix of the workload sized to about ``budget_s`` seconds."""
    import oracle

    oracle.build()
    cores = oracle.threads()
    n = omega.size

    def run(m):
        st = [x0[:m].copy(), np.zeros(m), np.zeros(m), np.zeros(m, np.uint8)]
        t0 = time.perf_counter()
        _, fin, longest, total = oracle.oscillator_run(omega[:m], *st, t_end=t_end[:m], dt=DT, max_steps=MAX_STEPS,
                                                       steps_out=False)
        return total, time.perf_counter() - t0

    m = min(n, 1 << 16)
    total, sec = run(m)
    rate = total / max(sec, 1e-9)
    per_sample = total / m
    m = int(min(n, max(m, budget_s * rate / per_sample)))
    m = max(4096, m // 4096 * 4096) if m < n else n
    total, sec = run(m)
    return {"value": total / sec, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"the first {m} of the {n} samples of one GPU shard ({total} sample-steps, {sec:.2f} s), "
                      f"run to completion on {cores} OpenMP threads"}


def reference(args):
    """The CPU arm: the oracle on the host cores, on bounded samples of the workload."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    omega, x0, t_end = _inputs(0, args.n)
    import oracle

    oracle.build()
    cores = oracle.threads()
    per_step = max(2.0, 150.0 / max(1, args.steps + args.warmup))
    # size one step's prefix from a calibration run
    m = 1 << 16
    st = [x0[:m].copy(), np.zeros(m), np.zeros(m), np.zeros(m, np.uint8)]
    t0 = time.perf_counter()
    _, _, _, total = oracle.oscillator_run(omega[:m], *st, t_end=t_end[:m], dt=DT, max_steps=MAX_STEPS,
                                           steps_out=False)
    rate = total / max(time.perf_counter() - t0, 1e-9)
    m = int(min(args.n, max(4096, per_step * rate / (total / m))))
    m = m // 4096 * 4096 if m < args.n else args.n
    times, totals = [], []
    for i in range(args.warmup + args.steps):
        st = [x0[:m].copy(), np.zeros(m), np.zeros(m), np.zeros(m, np.uint8)]
        t0 = time.perf_counter()
        _, fin, longest, total = oracle.oscillator_run(omega[:m], *st, t_end=t_end[:m], dt=DT, max_steps=MAX_STEPS,
                                                       steps_out=False)
        s = oracle.reduce(st[0])
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(dt)
            totals.append(total)
    value = sum(totals) / sum(times)
    sample = (f"the first {m} of the {args.n} samples per GPU shard ({totals[0]} sample-steps per step), "
              f"{cores} OpenMP threads, each sample run to completion then the canonical sum of x")
    line = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(times) / len(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (seeded numpy)",
            "config": {"workload": WORKLOAD, "n_per_gpu": args.n, "max_steps": MAX_STEPS, "dt": DT,
                       "sampled_n": m},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def engine(args):
    import torch

    import eagle_b200 as eb
    from eagle_b200 import _abi

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    n = args.n
    mode = "persist" if args.mode == "auto" else args.mode
    fma = not args.no_fma
    omega, x0, t_end = _inputs(rank, n)
    dev = torch.device("cuda", local)
    d_om = torch.from_numpy(omega).to(dev)
    d_te = torch.from_numpy(t_end).to(dev)
    d_x0 = torch.from_numpy(x0).to(dev)
    x = torch.empty_like(d_x0)
    v = torch.zeros_like(d_x0)
    t = torch.zeros_like(d_x0)
    mask = torch.zeros(n, dtype=torch.uint8, device=dev)
    runner = eb.until_done(eb.oscillator, max_steps=MAX_STEPS, mode=mode, fma=fma, terminated=mask, omega=d_om,
                           t_end=d_te, dt=DT, x=x, v=v, t=t)
    red = eb.Reducer(x, pair_out=True)
    gathered = torch.zeros(2 * world, dtype=torch.float64, device=dev)
    combine_work = torch.zeros(2 * world + 2, dtype=torch.float64, device=dev)
    result = torch.zeros(3, dtype=torch.float64, device=dev)
    lib = _abi.lib()

    def step(stream):
        x.copy_(d_x0)
        v.zero_()
        t.zero_()
        mask.zero_()
        runner.launch(stream)
        red(stream)
        if dist is not None:
            dist.all_gather_into_tensor(gathered, red.out)
            src = gathered
        else:
            src = red.out
        _abi.check(lib.eagle_backend_x_b200_combine_partials(src.data_ptr(), world, combine_work.data_ptr(),
                                                             result.data_ptr(), stream.cuda_stream))

    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        step(stream)
    rep = runner.report(stream)  # raises if the device reported an error word
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with _Clocks(local) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            step(stream)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist is not None:
        dist.barrier()
    rep = runner.report(stream)
    steps_per_run = rep.step_sum
    # engine-only time per run (the dominant kernel's launches), for the roofline
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    eng_ms = []
    for _ in range(3):
        x.copy_(d_x0)
        v.zero_()
        t.zero_()
        mask.zero_()
        f0.record(stream)
        runner.launch(stream)
        f1.record(stream)
        torch.cuda.synchronize()
        eng_ms.append(f0.elapsed_time(f1))
    eng = statistics.median(eng_ms)
    mx = torch.tensor([ms, eng], dtype=torch.float64, device=dev)
    tot = torch.tensor([float(steps_per_run)], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
    ms, eng = float(mx[0]), float(mx[1])
    all_steps = float(tot[0])
    value = all_steps * args.steps / (ms / 1e3)

    # e2e: the same runs through the C-ABI with the inputs in pinned host memory
    e2e = None
    result_dev = result.cpu().numpy().copy()
    if not args.no_e2e:
        h_om = torch.from_numpy(omega).pin_memory()
        h_te = torch.from_numpy(t_end).pin_memory()
        h_x0 = torch.from_numpy(x0).pin_memory()
        h_zero = torch.zeros(n, dtype=torch.float64).pin_memory()
        h_res = torch.zeros(3, dtype=torch.float64).pin_memory()
        s = stream.cuda_stream
        plane_bytes = 8 * n

        staged = eb.StagedRunner(eb.oscillator, max_steps=MAX_STEPS, chunks=args.e2e_chunks, mode=mode, fma=fma,
                                 terminated=mask, omega=d_om, t_end=d_te, dt=DT, x=x, v=v, t=t)
        host = {"omega": h_om, "t_end": h_te, "x": h_x0, "v": h_zero, "t": h_zero}

        def e2e_step():
            staged.launch(host, stream)  # chunked copies in, each chunk stepped as soon as it lands
            red(stream)
            if dist is not None:
                dist.all_gather_into_tensor(gathered, red.out)
                src = gathered
            else:
                src = red.out
            _abi.check(lib.eagle_backend_x_b200_combine_partials(src.data_ptr(), world, combine_work.data_ptr(),
                                                                 result.data_ptr(), s))
            _abi.check(lib.eagle_backend_memcpy(h_res.data_ptr(), result.data_ptr(), 24, _abi.COPY_D2H, s))
            return staged.report(stream)  # the run report: one small device-to-host read per chunk

        for _ in range(max(1, args.warmup)):
            e2e_step()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for _ in range(args.steps):
            r2 = e2e_step()
        g1.record(stream)
        torch.cuda.synchronize()
        ems = torch.tensor([g0.elapsed_time(g1)], dtype=torch.float64, device=dev)
        if dist is not None:
            dist.all_reduce(ems, op=dist.ReduceOp.MAX)
        e2e = {"value": all_steps * args.steps / (float(ems[0]) / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": 5 * plane_bytes, "d2h_bytes_per_step": 24 + int(r2.report_bytes),
               "ms_per_step": float(ems[0]) / args.steps, "chunks": args.e2e_chunks,
               "path": "StagedRunner: pinned host planes copied in chunks on a copy stream, each chunk's "
                       "persistent run enqueued behind its copy; canonical sum, combine, result read back",
               "sum_matches_device_run": bool(np.array_equal(h_res.numpy(), result_dev))}

    if rank != 0:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return
    peak, peak_kind = _peaks()
    achieved = B_STEP * steps_per_run / (eng / 1e3) / 1e9
    passes = rep.launches
    # engine kernels (persist: mask count, the claim order, the persistent run), the sum, the combine
    launches_per_step = (passes + 2 if mode == "band" else 3 if mode == "persist" else 2) + 1 + 1
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        try:
            with open(tpath) as f:
                traffic = json.load(f).get(f"{mode}_{'fma' if fma else 'exact'}")
        except Exception:
            traffic = None
    # the physical bounds beside the effective figure: DRAM bytes per launch (ncu) over the
    # engine time, and FP64 issue -- 2 DFMA lane-instructions per sample-step on the known-stop
    # path (x and v; t is not added per step), one more (the t add) on the step-by-step one;
    # twice as many uncontracted
    fp64_per_step = (2 if fma else 4) + (0 if mode == "persist" else 1)
    fp64_peak = _fp64_peak()
    fp64_rate = fp64_per_step * steps_per_run / (eng / 1e3) / 1e12
    physical = {"dram_gbs": traffic / (eng / 1e3) / 1e9 if traffic else None,
                "fp64": {"achieved": fp64_rate, "peak": fp64_peak, "unit": "T FP64 lane-instructions/s",
                         "frac": fp64_rate / fp64_peak, "per_sample_step": fp64_per_step,
                         "peak_kind": "derived: 64 FP64 lanes per SM per cycle x SMs x the measured max SM clock"}}
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded numpy, see bench.py)",
        "config": {"workload": WORKLOAD, "n_per_gpu": n, "n_total": n * world, "max_steps": MAX_STEPS, "dt": DT,
                   "mode": mode, "arith": "fma" if fma else "exact", "sample_steps_per_gpu_step": steps_per_run,
                   "status": "finished" if rep.done else "max_steps", "passes": passes,
                   "l2": "inputs larger than L2 (5 x 128 MiB planes per GPU, re-initialised every step)",
                   "parallelism": f"shard{world}"},
        "e2e": e2e,
        "gpu_launches": launches_per_step * args.steps,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic, "peak_kind": peak_kind,
                     "basis": "66 B per sample-step (eagle's unfused per-step plane traffic) x sample-steps "
                              "per run / engine time per run; the fused kernel keeps state in registers, so "
                              "this effective figure exceeds the physical DRAM rate",
                     "physical": physical},
        "clocks": clocks.summary(),
    }
    res = result.cpu().numpy()
    line["result"] = {"sum_x": float(res[2]), "mean_x": float(res[2]) / (n * world),
                      "finished_rank0": rep.finished, "steps_rank0": rep.steps}
    if world == 1 and not args.no_cpu:
        line["cpu_baseline"] = _cpu_baseline(omega, x0, t_end, args.cpu_seconds)
    print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# ----------------------------------------------------------------- the other configurations

def _timed(fn, steps, warmup, stream, reset=None):
    """CUDA-event time of ``steps`` calls of ``fn`` after ``warmup`` (``reset`` runs
    before every call, inside the timed region, as a run's re-initialisation)."""
    import torch

    for _ in range(warmup):
        if reset:
            reset()
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        if reset:
            reset()
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def _profile_value(key):
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f).get(key)
    except Exception:
        return None


def side_workload(args):
    """One JSON line for the Lorenz, gambler or compact-then-sum configuration on
    one GPU, with its CPU baseline (the oracle on a bounded prefix)."""
    import torch

    import eagle_b200 as eb
    import oracle

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream()
    oracle.build()
    cores = oracle.threads()
    line = {"n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "data": "synthetic (seeded numpy, see bench.py)"}
    if args.workload == "lorenz":
        n = args.n or (1 << 22)
        rng = np.random.default_rng
        rho = rng(1).uniform(20.0, 40.0, n)
        xyz = [rng(s).normal(1.0, 0.1, n) for s in (2, 3, 4)]
        init = {"rho": rho, "x": xyz[0], "y": xyz[1], "z": xyz[2], "t": np.zeros(n), "h": np.full(n, 1e-3)}
        d0 = {k: torch.from_numpy(v).to(dev) for k, v in init.items()}
        planes = {k: v.clone() for k, v in d0.items()}
        planes["n_acc"] = torch.zeros(n, dtype=torch.int32, device=dev)
        planes["n_rej"] = torch.zeros(n, dtype=torch.int32, device=dev)
        mask = torch.zeros(n, dtype=torch.uint8, device=dev)
        prm = dict(sigma=10.0, beta=8.0 / 3.0, t_final=10.0, rtol=1e-9, atol=1e-12)
        runner = eb.until_done(eb.lorenz, max_steps=200_000, mode="persist", terminated=mask, **planes, **prm)
        red = eb.Reducer(planes["z"])

        def reset():
            for k in ("x", "y", "z", "t", "h"):
                planes[k].copy_(d0[k])
            planes["n_acc"].zero_()
            planes["n_rej"].zero_()
            mask.zero_()

        def step():
            runner.launch(stream)
            red(stream)

        with _Clocks(0) as clocks:
            ms = _timed(step, args.steps, args.warmup, stream, reset)
        rep = runner.report(stream)
        instr = _profile_value("lorenz_fp64_instr_per_attempt")
        achieved = instr * rep.step_sum / (ms / 1e3) / 1e12 if instr else None
        fp64_peak = _fp64_peak()
        m = min(n, 1 << 15)
        host = {k: v[:m].copy() for k, v in init.items()}
        na, nr, term = np.zeros(m, np.uint32), np.zeros(m, np.uint32), np.zeros(m, np.uint8)
        t0 = time.perf_counter()
        _, _, total = oracle.lorenz_run(host["rho"], host["x"], host["y"], host["z"], host["t"], host["h"], na, nr,
                                        term, max_steps=200_000, **prm)
        sec = time.perf_counter() - t0
        line.update({"metric": "attempts/s, 4M-sample Lorenz-63 adaptive RKF7(8)", "value": rep.step_sum / (ms / 1e3),
                     "unit": "attempts/s", "ms_per_step": ms, "dtype": "f64",
                     "config": {"workload": "lorenz63-rkf78", "n": n, "max_steps": 200_000, **prm, "h0": 1e-3,
                                "attempts_per_run": rep.step_sum, "longest": rep.steps,
                                "status": "finished" if rep.done else "max_steps",
                                "l2": "state 8 planes x 32 MiB, re-initialised every step (the kernel is FP64-bound)"},
                     "result": {"sum_z": float(red.out[0].item())},
                     "roofline": {"bound": "fp64", "achieved": achieved, "peak": fp64_peak,
                                  "unit": "T FP64 lane-instructions/s",
                                  "frac": achieved / fp64_peak if achieved else None, "traffic": None,
                                  "peak_kind": "derived: 64 FP64 lanes per SM per cycle x SMs x the measured max SM "
                                               "clock (no FP64 figure is measured on this pool)",
                                  "basis": "FP64 thread instructions per attempt counted by ncu (profiles/"
                                           "traffic.json) x attempts per run / run time"},
                     "cpu_baseline": {"value": total / sec, "unit": "attempts/s", "cores": cores, "kind": "port",
                                      "sample": f"the first {m} samples run to t_final ({total} attempts, {sec:.2f} s)"},
                     "gpu_launches": 4 * args.steps, "clocks": clocks.summary()})
    elif args.workload == "gambler":
        n = args.n or (1 << 26)
        pos0 = np.random.default_rng(1).integers(1, 100, n).astype(np.int32)
        seed = 2026
        d_pos0 = torch.from_numpy(pos0).to(dev)
        pos, tm = d_pos0.clone(), torch.zeros(n, dtype=torch.int64, device=dev)
        mask = torch.zeros(n, dtype=torch.uint8, device=dev)
        runner = eb.until_done(eb.gambler, max_steps=1_000_000, mode="persist", terminated=mask, pos=pos, time=tm,
                               seed=seed)
        red = eb.Reducer(tm)

        def reset():
            pos.copy_(d_pos0)
            tm.zero_()
            mask.zero_()

        def step():
            runner.launch(stream)
            red(stream)

        with _Clocks(0) as clocks:
            ms = _timed(step, args.steps, args.warmup, stream, reset)
        rep = runner.report(stream)
        m = min(n, 1 << 18)
        hp, ht, term = pos0[:m].copy(), np.zeros(m, np.int64), np.zeros(m, np.uint8)
        t0 = time.perf_counter()
        _, _, total = oracle.gambler_run(hp, ht, term, seed=seed, max_steps=1_000_000)
        sec = time.perf_counter() - t0
        line.update({"metric": "sample-steps/s, 64M gambler's-ruin walk (Philox-4x32-10)",
                     "value": rep.step_sum / (ms / 1e3), "unit": "sample-steps/s", "ms_per_step": ms,
                     "dtype": "int32 position, int64 time",
                     "config": {"workload": "gamblers-ruin-philox", "n": n, "max_steps": 1_000_000, "seed": seed,
                                "absorb": [0, 100], "sample_steps_per_run": rep.step_sum, "longest": rep.steps,
                                "status": "finished" if rep.done else "max_steps",
                                "l2": "inputs 768 MiB, re-initialised every step"},
                     "result": {"sum_time": int(red.out[0].item()), "mean_time": float(red.out[0].item()) / n},
                     "roofline": {"bound": "integer ALU", "achieved": None, "peak": None, "unit": None,
                                  "frac": None, "traffic": None,
                                  "basis": "Philox-4x32-10 per 128 steps plus a compare per step: integer-issue "
                                           "bound; the ncu pipe shares are in profiles/"},
                     "cpu_baseline": {"value": total / sec, "unit": "sample-steps/s", "cores": cores, "kind": "port",
                                      "sample": f"the first {m} samples run to absorption ({total} steps, {sec:.2f} s)"},
                     "gpu_launches": 4 * args.steps, "clocks": clocks.summary()})
    elif args.workload == "reorder":
        n = args.n or (1 << 24)
        g = np.random.default_rng(11)
        names = ("omega", "t_end", "x", "v", "t")
        planes = [torch.from_numpy(g.standard_normal(n)).to(dev) for _ in names]
        mask0 = torch.from_numpy((g.random(n) < 0.5).astype(np.uint8)).to(dev)
        cls0 = torch.from_numpy(g.integers(0, 8, n).astype(np.uint8)).to(dev)
        mask, cls = mask0.clone(), cls0.clone()
        perm = torch.arange(n, dtype=torch.int32, device=dev)
        inv = perm.clone()
        im = torch.zeros(n, dtype=torch.int32, device=dev)
        cells = torch.zeros(8, dtype=torch.int32, device=dev)
        offsets = torch.zeros(9, dtype=torch.int32, device=dev)
        count, span, sorts = cells[0:1], cells[1:2], cells[2:3]
        every = planes + [mask, cls]

        def reset():
            eb.restore(every, perm, inv)
            span.fill_(n)

        times = {"reorder": [], "classes": []}
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with _Clocks(0) as clocks:
            for step in range(args.warmup + args.steps):
                for kind in ("reorder", "classes"):
                    reset()
                    torch.cuda.synchronize()
                    e0.record(stream)
                    if kind == "reorder":
                        keep = eb.reorder(every, mask, perm, inv, im, count, span, stream=stream)
                    else:
                        keep = eb.reorder_classes(every, mask, cls, perm, inv, im, count, span, offsets, sorts, 8,
                                                  stream=stream)
                    e1.record(stream)
                    torch.cuda.synchronize()
                    if step >= args.warmup:
                        times[kind].append(e0.elapsed_time(e1))
                    del keep
        ms = {k: statistics.median(v) for k, v in times.items()}
        # the in-place minimum: every moved plane read once and written once, the mask (and the class plane)
        # read for the keys, perm read and written, inv and index_map written
        moved = 5 * 8 + 1 + 1
        alg = {"reorder": n * (2 * moved + 1 + 8 + 4 + 4 * 0.5),
               "classes": n * (2 * moved + 2 + 8 + 4 + 4 * 0.5)}
        peak, peak_kind = _peaks()
        rate = {k: alg[k] / (ms[k] / 1e3) / 1e9 for k in ms}
        m = min(n, 1 << 22)
        hp = [p[:m].cpu().numpy().copy() for p in planes] + [mask0[:m].cpu().numpy().copy(),
                                                            cls0[:m].cpu().numpy().copy()]
        hperm, hinv, him = np.arange(m, dtype=np.int32), np.arange(m, dtype=np.int32), np.zeros(m, np.int32)
        t0 = time.perf_counter()
        oracle.reorder(hp, 5, hperm, hinv, him, m)
        sec = time.perf_counter() - t0
        line.update({"metric": "GB/s, 2^24-slot physical reorder (5 f64 planes + mask + class plane) vs HBM",
                     "value": rate["reorder"], "unit": "GB/s", "ms_per_step": ms["reorder"] + ms["classes"],
                     "dtype": "f64 planes, u8 mask and class, int32 perm",
                     "config": {"workload": "physical-reorder", "n": n, "p_keep": 0.5, "classes": 8,
                                "reorder_ms": ms["reorder"], "class_sort_ms": ms["classes"],
                                "class_sort_GBps": rate["classes"],
                                "l2": "7 planes of 16-128 MiB, restored to sample order before every timed call"},
                     "roofline": {"bound": "hbm", "achieved": rate["reorder"], "peak": peak, "unit": "GB/s",
                                  "frac": rate["reorder"] / peak, "traffic": None, "peak_kind": peak_kind,
                                  "basis": "the in-place minimum: each moved plane read and written once, the keys "
                                           "read, perm read and written, inv and index_map written; the stage copy "
                                           "that makes the move in place doubles the plane traffic by design"},
                     "cpu_baseline": {"value": m * (2 * moved + 13) / sec / 1e9, "unit": "GB/s", "cores": 1,
                                      "kind": "port", "sample": f"the first {m} slots, numpy stable partition "
                                                                f"({sec:.2f} s)"},
                     "gpu_launches": (2 + 2 * 8 + 1) + (3 + 2 * 8 + 2), "clocks": clocks.summary()})
    elif args.workload == "compact":
        # the active-set compaction alone (compact_device: ascending index map + count),
        # 2^28 samples, keep masks Bernoulli(p), p in {0.9, 0.5, 0.1, 0.01} (seeds 7 + i)
        n = args.n or (1 << 28)
        ps = (0.9, 0.5, 0.1, 0.01)
        masks = [torch.from_numpy(np.random.default_rng(7 + i).random(n) < p).to(dev) for i, p in enumerate(ps)]
        comps = [eb.Compactor(mk, drop=False) for mk in masks]
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # 256 MiB: evicts the 126 MB L2

        def step():
            for c in comps:
                flush.zero_()
                c(stream)

        with _Clocks(0) as clocks:
            ms = _timed(step, args.steps, args.warmup, stream)
        flush_ms = _timed(lambda: [flush.zero_() for _ in ps], 3, 1, stream)
        work_ms = max(ms - flush_ms, 1e-6)
        counts = [int(c.count.item()) for c in comps]
        alg = sum(n + 4 * k for k in counts)  # the mask read, the index map written
        peak, peak_kind = _peaks()
        m = min(n, 1 << 24)
        t0 = time.perf_counter()
        for i, p in enumerate(ps):
            oracle.compact(np.random.default_rng(7 + i).random(m) < p, drop=False)
        sec = time.perf_counter() - t0
        kept_sample = sum(int(m * p) for p in ps)
        line.update({"metric": "GB/s, 2^28 active-set compaction vs the HBM roofline",
                     "value": alg / (work_ms / 1e3) / 1e9, "unit": "GB/s", "ms_per_step": ms,
                     "dtype": "u8 mask, int32 map",
                     "config": {"workload": "active-set-compaction", "n": n, "p": list(ps), "kept": counts,
                                "l2": "a 256 MiB buffer is written before every compaction (its time is measured "
                                      "apart and taken out)", "flush_ms_per_step": flush_ms},
                     "roofline": {"bound": "hbm", "achieved": alg / (work_ms / 1e3) / 1e9, "peak": peak,
                                  "unit": "GB/s", "frac": alg / (work_ms / 1e3) / 1e9 / peak, "traffic": None,
                                  "peak_kind": peak_kind,
                                  "basis": "n mask bytes read + 4 bytes per kept index written, summed over the "
                                           "four masks / compaction time"},
                     "cpu_baseline": {"value": (4 * m + 4 * kept_sample) / sec / 1e9, "unit": "GB/s",
                                      "cores": 1, "kind": "port",
                                      "sample": f"the first {m} samples of each mask ({sec:.2f} s)"},
                     "gpu_launches": 4 * args.steps, "clocks": clocks.summary()})
    else:
        n = args.n or (1 << 28)
        rng = np.random.default_rng(4)
        vals = rng.standard_normal(n)
        big = np.random.default_rng(5).choice(n, size=max(1, n // 1_000_000), replace=False)
        sign = np.where(np.random.default_rng(6).random(big.size) < 0.5, -1.0, 1.0)
        vals[big] = sign * 1e12
        x = torch.from_numpy(vals).to(dev)
        ps = (0.9, 0.5, 0.1, 0.01)
        masks = [torch.from_numpy(np.random.default_rng(7 + i).random(n) < p).to(dev) for i, p in enumerate(ps)]
        sums = [eb.CompactSum(mk, x) for mk in masks]
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # 256 MiB: evicts the 126 MB L2

        def step():
            for cs in sums:
                flush.zero_()
                cs(stream)

        with _Clocks(0) as clocks:
            ms = _timed(step, args.steps, args.warmup, stream)
        flush_ms = _timed(lambda: [flush.zero_() for _ in ps], 3, 1, stream)
        work_ms = max(ms - flush_ms, 1e-6)
        counts = [int(cs.count.item()) for cs in sums]
        alg = sum(n + 8 * n * (1 - (1 - p) ** 4) for p in ps)  # mask + every 32 B value sector with a survivor
        peak, peak_kind = _peaks()
        m = min(n, 1 << 24)
        t0 = time.perf_counter()
        for i, p in enumerate(ps):
            keep = np.random.default_rng(7 + i).random(m) < p
            idx, _ = oracle.compact(keep, drop=False)
            oracle.reduce(vals[:m][idx])
        sec = time.perf_counter() - t0
        line.update({"metric": "GB/s, 2^28 compact-then-sum vs the HBM roofline", "value": alg / (work_ms / 1e3) / 1e9,
                     "unit": "GB/s", "ms_per_step": ms, "dtype": "f64 values, u8 mask",
                     "config": {"workload": "compact-then-sum", "n": n, "p": list(ps), "kept": counts,
                                "l2": "a 256 MiB buffer is written before every compaction (its time is measured "
                                      "apart and taken out)", "flush_ms_per_step": flush_ms},
                     "result": {"sums": [float(cs.out[0].item()) for cs in sums]},
                     "roofline": {"bound": "hbm", "achieved": alg / (work_ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                                  "frac": alg / (work_ms / 1e3) / 1e9 / peak, "traffic": None, "peak_kind": peak_kind,
                                  "basis": "n mask bytes + 8 n (1 - (1 - p)^4) value bytes per mask (the sectors "
                                           "holding a survivor), summed over the four masks / compaction time"},
                     "cpu_baseline": {"value": 4 * (m + 8 * m) / sec / 1e9, "unit": "GB/s", "cores": cores,
                                      "kind": "port",
                                      "sample": f"the first {m} samples of each mask: compaction then canonical "
                                                f"sum ({sec:.2f} s; mask + values read)"},
                     "gpu_launches": 4 * 2 * args.steps, "clocks": clocks.summary()})
    print(json.dumps(line), flush=True)


def main():
    args = _args()
    if args.workload != "oscillator":
        side_workload(args)
        return
    if args.n is None:
        args.n = N_PER_GPU
    if args.impl == "reference":
        reference(args)
    else:
        engine(args)


if __name__ == "__main__":
    main()
