"""Test infrastructure: NumPy face of the CPU restatement in ``oracle.cpp``.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
import this package; the engine in ``eagle_b200`` never does. Each function says
which part of eagle it restates (paths relative to the eagle source tree).
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

F32, F64, I32, I64, U8 = 0, 1, 2, 3, 4
OP_SUM, OP_MAX, OP_ALL, OP_MIN = 0, 1, 2, 3
MASK_IS_DROP = 1
_DTYPE_CODE = {np.dtype(np.float32): F32, np.dtype(np.float64): F64, np.dtype(np.int32): I32,
               np.dtype(np.int64): I64, np.dtype(np.uint8): U8, np.dtype(np.bool_): U8}
_OPS = {"sum": OP_SUM, "max": OP_MAX, "all": OP_ALL, "min": OP_MIN}

_P = ctypes.c_void_p
_I64 = ctypes.c_int64


def build() -> str:
    """Compile ``liboracle.so`` with the committed Makefile (g++ -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.oracle_threads.argtypes = [ctypes.c_int]
        L.oracle_reduce.argtypes = [_P, _I64, _I64, ctypes.c_int, ctypes.c_int, _P, _P, ctypes.c_int]
        L.oracle_leaf_partials_f64.argtypes = [_P, _I64, _P]
        L.oracle_reduce_fixed.argtypes = [_P, _I64, _I64, _P, _P]
        L.oracle_ladder.argtypes = [_I64, ctypes.c_int, ctypes.c_int, _P, _P]
        L.oracle_leaf_partials_f64.restype = _I64
        L.oracle_pairwise_f64.argtypes = [_P, _I64, _P]
        L.oracle_partial_value_f64.argtypes = [ctypes.c_double, ctypes.c_double]
        L.oracle_partial_value_f64.restype = ctypes.c_double
        L.oracle_compact.argtypes = [_P, _I64, ctypes.c_uint32, _P, _P, ctypes.c_uint32, ctypes.c_float, _P, _P]
        L.oracle_mask_count.argtypes = [_P, _I64]
        L.oracle_mask_count.restype = ctypes.c_uint32
        L.oracle_band_k.argtypes = [ctypes.c_double, _I64, _I64, _I64, _I64, _I64]
        L.oracle_band_k.restype = _I64
        L.oracle_policy_step.argtypes = [ctypes.c_uint32, ctypes.c_uint32, _P, _P, _P, _P, _I64, _I64] + \
            [ctypes.c_int] * 7
        L.oracle_oscillator_run.argtypes = [_I64, _P, _P, ctypes.c_double, ctypes.c_double, _P, _P, _P, _P, _P,
                                            _I64, ctypes.c_int, _I64, _P]
        L.oracle_philox4x32_10.argtypes = [_P, ctypes.c_uint64, _P]
        L.oracle_gambler_run.argtypes = [_I64, _P, _P, _P, _I64, ctypes.c_uint64, _I64, _P]
        L.oracle_det_pow.argtypes = [ctypes.c_double, ctypes.c_double]
        L.oracle_det_pow.restype = ctypes.c_double
        L.oracle_lorenz_stages.argtypes = [_P, ctypes.c_double, ctypes.c_double, ctypes.c_double, ctypes.c_double,
                                           ctypes.c_double, ctypes.c_double, _P, _P, _P]
        L.oracle_lorenz_run.argtypes = [_I64, _P] + [ctypes.c_double] * 5 + [_P] * 8 + [_I64, _P]
        L.oracle_corpus_f64.argtypes = [_I64, ctypes.c_uint64, _P]
        L.oracle_corpus_f32.argtypes = [_I64, ctypes.c_uint64, _P]
        L.oracle_fixture_f64.argtypes = [_I64, ctypes.c_double, _P, _P]
        L.oracle_fixture_f64.restype = ctypes.c_double
        L.oracle_fixture_f32.argtypes = [_I64, ctypes.c_double, _P, _P]
        L.oracle_fixture_f32.restype = ctypes.c_double
        _lib = L
    return _lib


def _ptr(a) -> int:
    return 0 if a is None else a.ctypes.data


def threads(n: int = 0) -> int:
    """Set (n > 0) and return the OpenMP team size."""
    return lib().oracle_threads(int(n))


def reduce(x, op: str = "sum", *, columns: int = 1, comp=None, pair_out: bool = False):
    """The canonical ``ordered`` reduction (eagle/reduce/canonical.h:10-32, :340-408)
    of each column of the row-major ``(n, columns)`` array ``x``."""
    x = np.ascontiguousarray(x)
    code = _DTYPE_CODE[x.dtype]
    if x.dtype == np.bool_:
        x = x.view(np.uint8)
    n = x.size // columns
    out = np.zeros(columns * (2 if pair_out else 1), dtype=x.dtype)
    c = None if comp is None else np.ascontiguousarray(comp, dtype=x.dtype)
    rc = lib().oracle_reduce(_ptr(x), n, columns, code, _OPS[op], _ptr(c), _ptr(out), int(pair_out))
    if rc != 0:
        raise ValueError(f"oracle_reduce refused (status {rc})")
    return out


def leaf_partials(x):
    """Per-leaf (hi, comp) partials of a float64 sum, leaf order: shape (leaves, 2)."""
    x = np.ascontiguousarray(x, dtype=np.float64)
    m = (x.size + 4095) // 4096
    hc = np.zeros((m, 2), dtype=np.float64)
    lib().oracle_leaf_partials_f64(_ptr(x), x.size, _ptr(hc))
    return hc


def pairwise(hc):
    """Level-by-level pairwise root of (hi, comp) partials (canonical.h:358-381)."""
    hc = np.ascontiguousarray(hc, dtype=np.float64).reshape(-1, 2)
    root = np.zeros(2, dtype=np.float64)
    lib().oracle_pairwise_f64(_ptr(hc), hc.shape[0], _ptr(root))
    return root


def partial_value(h: float, c: float) -> float:
    return lib().oracle_partial_value_f64(h, c)


def compact(mask, *, drop: bool = True, span: int = 0, theta: float = 0.0, trigger: bool = False):
    """Ascending map of the kept samples and its count (eagle/filtering/Compact.h:23-47);
    with ``trigger`` also ``(live32, fire)`` (Compact.h:113-118)."""
    m = np.ascontiguousarray(mask).view(np.uint8) if np.asarray(mask).dtype == np.bool_ \
        else np.ascontiguousarray(mask, dtype=np.uint8)
    n = m.size
    index_map = np.zeros(max(n, 1), dtype=np.int32)
    count = np.zeros(1, dtype=np.uint32)
    live32 = np.zeros(1, dtype=np.uint32) if trigger else None
    fire = np.zeros(1, dtype=np.uint32) if trigger else None
    rc = lib().oracle_compact(_ptr(m), n, MASK_IS_DROP if drop else 0, _ptr(index_map), _ptr(count), span,
                              theta, _ptr(live32), _ptr(fire))
    if rc != 0:
        raise ValueError(f"oracle_compact refused (status {rc})")
    c = int(count[0])
    if trigger:
        return index_map[:c].copy(), c, int(live32[0]), int(fire[0])
    return index_map[:c].copy(), c


def mask_count(mask) -> int:
    m = np.ascontiguousarray(mask).view(np.uint8)
    return int(lib().oracle_mask_count(_ptr(m), m.size))


def band_k(rate, newly, live, k, k_max, k_min=8) -> int:
    """eagle/policy/Launch.h:184-190."""
    return int(lib().oracle_band_k(float(rate), int(newly), int(live), int(k), int(k_max), int(k_min)))


def policy_step(finished, total, cells, word, go, hist, k_min, k_max, idx=(0, 1, 2, 3, 4, 5), scale=1000):
    """One POLICY cell op (python/src/plugin/eagle_cuda.cu:1990-2025) on int64 host cells, in place."""
    lib().oracle_policy_step(int(finished), int(total), _ptr(cells), _ptr(word), _ptr(go), _ptr(hist),
                             int(k_min), int(k_max), *[int(i) for i in idx], int(scale))


def oscillator_run(omega, x, v, t, terminated, *, t_end, dt, max_steps, fused=False, tile=1024,
                   steps_out=True):
    """Run every live sample of the README Euler oscillator (README.md:89-97) until its
    ``t >= t_end`` or ``max_steps`` steps, in place. ``t_end`` is a number (a Param) or a
    per-sample array. Returns ``(steps_per_sample or None, finished, longest, total)``."""
    n = omega.size
    for a in (omega, x, v, t):
        assert a.dtype == np.float64 and a.flags.c_contiguous and a.size == n
    assert terminated.dtype in (np.uint8, np.bool_) and terminated.size == n
    te_arr = None
    te_uniform = 0.0
    if np.ndim(t_end) == 0:
        te_uniform = float(t_end)
    else:
        te_arr = np.ascontiguousarray(t_end, dtype=np.float64)
    steps = np.zeros(n, dtype=np.int32) if steps_out else None
    stats = np.zeros(3, dtype=np.int64)
    rc = lib().oracle_oscillator_run(n, _ptr(omega), _ptr(te_arr), te_uniform, float(dt), _ptr(x), _ptr(v),
                                     _ptr(t), _ptr(terminated.view(np.uint8)), _ptr(steps), int(max_steps),
                                     int(bool(fused)), int(tile), _ptr(stats))
    if rc != 0:
        raise ValueError(f"oracle_oscillator_run refused (status {rc})")
    return steps, int(stats[0]), int(stats[1]), int(stats[2])


def corpus(n: int, seed: int, dtype=np.float64):
    """The adversarial corpus of eagle's reduction tests (tests/CanonicalReduceCases.h:49-60):
    normal values scaled by 10^U{-8..8}, std::mt19937_64(seed)."""
    out = np.zeros(n, dtype=dtype)
    if dtype == np.float64:
        lib().oracle_corpus_f64(n, seed, _ptr(out))
    else:
        lib().oracle_corpus_f32(n, seed, _ptr(out))
    return out


def reduce_fixed(x, *, columns: int = 1, comp=None):
    """eagle's fixed-point float64 sum (eagle/reduce/canonical.h:153-302): the canonical
    tree over 128-bit fixed-point partials, one value per column of the row-major
    ``(n, columns)`` array ``x`` -- what eagle computes on a device whose FP32:FP64
    ratio is 8 or worse (canonical.h:304-313)."""
    x = np.ascontiguousarray(x, dtype=np.float64)
    n = x.size // columns
    out = np.zeros(columns, dtype=np.float64)
    c = None if comp is None else np.ascontiguousarray(comp, dtype=np.float64)
    rc = lib().oracle_reduce_fixed(_ptr(x), n, columns, _ptr(c), _ptr(out))
    if rc != 0:
        raise ValueError(f"oracle_reduce_fixed refused (status {rc})")
    return out


def fixed_leaf(fp32_per_fp64: int) -> bool:
    """Whether eagle reduces float64 sums on the fixed-point leaf on a device with
    this FP32:FP64 throughput ratio (canonical.h:304-313: 8 or worse)."""
    return fp32_per_fp64 >= 8


def ladder(n: int, er: int, g: int):
    """The cancellation ladder of eagle's fixed-point tests
    (tests/test_CanonicalReduce.cu:88-119): returns (values, exact sum in units of 2^-10)."""
    x = np.zeros(n, dtype=np.float64)
    units = np.zeros(1, dtype=np.int64)
    lib().oracle_ladder(n, int(er), int(g), _ptr(x), _ptr(units))
    return x, int(units[0])


def fixture(n: int, kappa: float, dtype=np.float64):
    """The exact-sum fixture of eagle's reduction tests (tests/CanonicalReduceCases.h:141-176):
    returns (values, exact sum, reached condition number)."""
    x = np.zeros(n, dtype=dtype)
    reached = np.zeros(1, dtype=np.float64)
    f = lib().oracle_fixture_f64 if dtype == np.float64 else lib().oracle_fixture_f32
    exact = f(n, float(kappa), _ptr(x), _ptr(reached))
    return x, float(exact), float(reached[0])


def philox4x32_10(counter, seed: int):
    """Philox-4x32-10 (Salmon et al., SC'11) of a 4-word counter under a 64-bit seed."""
    c = np.ascontiguousarray(counter, dtype=np.uint32)
    out = np.zeros(4, dtype=np.uint32)
    lib().oracle_philox4x32_10(_ptr(c), int(seed), _ptr(out))
    return out


def lorenz_stages(s0, step, *, rho, sigma, beta, rtol, atol):
    """The scheme of one RKF7(8) attempt of Lorenz-63 from ``s0`` with ``step``
    (benchmarks/perf_card/perf_card.py:289-309 rkf78_stages and error_ratio, with
    Lorenz's right-hand side): ``(s8, err, ratio)``."""
    s = np.ascontiguousarray(s0, dtype=np.float64)
    s8 = np.zeros(3)
    err = np.zeros(3)
    ratio = np.zeros(1)
    lib().oracle_lorenz_stages(_ptr(s), float(step), float(rho), float(sigma), float(beta), float(rtol),
                               float(atol), _ptr(s8), _ptr(err), _ptr(ratio))
    return s8, err, float(ratio[0])


def curand_philox4x32_10(counters, keys):
    """cuRAND's Philox-4x32-10 (``curand_Philox4x32_10`` of its device API) of each
    row of ``counters`` (n x 4 uint32) under the key in the same row of ``keys``
    (n x 2 uint32), computed on the GPU: the check of :func:`philox4x32_10`. Needs a
    CUDA device."""
    c = np.ascontiguousarray(counters, dtype=np.uint32).reshape(-1, 4)
    k = np.ascontiguousarray(keys, dtype=np.uint32).reshape(-1, 2)
    if c.shape[0] != k.shape[0]:
        raise ValueError("one key per counter")
    path = os.path.join(_HERE, "libcurand_philox.so")
    if not os.path.exists(path):
        build()
    L = ctypes.CDLL(path)
    L.curand_philox_ref.argtypes = [_P, _P, _P, ctypes.c_int]
    out = np.zeros_like(c)
    err = L.curand_philox_ref(_ptr(c), _ptr(k), _ptr(out), int(c.shape[0]))
    if err != 0:
        raise RuntimeError(f"curand_philox_ref: CUDA error {err}")
    return out


def gambler_run(pos, time, terminated, *, seed: int, max_steps: int, id_base: int = 0):
    """Every live sample's walk until it reaches 0 or 100 or has taken ``max_steps``
    steps in this run, in place. Returns ``(finished, longest, total)``."""
    n = pos.size
    assert pos.dtype == np.int32 and time.dtype == np.int64 and terminated.dtype in (np.uint8, np.bool_)
    stats = np.zeros(3, dtype=np.int64)
    rc = lib().oracle_gambler_run(n, _ptr(pos), _ptr(time), _ptr(terminated.view(np.uint8)), int(id_base),
                                  int(seed), int(max_steps), _ptr(stats))
    if rc != 0:
        raise ValueError(f"oracle_gambler_run refused (status {rc})")
    return int(stats[0]), int(stats[1]), int(stats[2])


def det_pow(r: float, e: float) -> float:
    """The controller's deterministic power r^e (ln by the atanh series, exp by Taylor)."""
    return lib().oracle_det_pow(float(r), float(e))


LORENZ = dict(sigma=10.0, beta=8.0 / 3.0, t_final=10.0, rtol=1e-9, atol=1e-12)


def lorenz_run(rho, x, y, z, t, h, n_acc, n_rej, terminated, *, max_steps, sigma=10.0, beta=8.0 / 3.0,
               t_final=10.0, rtol=1e-9, atol=1e-12):
    """Adaptive RKF7(8) attempts of Lorenz-63 (benchmarks/perf_card/perf_card.py:131-348
    with the Lorenz right-hand side) until t reaches t_final or ``max_steps`` attempts,
    in place. Returns ``(finished, longest, total)`` in attempts."""
    n = rho.size
    for a in (rho, x, y, z, t, h):
        assert a.dtype == np.float64 and a.flags.c_contiguous and a.size == n
    assert n_acc.dtype == np.uint32 and n_rej.dtype == np.uint32
    stats = np.zeros(3, dtype=np.int64)
    rc = lib().oracle_lorenz_run(n, _ptr(rho), sigma, beta, t_final, rtol, atol, _ptr(x), _ptr(y), _ptr(z), _ptr(t),
                                 _ptr(h), _ptr(n_acc), _ptr(n_rej), _ptr(terminated.view(np.uint8)), int(max_steps),
                                 _ptr(stats))
    if rc != 0:
        raise ValueError(f"oracle_lorenz_run refused (status {rc})")
    return int(stats[0]), int(stats[1]), int(stats[2])


def reorder(planes, mask_plane: int, perm, inv, index_map, span: int, *, drop: bool = True, fire=None):
    """The physical reorder of eagle/filtering/Reorder.h (reorderDst :171-175; the
    stage / place / fin kernels :177-430): over slots [0, span) the kept samples move
    to [0, count) in ascending order and the dropped ones follow in ascending order,
    every plane (the mask among them, ``planes[mask_plane]``) and ``perm`` in place;
    ``inv[perm[s]] = s`` for the moved slots; ``index_map[0:count]`` is the identity.
    With ``fire == 0`` nothing happens. Returns ``(count, span, fire)`` after."""
    if fire is not None and fire == 0:
        return None, span, fire
    n = perm.size
    sp = min(int(span), n)
    mask = planes[mask_plane][:sp].copy()
    keep = (mask == 0) if drop else (mask != 0)
    order = np.concatenate([np.flatnonzero(keep), np.flatnonzero(~keep)])
    for p in planes:
        p[:sp] = p[:sp][order]
    perm[:sp] = perm[:sp][order]
    inv[perm[:sp]] = np.arange(sp, dtype=inv.dtype)
    cnt = int(keep.sum())
    index_map[:cnt] = np.arange(cnt, dtype=index_map.dtype)
    return cnt, cnt, (0 if fire is not None else None)


def restore(planes, perm, inv):
    """Reorder.h restoreDevice (:612-629): each plane back in sample order
    (``plane[perm[s]] = stage[s]``), then ``perm`` and ``inv`` the identity."""
    for p in planes:
        stage = p.copy()
        p[perm] = stage
    perm[:] = np.arange(perm.size, dtype=perm.dtype)
    inv[:] = np.arange(inv.size, dtype=inv.dtype)


def class_key(mask, cls, classes: int, *, drop: bool = True, within: bool = False):
    """ReorderClasses.h classKey (:58-67): the class clamped to K-1; with ``within``
    that alone, else K for a dead sample (dead sorts last)."""
    cc = np.minimum(cls.astype(np.int64), classes - 1)
    if within:
        return cc
    live = (mask == 0) if drop else (mask != 0)
    return np.where(live, cc, classes)


def reorder_classes(planes, mask_plane: int, class_plane: int, perm, inv, index_map, count: int, span: int,
                    classes: int, *, drop: bool = True, within: bool = False, fire=None):
    """ReorderClasses.h reorderClassesHost (:303-360): a stable counting sort of slots
    [0, lim) by key (lim = count within the live prefix, else span), every plane and
    perm in place; inv rebuilt for the moved slots; index_map the identity over the
    live samples; offsets[0..K] the keys' first slots. Returns
    ``(offsets, count, span, fire, sorted)``."""
    if fire is not None and fire == 0:
        return None, count, span, fire, False
    n = perm.size
    lim = min(int(count if within else span), n)
    key = class_key(planes[mask_plane][:lim], planes[class_plane][:lim], classes, drop=drop, within=within)
    order = np.argsort(key, kind="stable")
    nkeys = classes if within else classes + 1
    counts = np.bincount(key, minlength=nkeys)
    off = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    for p in planes:
        p[:lim] = p[:lim][order]
    perm[:lim] = perm[:lim][order]
    inv[perm[:lim]] = np.arange(lim, dtype=inv.dtype)
    live = int(count) if within else int(off[classes])
    index_map[:live] = np.arange(live, dtype=index_map.dtype)
    offsets = off[:classes + 1].copy()
    if not within:
        count = span = live
    return offsets, count, span, (0 if fire is not None else None), True


def class_trigger(mask, cls, *, drop: bool, live32: int, span: int, count: int, live_fire: int, class_theta: float,
                  stale: int = 0):
    """ReorderClasses.h classTriggerHost (:262-281) and classTriggerFires (:46-52):
    ``mixed32`` = 32-slot groups of [0, n) holding two or more live classes, and the
    class trigger."""
    n = mask.size
    live = (mask == 0) if drop else (mask != 0)
    mixed = 0
    for g in range(0, n, 32):
        c = cls[g:g + 32][live[g:g + 32]]
        if c.size and c.min() < c.max():
            mixed += 1
    warp_mix = mixed > 0 and float(mixed) >= float(np.float32(class_theta)) * float(live32) and span >= 4096
    drift = float(stale) > 0.05 * float(count)
    return mixed, int(warp_mix or drift or live_fire != 0)
