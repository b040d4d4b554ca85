"""The gambler's-ruin walk (the 2^26-sample random-walk configuration, Philox-4x32-10
steps, absorbing at 0 and 100) on the GPU against the oracle: positions, int64
absorption times and the mask bit for bit, the report exactly, the canonical
int64 sum of the times exact; both schedules; the cap and a continued run; shards
keyed by id_base draw the numbers of the whole; the hawk-ABI entry through
launch_raw; and the oracle's Philox itself against cuRAND's."""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from eagle_b200 import _abi  # noqa: E402

SEED = 2026


def _start(n, seed=8):
    return np.random.default_rng(seed).integers(1, 100, n).astype(np.int32)


def _device(eb, pos0, max_steps, mode, time0=None, runs=1, **kw):
    n = pos0.size
    pos = torch.from_numpy(pos0.copy()).cuda()
    time = torch.zeros(n, dtype=torch.int64, device="cuda") if time0 is None else torch.from_numpy(time0.copy()).cuda()
    term = torch.zeros(n, dtype=torch.uint8, device="cuda")
    r = eb.until_done(eb.gambler, max_steps=max_steps, mode=mode, terminated=term, pos=pos, time=time, seed=SEED,
                      **kw)
    reps = [r.run() for _ in range(runs)]
    return pos.cpu().numpy(), time.cpu().numpy(), term.cpu().numpy(), reps, time


def _oracle(orc, pos0, max_steps, runs=1, id_base=0):
    pos, time, term = pos0.copy(), np.zeros(pos0.size, np.int64), np.zeros(pos0.size, np.uint8)
    outs = [orc.gambler_run(pos, time, term, seed=SEED, max_steps=max_steps, id_base=id_base) for _ in range(runs)]
    return pos, time, term, outs


@pytest.mark.parametrize("mode", ("persist", "fused"))
@pytest.mark.parametrize("n", (1, 1000, 100_003))
def test_walk_bitwise(eb, orc, mode, n):
    pos0 = _start(n)
    p, t, m, (rep,), dtime = _device(eb, pos0, 1_000_000, mode)
    rp, rt, rm, ((fin, longest, total),) = _oracle(orc, pos0, 1_000_000)
    assert p.tobytes() == rp.tobytes() and t.tobytes() == rt.tobytes() and m.tobytes() == rm.tobytes()
    assert (rep.finished, rep.steps, rep.step_sum, rep.done) == (fin, longest, total, fin == n)
    assert int(eb.reduce(dtime).item()) == int(rt.sum())


def test_large_batch_and_exact_sum(eb, orc):
    n = 1 << 22
    pos0 = _start(n, 9)
    p, t, m, (rep,), dtime = _device(eb, pos0, 1_000_000, "persist")
    rp, rt, rm, ((fin, longest, total),) = _oracle(orc, pos0, 1_000_000)
    assert t.tobytes() == rt.tobytes() and m.tobytes() == rm.tobytes()
    assert rep.finished == n and int(eb.reduce(dtime).item()) == int(orc.reduce(rt)[0]) == int(rt.sum())
    assert abs(rt.mean() - 1683) < 10  # E[s (100 - s)] over s ~ U{1..99}


@pytest.mark.parametrize("mode", ("persist", "fused"))
def test_cap_and_continue(eb, orc, mode):
    n = 50_000
    pos0 = _start(n, 10)
    p, t, m, reps, _ = _device(eb, pos0, 700, mode, runs=3)
    rp, rt, rm, outs = _oracle(orc, pos0, 700, runs=3)
    assert t.tobytes() == rt.tobytes() and p.tobytes() == rp.tobytes() and m.tobytes() == rm.tobytes()
    for rep, (fin, longest, total) in zip(reps, outs):
        assert (rep.finished, rep.steps, rep.step_sum) == (fin, longest, total)
    assert not reps[0].done


def test_shards_draw_the_numbers_of_the_whole(eb, orc):
    n = 20_000
    pos0 = _start(n, 11)
    rp, rt, rm, _ = _oracle(orc, pos0, 1_000_000)
    half = n // 2
    for lo, hi in ((0, half), (half, n)):
        p, t, m, _, _ = _device(eb, pos0[lo:hi], 1_000_000, "persist", id_base=lo)
        assert t.tobytes() == rt[lo:hi].tobytes() and p.tobytes() == rp[lo:hi].tobytes()


def test_hawk_abi_persist_entry(eb, orc):
    n = 30_011
    pos0 = _start(n, 12)
    pos = torch.from_numpy(pos0.copy()).cuda()
    time = torch.zeros(n, dtype=torch.int64, device="cuda")
    term = torch.zeros(n, dtype=torch.uint8, device="cuda")
    fin = torch.zeros(1, dtype=torch.int32, device="cuda")
    budget = torch.tensor([1_000_000], dtype=torch.int64, device="cuda")
    words = torch.zeros(4, dtype=torch.int64, device="cuda")

    def h(tn, k):
        return _abi.ScalarHandle(tn.data_ptr(), k, 1, 2, 0)

    args = [h(pos, n), h(time, n), h(term, n), ctypes.c_int64(SEED), ctypes.c_int64(0), h(fin, 1), h(budget, 1),
            ctypes.c_int64(0), ctypes.c_int64(n), ctypes.c_int64(n), ctypes.c_uint64(words.data_ptr()),
            ctypes.c_uint64(0), ctypes.c_uint64(words.data_ptr() + 4), ctypes.c_uint64(words.data_ptr() + 8),
            ctypes.c_uint32(64)]
    ptrs = (ctypes.c_void_p * len(args))(*[ctypes.addressof(a) for a in args])
    d = _abi.new(_abi.LaunchRawDesc, device=-1, function=eb.entry("gambler_persist"),
                 stream=torch.cuda.current_stream().cuda_stream, args=ctypes.addressof(ptrs), arg_count=len(args))
    d.grid[:] = (148 * 2, 1, 1)
    d.block[:] = (256, 1, 1)
    _abi.check(_abi.lib().eagle_backend_launch_raw(ctypes.byref(d)))
    torch.cuda.synchronize()
    rp, rt, rm, ((f, longest, total),) = _oracle(orc, pos0, 1_000_000)
    assert time.cpu().numpy().tobytes() == rt.tobytes() and int(fin.item()) == f
    assert int(words.cpu().numpy()[1]) == total


def test_oracle_philox_is_curands(orc):
    """The oracle's Philox-4x32-10 -- the generator the walk's steps come from, and
    the check of the GPU walk above -- against cuRAND's own block function
    (curand_Philox4x32_10) on the same counters and keys: random ones, the walk's own
    (step / 128 and the sample id as two words each, under the seed used above), and
    the all-zero and all-ones edges."""
    g = np.random.default_rng(3)
    n = 4096
    counters = g.integers(0, 1 << 32, (n, 4), dtype=np.uint64).astype(np.uint32)
    keys = g.integers(0, 1 << 32, (n, 2), dtype=np.uint64).astype(np.uint32)
    blocks = g.integers(0, 1 << 20, 256, dtype=np.uint64)
    ids = g.integers(0, 1 << 26, 256, dtype=np.uint64)
    walk = np.stack([blocks & 0xffffffff, blocks >> 32, ids & 0xffffffff, ids >> 32], axis=1).astype(np.uint32)
    counters = np.concatenate([counters, walk, np.zeros((1, 4), np.uint32), np.full((1, 4), 0xffffffff, np.uint32)])
    seed_words = np.array([SEED & 0xffffffff, SEED >> 32], np.uint32)
    keys = np.concatenate([keys, np.tile(seed_words, (256, 1)), np.zeros((1, 2), np.uint32),
                           np.full((1, 2), 0xffffffff, np.uint32)])
    want = orc.curand_philox4x32_10(counters, keys)
    got = np.stack([orc.philox4x32_10(c, int(k[0]) | (int(k[1]) << 32)) for c, k in zip(counters, keys)])
    assert got.dtype == want.dtype and (got == want).all()
