"""Active-set compaction on the GPU (eagle_backend_compact_device): the map is the
ascending kept indices and the count their number, bit for bit against the oracle
and numpy's flatnonzero, over the sizes that hit the scan's edges (python/tests/
test_active_set.py:49 and tests/test_Compact.cu:46-53,145 of the eagle source tree),
with the reorder trigger, the keep-mask form, and a captured replay that follows
a mask changed between replays."""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SIZES = (0, 1, 7, 31, 32, 33, 63, 64, 65, 256, 257, 4095, 4096, 4097, 16383, 16384, 16385, 100_003, (1 << 20) + 37,
         1 << 24)


def _mask(n, seed, p):
    return np.random.default_rng([seed, n]).random(n) < p


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("p", (0.0, 0.01, 0.6, 0.99, 1.0))
def test_map_is_flatnonzero(eb, n, p):
    mask = _mask(n, 3, p)
    md = torch.from_numpy(mask).cuda()
    index_map, count = eb.compact(md)
    c = int(count.item())
    want = np.flatnonzero(~mask)
    assert c == want.size
    assert np.array_equal(index_map[:c].cpu().numpy(), want)


@pytest.mark.parametrize("n", (1, 257, 100_003))
def test_keep_mask(eb, n):
    mask = _mask(n, 5, 0.3)
    index_map, count = eb.compact(torch.from_numpy(mask).cuda(), drop=False)
    c = int(count.item())
    assert np.array_equal(index_map[:c].cpu().numpy(), np.flatnonzero(mask))


@pytest.mark.parametrize("n,p", ((100_003, 0.9), (100_003, 0.2), (4096, 0.99), (1 << 20, 0.97)))
def test_trigger_matches_oracle(eb, orc, n, p):
    mask = _mask(n, 9, p)
    comp = eb.Compactor(torch.from_numpy(mask).cuda(), trigger=True, theta=0.5)
    index_map, count = comp()
    m, c, live32, fire = orc.compact(mask, span=n, theta=0.5, trigger=True)
    assert int(count.item()) == c
    assert int(comp.live32.item()) == live32
    assert int(comp.fire.item()) == fire


def test_unaligned_mask_view(eb):
    n = 100_003
    base = torch.from_numpy(_mask(n + 3, 4, 0.5)).cuda()
    view = base[3:]  # not 16-byte aligned
    index_map, count = eb.compact(view)
    want = np.flatnonzero(~view.cpu().numpy())
    assert int(count.item()) == want.size and np.array_equal(index_map[:want.size].cpu().numpy(), want)


def test_captured_replay_follows_the_mask(eb):
    n = 100_003
    md = torch.from_numpy(_mask(n, 1, 0.5)).cuda()
    comp = eb.Compactor(md)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        comp(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        comp(s)
    for seed in (2, 3, 4):
        mask = _mask(n, seed, 0.3 * seed / 2)
        md.copy_(torch.from_numpy(mask))
        g.replay()
        torch.cuda.synchronize()
        want = np.flatnonzero(~mask)
        assert int(comp.count.item()) == want.size
        assert np.array_equal(comp.index_map[:want.size].cpu().numpy(), want)


def test_mask_count_cell_op(eb):
    for n in (1, 15, 16, 17, 100_003):
        mask = _mask(n, 8, 0.4)
        cell = eb.mask_count(torch.from_numpy(mask).cuda())
        assert int(cell.item()) == int(mask.sum())


def test_small_cell_ops(eb):
    from eagle_b200 import _abi

    cell = torch.zeros(4, dtype=torch.int32, device="cuda")
    eb.cell_op(_abi.CELL_BUMP, 1, [cell.data_ptr()])
    eb.cell_op(_abi.CELL_BUMP, 1, [cell.data_ptr()])
    ident = torch.full((1000,), -1, dtype=torch.int32, device="cuda")
    eb.cell_op(_abi.CELL_IDENTITY, 1000, [ident.data_ptr()])
    fire = torch.tensor([3], dtype=torch.int32, device="cuda")
    eb.cell_op(_abi.CELL_COUNT_FIRED, 1, [fire.data_ptr(), cell.data_ptr() + 4])
    eb.cell_op(_abi.CELL_SCALE_COUNT, 1, [cell.data_ptr(), cell.data_ptr() + 8], ints=[32])
    m = torch.tensor([1, 1, 0, 1, 1, 1, 1], dtype=torch.uint8, device="cuda")
    d = torch.zeros(3, dtype=torch.uint8, device="cuda")
    eb.cell_op(_abi.CELL_GROUP_AND, 3, [m.data_ptr(), d.data_ptr()], ints=[7, 3])
    torch.cuda.synchronize()
    assert cell.tolist()[:3] == [2, 1, 64]
    assert torch.equal(ident.cpu(), torch.arange(1000, dtype=torch.int32))
    assert d.tolist() == [0, 1, 1]


def test_policy_cell_op_matches_oracle(eb, orc):
    from eagle_b200 import _abi

    rng = np.random.default_rng(3)
    kmax = 64
    for _ in range(20):
        total = int(rng.integers(1, 1 << 20))
        fin = int(rng.integers(0, total + 1))
        cells = np.array([int(2 ** rng.integers(3, 7)), int(rng.integers(0, fin + 1)), int(rng.integers(0, 900)),
                          1000, int(rng.integers(1, 20000)), 0], dtype=np.int64)
        word = np.array([int(rng.integers(1, 64))], dtype=np.int64)
        go = np.zeros(1, dtype=np.uint32)
        hist = np.zeros(kmax + 1, dtype=np.int64)
        dcells, dword = torch.from_numpy(cells.copy()).cuda(), torch.from_numpy(word.copy()).cuda()
        dgo = torch.zeros(1, dtype=torch.int32, device="cuda")
        dhist = torch.zeros(kmax + 1, dtype=torch.int64, device="cuda")
        dfin = torch.tensor([fin], dtype=torch.int32, device="cuda")
        dtot = torch.tensor([total], dtype=torch.int32, device="cuda")
        eb.cell_op(_abi.CELL_POLICY, 1, [dfin.data_ptr(), dtot.data_ptr(), dcells.data_ptr(), dword.data_ptr(),
                                         dgo.data_ptr(), dhist.data_ptr()], ints=[8, kmax, 0, 1, 2, 3, 4, 5, 1000])
        orc.policy_step(fin, total, cells, word, go, hist, 8, kmax)
        torch.cuda.synchronize()
        assert np.array_equal(dcells.cpu().numpy(), cells)
        assert int(dgo.item()) == int(go[0])
        if go[0]:
            assert np.array_equal(dword.cpu().numpy(), word) and np.array_equal(dhist.cpu().numpy(), hist)


def test_reset_device(eb):
    from eagle_b200 import _abi

    n = 5000
    perm = torch.zeros(n, dtype=torch.int32, device="cuda")
    inv = torch.zeros(n, dtype=torch.int32, device="cuda")
    imap = torch.zeros(n, dtype=torch.int32, device="cuda")
    words = torch.zeros(2, dtype=torch.int32, device="cuda")
    d = _abi.new(_abi.ReorderDesc, perm=perm.data_ptr(), inv=inv.data_ptr(), index_map=imap.data_ptr(),
                 count=words.data_ptr(), span=words.data_ptr() + 4, n=n, device=-1,
                 stream=torch.cuda.current_stream().cuda_stream)
    _abi.check(_abi.lib().eagle_backend_reset_device(ctypes.byref(d)))
    torch.cuda.synchronize()
    ar = torch.arange(n, dtype=torch.int32)
    assert torch.equal(perm.cpu(), ar) and torch.equal(inv.cpu(), ar) and torch.equal(imap.cpu(), ar)
    assert words.tolist() == [n, n]


@pytest.mark.parametrize("tiles", (2, 5, 40))
def test_bounded_wait_gives_up(eb, tiles):
    """The look-back's bounded wait (eagle_b200/csrc/common.cuh lbExclusivePrefix):
    with the first tile withheld nothing ever publishes its status word, so each
    tile whose look-back reaches it polls ``spin_limit`` times, gives up and sets the
    error word; the count comes back 0xffffffff (above n) instead of a hang. The
    same scratch then serves a normal compaction bit for bit."""
    from eagle_b200 import _abi

    n = tiles * 32768 + 123
    mask = _mask(n, 21, 0.5)
    comp = eb.Compactor(torch.from_numpy(mask).cuda())
    d = _abi.new(_abi.CompactDesc)
    ctypes.memmove(ctypes.byref(d), ctypes.byref(comp.desc), ctypes.sizeof(d))
    d.stream = torch.cuda.current_stream().cuda_stream
    comp.count.fill_(7)
    _abi.check(_abi.lib().eagle_backend_x_b200_compact_wait_check(ctypes.byref(d), 1024))
    torch.cuda.synchronize()
    assert int(comp.count.item()) & 0xffffffff == 0xffffffff
    index_map, count = comp()
    c = int(count.item())
    want = np.flatnonzero(~mask)
    assert c == want.size and np.array_equal(index_map[:c].cpu().numpy(), want)


def test_bounded_wait_check_refusals(eb):
    from eagle_b200 import _abi

    d = _abi.new(_abi.CompactDesc, n=32768, mask=1, index_map=1, count=1, scratch=1)
    assert _abi.lib().eagle_backend_x_b200_compact_wait_check(ctypes.byref(d), 1024) == _abi.INVALID_ARGUMENT
    d.n = 70000
    assert _abi.lib().eagle_backend_x_b200_compact_wait_check(ctypes.byref(d), 0) == _abi.INVALID_ARGUMENT
    assert _abi.lib().eagle_backend_x_b200_compact_wait_check(ctypes.byref(d), (1 << 22) + 1) == \
        _abi.INVALID_ARGUMENT
