"""The device-side ragged exchange of compact-then-sum on one GPU, with the ranks
emulated: the batch is split into W shards, each shard compacted on its own, the
head blocks (first 4095 survivors and the count) stacked as the first all-gather
would stack them, then every rank's partial block and the rank-order fold (eagle_backend_x_b200_ragged_fold) -- bit for bit the
one-device compact-then-sum of the whole batch and the oracle's compaction +
canonical sum, for even and uneven splits, empty shards, and shards so sparse that
one leaf spans many ranks. Both forms of the leaves: from the gathered survivors
(eagle_backend_x_b200_ragged_leaves) and fused, straight from the values
(eagle_backend_x_b200_compact_sum_count / _head / _leaves / _straddle)."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

LEAF = 4096


def _fold(lib, gathered, world, cap, s):
    from eagle_b200 import _abi

    work = torch.zeros(2 * ((world * cap + 511) // 512) + 2, dtype=torch.float64, device="cuda")
    out = torch.zeros(3, dtype=torch.float64, device="cuda")
    _abi.check(lib.eagle_backend_x_b200_ragged_fold(gathered.data_ptr(), world, cap, work.data_ptr(),
                                                    out.data_ptr(), s))
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _emulated(eb, vals, keep, bounds):
    """Every rank's head block stacked as the first all-gather stacks them, every
    rank's partial block as the second does."""
    from eagle_b200 import _abi

    lib = _abi.lib()
    s = torch.cuda.current_stream().cuda_stream
    world = len(bounds) - 1
    sums = []
    for r in range(world):
        b, e = bounds[r], bounds[r + 1]
        cs = eb.CompactSum(torch.from_numpy(keep[b:e].copy()).cuda(), torch.from_numpy(vals[b:e].copy()).cuda())
        cs.gather()
        sums.append(cs)
    cap = max((bounds[r + 1] - bounds[r] + LEAF - 1) // LEAF + 1 for r in range(world))
    pb = 2 * cap + 2
    blocks = torch.zeros(world * LEAF, dtype=torch.float64, device="cuda")
    for r, cs in enumerate(sums):
        _abi.check(lib.eagle_backend_x_b200_ragged_head(cs.kept.data_ptr(), cs.count.data_ptr(),
                                                        blocks.data_ptr() + 8 * LEAF * r, s))
    gathered = torch.zeros(world * pb, dtype=torch.float64, device="cuda")
    for r, cs in enumerate(sums):
        _abi.check(lib.eagle_backend_x_b200_ragged_leaves(
            cs.kept.data_ptr(), blocks.data_ptr(), r, world, gathered.data_ptr() + 8 * pb * r, cap, s))
    return _fold(lib, gathered, world, cap, s)


def _emulated_fused(eb, vals, keep, bounds):
    import ctypes

    from eagle_b200 import _abi

    lib = _abi.lib()
    s = torch.cuda.current_stream().cuda_stream
    world = len(bounds) - 1
    cap = max((bounds[r + 1] - bounds[r] + LEAF - 1) // LEAF + 1 for r in range(world))
    pb = 2 * cap + 2
    blocks = torch.zeros(world * LEAF, dtype=torch.float64, device="cuda")
    sums, vdev = [], []
    for r in range(world):
        b, e = bounds[r], bounds[r + 1]
        v = torch.from_numpy(vals[b:e].copy()).cuda()
        cs = eb.CompactSum(torch.from_numpy(keep[b:e].copy()).cuda(), v)
        cs.sdesc.stream = s
        _abi.check(lib.eagle_backend_x_b200_compact_sum_count(ctypes.byref(cs.sdesc)))
        _abi.check(lib.eagle_backend_x_b200_compact_sum_head(ctypes.byref(cs.sdesc), v.data_ptr(),
                                                              blocks.data_ptr() + 8 * LEAF * r))
        sums.append(cs)
        vdev.append(v)
    gathered = torch.zeros(world * pb, dtype=torch.float64, device="cuda")
    for r, cs in enumerate(sums):
        _abi.check(lib.eagle_backend_x_b200_compact_sum_leaves(
            ctypes.byref(cs.sdesc), vdev[r].data_ptr(), blocks.data_ptr(), r, world,
            gathered.data_ptr() + 8 * pb * r, cap))
        _abi.check(lib.eagle_backend_x_b200_compact_sum_straddle(
            ctypes.byref(cs.sdesc), blocks.data_ptr(), r, world, gathered.data_ptr() + 8 * pb * r, cap))
    return _fold(lib, gathered, world, cap, s)


CASES = [
    (1 << 20, 0.37, (0, 1 << 19, 1 << 20)),                    # two even shards
    ((1 << 20) + 777, 0.61, None),                             # four uneven shards
    (300_000, 0.002, None),                                    # sparse: leaves span many ranks
    (200_000, 0.5, (0, 0, 100_000, 100_000, 200_000)),         # empty shards
    (100_000, 0.0, None),                                      # nothing kept
    (65_536, 1.0, (0, 1, 2, 3, 65_536)),                       # one-survivor shards
    (1 << 22, 0.9, (0, 1 << 20, 2 << 20, 3 << 20, 4 << 20)),  # dense: leaves on the warp path
    (1 << 22, 0.004, (0, 1 << 21, 1 << 22)),                   # sparse: leaves over many bitmap tiles
    (3 * 4096 + 17, 1.0, (0, 4096, 8192, 3 * 4096 + 17)),      # shards of exactly one leaf, then a ragged one
]


@pytest.mark.parametrize("n,p,bounds", CASES)
def test_emulated_ranks_equal_the_whole(eb, orc, n, p, bounds):
    g = np.random.default_rng([n, int(p * 1000)])
    vals = orc.corpus(n, 91)
    keep = g.random(n) < p
    if bounds is None:
        w = 8 if p < 0.01 else 4
        cuts = np.sort(g.integers(0, n, w - 1))
        bounds = (0, *[int(c) for c in cuts], n)
    got = _emulated(eb, vals, keep, list(bounds))
    fused = _emulated_fused(eb, vals, keep, list(bounds))
    whole = eb.CompactSum(torch.from_numpy(keep).cuda(), torch.from_numpy(vals).cuda())().cpu().numpy()
    want = orc.reduce(vals[keep])[0] if keep.any() else np.float64(0.0)  # the oracle refuses an empty sum
    assert np.float64(got[2]).tobytes() == np.float64(want).tobytes() == whole[-1].tobytes()
    assert np.float64(fused[2]).tobytes() == np.float64(want).tobytes()


def test_leaf_capacity_overflow_is_reported(eb):
    """A rank handed too small a ``cap`` for its leaves: every rank's fold gives NaN
    instead of a sum missing leaves."""
    from eagle_b200 import _abi

    lib = _abi.lib()
    s = torch.cuda.current_stream().cuda_stream
    n = 5 * LEAF
    cs = eb.CompactSum(torch.ones(n, dtype=torch.bool, device="cuda"),
                       torch.ones(n, dtype=torch.float64, device="cuda"))
    cs.gather()
    block = torch.zeros(LEAF, dtype=torch.float64, device="cuda")
    _abi.check(lib.eagle_backend_x_b200_ragged_head(cs.kept.data_ptr(), cs.count.data_ptr(), block.data_ptr(), s))
    partials = torch.zeros(2 * 2 + 2, dtype=torch.float64, device="cuda")
    _abi.check(lib.eagle_backend_x_b200_ragged_leaves(cs.kept.data_ptr(), block.data_ptr(), 0, 1,
                                                      partials.data_ptr(), 2, s))
    out = _fold(lib, partials, 1, 2, s)
    assert int(partials[4:5].view(torch.int64).item()) & 0xffffffff == 5
    assert np.isnan(out).all()
