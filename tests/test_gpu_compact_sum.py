"""Compact the survivors, then their canonical ordered sum (the 2^28-value
microbenchmark configuration: N(0, 1) values with one in 10^6 replaced by +-1e12,
Bernoulli(p) keep-masks for p in {0.9, 0.5, 0.1, 0.01}): the count, the kept
values in sample order and the sum's bits against the oracle (flatnonzero and
the canonical tree of eagle/reduce/canonical.h over the kept values)."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

PS = (0.9, 0.5, 0.1, 0.01)


def microbench_inputs(n, i):
    """Values (seed 4), outlier positions (seed 5) and signs (seed 6), mask i (seed 7 + i)."""
    x = np.random.default_rng(4).standard_normal(n)
    k = max(1, n // 1_000_000)
    pos = np.random.default_rng(5).choice(n, size=k, replace=False)
    sign = np.where(np.random.default_rng(6).random(k) < 0.5, -1.0, 1.0)
    x[pos] = sign * 1e12
    keep = np.random.default_rng(7 + i).random(n) < PS[i]
    return x, keep


@pytest.mark.parametrize("n", (1, 4097, (1 << 20) + 37, 1 << 24))
@pytest.mark.parametrize("i", range(4))
def test_compact_then_sum(eb, orc, n, i):
    x, keep = microbench_inputs(n, i)
    cs = eb.CompactSum(torch.from_numpy(keep).cuda(), torch.from_numpy(x).cuda())
    got = cs().cpu().numpy()
    kept = x[keep]
    assert int(cs.count.item()) == kept.size
    want = orc.reduce(kept) if kept.size else np.zeros(1)
    assert got.tobytes() == want.tobytes(), (n, PS[i])
    cs.gather()  # the compacted plane itself
    c = int(cs.count.item())
    assert c == kept.size
    assert cs.kept[:c].cpu().numpy().tobytes() == kept.tobytes()


def _patterns(n):
    """Masks whose survivors put leaf starts on word, row and tile edges."""
    i = np.arange(n)
    yield "all", np.ones(n, bool)
    yield "even", i % 2 == 0
    yield "every 33rd", i % 33 == 0
    yield "one run", (i >= n // 3) & (i < n // 3 + 3 * 4096 + 5)
    yield "first and last", (i == 0) | (i == n - 1)
    yield "runs of 4096", (i // 4096) % 2 == 1
    yield "tile edges", (i % 16384 == 16383) | (i % 16384 == 0)


@pytest.mark.parametrize("n", (31, 4096, 16384, 3 * 16384 + 7, 8 * 4096 * 33 + 1, (1 << 20) + 3))
def test_fused_sum_on_edge_masks(eb, orc, n):
    x = orc.corpus(n, n + 1)
    xd = torch.from_numpy(x).cuda()
    for name, keep in _patterns(n):
        cs = eb.CompactSum(torch.from_numpy(keep).cuda(), xd)
        got = cs().cpu().numpy()
        want = orc.reduce(x[keep]) if keep.any() else np.zeros(1)
        assert int(cs.count.item()) == int(keep.sum()), name
        assert got.tobytes() == want.tobytes(), (n, name)


@pytest.mark.parametrize("case", ("inf", "-inf then inf", "nan", "huge"))
def test_fused_sum_non_finite(eb, orc, case):
    """Infinities and NaNs among the kept values: a slot whose hi leaves the finite
    range ends with a zero comp, exactly as the step-by-step join gives it."""
    n = 3 * 4096 * 5 + 123
    x = orc.corpus(n, 77)
    keep = np.random.default_rng(78).random(n) < 0.7
    kept_at = np.flatnonzero(keep)
    if case == "inf":
        x[kept_at[[5, 4096 + 300]]] = np.inf
    elif case == "-inf then inf":
        x[kept_at[[17, 17 + 256 * 3]]] = (-np.inf, np.inf)
    elif case == "nan":
        x[kept_at[[0, 9000]]] = np.nan
    else:
        x[kept_at[::97]] = 1.7e308
    cs = eb.CompactSum(torch.from_numpy(keep).cuda(), torch.from_numpy(x).cuda(), pair_out=True)
    got = cs().cpu().numpy()
    want = orc.reduce(x[keep], pair_out=True)
    if np.isnan(want[0]):  # a NaN's payload is the hardware's; that it is NaN, and comp 0, is the contract
        assert np.isnan(got[0]) and got[1] == 0.0, case
    else:
        assert got.tobytes() == want.tobytes(), case


def test_fused_sum_unaligned_mask(eb, orc):
    """A mask that does not start on a 16-byte boundary takes the byte-wise loads."""
    n = 200_003
    x, keep = microbench_inputs(n, 1)
    buf = torch.zeros(n + 1, dtype=torch.uint8, device="cuda")
    buf[1:] = torch.from_numpy(keep.astype(np.uint8)).cuda()
    cs = eb.CompactSum(buf[1:], torch.from_numpy(x).cuda())
    assert cs().cpu().numpy().tobytes() == orc.reduce(x[keep]).tobytes()


def test_fused_sum_refusals(eb):
    from eagle_b200 import _abi
    import ctypes
    d = _abi.new(_abi.CompactDesc, device=0, n=10)
    with pytest.raises(eb.BackendUnsupported):
        _abi.check(_abi.lib().eagle_backend_x_b200_compact_sum(ctypes.byref(d), 0, 0, 4))
    d.index_map = 256
    with pytest.raises(eb.BackendUnsupported):
        _abi.check(_abi.lib().eagle_backend_x_b200_compact_sum(ctypes.byref(d), 0, 0, 0))
    d.index_map = 0
    d.n = 1 << 31
    with pytest.raises(eb.BackendUnsupported):
        _abi.check(_abi.lib().eagle_backend_x_b200_compact_sum(ctypes.byref(d), 0, 0, 0))


def test_drop_mask_and_pair_out(eb, orc):
    n = 100_003
    x, keep = microbench_inputs(n, 1)
    cs = eb.CompactSum(torch.from_numpy(~keep).cuda(), torch.from_numpy(x).cuda(), drop=True, pair_out=True)
    got = cs().cpu().numpy()
    assert got.tobytes() == orc.reduce(x[keep], pair_out=True).tobytes()


def test_nothing_kept_sums_to_zero(eb):
    n = 5000
    cs = eb.CompactSum(torch.zeros(n, dtype=torch.bool, device="cuda"),
                       torch.ones(n, dtype=torch.float64, device="cuda"))
    assert cs().item() == 0.0 and int(cs.count.item()) == 0


def test_captured_replay(eb, orc):
    n = 300_007
    x, keep = microbench_inputs(n, 2)
    md, xd = torch.from_numpy(keep).cuda(), torch.from_numpy(x).cuda()
    cs = eb.CompactSum(md, xd)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        cs(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        cs(s)
    for j in (0, 3):
        x2, keep2 = microbench_inputs(n, j)
        md.copy_(torch.from_numpy(keep2))
        xd.copy_(torch.from_numpy(x2))
        g.replay()
        torch.cuda.synchronize()
        assert cs.out.cpu().numpy().tobytes() == orc.reduce(x2[keep2]).tobytes()


def test_full_size_one_mask(eb, orc):
    n = 1 << 28
    x, keep = microbench_inputs(n, 2)
    cs = eb.CompactSum(torch.from_numpy(keep).cuda(), torch.from_numpy(x).cuda())
    got = cs().cpu().numpy()
    assert got.tobytes() == orc.reduce(x[keep]).tobytes()


def test_leaf_partials_join_to_the_canonical_sum(orc):
    """The leaf-partial entry gives the oracle's leaves, and joining them with the
    pairwise levels gives the canonical sum's bits."""
    from eagle_b200 import shard

    for n in (1, 4095, 4096, 4097, 100_003):
        x = orc.corpus(n, n)
        got = shard.device_leaf_partials(torch.from_numpy(x).cuda())
        assert got.cpu().numpy().tobytes() == orc.leaf_partials(x).tobytes()
        folded = shard.fold_partials(got.reshape(-1))
        assert folded[2].item() == orc.reduce(x)[0]
