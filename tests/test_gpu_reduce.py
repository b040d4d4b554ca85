"""The canonical reduction on the GPU, bit for bit against the oracle (which is
pinned to the reference's test oracle in test_oracle.py) and the golden fixtures.
Rows follow tests/CanonicalReduceCases.h and tests/test_CanonicalReduce.cu:48-85 of
the eagle source tree: every tree edge size, float and integer sums, min/max/all,
columns, the companion input, PAIR_OUT, non-finite terms, and a captured replay."""

import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SIZES = (1, 2, 3, 255, 256, 257, 4095, 4096, 4097, 8193, 12345, 65536, 65537, 100003, (1 << 20) + 37)
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.json")


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _same(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return a.dtype == b.dtype and a.tobytes() == b.tobytes()


@pytest.mark.parametrize("n", SIZES)
def test_f64_sum_bitwise(eb, orc, n):
    x = orc.corpus(n, 1000 + n)
    got = eb.reduce(_dev(x)).cpu().numpy()
    assert _same(got, orc.reduce(x)), n


def test_f64_sum_matches_golden(eb, orc):
    with open(GOLDEN) as f:
        cases = json.load(f)["reduce"]
    for c in cases:
        x = orc.corpus(c["n"], c["seed"])
        got = eb.reduce(_dev(x)).cpu().numpy().view(np.uint64)[0]
        assert int(got) == int(c["bits"], 16), c


@pytest.mark.parametrize("n", (257, 70001, 300000))
def test_f32_sum_bitwise(eb, orc, n):
    x = orc.corpus(n, 7 + n, np.float32)
    assert _same(eb.reduce(_dev(x)).cpu().numpy(), orc.reduce(x))


@pytest.mark.parametrize("n", (1, 4097, 1 << 24))
def test_large_and_tiny_sums(eb, orc, n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n)
    x[rng.choice(n, size=max(1, n // 1_000_000), replace=False)] = 1e12
    assert _same(eb.reduce(_dev(x)).cpu().numpy(), orc.reduce(x))


@pytest.mark.parametrize("n", (8192, 12289, (1 << 23) + 12345))
def test_staged_and_direct_leaf_loads(eb, orc, n):
    """A float64 plane gives the oracle's bits whether it starts on a 16-byte boundary
    or 8 bytes off one (a view one element into its buffer), at sizes whose CTAs own
    one leaf each and whose CTAs own groups of several."""
    x = orc.corpus(n, 77 + n)
    want = orc.reduce(x)
    assert _same(eb.reduce(_dev(x)).cpu().numpy(), want)
    base = torch.empty(n + 1, dtype=torch.float64, device="cuda")
    base[1:].copy_(torch.from_numpy(x))
    off = base[1:]
    assert off.data_ptr() % 16 == 8
    assert _same(eb.reduce(off).cpu().numpy(), want)


@pytest.mark.parametrize("n", ((1 << 22) + 37, 700 * 4096 + 1, 8000 * 4096 - 5))
def test_leaf_by_leaf_kernel_every_kind(eb, orc, n):
    """One column with more leaves than the device holds CTAs takes the leaf-by-leaf
    kernel (leaves claimed in order, each 512-leaf chunk joined by the CTA completing
    it, the chunk partials by the last): the oracle's bits for float64 (also with a
    companion and PAIR_OUT), float32, int64 sums, min, max and all, with a ragged last
    leaf and chunk."""
    x = orc.corpus(n, 5 + n)
    assert _same(eb.reduce(_dev(x)).cpu().numpy(), orc.reduce(x))
    c = orc.corpus(n, 6 + n) * 1e-17
    assert _same(eb.reduce(_dev(x), comp=_dev(c), pair_out=True).cpu().numpy(),
                 orc.reduce(x, comp=c, pair_out=True))
    xf = orc.corpus(n, 7 + n, np.float32)
    assert _same(eb.reduce(_dev(xf)).cpu().numpy(), orc.reduce(xf))
    xi = np.random.default_rng(n).integers(-10 ** 9, 10 ** 9, size=n)
    for op in ("sum", "max", "min"):
        assert _same(eb.reduce(_dev(xi), op).cpu().numpy(), orc.reduce(xi, op)), op
    m = (np.random.default_rng(n + 1).random(n) < 0.9999999).astype(np.uint8)
    assert _same(eb.reduce(_dev(m), "all").cpu().numpy(), orc.reduce(m, "all"))


@pytest.mark.parametrize("dtype", [np.int32, np.int64])
def test_integer_sums_min_max(eb, orc, dtype):
    rng = np.random.default_rng(1)
    for n in (1, 4095, 100003):
        x = rng.integers(-10 ** 6, 10 ** 6, size=n).astype(dtype)
        for op in ("sum", "max", "min"):
            assert _same(eb.reduce(_dev(x), op).cpu().numpy(), orc.reduce(x, op)), (n, op)


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_min_max_with_infinities(eb, orc, dtype):
    x = orc.corpus(9001, 5, dtype)
    for op in ("min", "max"):
        assert _same(eb.reduce(_dev(x), op).cpu().numpy(), orc.reduce(x, op))
    x[1000], x[7000] = np.inf, -np.inf
    assert eb.reduce(_dev(x), "min").item() == -np.inf
    assert eb.reduce(_dev(x), "max").item() == np.inf


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_non_finite_sum(eb, dtype, orc):
    x = orc.corpus(9001, 5, dtype)
    x[1000] = np.inf
    assert eb.reduce(_dev(x)).item() == np.inf
    x[7000] = -np.inf
    assert np.isnan(eb.reduce(_dev(x)).item())


def test_all_u8(eb, orc):
    for n in (1, 300, 100003):
        m = (np.random.default_rng(n).random(n) < 0.999).astype(np.uint8)
        assert _same(eb.reduce(_dev(m), "all").cpu().numpy(), orc.reduce(m, "all"))
        m[:] = 1
        assert eb.reduce(_dev(m), "all").item() == 1


def test_columns(eb, orc):
    rows, cols = 9001, 7
    x = orc.corpus(rows * cols, 21).reshape(rows, cols)
    assert _same(eb.reduce(_dev(x)).cpu().numpy(), orc.reduce(x, columns=cols))


def test_companion_and_pair_out(eb, orc):
    n = 100003
    x = orc.corpus(n, 3)
    c = orc.corpus(n, 4) * 1e-17
    assert _same(eb.reduce(_dev(x), comp=_dev(c)).cpu().numpy(), orc.reduce(x, comp=c))
    assert _same(eb.reduce(_dev(x), pair_out=True).cpu().numpy(), orc.reduce(x, pair_out=True))


def test_policies_agree(eb, orc):
    x = orc.corpus(65537, 9)
    want = orc.reduce(x)
    for policy in ("ordered", "compensated", "auto"):
        assert _same(eb.reduce(_dev(x), policy=policy).cpu().numpy(), want)


def test_captured_replay_follows_the_input(eb, orc):
    n = 100003
    x = orc.corpus(n, 11)
    xd = _dev(x)
    red = eb.Reducer(xd)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        red(s)  # warm (no allocation happens in the call)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        red(s)
    for seed in (12, 13):
        y = orc.corpus(n, seed)
        xd.copy_(torch.from_numpy(y))
        g.replay()
        torch.cuda.synchronize()
        assert _same(red.out.cpu().numpy(), orc.reduce(y))


def test_leaf_by_leaf_replay_follows_the_input(eb, orc):
    """The leaf-by-leaf kernel (one column of more leaves than the device holds CTAs)
    captured in a CUDA graph: each replay zeroes its chunk counters first and gives the
    oracle's bits for the plane's current values."""
    n = (1 << 22) + 37
    xd = _dev(orc.corpus(n, 21))
    red = eb.Reducer(xd, pair_out=True)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        red(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        red(s)
    for seed in (22, 23, 24):
        y = orc.corpus(n, seed)
        xd.copy_(torch.from_numpy(y))
        g.replay()
        torch.cuda.synchronize()
        assert _same(red.out.cpu().numpy(), orc.reduce(y, pair_out=True)), seed
    del g


def test_chunk_partials_combine_to_the_whole(eb, orc):
    """Aligned chunks (leafSize * 2^q) are subtrees: their PAIR_OUT partials combined
    by the pairwise levels give the bits of the whole (canonical.h:30-32, :424-439)."""
    n = 1 << 22
    x = orc.corpus(n, 77)
    whole = orc.reduce(x)[0]
    for ranks in (2, 4, 8):
        parts = np.stack([eb.reduce(_dev(x[r * n // ranks:(r + 1) * n // ranks]), pair_out=True).cpu().numpy()
                          for r in range(ranks)])
        root = orc.pairwise(parts)
        assert orc.partial_value(root[0], root[1]) == whole or np.isnan(whole)
        assert np.float64(orc.partial_value(root[0], root[1])).tobytes() == np.float64(whole).tobytes()
