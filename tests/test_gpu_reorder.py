"""The physical reorder of the active set (eagle/filtering/Reorder.h,
``eagle_backend_reorder_device``) and its undo (``eagle_backend_x_restore_device``)
on the GPU against the oracle's restatement: every plane (1, 2, 4, 8 and 16-byte
elements, the mask among them), perm, inv, index_map, count and span bit for bit,
over edge sizes, partial spans, two reorders in a row, the fire gate, and a
restore back to sample order."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _host(n, seed, p_drop):
    g = np.random.default_rng(seed)
    return [g.standard_normal(n),                                    # 8 bytes
            g.integers(-2**31, 2**31 - 1, n, dtype=np.int64).astype(np.int32),  # 4
            g.integers(-2**15, 2**15 - 1, n, dtype=np.int64).astype(np.int16),  # 2
            (g.random(n) < p_drop).astype(np.uint8),                 # 1: the mask
            (g.standard_normal(n) + 1j * g.standard_normal(n)),      # 16
            g.standard_normal(n).astype(np.float32)]                 # 4


MASK = 3


def _dev(host):
    return [torch.from_numpy(h.copy()).cuda() for h in host]


def _cells(n, span):
    perm = torch.arange(n, dtype=torch.int32, device="cuda")
    inv = torch.arange(n, dtype=torch.int32, device="cuda")
    im = torch.zeros(max(n, 1), dtype=torch.int32, device="cuda")
    count = torch.zeros(1, dtype=torch.int32, device="cuda")
    sp = torch.tensor([span], dtype=torch.int32, device="cuda")
    return perm, inv, im, count, sp


def _same(dev, host):
    for d, h in zip(dev, host):
        assert d.cpu().numpy().tobytes() == h.tobytes()


@pytest.mark.parametrize("drop", (True, False))
@pytest.mark.parametrize("n", (1, 7, 4096, 4097, 100_003))
def test_reorder_matches_oracle(eb, orc, n, drop):
    host = _host(n, n, 0.35)
    dev = _dev(host)
    perm, inv, im, count, span = _cells(n, n)
    hp, hi, him = np.arange(n, dtype=np.int32), np.arange(n, dtype=np.int32), np.zeros(max(n, 1), np.int32)
    keep_alive = eb.reorder(dev, dev[MASK], perm, inv, im, count, span, drop=drop)
    c, sp, _ = orc.reorder(host, MASK, hp, hi, him, n, drop=drop)
    torch.cuda.synchronize()
    _same(dev, host)
    assert perm.cpu().numpy().tobytes() == hp.tobytes() and inv.cpu().numpy().tobytes() == hi.tobytes()
    assert int(count.item()) == c and int(span.item()) == sp
    assert im.cpu().numpy()[:c].tobytes() == him[:c].tobytes()
    # a second reorder over the live prefix, after some live samples are dropped
    m2 = host[MASK].copy()
    m2[:c][::5] = 1 if drop else 0
    host[MASK][:] = m2
    dev[MASK].copy_(torch.from_numpy(m2))
    keep_alive = eb.reorder(dev, dev[MASK], perm, inv, im, count, span, drop=drop)
    c2, sp2, _ = orc.reorder(host, MASK, hp, hi, him, sp, drop=drop)
    torch.cuda.synchronize()
    _same(dev, host)
    assert perm.cpu().numpy().tobytes() == hp.tobytes() and inv.cpu().numpy().tobytes() == hi.tobytes()
    assert int(count.item()) == c2 and int(span.item()) == sp2
    del keep_alive


@pytest.mark.parametrize("pattern", ("keep_most", "keep_few", "all", "none", "runs", "front"))
def test_reorder_densities_and_runs(eb, orc, pattern):
    """Masks that move the kept runs by little (a tile's kept run then lands in its
    own tile and the one before, which it has to wait on) and by much, with the
    dropped runs staged and copied back: every plane, perm, inv and the count bit
    for bit against the oracle, on 2^21 + 123 slots (513 tiles)."""
    n = (1 << 21) + 123
    host = _host(n, 99, 0.5)
    g = np.random.default_rng(7)
    drop = {"keep_most": g.random(n) < 0.001, "keep_few": g.random(n) < 0.999, "all": np.zeros(n, bool),
            "none": np.ones(n, bool), "runs": (np.arange(n) // 5000) % 2 == 1,
            "front": np.arange(n) >= n // 3}[pattern]
    host[MASK] = drop.astype(np.uint8)
    dev = _dev(host)
    perm, inv, im, count, span = _cells(n, n)
    hp, hi, him = np.arange(n, dtype=np.int32), np.arange(n, dtype=np.int32), np.zeros(n, np.int32)
    keep_alive = eb.reorder(dev, dev[MASK], perm, inv, im, count, span, drop=True)
    c, sp, _ = orc.reorder(host, MASK, hp, hi, him, n, drop=True)
    torch.cuda.synchronize()
    _same(dev, host)
    assert perm.cpu().numpy().tobytes() == hp.tobytes() and inv.cpu().numpy().tobytes() == hi.tobytes()
    assert int(count.item()) == c and int(span.item()) == sp
    assert im.cpu().numpy()[:c].tobytes() == him[:c].tobytes()
    del keep_alive


@pytest.mark.parametrize("n", (4097, (1 << 20) + 3))
def test_reorder_paired_planes_and_a_narrow_stage(eb, orc, n):
    """Planes of one element size move two at a time when both dropped runs fit the
    stage: with no plane wider than 4 bytes the stage holds 4 bytes a slot, so the two
    byte planes pair and the int32 and float32 planes move alone; every plane, perm, inv
    and the count bit for bit against the oracle, a second reorder after it too."""
    g = np.random.default_rng(n)
    host = [(g.random(n) < 0.4).astype(np.uint8),                            # the mask
            g.integers(0, 256, n, dtype=np.int64).astype(np.uint8),
            g.integers(-2**31, 2**31 - 1, n, dtype=np.int64).astype(np.int32),
            g.standard_normal(n).astype(np.float32),
            g.integers(-2**15, 2**15 - 1, n, dtype=np.int64).astype(np.int16)]
    dev = _dev(host)
    perm, inv, im, count, span = _cells(n, n)
    hp, hi, him = np.arange(n, dtype=np.int32), np.arange(n, dtype=np.int32), np.zeros(n, np.int32)
    for r in range(2):
        keep_alive = eb.reorder(dev, dev[0], perm, inv, im, count, span, drop=True)
        c, sp, _ = orc.reorder(host, 0, hp, hi, him, n if r == 0 else sp, drop=True)
        torch.cuda.synchronize()
        _same(dev, host)
        assert perm.cpu().numpy().tobytes() == hp.tobytes() and inv.cpu().numpy().tobytes() == hi.tobytes()
        assert int(count.item()) == c and int(span.item()) == sp
        m2 = host[0].copy()
        m2[:c][::3] = 1
        host[0][:] = m2
        dev[0].copy_(torch.from_numpy(m2))
        del keep_alive


def test_partial_span_leaves_the_tail(eb, orc):
    n = 50_001
    host = _host(n, 3, 0.5)
    dev = _dev(host)
    perm, inv, im, count, span = _cells(n, 30_017)
    hp, hi, him = np.arange(n, dtype=np.int32), np.arange(n, dtype=np.int32), np.zeros(n, np.int32)
    eb.reorder(dev, dev[MASK], perm, inv, im, count, span)
    c, sp, _ = orc.reorder(host, MASK, hp, hi, him, 30_017)
    torch.cuda.synchronize()
    _same(dev, host)
    assert perm.cpu().numpy().tobytes() == hp.tobytes() and int(count.item()) == c and int(span.item()) == sp


def test_fire_gates_the_reorder(eb, orc):
    n = 20_000
    host = _host(n, 4, 0.5)
    dev = _dev(host)
    perm, inv, im, count, span = _cells(n, n)
    fire = torch.zeros(1, dtype=torch.int32, device="cuda")
    eb.reorder(dev, dev[MASK], perm, inv, im, count, span, fire=fire)
    torch.cuda.synchronize()
    _same(dev, host)  # fire == 0: nothing moved
    assert int(span.item()) == n and int(count.item()) == 0
    fire.fill_(1)
    eb.reorder(dev, dev[MASK], perm, inv, im, count, span, fire=fire)
    hp, hi, him = np.arange(n, dtype=np.int32), np.arange(n, dtype=np.int32), np.zeros(n, np.int32)
    c, sp, f = orc.reorder(host, MASK, hp, hi, him, n, fire=1)
    torch.cuda.synchronize()
    _same(dev, host)
    assert int(fire.item()) == f == 0 and int(count.item()) == c


def test_restore_returns_sample_order(eb, orc):
    n = 70_001
    host = _host(n, 5, 0.4)
    orig = [h.copy() for h in host]
    dev = _dev(host)
    perm, inv, im, count, span = _cells(n, n)
    eb.reorder(dev, dev[MASK], perm, inv, im, count, span)
    m = dev[MASK].cpu().numpy()
    c = int(count.item())
    m[:c][::3] = 1
    dev[MASK].copy_(torch.from_numpy(m))
    orig[MASK][perm.cpu().numpy()] = m  # the mask edit, in sample order
    eb.reorder(dev, dev[MASK], perm, inv, im, count, span)
    eb.restore(dev, perm, inv)
    torch.cuda.synchronize()
    _same(dev, orig)
    ident = np.arange(n, dtype=np.int32).tobytes()
    assert perm.cpu().numpy().tobytes() == ident and inv.cpu().numpy().tobytes() == ident


def test_empty_batch(eb):
    perm, inv, im, count, span = _cells(0, 0)
    count.fill_(5)
    span.fill_(5)
    mask = torch.zeros(0, dtype=torch.uint8, device="cuda")
    eb.reorder([mask], mask, perm, inv, im, count, span)
    torch.cuda.synchronize()
    assert int(count.item()) == 0 and int(span.item()) == 0
