"""The K-class physical sort (eagle/filtering/ReorderClasses.h;
``eagle_backend_reorder_classes_device``) and the compaction with the class
trigger (``eagle_backend_compact_classes_device``) on the GPU against the oracle:
planes, perm, inv, index_map, offsets, count, span and the sort counter bit for
bit over class counts 2..255 (class values past K clamp to K-1), both key forms
(live-then-class, class within the live prefix), the fire gate; mixed32 and the
class trigger word."""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from eagle_b200 import _abi  # noqa: E402

MASK, CLS = 1, 2


def _host(n, K, seed, p_drop):
    g = np.random.default_rng(seed)
    cls = g.integers(0, K + 2, n).astype(np.uint8)  # some past K: clamped to K - 1
    return [g.standard_normal(n), (g.random(n) < p_drop).astype(np.uint8), cls,
            g.integers(-2**15, 2**15 - 1, n, dtype=np.int64).astype(np.int16),
            g.standard_normal(n) + 1j * g.standard_normal(n),
            g.standard_normal(n).astype(np.float32),                            # a pair of 4-byte planes,
            g.integers(-2**31, 2**31 - 1, n, dtype=np.int64).astype(np.int32)]  # moved together


def _cells(n, count, span, K):
    d = dict(perm=torch.arange(n, dtype=torch.int32, device="cuda"),
             inv=torch.arange(n, dtype=torch.int32, device="cuda"),
             im=torch.zeros(max(n, 1), dtype=torch.int32, device="cuda"),
             count=torch.tensor([count], dtype=torch.int32, device="cuda"),
             span=torch.tensor([span], dtype=torch.int32, device="cuda"),
             off=torch.zeros(K + 1, dtype=torch.int32, device="cuda"),
             sorts=torch.zeros(1, dtype=torch.int32, device="cuda"))
    return d


def _run(eb, dev, c, K, **kw):
    return eb.reorder_classes(dev, dev[MASK], dev[CLS], c["perm"], c["inv"], c["im"], c["count"], c["span"],
                              c["off"], c["sorts"], K, **kw)


def _check(dev, host, c, hp, hi, him, off, count, span, live):
    torch.cuda.synchronize()
    for d, h in zip(dev, host):
        assert d.cpu().numpy().tobytes() == h.tobytes()
    assert c["perm"].cpu().numpy().tobytes() == hp.tobytes()
    assert c["inv"].cpu().numpy().tobytes() == hi.tobytes()
    assert c["im"].cpu().numpy()[:live].tobytes() == him[:live].tobytes()
    assert c["off"].cpu().numpy().astype(np.int64).tolist() == list(off)
    assert int(c["count"].item()) == count and int(c["span"].item()) == span


@pytest.mark.parametrize("drop", (True, False))
@pytest.mark.parametrize("K", (2, 7, 255))
@pytest.mark.parametrize("n", (1, 4097, 100_003))
def test_class_sort_matches_oracle(eb, orc, n, K, drop):
    host = _host(n, K, n + K, 0.4)
    dev = [torch.from_numpy(h.copy()).cuda() for h in host]
    c = _cells(n, 0, n, K)
    hp, hi, him = np.arange(n, dtype=np.int32), np.arange(n, dtype=np.int32), np.zeros(max(n, 1), np.int32)
    keep = _run(eb, dev, c, K, drop=drop)
    off, cnt, sp, _, _ = orc.reorder_classes(host, MASK, CLS, hp, hi, him, 0, n, K, drop=drop)
    _check(dev, host, c, hp, hi, him, off, cnt, sp, cnt)
    assert int(c["sorts"].item()) == 1
    # now by class only within the live prefix, after some classes changed
    cls = host[CLS].copy()
    cls[:cnt][::3] = (cls[:cnt][::3] + 1) % K
    host[CLS][:] = cls
    dev[CLS].copy_(torch.from_numpy(cls))
    keep = _run(eb, dev, c, K, drop=drop, within=True)
    off2, cnt2, sp2, _, _ = orc.reorder_classes(host, MASK, CLS, hp, hi, him, cnt, sp, K, drop=drop, within=True)
    _check(dev, host, c, hp, hi, him, off2, cnt2, sp2, cnt2)
    assert int(c["sorts"].item()) == 2
    del keep


def test_class_sort_fire_gate(eb, orc):
    n, K = 30_000, 4
    host = _host(n, K, 3, 0.5)
    dev = [torch.from_numpy(h.copy()).cuda() for h in host]
    c = _cells(n, 0, n, K)
    fire = torch.zeros(1, dtype=torch.int32, device="cuda")
    _run(eb, dev, c, K, fire=fire)
    torch.cuda.synchronize()
    for d, h in zip(dev, host):
        assert d.cpu().numpy().tobytes() == h.tobytes()
    assert int(c["sorts"].item()) == 0
    fire.fill_(1)
    _run(eb, dev, c, K, fire=fire)
    hp, hi, him = np.arange(n, dtype=np.int32), np.arange(n, dtype=np.int32), np.zeros(n, np.int32)
    off, cnt, sp, f, _ = orc.reorder_classes(host, MASK, CLS, hp, hi, him, 0, n, K, fire=1)
    _check(dev, host, c, hp, hi, him, off, cnt, sp, cnt)
    assert int(fire.item()) == f == 0 and int(c["sorts"].item()) == 1


@pytest.mark.parametrize("stale", (0, 10_000))
@pytest.mark.parametrize("K", (2, 16))
def test_compact_with_class_trigger(eb, orc, K, stale):
    n = 65_537
    g = np.random.default_rng(K + stale)
    # runs of one class so some 32-slot groups are pure and some mixed
    cls = np.repeat(g.integers(0, K, n // 64 + 1), 64)[:n].astype(np.uint8)
    cls[g.random(n) < 0.02] = g.integers(0, K)
    mask = (g.random(n) < 0.3).astype(np.uint8)
    d_mask, d_cls = torch.from_numpy(mask).cuda(), torch.from_numpy(cls).cuda()
    cells = torch.zeros(8, dtype=torch.int32, device="cuda")  # count, live32, span, fire, mixed, class_fire, stale
    cells[2] = n
    cells[6] = stale
    im = torch.zeros(n, dtype=torch.int32, device="cuda")
    a = lambda k: cells.data_ptr() + 4 * k  # noqa: E731
    d = _abi.new(_abi.CompactClassesDesc, flags=_abi.COMPACT_MASK_IS_DROP, device=0, mask=d_mask.data_ptr(),
                 index_map=im.data_ptr(), count=a(0), n=n, live32=a(1), span=a(2), fire=a(3), theta=0.9,
                 class_plane=d_cls.data_ptr(), classes=K, class_theta=0.25, mixed32=a(4), stale_count=a(6),
                 class_fire=a(5))
    _abi.check(_abi.lib().eagle_backend_compact_classes_device(ctypes.byref(d)))
    scratch = torch.zeros(int(d.scratch_bytes), dtype=torch.uint8, device="cuda")
    d.scratch = scratch.data_ptr()
    _abi.check(_abi.lib().eagle_backend_compact_classes_device(ctypes.byref(d)))
    torch.cuda.synchronize()
    v = cells.cpu().numpy()
    idx, c, live32, fire = orc.compact(mask, drop=True, span=n, theta=0.9, trigger=True)
    assert im.cpu().numpy()[:c].tobytes() == idx.tobytes()
    assert (v[0], v[1], v[3]) == (c, live32, fire)
    mixed, cfire = orc.class_trigger(mask, cls, drop=True, live32=live32, span=n, count=c, live_fire=fire,
                                     class_theta=0.25, stale=stale)
    assert (v[4], v[5]) == (mixed, cfire)
    assert mixed > 0
