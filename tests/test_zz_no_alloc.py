"""The allocation-free compaction (eagle_backend_x_b200_compact_device_noalloc),
for callers that cannot allocate device memory: through the C-ABI it must give
the same index map and count as the regular entry (eagle_backend_compact_device,
which takes caller scratch) and as numpy's flatnonzero of the kept samples, on two
calls in a row, since every call reuses the one built-in scratch array; and it
must refuse a batch past its 2^28-sample limit.

This file is collected last so that a failure here stops a -x run only after
every other test has run."""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from eagle_b200 import _abi  # noqa: E402


def _noalloc(mask, drop=True, trigger=False):
    n = mask.numel()
    index_map = torch.full((max(n, 1),), -1, dtype=torch.int32, device=mask.device)
    count = torch.full((1,), -1, dtype=torch.int32, device=mask.device)
    d = _abi.new(_abi.CompactDesc, flags=_abi.COMPACT_MASK_IS_DROP if drop else 0, device=-1, mask=mask.data_ptr(),
                 index_map=index_map.data_ptr(), count=count.data_ptr(), n=n,
                 stream=torch.cuda.current_stream().cuda_stream)
    extra = None
    if trigger:
        extra = torch.zeros(3, dtype=torch.int32, device=mask.device)  # live32, fire, span
        extra[2] = n
        d.live32, d.fire, d.span, d.theta = extra.data_ptr(), extra.data_ptr() + 4, extra.data_ptr() + 8, 0.5
    _abi.check(_abi.lib().eagle_backend_x_b200_compact_device_noalloc(ctypes.byref(d)))
    torch.cuda.synchronize()
    return index_map, count, extra


@pytest.mark.parametrize("n", (0, 1, 4097, (1 << 20) + 37, 1 << 24))
@pytest.mark.parametrize("drop", (True, False))
def test_matches_the_scratch_entry_twice(eb, n, drop):
    for seed, p in ((1, 0.4), (2, 0.9)):  # two calls in a row over the shared array
        mask = torch.from_numpy(np.random.default_rng([seed, n]).random(n) < p).cuda()
        m0, c0, _ = _noalloc(mask, drop=drop)
        ref = eb.Compactor(mask, drop=drop)
        m1, c1 = ref()
        torch.cuda.synchronize()
        c = int(c1.item())
        assert int(c0.item()) == c
        assert torch.equal(m0[:c], m1[:c])
        keep = mask.cpu().numpy()
        want = np.flatnonzero(~keep if drop else keep)
        assert c == want.size and np.array_equal(m0[:c].cpu().numpy(), want)


def test_trigger_matches(eb):
    n = 100_003
    for seed in (3, 4):
        mask = torch.from_numpy(np.random.default_rng(seed).random(n) < 0.95).cuda()
        m0, c0, extra = _noalloc(mask, trigger=True)
        ref = eb.Compactor(mask, trigger=True, theta=0.5)
        m1, c1 = ref()
        torch.cuda.synchronize()
        assert int(c0.item()) == int(c1.item())
        assert int(extra[0].item()) == int(ref.live32.item()) and int(extra[1].item()) == int(ref.fire.item())


def test_largest_batch_and_refusal(eb):
    n = 1 << 28
    mask = torch.from_numpy(np.random.default_rng(5).random(1 << 20) < 0.5).cuda().repeat(256)
    m0, c0, _ = _noalloc(mask)
    m1, c1 = eb.Compactor(mask)()
    torch.cuda.synchronize()
    c = int(c1.item())
    assert int(c0.item()) == c and torch.equal(m0[:c], m1[:c])
    want = np.flatnonzero(~mask[: 1 << 20].cpu().numpy())
    assert c == 256 * want.size
    assert np.array_equal(m0[:want.size].cpu().numpy(), want)
    assert np.array_equal(m0[c - want.size:c].cpu().numpy(), want + (255 << 20))
    del m0, m1, mask
    d = _abi.new(_abi.CompactDesc, flags=_abi.COMPACT_MASK_IS_DROP, mask=1, index_map=1, count=1, n=n + 1)
    assert _abi.lib().eagle_backend_x_b200_compact_device_noalloc(ctypes.byref(d)) == _abi.UNSUPPORTED
    assert "2^28" in _abi.last_error() or str(n) in _abi.last_error()
