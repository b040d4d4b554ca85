"""The seam's interop group (python/src/seam/eagle_backend.h:396-440) on the GPU:
the DLPack stream fence orders a producer stream's work before a consumer's
without blocking the host, events come from a reused pool, page-locked host
memory from host_alloc feeds asynchronous copies, and host_func runs a callback
in stream order."""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from eagle_b200 import _abi  # noqa: E402


def test_fence_orders_producer_before_consumer():
    L = _abi.lib()
    a, b = torch.cuda.Stream(), torch.cuda.Stream()
    x = torch.zeros(1 << 20, device="cuda")
    y = torch.empty_like(x)
    torch.cuda.synchronize()
    for value in (7.0, 9.0):
        with torch.cuda.stream(a):
            torch.cuda._sleep(20_000_000)  # a slow producer: ~10 ms of spinning
            x.fill_(value)
        _abi.check(L.eagle_backend_fence(2, 0, a.cuda_stream, b.cuda_stream))
        with torch.cuda.stream(b):
            y.copy_(x)
        b.synchronize()
        assert bool((y == value).all())
    n = ctypes.c_int64()
    _abi.check(L.eagle_backend_event_pool_created(ctypes.byref(n)))
    assert n.value >= 1
    before = n.value
    _abi.check(L.eagle_backend_fence(2, 0, a.cuda_stream, b.cuda_stream))
    _abi.check(L.eagle_backend_event_pool_created(ctypes.byref(n)))
    assert n.value == before  # the pool reuses its events
    torch.cuda.synchronize()


def test_host_alloc_feeds_async_copies():
    L = _abi.lib()
    nbytes = 1 << 22
    ptr = ctypes.c_uint64()
    _abi.check(L.eagle_backend_host_alloc(nbytes, ctypes.byref(ptr)))
    assert ptr.value != 0
    host = np.ctypeslib.as_array((ctypes.c_uint8 * nbytes).from_address(ptr.value))
    host[:] = np.arange(nbytes, dtype=np.uint64).astype(np.uint8)
    dev = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    _abi.check(L.eagle_backend_memcpy(dev.data_ptr(), ptr.value, nbytes, _abi.COPY_H2D, s))
    torch.cuda.synchronize()
    assert dev.cpu().numpy().tobytes() == host.tobytes()
    _abi.check(L.eagle_backend_host_free(ptr.value))


def test_host_func_runs_in_stream_order():
    L = _abi.lib()
    seen = []
    x = torch.zeros(4, device="cuda")
    proto = ctypes.CFUNCTYPE(None, ctypes.c_void_p)
    cb = proto(lambda arg: seen.append(int(arg or 0)))  # kept alive until the stream is past it
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        torch.cuda._sleep(10_000_000)
        x.fill_(3.0)
    _abi.check(L.eagle_backend_host_func(s.cuda_stream, ctypes.cast(cb, ctypes.c_void_p), ctypes.c_void_p(42)))
    assert seen == [] or seen == [42]
    _abi.check(L.eagle_backend_stream_sync(-1, s.cuda_stream))  # the foreign call drops the GIL while it waits
    assert seen == [42]
    assert bool((x == 3.0).all())
