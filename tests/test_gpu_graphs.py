"""The seam's graph groups (capturer, captured, fork, conditional, attribution,
graph, launcher; python/src/seam/eagle_backend.h:286-383 of the eagle source tree)
on the GPU: device-evaluated IF / IF-ELSE / SWITCH / WHILE nodes woven into a live
capture with the loop terms of eagle/conditional/ConditionalGroup.h (cap, runtime
trip count, break cell, the {remaining, ran} cell), graph chaining and launcher
patches, and eagle's captured until-done loop shape — WHILE(finished != n) over the
step entry — against the oracle bit for bit."""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from eagle_b200 import _abi  # noqa: E402
from eagle_b200.graphs import (CaptureConditional, CaptureFork, Graph, Launcher, StreamCapturer,  # noqa: E402
                               capture_add_child, capture_snapshot_nodes, is_node_toggleable)


def _cells(k):
    return torch.zeros(k, dtype=torch.int32, device="cuda")


def _addr(t, i=0):
    return t.data_ptr() + 4 * i


def _bump(ptr, stream):
    d = _abi.new(_abi.CellOpDesc, op=_abi.CELL_BUMP, device=-1, stream=int(stream))
    d.p[0] = int(ptr)
    _abi.check(_abi.lib().eagle_backend_cell_op(ctypes.byref(d)))


def _vals(t):
    torch.cuda.synchronize()
    return [int(v) for v in t.cpu().numpy().view(np.uint32)]


@pytest.fixture
def origin():
    s = torch.cuda.Stream()
    return s.cuda_stream, s


def _run(cap, launcher, stream, replays=1):
    torch.cuda.synchronize()  # cells set by torch on its own stream land first
    for _ in range(replays):
        launcher.launch()
    launcher.synchronize()


def test_while_runs_until_the_guard_and_counts(origin):
    s, keep = origin
    c = _cells(4)  # count, baseline, counter[2]
    c[1] = 5
    loop = CaptureConditional(s, count_ptr=_addr(c, 0), baseline_ptr=_addr(c, 1), loop_cap=100,
                              counter_ptr=_addr(c, 2))
    assert loop.is_loop()
    cap = StreamCapturer(s)
    cap.begin()
    assert cap.graph() != 0
    body = loop.begin()
    assert body == loop.body_stream() == loop.arm_stream(0)
    _bump(_addr(c, 0), body)
    loop.end()
    assert len(loop.nodes(-1)) == 2 and len(loop.nodes(0)) == 2  # head + tail; bump + tail
    launcher = Graph.from_captured(cap.end()).launcher()
    launcher.stream(s)
    _run(cap, launcher, s)
    assert _vals(c) == [5, 5, 95, 5]
    _run(cap, launcher, s)  # the guard already fails: the head resets the cell, the body never runs
    assert _vals(c) == [5, 5, 100, 0]


@pytest.mark.parametrize("terms", ("cap", "limit", "brk"))
def test_while_loop_terms(origin, terms):
    s, keep = origin
    c = _cells(6)  # count, baseline, counter[2], limit, brk
    c[1] = 1000
    c[4] = 2
    loop = CaptureConditional(s, count_ptr=_addr(c, 0), baseline_ptr=_addr(c, 1), loop_cap=3 if terms == "cap" else 50,
                              counter_ptr=_addr(c, 2), limit_ptr=_addr(c, 4) if terms == "limit" else 0,
                              brk_ptr=_addr(c, 5) if terms == "brk" else 0)
    cap = StreamCapturer(s)
    cap.begin()
    body = loop.begin()
    _bump(_addr(c, 0), body)
    if terms == "brk":
        _bump(_addr(c, 5), body)
    loop.end()
    launcher = Graph.from_captured(cap.end()).launcher()
    launcher.stream(s)
    _run(cap, launcher, s)
    want = {"cap": 3, "limit": 2, "brk": 1}[terms]
    v = _vals(c)
    assert v[0] == want and v[3] == want


@pytest.mark.parametrize("negate", (False, True))
def test_if_guard(origin, negate):
    s, keep = origin
    c = _cells(3)  # count, baseline, hits
    loop = CaptureConditional(s, count_ptr=_addr(c, 0), baseline_ptr=_addr(c, 1), negate=negate)
    assert not loop.is_loop()
    cap = StreamCapturer(s)
    cap.begin()
    body = loop.begin()
    _bump(_addr(c, 2), body)
    loop.end()
    launcher = Graph.from_captured(cap.end()).launcher()
    launcher.stream(s)
    _run(cap, launcher, s)  # count == baseline: the guard fails (holds when negated)
    assert _vals(c)[2] == (1 if negate else 0)
    c[0] = 7
    _run(cap, launcher, s)
    assert _vals(c)[2] == 1


def _has(flag):
    g = ctypes.c_uint64()
    _abi.check(_abi.lib().eagle_backend_capabilities(ctypes.byref(g)))
    return bool(g.value & flag)


def test_if_else_and_switch(origin):
    if not (_has(_abi.CAP_CONDITIONAL_IF_ELSE) and _has(_abi.CAP_CONDITIONAL_SWITCH)):
        pytest.skip("driver without IF/ELSE and SWITCH nodes")
    s, keep = origin
    c = _cells(8)  # count, baseline, arm, a, b, s0, s1, s2
    ie = CaptureConditional(s, count_ptr=_addr(c, 0), baseline_ptr=_addr(c, 1), kind="if_else")
    sw = CaptureConditional(s, count_ptr=_addr(c, 2), kind="switch", arms=3)
    cap = StreamCapturer(s)
    cap.begin()
    ie.begin()
    _bump(_addr(c, 3), ie.arm_stream(0))
    _bump(_addr(c, 4), ie.arm_stream(1))
    ie.end()
    sw.begin()
    for k in range(3):
        _bump(_addr(c, 5 + k), sw.arm_stream(k))
    sw.end()
    launcher = Graph.from_captured(cap.end()).launcher()
    launcher.stream(s)
    _run(cap, launcher, s)  # guard fails -> else arm; switch arm 0
    assert _vals(c)[3:] == [0, 1, 1, 0, 0]
    c[0] = 1
    c[2] = 2
    _run(cap, launcher, s)
    assert _vals(c)[3:] == [1, 1, 1, 0, 1]
    c[2] = 9  # past the last arm: none runs
    _run(cap, launcher, s)
    assert _vals(c)[3:] == [2, 1, 1, 0, 1]


def test_conditional_refusals(origin):
    s, keep = origin
    c = _cells(4)
    with pytest.raises(ValueError, match="loop_cap"):
        CaptureConditional(s, count_ptr=_addr(c, 0), counter_ptr=_addr(c, 2), loop_cap=0)
    with pytest.raises(ValueError, match="one arm"):
        CaptureConditional(s, count_ptr=_addr(c, 0), kind="if", arms=2)
    with pytest.raises(ValueError, match="arm-index"):
        CaptureConditional(s, count_ptr=0, kind="switch", arms=2)
    loop = CaptureConditional(s, count_ptr=_addr(c, 0))
    with pytest.raises(ValueError, match="not capturing"):
        loop.begin()
    # an arm that launched nothing is refused at end; the outer capture is then discarded
    empty = CaptureConditional(s, count_ptr=_addr(c, 0), counter_ptr=_addr(c, 2), loop_cap=4)
    cap = StreamCapturer(s)
    cap.begin()
    empty.begin()
    with pytest.raises(ValueError, match="no work"):
        empty.end()
    try:
        cap.end()
    except (ValueError, _abi.BackendError):
        pass


def test_graph_chain_and_launcher_patches(origin):
    s, keep = origin
    c = _cells(4)
    parts = []
    for k in (0, 1):
        cap = StreamCapturer(s)
        cap.begin()
        _bump(_addr(c, k), s)
        parts.append(cap.end())
    assert all(parts)
    g = Graph()
    assert g.last_node() == 0  # the empty root
    for p in parts:
        g.add_node(p)
    assert g.last_node() == 2 and not parts[0]
    g.stream(s)
    launcher = g.launcher()
    assert launcher.kernel_node_count() == 2
    _run(None, launcher, s, replays=3)
    assert _vals(c) == [3, 3, 0, 0]
    launcher.set_logical_size(1)  # 1x1 kernels keep their shape
    _run(None, launcher, s)
    assert _vals(c) == [4, 4, 0, 0]

    # argument patch: re-point a captured bump at another cell
    cap = StreamCapturer(s)
    cap.begin()
    _bump(_addr(c, 0), s)
    node = capture_snapshot_nodes(s)[-1]
    assert is_node_toggleable(node)
    one = Graph.from_captured(cap.end())
    one.stream(s)
    lz = one.launcher()
    assert one.last_node() == -1 and lz.kernel_node_count() == 0
    target = ctypes.c_uint64(_addr(c, 2))
    lz.set_kernel_params(node, [ctypes.addressof(target)])
    _run(None, lz, s)
    assert _vals(c) == [4, 4, 1, 0]
    lz.set_node_enabled(node, False)
    _run(None, lz, s)
    assert _vals(c) == [4, 4, 1, 0]
    lz.set_node_enabled(node, True)

    # exec update from a capture of the same shape, refused for another shape
    cap = StreamCapturer(s)
    cap.begin()
    _bump(_addr(c, 3), s)
    same = cap.end()
    assert lz.try_exec_update(same)
    _run(None, lz, s)
    assert _vals(c) == [4, 4, 1, 1]
    cap = StreamCapturer(s)
    cap.begin()
    _bump(_addr(c, 3), s)
    _bump(_addr(c, 3), s)
    other = cap.end()
    assert not lz.try_exec_update(other)

    # a clone of the source graph (argument patches reach it; exec updates do not)
    # runs as a child of another capture
    clone = lz.clone_graph()
    cap = StreamCapturer(s)
    cap.begin()
    capture_add_child(s, clone, conditional_body=True)
    host = Graph.from_captured(cap.end())
    host.stream(s)
    hl = host.launcher()
    _run(None, hl, s)
    assert _vals(c) == [4, 4, 2, 1]
    Launcher.destroy_graph(clone)


def test_memcpy_source_patch(origin):
    s, keep = origin
    a = torch.arange(16, dtype=torch.int32, device="cuda")
    b = torch.arange(100, 116, dtype=torch.int32, device="cuda")
    out = torch.zeros(16, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    cap = StreamCapturer(s)
    cap.begin()
    _abi.check(_abi.lib().eagle_backend_memcpy_device(out.data_ptr(), a.data_ptr(), 64, s))
    node = capture_snapshot_nodes(s)[-1]
    g = Graph.from_captured(cap.end())
    g.stream(s)
    lz = g.launcher()
    lz.set_memcpy_source(node, b.data_ptr())
    _run(None, lz, s)
    assert out.cpu().tolist() == list(range(100, 116))


def test_fork_join_marks(origin):
    s, keep = origin
    c = _cells(4)
    f = CaptureFork(s, 2, waits=1)
    assert len(f) == 2 and f.origin() == s and not f.forked()
    cap = StreamCapturer(s)
    cap.begin()
    f.fork()
    assert f.forked()
    _bump(_addr(c, 0), f.branch(0))
    m = f.mark(0)
    f.wait(1, m)
    _bump(_addr(c, 1), f.branch(1))
    f.join()
    assert not f.forked()
    _bump(_addr(c, 2), s)
    with pytest.raises(IndexError):
        f.mark(0)  # the one pre-made mark is used
    g = Graph.from_captured(cap.end())
    g.stream(s)
    lz = g.launcher()
    _run(None, lz, s, replays=2)
    assert _vals(c) == [2, 2, 2, 0]
    with pytest.raises(IndexError):
        f.branch(5)


def test_clone_refuses_a_conditional(origin):
    s, keep = origin
    c = _cells(4)
    loop = CaptureConditional(s, count_ptr=_addr(c, 0))
    cap = StreamCapturer(s)
    cap.begin()
    _bump(_addr(c, 1), loop.begin())
    loop.end()
    lz = Graph.from_captured(cap.end()).launcher()
    with pytest.raises(_abi.BackendUnsupported, match="conditional node"):
        lz.clone_graph()


@pytest.mark.parametrize("fma", (False, True))
def test_captured_until_done_loop(eb, orc, origin, fma):
    """eagle's captured until-done shape: WHILE(finished != n), capped at
    max_steps / K iterations, over the step entry run for K steps a launch."""
    s, keep = origin
    n, K, max_steps = 50_000, 100, 10_000
    rng = np.random.default_rng(21)
    om = rng.uniform(1, 3, n)
    te = 10.0 ** rng.uniform(-2, 1, n)
    x0 = rng.normal(1.0, 0.1, n)
    dev = dict(om=torch.from_numpy(om).cuda(), te=torch.from_numpy(te).cuda(), x=torch.from_numpy(x0).cuda(),
               v=torch.zeros(n, dtype=torch.float64, device="cuda"), t=torch.zeros(n, dtype=torch.float64, device="cuda"),
               m=torch.zeros(n, dtype=torch.uint8, device="cuda"))
    cells = _cells(4)  # finished, n, counter[2]
    cells[1] = n
    budget = torch.tensor([K], dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()

    def h(t, k):
        return _abi.ScalarHandle(t.data_ptr(), k, 1, 2, t.device.index)

    args = [h(dev["om"], n), h(dev["te"], n), ctypes.c_double(1e-3), h(dev["m"], n), h(dev["x"], n), h(dev["v"], n),
            h(dev["t"], n), _abi.ScalarHandle(_addr(cells, 0), 1, 1, 2, 0), h(budget, 1)]
    addrs = (ctypes.c_uint64 * len(args))(*[ctypes.addressof(a) for a in args])
    fn = eb.entry("oscillator_spread" + ("_fma" if fma else ""))
    loop = CaptureConditional(s, count_ptr=_addr(cells, 0), baseline_ptr=_addr(cells, 1),
                              loop_cap=max_steps // K, counter_ptr=_addr(cells, 2))
    cap = StreamCapturer(s)
    cap.begin()
    body = loop.begin()
    d = _abi.new(_abi.LaunchDesc, device=-1, block=256, function=fn, nparams=len(args), base=0, count=n,
                 n_samples=n, stream=body)
    d.params = ctypes.cast(addrs, ctypes.POINTER(ctypes.c_uint64))
    launched = ctypes.c_int32()
    _abi.check(_abi.lib().eagle_backend_run_device(ctypes.byref(d), ctypes.byref(launched)))
    loop.end()
    launcher = Graph.from_captured(cap.end()).launcher()
    launcher.stream(s)
    _run(None, launcher, s)
    st = [x0.copy(), np.zeros(n), np.zeros(n), np.zeros(n, np.uint8)]
    _, fin, longest, total = orc.oscillator_run(om, *st, t_end=te, dt=1e-3, max_steps=max_steps, fused=fma)
    for k, r in zip(("x", "v", "t", "m"), st):
        assert dev[k].cpu().numpy().tobytes() == r.tobytes(), k
    v = _vals(cells)
    assert v[0] == fin and fin > 0.99 * n
    assert v[3] == -(-longest // K)  # iterations ran: ceil(longest / K), at most the cap
    if fin == n:
        _run(None, launcher, s)  # a replay of a finished loop runs no iteration
        assert _vals(cells)[3] == 0
