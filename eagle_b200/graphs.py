"""Python faces of the seam's graph groups, with the names and arguments eagle's
``_core`` binds them under (python/src/eagle_core.cpp:2161-2770 of the eagle
source tree): ``StreamCapturer`` / ``CapturedGraph``, ``CaptureFork``,
``CaptureConditional``, ``Graph`` and ``Launcher``. Streams are raw
``cudaStream_t`` integers, device cells raw device addresses, as there.

The usual shape of eagle's captured until-done loop on top of them::

    loop = CaptureConditional(origin, count_ptr=finished, baseline_ptr=n_cell,
                              loop_cap=cap, counter_ptr=counter)   # before capture
    cap = StreamCapturer(origin); cap.begin()
    body = loop.begin()          # launch the step (+ mask count) on `body`
    ...
    loop.end()
    launcher = Graph.from_captured(cap.end()).launcher()
    launcher.launch(); launcher.synchronize()
"""

from __future__ import annotations

import ctypes

from . import _abi

_KINDS = {"": 0, "if": _abi.COND_IF, "if_else": _abi.COND_IF_ELSE, "while": _abi.COND_WHILE,
          "switch": _abi.COND_SWITCH}


def _lib():
    return _abi.lib()


def _need(h, what):
    if not h:
        raise ValueError(f"{what}: the handle was released or consumed")
    return h


def _nodes(fn, *args):
    buf = ctypes.POINTER(ctypes.c_uint64)()
    n = ctypes.c_int64()
    _abi.check(fn(*args, ctypes.byref(buf), ctypes.byref(n)))
    try:
        return [int(buf[i]) for i in range(n.value)]
    finally:
        _lib().eagle_backend_free(ctypes.cast(buf, ctypes.c_void_p))


class CapturedGraph:
    """A finished capture (owns its ``cudaGraph_t`` until a Graph consumes it)."""

    def __init__(self, h):
        self._h = h

    def __bool__(self):
        if not self._h:
            return False
        v = ctypes.c_int32()
        _abi.check(_lib().eagle_backend_captured_is_valid(self._h, ctypes.byref(v)))
        return v.value != 0

    def _take(self):
        h, self._h = _need(self._h, "CapturedGraph"), None
        return h

    def __del__(self):
        if getattr(self, "_h", None):
            _lib().eagle_backend_captured_release(self._h)
            self._h = None


class StreamCapturer:
    """A thread-local capture of ``stream``."""

    def __init__(self, stream: int, device: int = -1):
        d = _abi.new(_abi.CapturerDesc, device=device, stream=int(stream))
        h = ctypes.c_void_p()
        _abi.check(_lib().eagle_backend_capturer_create(ctypes.byref(d), ctypes.byref(h)))
        self._h = h

    def begin(self):
        _abi.check(_lib().eagle_backend_capturer_begin(_need(self._h, "StreamCapturer")))

    def end(self) -> CapturedGraph:
        g = ctypes.c_void_p()
        _abi.check(_lib().eagle_backend_capturer_end(_need(self._h, "StreamCapturer"), ctypes.byref(g)))
        return CapturedGraph(g)

    def graph(self) -> int:
        g = ctypes.c_uint64()
        _abi.check(_lib().eagle_backend_capturer_graph(_need(self._h, "StreamCapturer"), ctypes.byref(g)))
        return g.value

    def __del__(self):
        if getattr(self, "_h", None):
            _lib().eagle_backend_capturer_release(self._h)
            self._h = None


class CaptureFork:
    """Branch streams of ``origin`` (made before the capture begins)."""

    def __init__(self, origin: int, branch_count: int, device: int = -1, waits: int = 0):
        d = _abi.new(_abi.ForkDesc, device=device, origin=int(origin), branch_count=branch_count, wait_count=waits)
        h = ctypes.c_void_p()
        _abi.check(_lib().eagle_backend_fork_create(ctypes.byref(d), ctypes.byref(h)))
        self._h = h

    def fork(self):
        _abi.check(_lib().eagle_backend_fork_fork(_need(self._h, "CaptureFork")))

    def join(self):
        _abi.check(_lib().eagle_backend_fork_join(_need(self._h, "CaptureFork")))

    def branch(self, index: int) -> int:
        s = ctypes.c_uint64()
        _abi.check(_lib().eagle_backend_fork_branch(_need(self._h, "CaptureFork"), index, ctypes.byref(s)))
        return s.value

    def origin(self) -> int:
        s = ctypes.c_uint64()
        _abi.check(_lib().eagle_backend_fork_origin(_need(self._h, "CaptureFork"), ctypes.byref(s)))
        return s.value

    def forked(self) -> bool:
        v = ctypes.c_int32()
        _abi.check(_lib().eagle_backend_fork_forked(_need(self._h, "CaptureFork"), ctypes.byref(v)))
        return v.value != 0

    def mark(self, producer: int) -> int:
        m = ctypes.c_uint64()
        _abi.check(_lib().eagle_backend_fork_mark(_need(self._h, "CaptureFork"), producer, ctypes.byref(m)))
        return m.value

    def wait(self, waiter: int, mark: int):
        _abi.check(_lib().eagle_backend_fork_wait(_need(self._h, "CaptureFork"), waiter, mark))

    def size(self) -> int:
        n = ctypes.c_uint64()
        _abi.check(_lib().eagle_backend_fork_size(_need(self._h, "CaptureFork"), ctypes.byref(n)))
        return n.value

    __len__ = size

    def __del__(self):
        if getattr(self, "_h", None):
            _lib().eagle_backend_fork_release(self._h)
            self._h = None


class CaptureConditional:
    """A device-evaluated IF / IF-ELSE / WHILE / SWITCH node woven into the
    capture on ``origin``; the guard is ``(*count != (*baseline or 0)) != negate``."""

    def __init__(self, origin: int, count_ptr: int, baseline_ptr: int = 0, loop_cap: int = 0, counter_ptr: int = 0,
                 device: int = -1, kind: str = "", arms: int = 0, negate: bool = False, brk_ptr: int = 0,
                 limit_ptr: int = 0):
        if kind not in _KINDS:
            raise ValueError(f"CaptureConditional: unknown kind {kind!r} (if, if_else, while, switch)")
        d = _abi.new(_abi.ConditionalDesc, device=device, origin=int(origin), count_ptr=int(count_ptr),
                     baseline_ptr=int(baseline_ptr), loop_cap=int(loop_cap), counter_ptr=int(counter_ptr),
                     kind=_KINDS[kind], arms=int(arms), negate=1 if negate else 0, brk_ptr=int(brk_ptr),
                     limit_ptr=int(limit_ptr))
        h = ctypes.c_void_p()
        _abi.check(_lib().eagle_backend_conditional_create(ctypes.byref(d), ctypes.byref(h)))
        self._h = h

    def begin(self) -> int:
        s = ctypes.c_uint64()
        _abi.check(_lib().eagle_backend_conditional_begin(_need(self._h, "CaptureConditional"), ctypes.byref(s)))
        return s.value

    def body_stream(self) -> int:
        s = ctypes.c_uint64()
        _abi.check(_lib().eagle_backend_conditional_body_stream(_need(self._h, "CaptureConditional"),
                                                                ctypes.byref(s)))
        return s.value

    def arm_stream(self, k: int) -> int:
        s = ctypes.c_uint64()
        _abi.check(_lib().eagle_backend_conditional_arm_stream(_need(self._h, "CaptureConditional"), k,
                                                               ctypes.byref(s)))
        return s.value

    def is_loop(self) -> bool:
        v = ctypes.c_int32()
        _abi.check(_lib().eagle_backend_conditional_is_loop(_need(self._h, "CaptureConditional"), ctypes.byref(v)))
        return v.value != 0

    def end(self):
        _abi.check(_lib().eagle_backend_conditional_end(_need(self._h, "CaptureConditional")))

    def nodes(self, which: int = 0) -> list[int]:
        return _nodes(_lib().eagle_backend_conditional_nodes, _need(self._h, "CaptureConditional"), which)

    def __del__(self):
        if getattr(self, "_h", None):
            _lib().eagle_backend_conditional_release(self._h)
            self._h = None


def capture_snapshot_nodes(stream: int) -> list[int]:
    """The nodes of the graph ``stream`` is capturing into."""
    return _nodes(_lib().eagle_backend_capture_snapshot_nodes, int(stream))


def is_node_toggleable(node: int) -> bool:
    v = ctypes.c_int32()
    _abi.check(_lib().eagle_backend_is_node_toggleable(int(node), ctypes.byref(v)))
    return v.value != 0


def capture_add_child(stream: int, child: int, conditional_body: bool = False):
    """Insert the graph ``child`` at the capture tip of ``stream`` as one node."""
    _abi.check(_lib().eagle_backend_capture_add_child(int(stream), int(child), 1 if conditional_body else 0))


class Launcher:
    """An instantiated graph."""

    def __init__(self, h):
        self._h = h

    def launch(self):
        _abi.check(_lib().eagle_backend_launcher_launch(_need(self._h, "Launcher")))

    def synchronize(self):
        _abi.check(_lib().eagle_backend_launcher_synchronize(_need(self._h, "Launcher")))

    def stream(self, stream: int):
        _abi.check(_lib().eagle_backend_launcher_stream(_need(self._h, "Launcher"), int(stream)))

    def set_logical_size(self, logical_size: int):
        _abi.check(_lib().eagle_backend_launcher_set_logical_size(_need(self._h, "Launcher"), int(logical_size)))

    def kernel_node_count(self) -> int:
        n = ctypes.c_int64()
        _abi.check(_lib().eagle_backend_launcher_kernel_node_count(_need(self._h, "Launcher"), ctypes.byref(n)))
        return n.value

    def set_node_enabled(self, node: int, enabled: bool):
        _abi.check(_lib().eagle_backend_launcher_set_node_enabled(_need(self._h, "Launcher"), int(node),
                                                                  1 if enabled else 0))

    def set_kernel_params(self, node: int, params):
        """``params``: addresses of the new argument values (0 keeps one)."""
        arr = (ctypes.c_uint64 * max(1, len(params)))(*[int(p) for p in params])
        _abi.check(_lib().eagle_backend_launcher_set_kernel_params(_need(self._h, "Launcher"), int(node), arr,
                                                                   len(params)))

    def set_memcpy_source(self, node: int, src: int):
        _abi.check(_lib().eagle_backend_launcher_set_memcpy_source(_need(self._h, "Launcher"), int(node), int(src)))

    def try_exec_update(self, captured: CapturedGraph) -> bool:
        ok = ctypes.c_int32()
        _abi.check(_lib().eagle_backend_launcher_exec_update(_need(self._h, "Launcher"),
                                                             _need(captured._h, "CapturedGraph"), ctypes.byref(ok)))
        return ok.value != 0

    def clone_graph(self) -> int:
        g = ctypes.c_uint64()
        _abi.check(_lib().eagle_backend_launcher_clone_graph(_need(self._h, "Launcher"), ctypes.byref(g)))
        return g.value

    @staticmethod
    def destroy_graph(graph: int):
        _abi.check(_lib().eagle_backend_launcher_graph_destroy(int(graph)))

    def __del__(self):
        if getattr(self, "_h", None):
            _lib().eagle_backend_launcher_release(self._h)
            self._h = None


class Graph:
    """A graph built from captures: ``Graph()`` starts with one empty node and
    ``add_node`` chains each capture after the last node; ``Graph.from_captured``
    adopts one capture whole."""

    def __init__(self, device: int = -1, _h=None):
        if _h is None:
            d = _abi.new(_abi.GraphDesc, device=device)
            _h = ctypes.c_void_p()
            _abi.check(_lib().eagle_backend_graph_create(ctypes.byref(d), ctypes.byref(_h)))
        self._h = _h

    @classmethod
    def from_captured(cls, captured: CapturedGraph) -> "Graph":
        h = ctypes.c_void_p()
        _abi.check(_lib().eagle_backend_graph_from_captured(_need(captured._h, "CapturedGraph"), ctypes.byref(h)))
        captured._h = None  # consumed
        return cls(_h=h)

    def stream(self, stream: int):
        _abi.check(_lib().eagle_backend_graph_stream(_need(self._h, "Graph"), int(stream)))

    def add_node(self, captured: CapturedGraph):
        _abi.check(_lib().eagle_backend_graph_add_node(_need(self._h, "Graph"), _need(captured._h, "CapturedGraph")))
        captured._h = None  # consumed

    def launcher(self) -> Launcher:
        h = ctypes.c_void_p()
        _abi.check(_lib().eagle_backend_graph_launcher(_need(self._h, "Graph"), ctypes.byref(h)))
        return Launcher(h)

    def last_node(self) -> int:
        i = ctypes.c_int64()
        _abi.check(_lib().eagle_backend_graph_last_node(_need(self._h, "Graph"), ctypes.byref(i)))
        return i.value

    def __del__(self):
        if getattr(self, "_h", None):
            _lib().eagle_backend_graph_release(self._h)
            self._h = None
