"""ctypes binding of ``libeagle_b200.so`` (declared in ``include/eagle_b200.h``).

The library is loaded from this package's directory only; a missing or unloadable
library raises ``BackendUnavailable`` (there is no fallback path). Every seam call
goes through :func:`check`, which turns a non-OK status into the matching
exception carrying ``eagle_backend_last_error()``.
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libeagle_b200.so")

OK, ERROR, INVALID_ARGUMENT, INDEX, INTEROP, UNAVAILABLE, CALLBACK_FAILED, BAD_HANDLE, UNSUPPORTED = range(9)

CAP_STREAM, CAP_EXEC, CAP_DEVICE, CAP_FILTERING = 1 << 0, 1 << 9, 1 << 10, 1 << 12
CAP_CAPTURER, CAP_CAPTURED, CAP_FORK, CAP_CONDITIONAL, CAP_ATTRIBUTION, CAP_GRAPH, CAP_LAUNCHER = (1 << k for k in range(1, 8))
CAP_CONDITIONAL_IF_ELSE, CAP_CONDITIONAL_SWITCH = 1 << 13, 1 << 14
CAP_INTEROP = 1 << 11
STREAM_NONE = -(1 << 63)
COND_IF, COND_IF_ELSE, COND_WHILE, COND_SWITCH = 1, 2, 3, 4
LOOP_UNCAPPED = 0xFFFFFFFF

CELL_BUMP, CELL_MASK_COUNT, CELL_POLICY, CELL_IDENTITY, CELL_COUNT_FIRED, CELL_GROUP_AND, CELL_SCALE_COUNT = range(7)
COMPACT_MASK_IS_DROP = 1
CLASSES_WITHIN_LIVE = 2
REDUCE_F32, REDUCE_F64, REDUCE_I32, REDUCE_I64, REDUCE_U8 = range(5)
REDUCE_OP_SUM, REDUCE_OP_MAX, REDUCE_OP_ALL, REDUCE_OP_MIN = range(4)
REDUCE_COMPENSATED, REDUCE_ORDERED, REDUCE_AUTO = range(3)
REDUCE_PAIR_OUT = 1
COPY_H2D, COPY_D2H, COPY_D2D, COPY_H2H = range(4)
MEM_DEVICE, MEM_PINNED = 0, 1

MODEL_OSCILLATOR, MODEL_OSCILLATOR_SPREAD, MODEL_GAMBLER, MODEL_LORENZ = 0, 1, 2, 3
MODE_BAND, MODE_PERSIST, MODE_FUSED, MODE_BAND_EAGER = 0, 1, 2, 3
FLAG_FMA = 1
FLAG_INDEX_ORDER = 2


class BackendError(RuntimeError):
    """A seam call failed; ``status`` is its ``eagle_backend_status``."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class BackendUnavailable(BackendError):
    pass


class BackendUnsupported(BackendError):
    pass


_u32, _i32, _u64, _i64, _f32, _f64 = (ctypes.c_uint32, ctypes.c_int32, ctypes.c_uint64, ctypes.c_int64,
                                      ctypes.c_float, ctypes.c_double)


class BuildInfo(ctypes.Structure):
    _fields_ = [("struct_size", _u32), ("abi_version", _u32), ("cudart_version", _i32), ("reserved0", _i32),
                ("eagle_version", ctypes.c_char * 32), ("archs", ctypes.c_char * 128),
                ("backend_kind", ctypes.c_char * 16)]


class DeviceProps(ctypes.Structure):
    _fields_ = [("struct_size", _u32), ("device", _i32), ("name", ctypes.c_char * 256),
                ("cc_major", _i32), ("cc_minor", _i32), ("sm_count", _i32), ("clock_rate_khz", _i32),
                ("memory_clock_rate_khz", _i32), ("memory_bus_width_bits", _i32),
                ("regs_per_block", _i32), ("regs_per_sm", _i32), ("warp_size", _i32), ("reserved0", _i32),
                ("shared_mem_per_block", _i64), ("shared_mem_per_sm", _i64),
                ("peak_bytes_per_s", _f64), ("peak_flops_sp", _f64), ("peak_flops_dp", _f64), ("fp64_ratio", _f64),
                ("ridge_flops_per_byte_sp", _f64), ("ridge_flops_per_byte_dp", _f64),
                ("total_mem_bytes", _i64), ("free_mem_bytes", _i64)]


class LaunchDesc(ctypes.Structure):
    _fields_ = [("struct_size", _u32), ("flags", _u32), ("device", _i32), ("block", _u32), ("function", _u64),
                ("params", ctypes.POINTER(_u64)), ("param_sizes", ctypes.POINTER(_u64)), ("nparams", _i64),
                ("base", _i64), ("count", _i64), ("n_samples", _i64), ("stream", _u64)]


class LaunchRawDesc(ctypes.Structure):
    _fields_ = [("struct_size", _u32), ("flags", _u32), ("device", _i32), ("shared_bytes", _u32),
                ("function", _u64), ("stream", _u64), ("grid", _u32 * 3), ("block", _u32 * 3), ("args", _u64),
                ("arg_count", _u32), ("reserved", _u32)]


class CellOpDesc(ctypes.Structure):
    _fields_ = [("struct_size", _u32), ("flags", _u32), ("op", _u32), ("device", _i32), ("stream", _u64),
                ("n", _i64), ("p", _u64 * 6), ("i", _i64 * 10), ("f", _f64 * 2), ("j", _i64 * 4)]


class CompactDesc(ctypes.Structure):
    _fields_ = [("struct_size", _u32), ("flags", _u32), ("device", _i32), ("reserved", _u32), ("mask", _u64),
                ("index_map", _u64), ("count", _u64), ("scratch", _u64), ("n", _i64), ("stream", _u64),
                ("scratch_bytes", _i64), ("live32", _u64), ("span", _u64), ("fire", _u64), ("theta", _f32),
                ("reserved2", _u32)]


class ReorderPlane(ctypes.Structure):
    _fields_ = [("data", _u64), ("elem_bytes", _u32), ("reserved", _u32)]


class ReorderDesc(ctypes.Structure):
    _fields_ = [("struct_size", _u32), ("flags", _u32), ("device", _i32), ("n_planes", _u32), ("planes", _u64),
                ("mask", _u64), ("perm", _u64), ("inv", _u64), ("index_map", _u64), ("count", _u64),
                ("span", _u64), ("fire", _u64), ("scratch", _u64), ("n", _i64), ("stream", _u64),
                ("scratch_bytes", _i64)]


class ReduceDesc(ctypes.Structure):
    _fields_ = [("struct_size", _u32), ("dtype", _u32), ("op", _u32), ("device", _i32), ("in_", _u64),
                ("out", _u64), ("work_a", _u64), ("work_b", _u64), ("n", _i64), ("stream", _u64),
                ("work_elems", _i64), ("policy", _u32), ("flags", _u32), ("columns", _i64), ("comp_in", _u64)]


class EngineDesc(ctypes.Structure):
    _fields_ = [("struct_size", _u32), ("flags", _u32), ("device", _i32), ("model", _u32), ("mode", _u32),
                ("reserved0", _u32), ("n", _i64), ("max_steps", _i64), ("planes", _u64 * 8),
                ("uniforms", _f64 * 4), ("terminated", _u64), ("k_first", _i64), ("k_min", _i64),
                ("k_max", _i64), ("chunk", _u32), ("block", _u32), ("overhead_steps", _f64),
                ("interval_steps", _f64), ("iuniforms", _i64 * 4), ("uniforms_ext", _f64 * 4),
                ("ctas_per_sm", _u32), ("reserved1", _u32)]


class ScalarHandle(ctypes.Structure):
    """The 32-byte per-sample plane handle of the hawk kernel ABI (plugin/gref_layout.h:115-122)."""
    _fields_ = [("data", _u64), ("samples", _u64), ("stride", _u64), ("device_type", _i32), ("device_id", _i32)]


class Report(ctypes.Structure):
    _fields_ = [("struct_size", _u32), ("done", _u32), ("n", _i64), ("finished", _i64), ("steps", _i64),
                ("launches", _i64), ("compactions", _i64), ("step_sum", _u64), ("error", _u32), ("mode", _u32),
                ("report_bytes", _u32), ("reserved0", _u32)]


class CompactClassesDesc(ctypes.Structure):
    _fields_ = [("struct_size", _u32), ("flags", _u32), ("device", _i32), ("reserved", _u32), ("mask", _u64),
                ("index_map", _u64), ("count", _u64), ("scratch", _u64), ("n", _i64), ("stream", _u64),
                ("scratch_bytes", _i64), ("live32", _u64), ("span", _u64), ("fire", _u64), ("theta", _f32),
                ("reserved2", _u32), ("class_plane", _u64), ("classes", _u32), ("class_theta", _f32),
                ("offsets", _u64), ("mixed32", _u64), ("stale_count", _u64), ("class_fire", _u64),
                ("reserved3", _u64)]


class ReorderClassesDesc(ctypes.Structure):
    _fields_ = [("struct_size", _u32), ("flags", _u32), ("device", _i32), ("n_planes", _u32), ("planes", _u64),
                ("mask", _u64), ("perm", _u64), ("inv", _u64), ("index_map", _u64), ("count", _u64),
                ("span", _u64), ("fire", _u64), ("scratch", _u64), ("n", _i64), ("stream", _u64),
                ("scratch_bytes", _i64), ("class_plane", _u64), ("classes", _u32), ("reserved3", _u32),
                ("offsets", _u64), ("class_sorts", _u64)]


class CapturerDesc(ctypes.Structure):
    _fields_ = [("struct_size", _u32), ("flags", _u32), ("device", _i32), ("reserved0", _i32), ("stream", _u64)]


class ForkDesc(ctypes.Structure):
    _fields_ = [("struct_size", _u32), ("flags", _u32), ("device", _i32), ("reserved0", _i32), ("origin", _u64),
                ("branch_count", _u64), ("wait_count", _u64)]


class ConditionalDesc(ctypes.Structure):
    _fields_ = [("struct_size", _u32), ("flags", _u32), ("device", _i32), ("loop_cap", _u32), ("origin", _u64),
                ("count_ptr", _u64), ("baseline_ptr", _u64), ("counter_ptr", _u64), ("kind", _u32), ("arms", _u32),
                ("negate", _u32), ("reserved1", _u32), ("brk_ptr", _u64), ("limit_ptr", _u64)]


class GraphDesc(ctypes.Structure):
    _fields_ = [("struct_size", _u32), ("flags", _u32), ("device", _i32), ("reserved0", _i32)]


def new(struct_type, **fields):
    """A zero-filled desc with ``struct_size`` set, then ``fields``."""
    s = struct_type()
    s.struct_size = ctypes.sizeof(struct_type)
    for k, v in fields.items():
        setattr(s, k, v)
    return s


_P = ctypes.c_void_p
_lib = None

# name -> (restype, argtypes); the library must export every one of them
SIGNATURES = {
    "eagle_backend_version": (_u32, []),
    "eagle_backend_last_error": (ctypes.c_char_p, []),
    "eagle_backend_build_info": (_i32, [ctypes.POINTER(BuildInfo)]),
    "eagle_backend_probe": (_i32, []),
    "eagle_backend_free": (None, [_P]),
    "eagle_backend_capabilities": (_i32, [ctypes.POINTER(_u64)]),
    "eagle_backend_device_types": (_i32, [ctypes.POINTER(_i32), _i32, ctypes.POINTER(_i32)]),
    "eagle_backend_stream_create": (_i32, [_P, ctypes.POINTER(_P)]),
    "eagle_backend_stream_ptr": (_i32, [_P, ctypes.POINTER(_u64)]),
    "eagle_backend_stream_synchronize": (_i32, [_P]),
    "eagle_backend_stream_release": (None, [_P]),
    "eagle_backend_x_b200_leaf_partials": (_i32, [_u64, _i64, _u64, _u64]),
    "eagle_backend_module_load": (_i32, [_P, _u64, _i32, ctypes.POINTER(_u64)]),
    "eagle_backend_module_load_jit": (_i32, [_P, _u64, _i32, _u32, ctypes.POINTER(_u64)]),
    "eagle_backend_link_ptx": (_i32, [_P, _u64, _i32, _u32, _P, _u64, ctypes.POINTER(_u64)]),
    "eagle_backend_module_function": (_i32, [_u64, ctypes.c_char_p, ctypes.POINTER(_u64)]),
    "eagle_backend_module_release": (None, [_u64, _i32]),
    "eagle_backend_memcpy_strided": (_i32, [_u64, _u64, _u64, _u64, _u64, _u64, _i32, _u64]),
    "eagle_backend_mem_alloc": (_i32, [_i32, _i32, _u64, _u64, ctypes.POINTER(_u64), ctypes.POINTER(_u64)]),
    "eagle_backend_mem_release": (None, [_u64]),
    "eagle_backend_mem_drain": (_i32, [ctypes.POINTER(_i64)]),
    "eagle_backend_pointer_device": (_i32, [_u64, ctypes.POINTER(_i32)]),
    "eagle_backend_fence": (_i32, [_i32, _i32, _i64, _i64]),
    "eagle_backend_event_pool_created": (_i32, [ctypes.POINTER(_i64)]),
    "eagle_backend_host_alloc": (_i32, [_u64, ctypes.POINTER(_u64)]),
    "eagle_backend_host_free": (_i32, [_u64]),
    "eagle_backend_host_func": (_i32, [_u64, _P, _P]),
    "eagle_backend_reorder_device": (_i32, [ctypes.POINTER(ReorderDesc)]),
    "eagle_backend_x_restore_device": (_i32, [ctypes.POINTER(ReorderDesc)]),
    "eagle_backend_pointer_residency": (_i32, [_i32, _u64, ctypes.POINTER(_i32)]),
    "eagle_backend_compact_classes_device": (_i32, [ctypes.POINTER(CompactClassesDesc)]),
    "eagle_backend_reorder_classes_device": (_i32, [ctypes.POINTER(ReorderClassesDesc)]),
    "eagle_backend_capturer_create": (_i32, [ctypes.POINTER(CapturerDesc), ctypes.POINTER(_P)]),
    "eagle_backend_capturer_begin": (_i32, [_P]),
    "eagle_backend_capturer_end": (_i32, [_P, ctypes.POINTER(_P)]),
    "eagle_backend_capturer_graph": (_i32, [_P, ctypes.POINTER(_u64)]),
    "eagle_backend_capturer_release": (None, [_P]),
    "eagle_backend_captured_is_valid": (_i32, [_P, ctypes.POINTER(_i32)]),
    "eagle_backend_captured_release": (None, [_P]),
    "eagle_backend_fork_create": (_i32, [ctypes.POINTER(ForkDesc), ctypes.POINTER(_P)]),
    "eagle_backend_fork_fork": (_i32, [_P]),
    "eagle_backend_fork_join": (_i32, [_P]),
    "eagle_backend_fork_branch": (_i32, [_P, _u64, ctypes.POINTER(_u64)]),
    "eagle_backend_fork_origin": (_i32, [_P, ctypes.POINTER(_u64)]),
    "eagle_backend_fork_forked": (_i32, [_P, ctypes.POINTER(_i32)]),
    "eagle_backend_fork_size": (_i32, [_P, ctypes.POINTER(_u64)]),
    "eagle_backend_fork_release": (None, [_P]),
    "eagle_backend_fork_mark": (_i32, [_P, _u64, ctypes.POINTER(_u64)]),
    "eagle_backend_fork_wait": (_i32, [_P, _u64, _u64]),
    "eagle_backend_conditional_create": (_i32, [ctypes.POINTER(ConditionalDesc), ctypes.POINTER(_P)]),
    "eagle_backend_conditional_begin": (_i32, [_P, ctypes.POINTER(_u64)]),
    "eagle_backend_conditional_body_stream": (_i32, [_P, ctypes.POINTER(_u64)]),
    "eagle_backend_conditional_is_loop": (_i32, [_P, ctypes.POINTER(_i32)]),
    "eagle_backend_conditional_end": (_i32, [_P]),
    "eagle_backend_conditional_release": (None, [_P]),
    "eagle_backend_conditional_arm_stream": (_i32, [_P, _u64, ctypes.POINTER(_u64)]),
    "eagle_backend_conditional_nodes": (_i32, [_P, _i64, ctypes.POINTER(ctypes.POINTER(_u64)), ctypes.POINTER(_i64)]),
    "eagle_backend_capture_snapshot_nodes": (_i32, [_u64, ctypes.POINTER(ctypes.POINTER(_u64)),
                                                    ctypes.POINTER(_i64)]),
    "eagle_backend_is_node_toggleable": (_i32, [_u64, ctypes.POINTER(_i32)]),
    "eagle_backend_capture_add_child": (_i32, [_u64, _u64, _i32]),
    "eagle_backend_graph_create": (_i32, [ctypes.POINTER(GraphDesc), ctypes.POINTER(_P)]),
    "eagle_backend_graph_from_captured": (_i32, [_P, ctypes.POINTER(_P)]),
    "eagle_backend_graph_stream": (_i32, [_P, _u64]),
    "eagle_backend_graph_add_node": (_i32, [_P, _P]),
    "eagle_backend_graph_launcher": (_i32, [_P, ctypes.POINTER(_P)]),
    "eagle_backend_graph_last_node": (_i32, [_P, ctypes.POINTER(_i64)]),
    "eagle_backend_graph_release": (None, [_P]),
    "eagle_backend_launcher_launch": (_i32, [_P]),
    "eagle_backend_launcher_synchronize": (_i32, [_P]),
    "eagle_backend_launcher_stream": (_i32, [_P, _u64]),
    "eagle_backend_launcher_set_logical_size": (_i32, [_P, _i64]),
    "eagle_backend_launcher_kernel_node_count": (_i32, [_P, ctypes.POINTER(_i64)]),
    "eagle_backend_launcher_set_node_enabled": (_i32, [_P, _u64, _i32]),
    "eagle_backend_launcher_release": (None, [_P]),
    "eagle_backend_launcher_set_kernel_params": (_i32, [_P, _u64, ctypes.POINTER(_u64), _i64]),
    "eagle_backend_launcher_set_memcpy_source": (_i32, [_P, _u64, _u64]),
    "eagle_backend_launcher_exec_update": (_i32, [_P, _P, ctypes.POINTER(_i32)]),
    "eagle_backend_launcher_clone_graph": (_i32, [_P, ctypes.POINTER(_u64)]),
    "eagle_backend_launcher_graph_destroy": (_i32, [_u64]),
    "eagle_backend_run_device": (_i32, [ctypes.POINTER(LaunchDesc), ctypes.POINTER(_i32)]),
    "eagle_backend_device_props": (_i32, [_i32, ctypes.POINTER(DeviceProps)]),
    "eagle_backend_memset_device": (_i32, [_u64, _u64, _u64]),
    "eagle_backend_memcpy_device": (_i32, [_u64, _u64, _u64, _u64]),
    "eagle_backend_memcpy": (_i32, [_u64, _u64, _u64, _i32, _u64]),
    "eagle_backend_device_count": (_i32, [ctypes.POINTER(_i32)]),
    "eagle_backend_set_device": (_i32, [_i32]),
    "eagle_backend_get_device": (_i32, [ctypes.POINTER(_i32)]),
    "eagle_backend_launch_status": (_i32, [_i32]),
    "eagle_backend_device_synchronize": (_i32, [_i32]),
    "eagle_backend_stream_is_capturing": (_i32, [_u64, ctypes.POINTER(_i32)]),
    "eagle_backend_function_attribute": (_i32, [_u64, _i32, ctypes.POINTER(_i32)]),
    "eagle_backend_launch_raw": (_i32, [ctypes.POINTER(LaunchRawDesc)]),
    "eagle_backend_cell_op": (_i32, [ctypes.POINTER(CellOpDesc)]),
    "eagle_backend_stream_sync": (_i32, [_i32, _u64]),
    "eagle_backend_event_create": (_i32, [_i32, ctypes.POINTER(_u64)]),
    "eagle_backend_event_create_timed": (_i32, [_i32, ctypes.POINTER(_u64)]),
    "eagle_backend_event_elapsed": (_i32, [_u64, _u64, ctypes.POINTER(_f32)]),
    "eagle_backend_event_record": (_i32, [_u64, _u64]),
    "eagle_backend_event_wait": (_i32, [_u64, _u64]),
    "eagle_backend_event_release": (None, [_u64, _i32]),
    "eagle_backend_compact_device": (_i32, [ctypes.POINTER(CompactDesc)]),
    "eagle_backend_x_b200_compact_device_noalloc": (_i32, [ctypes.POINTER(CompactDesc)]),
    "eagle_backend_x_b200_compact_wait_check": (_i32, [ctypes.POINTER(CompactDesc), _u32]),
    "eagle_backend_x_b200_ragged_head": (_i32, [_u64, _u64, _u64, _u64]),
    "eagle_backend_x_b200_ragged_leaves": (_i32, [_u64, _u64, _i32, _i32, _u64, _i64, _u64]),
    "eagle_backend_x_b200_ragged_fold": (_i32, [_u64, _i32, _i64, _u64, _u64, _u64]),
    "eagle_backend_x_b200_compact_sum_count": (_i32, [ctypes.POINTER(CompactDesc)]),
    "eagle_backend_x_b200_compact_sum_head": (_i32, [ctypes.POINTER(CompactDesc), _u64, _u64]),
    "eagle_backend_x_b200_compact_sum_leaves": (_i32, [ctypes.POINTER(CompactDesc), _u64, _u64, _i32, _i32, _u64,
                                                       _i64]),
    "eagle_backend_x_b200_compact_sum_straddle": (_i32, [ctypes.POINTER(CompactDesc), _u64, _i32, _i32, _u64,
                                                         _i64]),
    "eagle_backend_reset_device": (_i32, [ctypes.POINTER(ReorderDesc)]),
    "eagle_backend_x_reduce_canonical": (_i32, [ctypes.POINTER(ReduceDesc)]),
    "eagle_backend_x_b200_entry": (_i32, [ctypes.c_char_p, _i32, ctypes.POINTER(_u64)]),
    "eagle_backend_x_b200_combine_partials": (_i32, [_u64, _i64, _u64, _u64, _u64]),
    "eagle_backend_x_b200_compact_gather": (_i32, [ctypes.POINTER(CompactDesc), _u64, _u64, _u32]),
    "eagle_backend_x_b200_reduce_counted": (_i32, [ctypes.POINTER(ReduceDesc), _u64]),
    "eagle_backend_x_b200_reduce_fixed": (_i32, [ctypes.POINTER(ReduceDesc)]),
    "eagle_backend_x_b200_compact_sum": (_i32, [ctypes.POINTER(CompactDesc), _u64, _u64, _u32]),
    "eagle_backend_x_b200_engine_create": (_i32, [ctypes.POINTER(EngineDesc), ctypes.POINTER(_P)]),
    "eagle_backend_x_b200_engine_launch": (_i32, [_P, _u64]),
    "eagle_backend_x_b200_engine_report": (_i32, [_P, _u64, ctypes.POINTER(Report)]),
    "eagle_backend_x_b200_engine_report_enqueue": (_i32, [_P, _u64]),
    "eagle_backend_x_b200_engine_report_read": (_i32, [_P, ctypes.POINTER(Report)]),
    "eagle_backend_x_b200_engine_run": (_i32, [_P, _u64, ctypes.POINTER(Report)]),
    "eagle_backend_x_b200_engine_release": (None, [_P]),
    "eagle_backend_x_b200_engine_time_kernel": (_i32, [_P, _i32]),
    "eagle_backend_x_b200_engine_kernel_ms": (_i32, [_P, ctypes.POINTER(_f32), _i32, ctypes.POINTER(_i32)]),
    "eagle_backend_x_b200_probe_fp64": (_i32, [_i32, _u32, _u32, _u64, ctypes.POINTER(ctypes.c_double)]),
}


def lib():
    """The loaded library (loaded once); raises BackendUnavailable when it is absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise BackendUnavailable(UNAVAILABLE, f"eagle_b200: {LIB_PATH} is not built; run "
                                                  "`python -c 'import __graft_entry__ as g; g.build()'` first")
        try:
            L = ctypes.CDLL(LIB_PATH)
        except OSError as e:
            raise BackendUnavailable(UNAVAILABLE, f"eagle_b200: cannot load {LIB_PATH}: {e}") from e
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    msg = lib().eagle_backend_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str = "") -> None:
    if status == OK:
        return
    msg = last_error() or what
    if status == UNAVAILABLE:
        raise BackendUnavailable(status, msg)
    if status == UNSUPPORTED:
        raise BackendUnsupported(status, msg)
    if status == INVALID_ARGUMENT:
        raise ValueError(msg)
    if status == INDEX:
        raise IndexError(msg)
    raise BackendError(status, msg)
