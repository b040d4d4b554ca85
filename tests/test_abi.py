"""The C-ABI library without a GPU: it loads, exports exactly the seam symbols the
header declares, its desc layouts match the C header, and the calls that need no
device (queries, argument refusals, the probe) behave as the seam specifies
(python/src/seam/eagle_backend.h of the eagle source tree)."""

import ctypes
import os
import re
import subprocess

import pytest

from eagle_b200 import _abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "eagle_b200.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(eagle_backend_\w+)\s*\(", text)))


def _exported():
    out = subprocess.run(["nm", "-D", "--defined-only", _abi.LIB_PATH], capture_output=True, text=True, check=True)
    return sorted(line.split()[-1] for line in out.stdout.splitlines() if " T " in line)


def test_library_loads_and_reports_its_version():
    L = _abi.lib()
    assert L.eagle_backend_version() == (1 << 16) | 8
    groups = ctypes.c_uint64()
    assert L.eagle_backend_capabilities(ctypes.byref(groups)) == _abi.OK
    base = (_abi.CAP_STREAM | _abi.CAP_CAPTURER | _abi.CAP_CAPTURED | _abi.CAP_FORK | _abi.CAP_CONDITIONAL
            | _abi.CAP_ATTRIBUTION | _abi.CAP_GRAPH | _abi.CAP_LAUNCHER | _abi.CAP_EXEC | _abi.CAP_DEVICE
            | _abi.CAP_INTEROP | _abi.CAP_FILTERING)
    arms = _abi.CAP_CONDITIONAL_IF_ELSE | _abi.CAP_CONDITIONAL_SWITCH
    assert groups.value & ~arms == base  # the arm kinds follow the driver's version
    info = _abi.new(_abi.BuildInfo)
    assert L.eagle_backend_build_info(ctypes.byref(info)) == _abi.OK
    assert info.backend_kind == b"cuda" and info.abi_version == (1 << 16) | 8


def test_exports_are_exactly_the_declared_seam():
    declared = _declared()
    exported = _exported()
    assert declared, "no declarations parsed"
    assert set(declared) == set(exported), (set(declared) ^ set(exported))
    assert all(name.startswith("eagle_backend_") for name in exported)
    assert set(_abi.SIGNATURES) == set(declared)


_LAYOUTS = {
    "eagle_backend_build_info": _abi.BuildInfo,
    "eagle_backend_device_props": _abi.DeviceProps,
    "eagle_backend_launch_desc": _abi.LaunchDesc,
    "eagle_backend_launch_raw_desc": _abi.LaunchRawDesc,
    "eagle_backend_cell_op_desc": _abi.CellOpDesc,
    "eagle_backend_compact_desc": _abi.CompactDesc,
    "eagle_backend_reorder_desc": _abi.ReorderDesc,
    "eagle_backend_reduce_desc": _abi.ReduceDesc,
    "eagle_b200_engine_desc": _abi.EngineDesc,
    "eagle_b200_report": _abi.Report,
    "eagle_backend_capturer_desc": _abi.CapturerDesc,
    "eagle_backend_fork_desc": _abi.ForkDesc,
    "eagle_backend_conditional_desc": _abi.ConditionalDesc,
    "eagle_backend_graph_desc": _abi.GraphDesc,
    "eagle_backend_compact_classes_desc": _abi.CompactClassesDesc,
    "eagle_backend_reorder_classes_desc": _abi.ReorderClassesDesc,
}


def test_desc_layouts_match_the_header(tmp_path):
    """Compile the header with gcc and compare every struct's size and field offsets
    with the ctypes mirrors (and the seam's sizes of eagle_backend.h:171-906)."""
    lines = ['#include <stddef.h>', '#include <stdio.h>', f'#include "{HEADER}"', "int main(void) {"]
    for cname, ct in _LAYOUTS.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof(struct {cname}));')
        for fname, _ in ct._fields_:
            cf = "in" if fname == "in_" else fname
            lines.append(f'printf("{cname}.{fname} %zu\\n", offsetof(struct {cname}, {cf}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-o", str(exe), str(src)], check=True)
    got = dict(line.rsplit(" ", 1) for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                               check=True).stdout.splitlines())
    for cname, ct in _LAYOUTS.items():
        assert int(got[cname]) == ctypes.sizeof(ct), cname
        for fname, _ in ct._fields_:
            assert int(got[f"{cname}.{fname}"]) == getattr(ct, fname).offset, (cname, fname)


# eagle's own seam header (test infrastructure: read where the eagle source tree lies,
# never shipped); the layouts of the structs both headers declare must be identical
REFERENCE = os.environ.get("EAGLE_REFERENCE", "/root/reference")
SEAM = os.path.join(REFERENCE, "python", "src", "seam", "eagle_backend.h")


def _struct_fields(text):
    """{struct name: [field names]} of every struct body in a C header."""
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    out = {}
    for name, body in re.findall(r"struct\s+(\w+)\s*\{(.*?)\}\s*;", text, flags=re.S):
        fields = []
        for decl in body.split(";"):
            decl = decl.strip()
            if not decl:
                continue
            for part in decl.split(","):
                part = re.sub(r"\[.*?\]", "", part).strip()
                fields.append(re.findall(r"\w+", part)[-1])
        out[name] = fields
    return out


def _layouts(header, structs, tmp_path, tag):
    lines = ["#include <stddef.h>", "#include <stdio.h>", f'#include "{header}"', "int main(void) {"]
    for cname, fields in structs.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof(struct {cname}));')
        for f in fields:
            lines.append(f'printf("{cname}.{f} %zu\\n", offsetof(struct {cname}, {f}));')
    lines.append("return 0; }")
    src = tmp_path / f"{tag}.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / tag
    subprocess.run(["gcc", "-std=c11", "-o", str(exe), str(src)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    return dict(line.rsplit(" ", 1) for line in out.splitlines())


@pytest.mark.skipif(not os.path.exists(SEAM), reason="the eagle source tree is not here")
def test_shared_structs_match_eagles_seam_header(tmp_path):
    """Every struct this header shares with eagle's seam header
    (python/src/seam/eagle_backend.h) has the same size and the same offset for every
    field, compiled from both headers with gcc."""
    theirs = _struct_fields(open(SEAM).read())
    ours = _struct_fields(open(HEADER).read())
    shared = {k: theirs[k] for k in theirs if k in ours}
    assert len(shared) >= 16, sorted(shared)
    for k in shared:
        assert ours[k] == theirs[k], k
    a = _layouts(SEAM, shared, tmp_path, "seam")
    b = _layouts(HEADER, shared, tmp_path, "ours")
    assert a == b, {k: (a.get(k), b.get(k)) for k in set(a) | set(b) if a.get(k) != b.get(k)}


def test_compact_query_needs_no_device():
    d = _abi.new(_abi.CompactDesc, n=100_003, flags=_abi.COMPACT_MASK_IS_DROP)
    assert _abi.lib().eagle_backend_compact_device(ctypes.byref(d)) == _abi.OK
    assert d.scratch_bytes >= 8 * ((100_003 + 32767) // 32768)  # one status word per 32768-sample tile


def test_compact_refuses_past_int32_and_negative():
    L = _abi.lib()
    d = _abi.new(_abi.CompactDesc, n=2 ** 31, scratch=1, mask=1, index_map=1, count=1)
    assert L.eagle_backend_compact_device(ctypes.byref(d)) == _abi.UNSUPPORTED
    assert "2^31-1" in _abi.last_error()
    d = _abi.new(_abi.CompactDesc, n=-1)
    assert L.eagle_backend_compact_device(ctypes.byref(d)) == _abi.INVALID_ARGUMENT


def test_unknown_flag_bits_are_refused():
    d = _abi.new(_abi.CompactDesc, n=10, flags=1 << 7)
    assert _abi.lib().eagle_backend_compact_device(ctypes.byref(d)) == _abi.UNSUPPORTED


def test_reduce_argument_refusals():
    L = _abi.lib()
    d = _abi.new(_abi.ReduceDesc, n=0)
    assert L.eagle_backend_x_reduce_canonical(ctypes.byref(d)) == _abi.INVALID_ARGUMENT
    d = _abi.new(_abi.ReduceDesc, n=10, dtype=_abi.REDUCE_F64, op=_abi.REDUCE_OP_ALL)
    assert L.eagle_backend_x_reduce_canonical(ctypes.byref(d)) == _abi.INVALID_ARGUMENT
    d = _abi.new(_abi.ReduceDesc, n=10, dtype=_abi.REDUCE_I64, op=_abi.REDUCE_OP_SUM, flags=_abi.REDUCE_PAIR_OUT,
                 columns=1)
    assert L.eagle_backend_x_reduce_canonical(ctypes.byref(d)) == _abi.INVALID_ARGUMENT


def test_cell_op_array_ops_unsupported():
    d = _abi.new(_abi.CellOpDesc, op=7, n=4)
    assert _abi.lib().eagle_backend_cell_op(ctypes.byref(d)) == _abi.UNSUPPORTED


def test_entry_lookup_unknown_name():
    f = ctypes.c_uint64()
    assert _abi.lib().eagle_backend_x_b200_entry(b"no_such_kernel", -1, ctypes.byref(f)) == _abi.INDEX


def test_probe_without_a_device():
    try:
        import torch

        if torch.cuda.is_available():
            pytest.skip("a device is visible")
    except ImportError:
        pass
    assert _abi.lib().eagle_backend_probe() == _abi.UNAVAILABLE
    assert "no CUDA device" in _abi.last_error()


def test_last_error_clears_on_success():
    L = _abi.lib()
    d = _abi.new(_abi.CompactDesc, n=-1)
    L.eagle_backend_compact_device(ctypes.byref(d))
    assert _abi.last_error()
    d = _abi.new(_abi.CompactDesc, n=5)
    assert L.eagle_backend_compact_device(ctypes.byref(d)) == _abi.OK
    assert _abi.last_error() == ""


def _reorder_desc(n, planes, mask, **kw):
    tab = (_abi.ReorderPlane * max(1, len(planes)))()
    for k, (addr, e) in enumerate(planes):
        tab[k].data, tab[k].elem_bytes = addr, e
    d = _abi.new(_abi.ReorderDesc, n=n, n_planes=len(planes), planes=ctypes.addressof(tab), mask=mask, **kw)
    return d, tab


def test_reorder_query_and_refusals():
    L = _abi.lib()
    d, tab = _reorder_desc(100_000, [(1 << 20, 8), (1 << 30, 1)], 1 << 30)
    assert L.eagle_backend_reorder_device(ctypes.byref(d)) == _abi.OK
    assert d.scratch_bytes >= 8 * 100_000  # the stage holds the widest plane
    d, tab = _reorder_desc(100, [(1 << 20, 3), (1 << 30, 1)], 1 << 30)
    assert L.eagle_backend_reorder_device(ctypes.byref(d)) == _abi.INVALID_ARGUMENT
    assert "3-byte" in _abi.last_error()
    d, tab = _reorder_desc(100, [(1 << 20, 8)], 1 << 30)
    assert L.eagle_backend_reorder_device(ctypes.byref(d)) == _abi.INVALID_ARGUMENT
    assert "mask must be one of the planes" in _abi.last_error()
    d, tab = _reorder_desc(100, [(1 << 20, 8), ((1 << 20) + 8, 8), (1 << 30, 1)], 1 << 30)
    assert L.eagle_backend_reorder_device(ctypes.byref(d)) == _abi.INVALID_ARGUMENT
    assert "overlap" in _abi.last_error()
    d, tab = _reorder_desc(100, [((1 << 20) + 4, 8), (1 << 30, 1)], 1 << 30)
    assert L.eagle_backend_reorder_device(ctypes.byref(d)) == _abi.INVALID_ARGUMENT
    assert "aligned" in _abi.last_error()
    d, tab = _reorder_desc(2 ** 31, [(1 << 20, 8), (1 << 30, 1)], 1 << 30)
    assert L.eagle_backend_reorder_device(ctypes.byref(d)) == _abi.UNSUPPORTED


def test_fence_refusals_need_no_device():
    L = _abi.lib()
    assert L.eagle_backend_fence(1, 0, 1, 2) == _abi.UNSUPPORTED  # a CPU buffer has no CUDA fence
    assert L.eagle_backend_fence(2, 0, 0, 2) == _abi.INVALID_ARGUMENT  # stream 0 is refused by DLPack
    assert "ambiguous" in _abi.last_error()
    assert L.eagle_backend_fence(2, 0, -5, 2) == _abi.INVALID_ARGUMENT
    assert L.eagle_backend_fence(2, 0, -1, 2) == _abi.OK  # no ordering asked for
    assert L.eagle_backend_fence(2, 0, 2, 2) == _abi.OK   # one stream orders itself
    assert L.eagle_backend_fence(2, 0, _abi.STREAM_NONE, 1) == _abi.OK  # none given: the legacy default
    out = ctypes.c_uint64(7)
    assert L.eagle_backend_host_alloc(0, ctypes.byref(out)) == _abi.OK and out.value == 0
    assert L.eagle_backend_host_free(0) == _abi.OK
