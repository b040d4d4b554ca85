"""Hawk artifact intake and the array layer's memory through the seam's per-symbol
entries (python/src/seam/eagle_backend.h:457-476, :612-646): a step kernel
compiled apart from this library (as hawk builds one: a cubin, or PTX JIT-linked
for the device) is loaded with ``module_load`` / ``module_load_jit`` /
``link_ptx``, found with ``module_function`` and launched through ``run_device``
with the hawk argument packing, bit for bit against the oracle; stream-ordered
allocations, their deferred frees and strided copies."""

import ctypes
import os
import shutil
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from eagle_b200 import _abi  # noqa: E402

# a finishing Euler step entry in the hawk kernel ABI: role handles, the Params by
# value, then the partition triple (eagle/exec/DeviceKernel.h:47-84); each operation
# rounds once, in the README body's order
SOURCE = r"""
struct Handle { void* data; unsigned long long samples, stride; int device_type, device_id; };
extern "C" __global__ void euler_step(Handle omega, double t_end, double dt, Handle terminated, Handle x,
                                      Handle v, Handle t, Handle finished, Handle fused,
                                      long long base, long long count, long long n_samples)
{
    const long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= count) return;
    const long long i = base + j;
    unsigned char* m = (unsigned char*)terminated.data;
    if (m[i]) return;
    double* X = (double*)x.data; double* V = (double*)v.data; double* T = (double*)t.data;
    const double om = ((const double*)omega.data)[i];
    const double c = __dmul_rn(__dmul_rn(dt, om), om);
    const long long budget = *(const long long*)fused.data;
    double xx = X[i], vv = V[i], tt = T[i];
    for (long long k = 0; k < budget; ++k) {
        const double x1 = __dadd_rn(xx, __dmul_rn(dt, vv));
        const double v1 = __dsub_rn(vv, __dmul_rn(c, xx));
        xx = x1; vv = v1; tt = __dadd_rn(tt, dt);
        if (tt >= t_end) { m[i] = 1; atomicAdd((unsigned int*)finished.data, 1u); break; }
    }
    X[i] = xx; V[i] = vv; T[i] = tt;
}
"""


def _nvcc():
    for c in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    pytest.skip("nvcc is not available to build the stand-in artifact")


@pytest.fixture(scope="module")
def artifact(tmp_path_factory):
    d = tmp_path_factory.mktemp("hawk_artifact")
    src = d / "euler.cu"
    src.write_text(SOURCE)
    nvcc = _nvcc()
    subprocess.run([nvcc, "-cubin", "-gencode", "arch=compute_100a,code=sm_100a", "-o", str(d / "euler.cubin"),
                    str(src)], check=True)
    subprocess.run([nvcc, "-ptx", "-gencode", "arch=compute_100a,code=compute_100a", "-o", str(d / "euler.ptx"),
                    str(src)], check=True)
    return (d / "euler.cubin").read_bytes(), (d / "euler.ptx").read_bytes()


def _function(L, image, how):
    module = ctypes.c_uint64()
    buf = ctypes.create_string_buffer(image, len(image))
    if how == "cubin":
        _abi.check(L.eagle_backend_module_load(buf, len(image), -1, ctypes.byref(module)))
    elif how == "jit":
        _abi.check(L.eagle_backend_module_load_jit(buf, len(image), -1, 64, ctypes.byref(module)))
    else:
        size = ctypes.c_uint64()
        _abi.check(L.eagle_backend_link_ptx(buf, len(image), -1, 0, None, 0, ctypes.byref(size)))
        assert size.value > 0
        out = ctypes.create_string_buffer(size.value)
        _abi.check(L.eagle_backend_link_ptx(buf, len(image), -1, 0, out, size.value, ctypes.byref(size)))
        _abi.check(L.eagle_backend_module_load(out, size.value, -1, ctypes.byref(module)))
    fn = ctypes.c_uint64()
    _abi.check(L.eagle_backend_module_function(module.value, b"euler_step", ctypes.byref(fn)))
    return module.value, fn.value


@pytest.mark.parametrize("how", ("cubin", "jit", "link"))
def test_loaded_artifact_runs_through_run_device(orc, artifact, how):
    L = _abi.lib()
    module, fn = _function(L, artifact[0] if how == "cubin" else artifact[1], how)
    n, t_end, dt, budget = 40_000, 1.0, 1e-3, 700
    om = np.random.default_rng(5).uniform(1, 3, n)
    dev = {k: torch.zeros(n, dtype=torch.float64, device="cuda") for k in ("x", "v", "t")}
    dev["x"].fill_(1.0)
    d_om = torch.from_numpy(om).cuda()
    mask = torch.zeros(n, dtype=torch.uint8, device="cuda")
    fin = torch.zeros(1, dtype=torch.int32, device="cuda")
    fused = torch.tensor([budget], dtype=torch.int64, device="cuda")

    def h(tn, k):
        return _abi.ScalarHandle(tn.data_ptr(), k, 1, 2, 0)

    args = [h(d_om, n), ctypes.c_double(t_end), ctypes.c_double(dt), h(mask, n), h(dev["x"], n), h(dev["v"], n),
            h(dev["t"], n), h(fin, 1), h(fused, 1)]
    addrs = (ctypes.c_uint64 * len(args))(*[ctypes.addressof(a) for a in args])
    for _ in range(2):  # two launches: the second continues from the mask and state
        d = _abi.new(_abi.LaunchDesc, device=-1, block=128, function=fn, nparams=len(args), base=0, count=n,
                     n_samples=n, stream=torch.cuda.current_stream().cuda_stream)
        d.params = ctypes.cast(addrs, ctypes.POINTER(ctypes.c_uint64))
        launched = ctypes.c_int32()
        _abi.check(L.eagle_backend_run_device(ctypes.byref(d), ctypes.byref(launched)))
    torch.cuda.synchronize()
    st = [np.ones(n), np.zeros(n), np.zeros(n), np.zeros(n, np.uint8)]
    _, f1, _, _ = orc.oscillator_run(om, *st, t_end=t_end, dt=dt, max_steps=budget)
    _, f2, _, _ = orc.oscillator_run(om, *st, t_end=t_end, dt=dt, max_steps=budget)
    for k, r in zip(("x", "v", "t"), st[:3]):
        assert dev[k].cpu().numpy().tobytes() == r.tobytes(), k
    assert mask.cpu().numpy().tobytes() == st[3].tobytes()
    assert int(fin.item()) == f1 + f2 == n
    value = ctypes.c_int32()
    _abi.check(L.eagle_backend_function_attribute(fn, 4, ctypes.byref(value)))  # registers per thread
    assert value.value > 0
    L.eagle_backend_module_release(module, -1)


def test_module_function_refusals(artifact):
    L = _abi.lib()
    module, _ = _function(L, artifact[0], "cubin")
    fn = ctypes.c_uint64()
    with pytest.raises(IndexError, match="no function named"):
        _abi.check(L.eagle_backend_module_function(module, b"not_there", ctypes.byref(fn)))
    L.eagle_backend_module_release(module, -1)
    with pytest.raises(ValueError):
        _abi.check(L.eagle_backend_module_load(None, 0, -1, ctypes.byref(fn)))


def test_stream_ordered_memory_and_strided_copies():
    L = _abi.lib()
    s = torch.cuda.Stream()
    chunk, ptr = ctypes.c_uint64(), ctypes.c_uint64()
    _abi.check(L.eagle_backend_mem_alloc(_abi.MEM_DEVICE, -1, 1 << 20, s.cuda_stream, ctypes.byref(chunk),
                                         ctypes.byref(ptr)))
    assert ptr.value != 0 and ptr.value % 256 == 0
    dev = ctypes.c_int32()
    _abi.check(L.eagle_backend_pointer_device(ptr.value, ctypes.byref(dev)))
    assert dev.value == torch.cuda.current_device()
    # a strided copy: 64 rows of 96 bytes out of a 128-byte pitched host block
    rows, width, pitch = 64, 96, 128
    host = (np.arange(rows * pitch) % 251).astype(np.uint8)
    pinned = torch.from_numpy(host).pin_memory()
    _abi.check(L.eagle_backend_memcpy_strided(ptr.value, width, pinned.data_ptr(), pitch, width, rows, _abi.COPY_H2D,
                                              s.cuda_stream))
    back = torch.zeros(rows * width, dtype=torch.uint8).pin_memory()
    _abi.check(L.eagle_backend_memcpy(back.data_ptr(), ptr.value, rows * width, _abi.COPY_D2H, s.cuda_stream))
    s.synchronize()
    assert back.numpy().tobytes() == host.reshape(rows, pitch)[:, :width].tobytes()
    L.eagle_backend_mem_release(chunk.value)
    left = ctypes.c_int64(-1)
    _abi.check(L.eagle_backend_mem_drain(ctypes.byref(left)))
    assert left.value == 0
    # pinned host memory, and a zero-byte allocation
    _abi.check(L.eagle_backend_mem_alloc(_abi.MEM_PINNED, -1, 4096, 0, ctypes.byref(chunk), ctypes.byref(ptr)))
    assert ptr.value != 0
    L.eagle_backend_mem_release(chunk.value)
    _abi.check(L.eagle_backend_mem_alloc(_abi.MEM_DEVICE, -1, 0, 0, ctypes.byref(chunk), ctypes.byref(ptr)))
    assert ptr.value == 0 and chunk.value == 0
    _abi.check(L.eagle_backend_pointer_device(0, ctypes.byref(dev)))
    assert dev.value == -1
    torch.cuda.synchronize()
