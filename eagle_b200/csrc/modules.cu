// The seam's per-symbol minor-7 entries outside the hot loop: device modules
// (hawk artifacts: a cubin, fatbin or PTX loaded in the device's primary context,
// a function taken from it and launched through launch_raw / run_device), and
// stream-ordered memory for eagle's array layer (python/src/seam/eagle_backend.h
// :457-476, :612-646).
#include "common.cuh"

#include <deque>
#include <mutex>
#include <string>

#define EB_API extern "C" __attribute__((visibility("default")))

namespace eb {
namespace {

struct ModuleDriver {
    CUresult (*load)(CUmodule*, const void*) = nullptr;
    CUresult (*loadEx)(CUmodule*, const void*, unsigned, CUjit_option*, void**) = nullptr;
    CUresult (*function)(CUfunction*, CUmodule, const char*) = nullptr;
    CUresult (*unload)(CUmodule) = nullptr;
    CUresult (*linkCreate)(unsigned, CUjit_option*, void**, CUlinkState*) = nullptr;
    CUresult (*linkAdd)(CUlinkState, CUjitInputType, void*, size_t, const char*, unsigned, CUjit_option*,
        void**) = nullptr;
    CUresult (*linkComplete)(CUlinkState, void**, size_t*) = nullptr;
    CUresult (*linkDestroy)(CUlinkState) = nullptr;
};

const ModuleDriver& moduleDriver()
{
    static ModuleDriver d;
    static std::once_flag once;
    std::call_once(once, [] {
        auto get = [](const char* sym, void** fn) {
            cudaDriverEntryPointQueryResult q{};
            if (cudaGetDriverEntryPointByVersion(sym, fn, CUDART_VERSION, cudaEnableDefault, &q) != cudaSuccess
                || q != cudaDriverEntryPointSuccess)
                *fn = nullptr;
            (void)cudaGetLastError();
        };
        get("cuModuleLoadData", reinterpret_cast<void**>(&d.load));
        get("cuModuleLoadDataEx", reinterpret_cast<void**>(&d.loadEx));
        get("cuModuleGetFunction", reinterpret_cast<void**>(&d.function));
        get("cuModuleUnload", reinterpret_cast<void**>(&d.unload));
        get("cuLinkCreate", reinterpret_cast<void**>(&d.linkCreate));
        get("cuLinkAddData", reinterpret_cast<void**>(&d.linkAdd));
        get("cuLinkComplete", reinterpret_cast<void**>(&d.linkComplete));
        get("cuLinkDestroy", reinterpret_cast<void**>(&d.linkDestroy));
    });
    return d;
}

template <class F>
F needFn(F fn, const char* name)
{
    if (fn == nullptr)
        fail(EAGLE_BACKEND_UNAVAILABLE, std::string("eagle_b200: the driver lacks ") + name);
    return fn;
}

/** Make ``device`` (-1: the current one) current with its primary context live. */
int enterDevice(int32_t device)
{
    requireDevice();
    int dev = device;
    if (dev < 0)
        cudaCheck(cudaGetDevice(&dev), "cudaGetDevice");
    return resolveDevice(dev, 0);
}

void primaryContext()
{
    cudaCheck(cudaFree(nullptr), "cudaFree(0)");  // the runtime makes the device's primary context current
}

// ---- stream-ordered memory -------------------------------------------------------

struct Chunk {
    int32_t kind;
    int device;
    void* ptr;
    cudaStream_t stream;
};

/** Frees queued while their stream was capturing; run at the next allocation or drain. */
struct Deferred {
    std::mutex mu;
    std::deque<Chunk*> queue;
};

Deferred& deferred()
{
    static Deferred* d = new Deferred();
    return *d;
}

bool capturing(cudaStream_t s)
{
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &st) != cudaSuccess) {
        (void)cudaGetLastError();
        return false;
    }
    return st != cudaStreamCaptureStatusNone;
}

void freeChunk(Chunk* c)
{
    int prev = -1;
    (void)cudaGetDevice(&prev);
    (void)cudaSetDevice(c->device);
    if (c->kind == EAGLE_BACKEND_MEM_PINNED)
        (void)cudaFreeHost(c->ptr);
    else
        (void)cudaFreeAsync(c->ptr, c->stream);
    (void)cudaGetLastError();
    if (prev >= 0)
        (void)cudaSetDevice(prev);
    delete c;
}

/** Run the queued frees whose streams are no longer capturing; the count left. */
int64_t drainDeferred()
{
    Deferred& d = deferred();
    std::deque<Chunk*> ready, waiting;
    {
        std::lock_guard<std::mutex> lock(d.mu);
        for (Chunk* c : d.queue)
            (capturing(c->stream) ? waiting : ready).push_back(c);
        d.queue.swap(waiting);
    }
    for (Chunk* c : ready)
        freeChunk(c);
    std::lock_guard<std::mutex> lock(d.mu);
    return int64_t(d.queue.size());
}

}  // namespace
}  // namespace eb

using namespace eb;

// ---- modules ------------------------------------------------------------------------

EB_API eagle_backend_status eagle_backend_module_load(const void* image, uint64_t bytes, int32_t device,
    uint64_t* module)
{
    return guarded([&] {
        if (image == nullptr || bytes == 0 || module == nullptr)
            invalid("eagle_backend_module_load: empty image or null output");
        DeviceScope scope(enterDevice(device));
        primaryContext();
        // PTX text must end in NUL; a cubin or fatbin ignores the byte after it
        const std::string copy(static_cast<const char*>(image), size_t(bytes));
        CUmodule m = nullptr;
        cuCheck(needFn(moduleDriver().load, "cuModuleLoadData")(&m, copy.c_str()), "cuModuleLoadData");
        *module = reinterpret_cast<uint64_t>(m);
    });
}

EB_API eagle_backend_status eagle_backend_module_load_jit(const void* image, uint64_t bytes, int32_t device,
    uint32_t max_registers, uint64_t* module)
{
    return guarded([&] {
        if (image == nullptr || bytes == 0 || module == nullptr)
            invalid("eagle_backend_module_load_jit: empty image or null output");
        DeviceScope scope(enterDevice(device));
        primaryContext();
        const std::string copy(static_cast<const char*>(image), size_t(bytes));
        CUjit_option option = CU_JIT_MAX_REGISTERS;
        void* value = reinterpret_cast<void*>(uintptr_t(max_registers));
        CUmodule m = nullptr;
        cuCheck(needFn(moduleDriver().loadEx, "cuModuleLoadDataEx")(&m, copy.c_str(), max_registers != 0 ? 1u : 0u,
                    &option, &value),
            "cuModuleLoadDataEx");
        *module = reinterpret_cast<uint64_t>(m);
    });
}

EB_API eagle_backend_status eagle_backend_link_ptx(const void* image, uint64_t bytes, int32_t device,
    uint32_t max_registers, void* out, uint64_t capacity, uint64_t* size)
{
    return guarded([&] {
        if (image == nullptr || bytes == 0 || size == nullptr)
            invalid("eagle_backend_link_ptx: empty image or null size");
        DeviceScope scope(enterDevice(device));
        primaryContext();
        const ModuleDriver& d = moduleDriver();
        std::string copy(static_cast<const char*>(image), size_t(bytes));
        CUjit_option option = CU_JIT_MAX_REGISTERS;
        void* value = reinterpret_cast<void*>(uintptr_t(max_registers));
        CUlinkState state = nullptr;
        cuCheck(needFn(d.linkCreate, "cuLinkCreate")(max_registers != 0 ? 1u : 0u, &option, &value, &state),
            "cuLinkCreate");
        auto destroy = needFn(d.linkDestroy, "cuLinkDestroy");
        try {
            cuCheck(needFn(d.linkAdd, "cuLinkAddData")(state, CU_JIT_INPUT_PTX, copy.data(), copy.size() + 1, "entry",
                        0, nullptr, nullptr),
                "cuLinkAddData");
            void* cubin = nullptr;
            size_t n = 0;
            cuCheck(needFn(d.linkComplete, "cuLinkComplete")(state, &cubin, &n), "cuLinkComplete");
            if (out != nullptr) {
                if (capacity < n)
                    invalid("eagle_backend_link_ptx: the output holds " + std::to_string(capacity)
                        + " bytes, the cubin " + std::to_string(n));
                std::memcpy(out, cubin, n);
            }
            *size = uint64_t(n);
        } catch (...) {
            destroy(state);
            throw;
        }
        destroy(state);
    });
}

EB_API eagle_backend_status eagle_backend_module_function(uint64_t module, const char* name, uint64_t* function)
{
    return guarded([&] {
        if (module == 0 || name == nullptr)
            fail(EAGLE_BACKEND_BAD_HANDLE, "eagle_backend_module_function: null module or name");
        if (function == nullptr)
            invalid("eagle_backend_module_function: null output");
        requireDevice();
        CUfunction f = nullptr;
        const CUresult r = needFn(moduleDriver().function, "cuModuleGetFunction")(&f, reinterpret_cast<CUmodule>(module),
            name);
        if (r == CUDA_ERROR_NOT_FOUND)
            fail(EAGLE_BACKEND_INDEX, std::string("eagle_backend_module_function: no function named '") + name + "'");
        cuCheck(r, "cuModuleGetFunction");
        *function = reinterpret_cast<uint64_t>(f);
    });
}

EB_API void eagle_backend_module_release(uint64_t module, int32_t device)
{
    if (module == 0)
        return;
    try {
        DeviceScope scope(enterDevice(device));
        if (auto unload = moduleDriver().unload)
            unload(reinterpret_cast<CUmodule>(module));
    } catch (...) {
        // a release never throws across the seam
    }
    (void)cudaGetLastError();
}

// ---- stream-ordered memory -------------------------------------------------------

EB_API eagle_backend_status eagle_backend_mem_alloc(int32_t kind, int32_t device, uint64_t bytes, uint64_t stream,
    uint64_t* chunk, uint64_t* ptr)
{
    return guarded([&] {
        if (chunk == nullptr || ptr == nullptr)
            invalid("eagle_backend_mem_alloc: null output");
        if (kind != EAGLE_BACKEND_MEM_DEVICE && kind != EAGLE_BACKEND_MEM_PINNED)
            invalid("eagle_backend_mem_alloc: unknown kind " + std::to_string(kind));
        *chunk = 0;
        *ptr = 0;
        if (bytes == 0)
            return;
        requireDevice();
        const cudaStream_t s = seamStream(stream);
        if (capturing(s))
            invalid("eagle_backend_mem_alloc: the stream is capturing, and an allocation is not capture-legal");
        drainDeferred();
        int dev = device;
        if (dev < 0) {
            if (stream != 0)
                cudaCheck(cudaStreamGetDevice(s, &dev), "cudaStreamGetDevice");
            else
                cudaCheck(cudaGetDevice(&dev), "cudaGetDevice");
        }
        DeviceScope scope(resolveDevice(dev, 0));
        void* p = nullptr;
        if (kind == EAGLE_BACKEND_MEM_PINNED)
            cudaCheck(cudaHostAlloc(&p, size_t(bytes), cudaHostAllocPortable), "cudaHostAlloc");
        else
            cudaCheck(cudaMallocAsync(&p, size_t(bytes), s), "cudaMallocAsync");
        auto* c = new Chunk{kind, resolveDevice(dev, 0), p, s};
        *chunk = reinterpret_cast<uint64_t>(c);
        *ptr = reinterpret_cast<uint64_t>(p);
    });
}

EB_API void eagle_backend_mem_release(uint64_t chunk)
{
    if (chunk == 0)
        return;
    auto* c = reinterpret_cast<Chunk*>(chunk);
    if (capturing(c->stream)) {
        Deferred& d = deferred();
        std::lock_guard<std::mutex> lock(d.mu);
        d.queue.push_back(c);
        return;
    }
    freeChunk(c);
}

EB_API eagle_backend_status eagle_backend_mem_drain(int64_t* left)
{
    return guarded([&] {
        const int64_t n = drainDeferred();
        if (left != nullptr)
            *left = n;
    });
}

EB_API eagle_backend_status eagle_backend_pointer_device(uint64_t ptr, int32_t* device)
{
    return guarded([&] {
        if (device == nullptr)
            invalid("eagle_backend_pointer_device: null output");
        *device = -1;
        cudaPointerAttributes a{};
        if (ptr == 0 || cudaPointerGetAttributes(&a, reinterpret_cast<const void*>(ptr)) != cudaSuccess) {
            (void)cudaGetLastError();
            return;
        }
        if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged)
            *device = a.device;
    });
}

EB_API eagle_backend_status eagle_backend_memcpy_strided(uint64_t dst, uint64_t dst_pitch, uint64_t src,
    uint64_t src_pitch, uint64_t width_bytes, uint64_t height, int32_t kind, uint64_t stream)
{
    return guarded([&] {
        cudaMemcpyKind k = cudaMemcpyDefault;
        switch (kind) {
        case EAGLE_BACKEND_COPY_H2D: k = cudaMemcpyHostToDevice; break;
        case EAGLE_BACKEND_COPY_D2H: k = cudaMemcpyDeviceToHost; break;
        case EAGLE_BACKEND_COPY_D2D: k = cudaMemcpyDeviceToDevice; break;
        default: invalid("eagle_backend_memcpy_strided: kind must be H2D, D2H or D2D");
        }
        if (width_bytes == 0 || height == 0)
            return;
        if (dst == 0 || src == 0)
            invalid("eagle_backend_memcpy_strided: null address");
        if (dst_pitch < width_bytes || src_pitch < width_bytes)
            invalid("eagle_backend_memcpy_strided: a pitch is narrower than the row");
        requireDevice();
        DeviceScope scope(resolveDevice(-1, kind == EAGLE_BACKEND_COPY_H2D ? dst : src));
        cudaCheck(cudaMemcpy2DAsync(reinterpret_cast<void*>(dst), size_t(dst_pitch), reinterpret_cast<const void*>(src),
                      size_t(src_pitch), size_t(width_bytes), size_t(height), k, seamStream(stream)),
            "cudaMemcpy2DAsync");
    });
}
