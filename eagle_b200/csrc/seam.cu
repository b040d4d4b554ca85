// The seam's plumbing entries: meta, device scope, streams, memory, events and
// the raw / partition launches of the hawk kernel ABI. Each entry keeps the
// meaning of the eagle-backend/1 declaration its header comment cites.
#include "common.cuh"

#include <mutex>
#include <unordered_map>
#include <vector>

namespace eb {

std::string& lastError()
{
    thread_local std::string message;
    return message;
}

int resolveDevice(int32_t device, uint64_t ptr)
{
    if (device >= 0) {
        int count = 0;
        cudaCheck(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
        if (device >= count)
            invalid("eagle_b200: device " + std::to_string(device) + " out of range (" + std::to_string(count)
                + " devices)");
        return device;
    }
    if (ptr != 0) {
        cudaPointerAttributes a{};
        if (cudaPointerGetAttributes(&a, reinterpret_cast<const void*>(ptr)) == cudaSuccess
            && (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged))
            return a.device;
        (void)cudaGetLastError();
    }
    int cur = 0;
    cudaCheck(cudaGetDevice(&cur), "cudaGetDevice");
    return cur;
}

const Driver& driver()
{
    static Driver d;
    static std::once_flag once;
    std::call_once(once, [] {
        auto get = [](const char* sym, void** fn) {
            cudaDriverEntryPointQueryResult q{};
            if (cudaGetDriverEntryPoint(sym, fn, cudaEnableDefault, &q) != cudaSuccess
                || q != cudaDriverEntryPointSuccess)
                *fn = nullptr;
            (void)cudaGetLastError();
        };
        get("cuLaunchKernel", reinterpret_cast<void**>(&d.launchKernel));
        get("cuFuncGetAttribute", reinterpret_cast<void**>(&d.funcGetAttribute));
        get("cuGetErrorName", reinterpret_cast<void**>(&d.getErrorName));
    });
    if (d.launchKernel == nullptr || d.funcGetAttribute == nullptr)
        fail(EAGLE_BACKEND_UNAVAILABLE, "eagle_b200: the CUDA driver's launch entry points are unavailable");
    return d;
}

int smCount()
{
    static std::mutex mu;
    static std::vector<int> cache;
    int dev = 0;
    cudaCheck(cudaGetDevice(&dev), "cudaGetDevice");
    std::lock_guard<std::mutex> lock(mu);
    if (int(cache.size()) <= dev)
        cache.resize(size_t(dev) + 1, 0);
    if (cache[size_t(dev)] == 0)
        cudaCheck(cudaDeviceGetAttribute(&cache[size_t(dev)], cudaDevAttrMultiProcessorCount, dev),
            "cudaDeviceGetAttribute");
    return cache[size_t(dev)];
}

void requireDevice()
{
    int count = 0;
    const cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) {
        (void)cudaGetLastError();
        fail(EAGLE_BACKEND_UNAVAILABLE, std::string("eagle_b200: no CUDA device visible")
            + (e != cudaSuccess ? std::string(" (") + cudaGetErrorName(e) + ")" : std::string()));
    }
}

namespace {

void copyText(char* dst, size_t n, const char* src)
{
    std::snprintf(dst, n, "%s", src);
}

struct Stream {
    int device;
    cudaStream_t s;
};

cudaMemcpyKind copyKind(int32_t kind)
{
    switch (kind) {
    case EAGLE_BACKEND_COPY_H2D: return cudaMemcpyHostToDevice;
    case EAGLE_BACKEND_COPY_D2H: return cudaMemcpyDeviceToHost;
    case EAGLE_BACKEND_COPY_D2D: return cudaMemcpyDeviceToDevice;
    case EAGLE_BACKEND_COPY_H2H: return cudaMemcpyHostToHost;
    default: invalid("eagle_backend_memcpy: unknown copy kind " + std::to_string(kind));
    }
}

}  // namespace
}  // namespace eb

using namespace eb;

#define EB_API extern "C" __attribute__((visibility("default")))

// ---- meta -----------------------------------------------------------------------

EB_API uint32_t eagle_backend_version(void) { return EAGLE_BACKEND_VERSION; }

EB_API const char* eagle_backend_last_error(void) { return lastError().c_str(); }

EB_API eagle_backend_status eagle_backend_build_info(struct eagle_backend_build_info* info)
{
    return guarded([&] {
        if (info == nullptr || info->struct_size < 8)
            invalid("eagle_backend_build_info: null or short struct");
        struct eagle_backend_build_info b{};
        b.struct_size = sizeof b;
        b.abi_version = EAGLE_BACKEND_VERSION;
        b.cudart_version = CUDART_VERSION;
        copyText(b.eagle_version, sizeof b.eagle_version, "0.7.9-b200");
        copyText(b.archs, sizeof b.archs, "100a/");
        copyText(b.backend_kind, sizeof b.backend_kind, "cuda");
        const uint32_t size = info->struct_size < sizeof b ? info->struct_size : uint32_t(sizeof b);
        std::memcpy(info, &b, size);
        info->struct_size = size;
    });
}

EB_API eagle_backend_status eagle_backend_probe(void)
{
    return guarded([&] {
        requireDevice();
        int major = 0, minor = 0;
        cudaCheck(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, 0), "cudaDeviceGetAttribute");
        cudaCheck(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, 0), "cudaDeviceGetAttribute");
        if (major != 10 || minor != 0)
            fail(EAGLE_BACKEND_UNAVAILABLE, "eagle_b200: device 0 is sm_" + std::to_string(major)
                + std::to_string(minor) + "; this build carries sm_100a code only");
    });
}

EB_API void eagle_backend_free(void* p) { std::free(p); }

EB_API eagle_backend_status eagle_backend_capabilities(uint64_t* groups)
{
    return guarded([&] {
        if (groups == nullptr)
            invalid("eagle_backend_capabilities: null output");
        *groups = EAGLE_BACKEND_CAP_STREAM | EAGLE_BACKEND_CAP_CAPTURER | EAGLE_BACKEND_CAP_CAPTURED
            | EAGLE_BACKEND_CAP_FORK | EAGLE_BACKEND_CAP_CONDITIONAL | EAGLE_BACKEND_CAP_ATTRIBUTION
            | EAGLE_BACKEND_CAP_GRAPH | EAGLE_BACKEND_CAP_LAUNCHER | EAGLE_BACKEND_CAP_EXEC | EAGLE_BACKEND_CAP_DEVICE
            | EAGLE_BACKEND_CAP_INTEROP | EAGLE_BACKEND_CAP_FILTERING;
        // IF/ELSE and SWITCH nodes exist from driver 12.8 on: the driver's version is their capability.
        int v = 0;
        if (cudaDriverGetVersion(&v) == cudaSuccess && v >= 12080)
            *groups |= EAGLE_BACKEND_CAP_CONDITIONAL_IF_ELSE | EAGLE_BACKEND_CAP_CONDITIONAL_SWITCH;
        (void)cudaGetLastError();
    });
}

EB_API eagle_backend_status eagle_backend_device_types(int32_t* types, int32_t cap, int32_t* count)
{
    return guarded([&] {
        if (count == nullptr)
            invalid("eagle_backend_device_types: null count");
        *count = 1;
        if (cap >= 1 && types != nullptr)
            types[0] = 2;  // kDLCUDA
    });
}

// ---- stream -------------------------------------------------------------------

EB_API eagle_backend_status eagle_backend_stream_create(const struct eagle_backend_stream_desc* desc,
    eagle_backend_stream* out)
{
    return guarded([&] {
        const auto d = readDesc(desc, EAGLE_BACKEND_STREAM_NON_BLOCKING, "eagle_backend_stream_create");
        if (out == nullptr)
            invalid("eagle_backend_stream_create: null output");
        requireDevice();
        const int dev = resolveDevice(d.device, 0);
        DeviceScope scope(dev);
        cudaStream_t s = nullptr;
        cudaCheck(cudaStreamCreateWithFlags(&s, (d.flags & EAGLE_BACKEND_STREAM_NON_BLOCKING) ? cudaStreamNonBlocking
                                                                                                : cudaStreamDefault),
            "cudaStreamCreateWithFlags");
        *out = reinterpret_cast<eagle_backend_stream>(new Stream{dev, s});
    });
}

EB_API eagle_backend_status eagle_backend_stream_ptr(eagle_backend_stream h, uint64_t* stream)
{
    return guarded([&] {
        if (h == nullptr)
            fail(EAGLE_BACKEND_BAD_HANDLE, "eagle_backend_stream_ptr: null handle");
        if (stream == nullptr)
            invalid("eagle_backend_stream_ptr: null output");
        *stream = reinterpret_cast<uint64_t>(reinterpret_cast<Stream*>(h)->s);
    });
}

EB_API eagle_backend_status eagle_backend_stream_synchronize(eagle_backend_stream h)
{
    return guarded([&] {
        if (h == nullptr)
            fail(EAGLE_BACKEND_BAD_HANDLE, "eagle_backend_stream_synchronize: null handle");
        auto* s = reinterpret_cast<Stream*>(h);
        DeviceScope scope(s->device);
        cudaCheck(cudaStreamSynchronize(s->s), "cudaStreamSynchronize");
    });
}

EB_API void eagle_backend_stream_release(eagle_backend_stream h)
{
    if (h == nullptr)
        return;
    auto* s = reinterpret_cast<Stream*>(h);
    {
        int prev = 0;
        if (cudaGetDevice(&prev) == cudaSuccess) {
            (void)cudaSetDevice(s->device);
            (void)cudaStreamDestroy(s->s);
            (void)cudaSetDevice(prev);
        }
    }
    delete s;
}

// ---- device ----------------------------------------------------------------------

EB_API eagle_backend_status eagle_backend_device_props(int32_t device, struct eagle_backend_device_props* props)
{
    return guarded([&] {
        if (props == nullptr || props->struct_size < 8)
            invalid("eagle_backend_device_props: null or short struct");
        requireDevice();
        const int dev = resolveDevice(device, 0);
        DeviceScope scope(dev);
        cudaDeviceProp p{};
        cudaCheck(cudaGetDeviceProperties(&p, dev), "cudaGetDeviceProperties");
        struct eagle_backend_device_props o{};
        o.struct_size = sizeof o;
        o.device = dev;
        copyText(o.name, sizeof o.name, p.name);
        o.cc_major = p.major;
        o.cc_minor = p.minor;
        o.sm_count = p.multiProcessorCount;
        int clockKhz = 0, memKhz = 0, ratio = 0;
        (void)cudaDeviceGetAttribute(&clockKhz, cudaDevAttrClockRate, dev);
        (void)cudaDeviceGetAttribute(&memKhz, cudaDevAttrMemoryClockRate, dev);
        (void)cudaDeviceGetAttribute(&ratio, cudaDevAttrSingleToDoublePrecisionPerfRatio, dev);
        (void)cudaGetLastError();
        o.clock_rate_khz = clockKhz;
        o.memory_clock_rate_khz = memKhz;
        o.memory_bus_width_bits = p.memoryBusWidth;
        o.regs_per_block = p.regsPerBlock;
        o.regs_per_sm = p.regsPerMultiprocessor;
        o.warp_size = p.warpSize;
        o.shared_mem_per_block = int64_t(p.sharedMemPerBlockOptin);
        o.shared_mem_per_sm = int64_t(p.sharedMemPerMultiprocessor);
        o.peak_bytes_per_s = double(memKhz) * 1e3 * double(p.memoryBusWidth) * 2.0 / 8.0;
        // sm_100: 128 fp32 lanes per SM, fp64 at the device's reported ratio
        o.peak_flops_sp = 2.0 * 128.0 * double(p.multiProcessorCount) * double(clockKhz) * 1e3;
        o.fp64_ratio = ratio > 0 ? double(ratio) : 0.0;
        o.peak_flops_dp = ratio > 0 ? o.peak_flops_sp / double(ratio) : 0.0;
        o.ridge_flops_per_byte_sp = o.peak_bytes_per_s > 0 ? o.peak_flops_sp / o.peak_bytes_per_s : 0.0;
        o.ridge_flops_per_byte_dp = o.peak_bytes_per_s > 0 ? o.peak_flops_dp / o.peak_bytes_per_s : 0.0;
        size_t freeB = 0, totalB = 0;
        cudaCheck(cudaMemGetInfo(&freeB, &totalB), "cudaMemGetInfo");
        o.total_mem_bytes = int64_t(totalB);
        o.free_mem_bytes = int64_t(freeB);
        const uint32_t size = props->struct_size < sizeof o ? props->struct_size : uint32_t(sizeof o);
        std::memcpy(props, &o, size);
        props->struct_size = size;
    });
}

EB_API eagle_backend_status eagle_backend_device_count(int32_t* count)
{
    return guarded([&] {
        if (count == nullptr)
            invalid("eagle_backend_device_count: null output");
        int c = 0;
        const cudaError_t e = cudaGetDeviceCount(&c);
        if (e != cudaSuccess) {
            (void)cudaGetLastError();
            c = 0;
        }
        *count = c;
    });
}

EB_API eagle_backend_status eagle_backend_set_device(int32_t device)
{
    return guarded([&] {
        requireDevice();
        cudaCheck(cudaSetDevice(resolveDevice(device, 0)), "cudaSetDevice");
    });
}

EB_API eagle_backend_status eagle_backend_get_device(int32_t* device)
{
    return guarded([&] {
        if (device == nullptr)
            invalid("eagle_backend_get_device: null output");
        int d = 0;
        cudaCheck(cudaGetDevice(&d), "cudaGetDevice");
        *device = d;
    });
}

EB_API eagle_backend_status eagle_backend_launch_status(int32_t device)
{
    return guarded([&] {
        const int dev = resolveDevice(device, 0);
        DeviceScope scope(dev);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess)
            fail(EAGLE_BACKEND_ERROR, std::string("eagle_backend_launch_status: ") + cudaGetErrorName(e) + " ("
                + cudaGetErrorString(e) + ")");
    });
}

EB_API eagle_backend_status eagle_backend_device_synchronize(int32_t device)
{
    return guarded([&] {
        DeviceScope scope(resolveDevice(device, 0));
        cudaCheck(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    });
}

EB_API eagle_backend_status eagle_backend_stream_is_capturing(uint64_t stream, int32_t* capturing)
{
    return guarded([&] {
        if (capturing == nullptr)
            invalid("eagle_backend_stream_is_capturing: null output");
        cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
        cudaCheck(cudaStreamIsCapturing(seamStream(stream), &st), "cudaStreamIsCapturing");
        *capturing = st == cudaStreamCaptureStatusActive ? 1 : 0;
    });
}

EB_API eagle_backend_status eagle_backend_stream_sync(int32_t device, uint64_t stream)
{
    return guarded([&] {
        DeviceScope scope(resolveDevice(device, 0));
        cudaCheck(cudaStreamSynchronize(seamStream(stream)), "cudaStreamSynchronize");
    });
}

// ---- memory ------------------------------------------------------------------------

EB_API eagle_backend_status eagle_backend_memset_device(uint64_t ptr, uint64_t bytes, uint64_t stream)
{
    return guarded([&] {
        if (bytes == 0)
            return;
        if (ptr == 0)
            invalid("eagle_backend_memset_device: null address");
        DeviceScope scope(resolveDevice(-1, ptr));
        cudaCheck(cudaMemsetAsync(reinterpret_cast<void*>(ptr), 0, bytes, seamStream(stream)), "cudaMemsetAsync");
    });
}

EB_API eagle_backend_status eagle_backend_memcpy_device(uint64_t dst, uint64_t src, uint64_t bytes, uint64_t stream)
{
    return guarded([&] {
        if (bytes == 0 || dst == src)
            return;
        if (dst == 0 || src == 0)
            invalid("eagle_backend_memcpy_device: null address");
        DeviceScope scope(resolveDevice(-1, dst));
        cudaCheck(cudaMemcpyAsync(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), bytes,
                      cudaMemcpyDeviceToDevice, seamStream(stream)),
            "cudaMemcpyAsync");
    });
}

EB_API eagle_backend_status eagle_backend_memcpy(uint64_t dst, uint64_t src, uint64_t bytes, int32_t kind,
    uint64_t stream)
{
    return guarded([&] {
        const cudaMemcpyKind k = copyKind(kind);
        if (bytes == 0 || dst == src)
            return;
        if (dst == 0 || src == 0)
            invalid("eagle_backend_memcpy: null address");
        const uint64_t devPtr = kind == EAGLE_BACKEND_COPY_H2D ? dst : src;
        DeviceScope scope(resolveDevice(-1, devPtr));
        cudaCheck(cudaMemcpyAsync(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), bytes, k,
                      seamStream(stream)),
            "cudaMemcpyAsync");
    });
}

// ---- interop (bit 11): the DLPack stream fence and host memory ---------------------

namespace {

constexpr int64_t kStreamNone = INT64_MIN;  // no stream argument given: the type's default
constexpr int32_t kDLCUDA = 2;

/** A DLPack ``__dlpack__(stream=)`` value of a CUDA buffer: 1 the legacy default
 *  stream, 2 the per-thread default, -1 no ordering, 0 refused, else a raw stream
 *  (python/src/seam/eagle_backend.h:90-93). ``order`` is false for -1. */
struct DlStream {
    bool order;
    cudaStream_t s;
    int64_t code;
};

DlStream dlStream(int64_t code, const char* who)
{
    if (code == kStreamNone)
        code = 1;
    if (code == 0)
        invalid(std::string(who) + ": stream 0 is ambiguous and refused by DLPack; pass 1 for the legacy default "
                                   "stream or 2 for the per-thread default stream");
    if (code == -1)
        return DlStream{false, nullptr, code};
    if (code < -1)
        invalid(std::string(who) + ": a stream must be -1, 1, 2 or a stream handle, got " + std::to_string(code));
    cudaStream_t s = code == 1 ? cudaStreamLegacy
        : code == 2            ? cudaStreamPerThread
                               : reinterpret_cast<cudaStream_t>(code);
    return DlStream{true, s, code};
}

/** Timing-free events reused per device; never destroyed (the process may outlive
 *  its contexts' teardown order). */
struct FenceEvents {
    std::mutex mu;
    std::unordered_map<int, std::vector<cudaEvent_t>> free;
    int64_t created = 0;

    cudaEvent_t acquire(int device)
    {
        {
            std::lock_guard<std::mutex> lock(mu);
            auto& f = free[device];
            if (!f.empty()) {
                cudaEvent_t e = f.back();
                f.pop_back();
                return e;
            }
            ++created;
        }
        cudaEvent_t e = nullptr;
        cudaCheck(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreateWithFlags");
        return e;
    }
    void release(int device, cudaEvent_t e)
    {
        std::lock_guard<std::mutex> lock(mu);
        free[device].push_back(e);
    }
};

FenceEvents& fenceEvents()
{
    static FenceEvents* pool = new FenceEvents();
    return *pool;
}

}  // namespace

EB_API eagle_backend_status eagle_backend_fence(int32_t dl_device_type, int32_t device_id, int64_t producer,
    int64_t consumer)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_fence";
        if (dl_device_type != kDLCUDA)
            unsupported(std::string(who) + ": this backend serves DLPack device type 2 (CUDA), not "
                + std::to_string(dl_device_type));
        const DlStream p = dlStream(producer, who), c = dlStream(consumer, who);
        if (!p.order || !c.order || p.code == c.code)
            return;  // no ordering asked for, or one stream orders itself
        requireDevice();
        const int dev = resolveDevice(device_id, 0);
        DeviceScope scope(dev);
        FenceEvents& pool = fenceEvents();
        cudaEvent_t e = pool.acquire(dev);
        const cudaError_t rec = cudaEventRecord(e, p.s);
        const cudaError_t wait = rec == cudaSuccess ? cudaStreamWaitEvent(c.s, e, 0) : rec;
        pool.release(dev, e);  // a recorded event may be recorded again: the wait keeps its own snapshot
        cudaCheck(rec, "cudaEventRecord");
        cudaCheck(wait, "cudaStreamWaitEvent");
    });
}

EB_API eagle_backend_status eagle_backend_event_pool_created(int64_t* count)
{
    return guarded([&] {
        if (count == nullptr)
            invalid("eagle_backend_event_pool_created: null output");
        FenceEvents& pool = fenceEvents();
        std::lock_guard<std::mutex> lock(pool.mu);
        *count = pool.created;
    });
}

EB_API eagle_backend_status eagle_backend_host_alloc(uint64_t bytes, uint64_t* out)
{
    return guarded([&] {
        if (out == nullptr)
            invalid("eagle_backend_host_alloc: null output");
        *out = 0;
        if (bytes == 0)
            return;
        requireDevice();
        void* p = nullptr;
        cudaCheck(cudaHostAlloc(&p, size_t(bytes), cudaHostAllocPortable), "cudaHostAlloc");
        *out = reinterpret_cast<uint64_t>(p);
    });
}

EB_API eagle_backend_status eagle_backend_host_free(uint64_t ptr)
{
    return guarded([&] {
        if (ptr != 0)
            cudaCheck(cudaFreeHost(reinterpret_cast<void*>(ptr)), "cudaFreeHost");
    });
}

EB_API eagle_backend_status eagle_backend_host_func(uint64_t stream, void (*fn)(void*), void* arg)
{
    return guarded([&] {
        if (fn == nullptr)
            invalid("eagle_backend_host_func: null function");
        requireDevice();
        cudaCheck(cudaLaunchHostFunc(seamStream(stream), fn, arg), "cudaLaunchHostFunc");
    });
}

// ---- events ------------------------------------------------------------------------

namespace {
eagle_backend_status eventCreate(int32_t device, uint64_t* event, unsigned flags)
{
    return guarded([&] {
        if (event == nullptr)
            invalid("eagle_backend_event_create: null output");
        DeviceScope scope(resolveDevice(device, 0));
        cudaEvent_t e = nullptr;
        cudaCheck(cudaEventCreateWithFlags(&e, flags), "cudaEventCreateWithFlags");
        *event = reinterpret_cast<uint64_t>(e);
    });
}
}  // namespace

EB_API eagle_backend_status eagle_backend_event_create(int32_t device, uint64_t* event)
{
    return eventCreate(device, event, cudaEventDisableTiming);
}

EB_API eagle_backend_status eagle_backend_event_create_timed(int32_t device, uint64_t* event)
{
    return eventCreate(device, event, cudaEventDefault);
}

EB_API eagle_backend_status eagle_backend_event_elapsed(uint64_t start, uint64_t end, float* ms)
{
    return guarded([&] {
        if (ms == nullptr || start == 0 || end == 0)
            invalid("eagle_backend_event_elapsed: null event or output");
        cudaCheck(cudaEventElapsedTime(ms, reinterpret_cast<cudaEvent_t>(start), reinterpret_cast<cudaEvent_t>(end)),
            "cudaEventElapsedTime");
    });
}

EB_API eagle_backend_status eagle_backend_event_record(uint64_t event, uint64_t stream)
{
    return guarded([&] {
        if (event == 0)
            invalid("eagle_backend_event_record: null event");
        cudaCheck(cudaEventRecord(reinterpret_cast<cudaEvent_t>(event), seamStream(stream)), "cudaEventRecord");
    });
}

EB_API eagle_backend_status eagle_backend_event_wait(uint64_t stream, uint64_t event)
{
    return guarded([&] {
        if (event == 0)
            invalid("eagle_backend_event_wait: null event");
        cudaCheck(cudaStreamWaitEvent(seamStream(stream), reinterpret_cast<cudaEvent_t>(event), 0),
            "cudaStreamWaitEvent");
    });
}

EB_API void eagle_backend_event_release(uint64_t event, int32_t device)
{
    if (event == 0)
        return;
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess)
        return;
    if (device >= 0)
        (void)cudaSetDevice(device);
    (void)cudaEventDestroy(reinterpret_cast<cudaEvent_t>(event));
    (void)cudaSetDevice(prev);
}

// ---- raw and partition launches ------------------------------------------------------

EB_API eagle_backend_status eagle_backend_function_attribute(uint64_t function, int32_t attribute, int32_t* value)
{
    return guarded([&] {
        if (function == 0 || value == nullptr)
            invalid("eagle_backend_function_attribute: null function or output");
        int v = 0;
        cuCheck(driver().funcGetAttribute(&v, static_cast<CUfunction_attribute>(attribute),
                    reinterpret_cast<CUfunction>(function)),
            "cuFuncGetAttribute");
        *value = v;
    });
}

EB_API eagle_backend_status eagle_backend_launch_raw(const struct eagle_backend_launch_raw_desc* desc)
{
    return guarded([&] {
        const auto d = readDesc(desc, 0u, "eagle_backend_launch_raw");
        if (d.function == 0)
            invalid("eagle_backend_launch_raw: null function");
        if (d.reserved != 0)
            invalid("eagle_backend_launch_raw: reserved must be zero");
        for (int a = 0; a < 3; ++a)
            if (d.grid[a] == 0 || d.block[a] == 0)
                invalid("eagle_backend_launch_raw: grid and block extents must be >= 1");
        const int dev = d.device >= 0 ? d.device : resolveDevice(-1, 0);
        DeviceScope scope(dev);
        cuCheck(driver().launchKernel(reinterpret_cast<CUfunction>(d.function), d.grid[0], d.grid[1], d.grid[2], d.block[0],
                    d.block[1], d.block[2], d.shared_bytes, reinterpret_cast<CUstream>(seamStream(d.stream)),
                    reinterpret_cast<void**>(d.args), nullptr),
            "cuLaunchKernel");
    });
}

EB_API eagle_backend_status eagle_backend_run_device(const struct eagle_backend_launch_desc* desc, int32_t* launched)
{
    return guarded([&] {
        const auto d = readDesc(desc, 0u, "eagle_backend_run_device");
        if (launched == nullptr)
            invalid("eagle_backend_run_device: null output");
        if (d.function == 0)
            invalid("eagle_backend_run_device: null function");
        if (d.nparams < 0 || (d.nparams > 0 && d.params == nullptr))
            invalid("eagle_backend_run_device: params must hold nparams addresses");
        if (d.base < 0 || d.count < 0 || d.n_samples < 0 || d.base + d.count > d.n_samples)
            fail(EAGLE_BACKEND_INDEX, "eagle_backend_run_device: the partition [base, base + count) must lie in "
                                      "[0, n_samples)");
        if (d.count == 0) {
            *launched = 0;
            return;
        }
        const uint32_t block = d.block == 0 ? 256u : d.block;
        const int64_t grid = (d.count + block - 1) / block;
        if (grid > INT64_C(2147483647))
            unsupported("eagle_backend_run_device: the grid exceeds 2^31 - 1 blocks");
        // the packed role arguments, then the partition triple by value
        std::vector<void*> args(size_t(d.nparams) + 3);
        for (int64_t i = 0; i < d.nparams; ++i)
            args[size_t(i)] = reinterpret_cast<void*>(d.params[i]);
        int64_t triple[3] = {d.base, d.count, d.n_samples};
        for (int i = 0; i < 3; ++i)
            args[size_t(d.nparams) + size_t(i)] = &triple[i];
        const int dev = d.device >= 0 ? d.device : resolveDevice(-1, 0);
        DeviceScope scope(dev);
        cuCheck(driver().launchKernel(reinterpret_cast<CUfunction>(d.function), unsigned(grid), 1, 1, block, 1, 1, 0,
                    reinterpret_cast<CUstream>(seamStream(d.stream)), args.data(), nullptr),
            "cuLaunchKernel");
        *launched = 1;
    });
}
