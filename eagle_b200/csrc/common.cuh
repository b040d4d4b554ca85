// Shared pieces of the B200 engine: status mapping for the C seam, the hawk
// argument-handle layout, device-resolution helpers and the device primitives
// (warp scans, the decoupled look-back) several kernels use.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>

#include "../../include/eagle_b200.h"

namespace eb {

// ------------------------------------------------------------------ host errors

/** A failure that maps to one seam status; the message goes to last_error. */
struct Failure : std::runtime_error {
    eagle_backend_status status;
    Failure(eagle_backend_status s, const std::string& m) : std::runtime_error(m), status(s) {}
};

[[noreturn]] inline void fail(eagle_backend_status s, const std::string& m) { throw Failure(s, m); }
[[noreturn]] inline void invalid(const std::string& m) { fail(EAGLE_BACKEND_INVALID_ARGUMENT, m); }
[[noreturn]] inline void unsupported(const std::string& m) { fail(EAGLE_BACKEND_UNSUPPORTED, m); }

inline void cudaCheck(cudaError_t e, const char* what)
{
    if (e != cudaSuccess)
        fail(EAGLE_BACKEND_ERROR, std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

/** The three driver functions the seam needs (raw launches of CUfunction
 *  handles), resolved through the runtime at first use so the library links no
 *  libcuda and loads on a machine without a driver. */
struct Driver {
    CUresult (*launchKernel)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned,
        CUstream, void**, void**) = nullptr;
    CUresult (*funcGetAttribute)(int*, CUfunction_attribute, CUfunction) = nullptr;
    CUresult (*getErrorName)(CUresult, const char**) = nullptr;
};
const Driver& driver();

inline void cuCheck(CUresult r, const char* what)
{
    if (r != CUDA_SUCCESS) {
        const char* name = "?";
        if (driver().getErrorName != nullptr)
            driver().getErrorName(r, &name);
        fail(EAGLE_BACKEND_ERROR, std::string(what) + ": " + name + " (" + std::to_string(int(r)) + ")");
    }
}

/** The thread's message of the last failed seam call. */
std::string& lastError();

/** Run ``body``; map what it throws to a status and leave the message in
 *  lastError(). A failure also clears the CUDA runtime's sticky-free last error
 *  so the next launch check names only its own launch. */
template <class Body>
eagle_backend_status guarded(Body&& body) noexcept
{
    try {
        body();
        lastError().clear();
        return EAGLE_BACKEND_OK;
    } catch (const Failure& f) {
        lastError() = f.what();
        (void)cudaGetLastError();
        return f.status;
    } catch (const std::bad_alloc&) {
        lastError() = "eagle_b200: host allocation failed";
        return EAGLE_BACKEND_ERROR;
    } catch (const std::exception& e) {
        lastError() = e.what();
        (void)cudaGetLastError();
        return EAGLE_BACKEND_ERROR;
    } catch (...) {
        lastError() = "eagle_b200: unknown exception";
        return EAGLE_BACKEND_ERROR;
    }
}

/** Copy ``min(in->struct_size, sizeof(D))`` bytes of an input desc; the rest
 *  stays zero. Unknown flag bits are refused. */
template <class D>
D readDesc(const D* in, uint32_t knownFlags, const char* who)
{
    if (in == nullptr)
        invalid(std::string(who) + ": null desc");
    if (in->struct_size < 8)
        invalid(std::string(who) + ": struct_size too small");
    D d;
    std::memset(&d, 0, sizeof d);
    std::memcpy(&d, in, in->struct_size < sizeof(D) ? in->struct_size : sizeof(D));
    if ((d.flags & ~knownFlags) != 0)
        unsupported(std::string(who) + ": unknown flag bits " + std::to_string(d.flags & ~knownFlags));
    return d;
}

/** A raw seam stream value as a runtime stream: 0 is the legacy default stream. */
inline cudaStream_t seamStream(uint64_t s)
{
    return s == 0 ? cudaStreamLegacy : reinterpret_cast<cudaStream_t>(s);
}

/** The device a desc names: ``device >= 0`` as given; -1 is the device owning
 *  ``ptr`` (the first non-zero address), else the current device. */
int resolveDevice(int32_t device, uint64_t ptr);

/** Make ``device`` current for a scope, restoring the previous one. */
struct DeviceScope {
    int prev = -1;
    explicit DeviceScope(int device)
    {
        cudaCheck(cudaGetDevice(&prev), "cudaGetDevice");
        if (device != prev)
            cudaCheck(cudaSetDevice(device), "cudaSetDevice");
    }
    ~DeviceScope()
    {
        if (prev >= 0)
            (void)cudaSetDevice(prev);
    }
};

/** Report a launch failure of the kernel just enqueued. */
inline void launchCheck(const char* who)
{
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        fail(EAGLE_BACKEND_ERROR, std::string(who) + ": launch failed: " + cudaGetErrorName(e) + " ("
            + cudaGetErrorString(e) + ")");
}

/** UNAVAILABLE unless a CUDA device is visible. */
void requireDevice();

/** SMs of the current device (cached per device). */
int smCount();

// ----------------------------------------------------------- device primitives

constexpr unsigned kFull = 0xffffffffu;

/** Inclusive warp scan (sum) of ``v``. */
template <class T>
__device__ __forceinline__ T warpInclusiveSum(T v)
{
    const unsigned lane = threadIdx.x & 31u;
#pragma unroll
    for (unsigned off = 1; off < 32; off <<= 1) {
        const T o = __shfl_up_sync(kFull, v, off);
        if (lane >= off)
            v += o;
    }
    return v;
}

template <class T>
__device__ __forceinline__ T warpSum(T v)
{
#pragma unroll
    for (unsigned off = 16; off > 0; off >>= 1)
        v += __shfl_xor_sync(kFull, v, off);
    return v;
}

template <class T>
__device__ __forceinline__ T warpMax(T v)
{
#pragma unroll
    for (unsigned off = 16; off > 0; off >>= 1) {
        const T o = __shfl_xor_sync(kFull, v, off);
        v = o > v ? o : v;
    }
    return v;
}

/** Block-wide exclusive scan of one value per thread (blockDim.x a multiple of
 *  32, at most 1024); returns the thread's exclusive prefix, ``total`` the sum.
 *  ``scratch`` holds 33 values of shared memory. */
template <class T>
__device__ __forceinline__ T blockExclusiveSum(T v, T& total, T* scratch)
{
    const unsigned lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const unsigned warps = blockDim.x >> 5;
    const T inc = warpInclusiveSum(v);
    if (lane == 31)
        scratch[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        T w = lane < warps ? scratch[lane] : T(0);
        const T winc = warpInclusiveSum(w);
        if (lane < warps)
            scratch[lane] = winc - w;  // exclusive prefix of each warp
        if (lane == warps - 1)
            scratch[32] = winc;  // the block total
    }
    __syncthreads();
    total = scratch[32];
    const T r = scratch[warp] + inc - v;
    __syncthreads();  // scratch may be reused by the caller
    return r;
}

// ------------------------------------------------------------ decoupled look-back
//
// Each tile of a single-pass scan publishes one 64-bit status word: first its own
// aggregate (flag 1), then the inclusive prefix through it (flag 2). Two codecs:
//
//   EpochCodec  [epoch:30 | flag:2 | payload:32] -- a loop's pass number tags the
//               word, so a word written in an earlier pass reads as "not yet
//               written" and the buffer never needs clearing between passes
//               (epoch 0 is never used: a zeroed buffer is unwritten for all).
//   PlainCodec  [flag:2 | payload:62] -- for a buffer zeroed before the launch; the
//               payload may pack several counters whose sums cannot carry into
//               one another.

constexpr uint32_t kLbAggregate = 1, kLbPrefix = 2;

struct EpochCodec {
    static __device__ __forceinline__ uint64_t make(uint32_t epoch, uint32_t flag, uint64_t payload)
    {
        return (uint64_t(epoch & 0x3fffffffu) << 34) | (uint64_t(flag) << 32) | (payload & 0xffffffffull);
    }
    static __device__ __forceinline__ bool ready(uint64_t w, uint32_t epoch)
    {
        return uint32_t(w >> 34) == (epoch & 0x3fffffffu) && ((w >> 32) & 3u) != 0;
    }
    static __device__ __forceinline__ uint32_t flag(uint64_t w) { return uint32_t((w >> 32) & 3u); }
    static __device__ __forceinline__ uint64_t payload(uint64_t w) { return w & 0xffffffffull; }
};

struct PlainCodec {
    static __device__ __forceinline__ uint64_t make(uint32_t, uint32_t flag, uint64_t payload)
    {
        return (uint64_t(flag) << 62) | (payload & ((1ull << 62) - 1));
    }
    static __device__ __forceinline__ bool ready(uint64_t w, uint32_t) { return (w >> 62) != 0; }
    static __device__ __forceinline__ uint32_t flag(uint64_t w) { return uint32_t(w >> 62); }
    static __device__ __forceinline__ uint64_t payload(uint64_t w) { return w & ((1ull << 62) - 1); }
};

template <class Codec>
__device__ __forceinline__ void lbPublish(uint64_t* status, uint32_t tile, uint32_t epoch, uint32_t flag,
    uint64_t payload)
{
    // flag and payload travel in one 64-bit word: a single atomic store publishes both
    atomicExch(reinterpret_cast<unsigned long long*>(status + tile),
        static_cast<unsigned long long>(Codec::make(epoch, flag, payload)));
}

__device__ __forceinline__ uint64_t lbLoad(const uint64_t* status, int64_t i)
{
    uint64_t w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(status + i) : "memory");
    return w;
}

/** The look-back spin bound: past it the wait gives up, sets bit 0 of ``*err``
 *  and takes the missing predecessors as empty (the result is then wrong and
 *  the host reports the error word; the GPU never hangs on it). */
constexpr uint32_t kLbSpinLimit = 1u << 22;

/** Called by one full warp of the CTA owning ``tile`` (> 0) after it published
 *  its aggregate. Returns the exclusive prefix payload of the tile in every lane.
 *  Each lane polls a predecessor at most ``spinLimit`` times.
 *  Lane l inspects tile ``end - 1 - l``: the nearest predecessor holding an
 *  inclusive prefix ends the walk. */
template <class Codec>
__device__ __forceinline__ uint64_t lbExclusivePrefix(const uint64_t* status, uint32_t tile, uint32_t epoch,
    uint32_t* err, uint32_t spinLimit = kLbSpinLimit)
{
    const unsigned lane = threadIdx.x & 31u;
    uint64_t exclusive = 0;
    int64_t end = int64_t(tile);
    while (end > 0) {
        const int64_t i = end - 1 - int64_t(lane);
        uint64_t w = 0;
        uint32_t flag = kLbPrefix;  // before tile 0: the empty prefix
        if (i >= 0) {
            uint32_t spins = 0;
            for (;;) {
                w = lbLoad(status, i);
                if (Codec::ready(w, epoch)) {
                    flag = Codec::flag(w);
                    break;
                }
                if (++spins > spinLimit) {
                    atomicOr(err, 1u);
                    w = 0;
                    flag = kLbPrefix;
                    break;
                }
                if (spins > 32)
                    __nanosleep(64);
            }
        }
        const uint64_t value = (i >= 0 && Codec::ready(w, epoch)) ? Codec::payload(w) : 0ull;
        const unsigned prefixLanes = __ballot_sync(kFull, flag == kLbPrefix);
        if (prefixLanes != 0) {
            const unsigned first = __ffs(prefixLanes) - 1;  // nearest predecessor with a prefix
            exclusive += warpSum(lane <= first ? value : 0ull);
            break;
        }
        exclusive += warpSum(value);
        end -= 32;
    }
    return exclusive;
}

// ------------------------------------------------------------------ bulk copies
//
// One thread asks the copy engine for a contiguous global -> shared copy that
// completes on an mbarrier (cp.async.bulk, no tensor map, never multicast: the
// source is always this GPU's own memory). Every wait on the barrier is bounded.

__device__ __forceinline__ uint32_t sharedAddr(const void* p) { return uint32_t(__cvta_generic_to_shared(p)); }

/** One-thread init of a CTA-local mbarrier expecting ``arrivals`` arrivals, made
 *  visible to the copy engine; the CTA must pass a barrier before using it. */
__device__ __forceinline__ void mbarInit(uint64_t* bar, uint32_t arrivals)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n"
                 "fence.mbarrier_init.release.cluster;\n" ::"r"(sharedAddr(bar)),
        "r"(arrivals)
        : "memory");
}

/** Arrive on ``bar`` announcing ``bytes`` still to land, then copy ``bytes`` (a
 *  multiple of 16, both addresses 16-byte aligned) from global ``src`` to this
 *  CTA's shared ``dst``; the copy engine counts them off the barrier's phase. */
__device__ __forceinline__ void bulkLoad(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n"
                 "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%2], [%3], %1, [%0];\n" ::"r"(
                     sharedAddr(bar)),
        "r"(bytes), "r"(sharedAddr(dst)), "l"(src)
        : "memory");
}

/** Wait for phase ``parity`` of ``bar`` to complete, at most ``limit`` polls (each
 *  may suspend the thread for a while in hardware). False if it gave up. */
__device__ __forceinline__ bool mbarWait(uint64_t* bar, uint32_t parity, uint32_t limit)
{
    for (uint32_t i = 0; i < limit; ++i) {
        uint32_t done = 0;
        asm volatile("{\n .reg .pred p;\n"
                     " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                     " selp.u32 %0, 1, 0, p;\n}\n"
                     : "=r"(done)
                     : "r"(sharedAddr(bar)), "r"(parity)
                     : "memory");
        if (done != 0)
            return true;
    }
    return false;
}

// ------------------------------------------------------------------ mask bytes

/** Bits of the non-zero bytes among the 16 in ``w`` (bit j: byte j). */
__device__ __forceinline__ uint32_t nonZero16(uint4 w)
{
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
    uint32_t set = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        // 0xff per non-zero byte; the multiply moves the top bits of bytes 0..3 (bits 7,
        // 15, 23, 31) to bits 28..31 -- every partial product lands on its own bit
        // position, so nothing carries into them
        const uint32_t nz = __vcmpne4(words[q], 0u) & 0x80808080u;
        set |= ((nz * 0x00204081u) >> 28) << (4 * q);
    }
    return set;
}

/** The 16 mask bytes of samples [i0, i0 + 16) as one 16-byte word (bytes past n read
 *  as 0): one vector load when the mask is 16-byte aligned and the run whole. Issue
 *  all of a thread's loads before the first keepOf16, so they are in flight together. */
template <bool Aligned>
__device__ __forceinline__ uint4 maskBytes16(const uint8_t* __restrict__ mask, int64_t i0, int64_t n)
{
    if (Aligned && i0 + 16 <= n)
        return __ldg(reinterpret_cast<const uint4*>(mask + i0));
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int j = 0; j < 16; ++j)
        if (i0 + j < n)
            w[j >> 2] |= uint32_t(mask[i0 + j]) << (8 * (j & 3));
    return make_uint4(w[0], w[1], w[2], w[3]);
}

/** Keep bits of 16 mask bytes already loaded by maskBytes16 (bit j: sample i0 + j kept). */
template <bool Drop>
__device__ __forceinline__ uint32_t keepOf16(uint4 raw, int64_t i0, int64_t n)
{
    const uint32_t set = nonZero16(raw);
    const uint32_t valid = i0 >= n ? 0u : (i0 + 16 <= n ? 0xffffu : ((1u << uint32_t(n - i0)) - 1u));
    return (Drop ? ~set : set) & valid;
}

// ------------------------------------------------------------- hawk handle ABI

/** The 32-byte per-sample plane handle of the hawk kernel ABI (a rank-1 array
 *  view: data, extent, stride, DLPack device type and id). */
struct ScalarHandle {
    void* data;
    uint64_t samples;
    uint64_t stride;
    int32_t deviceType;
    int32_t deviceId;
};
static_assert(sizeof(ScalarHandle) == 32, "ScalarHandle is 32 bytes");

}  // namespace eb
