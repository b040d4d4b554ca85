// Active-set compaction and the until-done loop's cell ops, on B200.
//
// compact_device keeps eagle's contract (eagle/filtering/Compact.h:23-47,
// python/src/seam/eagle_backend.h:666-701): index_map[0, count) = the kept sample
// indices, ascending; count; optionally the reorder trigger (live32, fire) of
// Compact.h:113-118. Eagle runs predicate -> multi-level int64 scan -> scatter
// (about 2 log256(n) + 2 launches over 8-byte planes). Here it is ONE kernel
// after a memset of its scratch: each CTA takes the next 32768-sample tile off a
// counter (so every tile it waits on is already owned by a running CTA), turns
// 8 x 16 mask bytes per thread into keep bit-sets, scans the counts across the CTA,
// finds the tile's global offset by a decoupled look-back over the earlier
// tiles' status words, stages the kept indices in shared memory and writes them
// with coalesced stores. The trigger's live32 rides in the same status words, so
// the last tile alone knows count and live32 and writes count, live32 and fire.
#include "common.cuh"

#include <mutex>

namespace eb {
namespace {

constexpr int kThreads = 256;
constexpr int kRows = 8;                               // a tile is eight rows of 4096 samples
constexpr int64_t kRow = int64_t(kThreads) * 16;       // 16 mask bytes per thread per row
constexpr int64_t kTile = kRow * kRows;                // 32768 samples per CTA
constexpr uint32_t kStage = uint32_t(kTile / 4);       // kept indices staged in the tile's mask bytes
constexpr int kCtasPerSm = 6;                          // 33 KB of shared memory and <= 40 registers each

struct CompactArgs {
    const uint8_t* mask;
    int64_t n;
    int32_t* map;
    uint32_t* count;
    uint64_t* status;      // one word per tile, zero on entry
    uint32_t* tileNext;    // zero on entry
    uint32_t* err;         // zero on entry
    uint32_t* live32;      // trigger outputs (Trigger only)
    const uint32_t* span;
    uint32_t* fire;
    float theta;
    uint32_t tiles;
    const void* values;  // Gather: the samples' values (elemBytes each)
    void* outValues;     // Gather: the kept samples' values, in sample order
    uint32_t elemBytes;  // Gather: 4 or 8
    uint32_t spinLimit;  // polls of one predecessor's status word before the look-back gives up
};

/** One 32768-sample tile per CTA, as eight rows of 4096: thread t holds the 16
 *  mask bytes at t * 16 of every row (eight coalesced 16-byte loads, all in flight
 *  before the first is used). Two CTA scans of the rows' counts, packed four at a
 *  time as 16-bit lanes of a 64-bit word, give each thread's place in every row,
 *  one decoupled look-back the tile's offset; each row's kept indices then go
 *  through shared memory to coalesced stores (the Gather values are read through
 *  the staged indices at the store). Eight rows per look-back keep eight times the
 *  bytes in flight per round trip, which is what a sparse mask (few kept, so
 *  little else to do) is bound by; a row at most a quarter kept is staged by its
 *  set bits alone, a denser one by all 16 bits predicated. */
template <bool Drop, bool Trigger, bool Aligned, bool Gather = false>
__global__ __launch_bounds__(kThreads, kCtasPerSm) void compactKernel(CompactArgs a)
{
    __shared__ uint32_t sTile;
    __shared__ uint64_t scan64[33];
    __shared__ uint32_t scan[33];
    __shared__ uint64_t sPrefix;
    __shared__ uint64_t sBar;  // completes when the tile's mask bytes have landed
    // the tile's mask bytes; once every thread holds its keep bits, the staging area
    __shared__ __align__(128) uint8_t sMask[kTile];
    int32_t* stage = reinterpret_cast<int32_t*>(sMask);
    const int t = int(threadIdx.x);
    if (t == 0) {
        sTile = atomicAdd(a.tileNext, 1u);
        mbarInit(&sBar, 1);
    }
    __syncthreads();
    const uint32_t tile = sTile;
    const int64_t tile0 = int64_t(tile) * kTile;
    if (Aligned && tile0 + kTile <= a.n) {
        // the whole tile in one bulk copy by the copy engine, issued by one thread
        if (t == 0)
            bulkLoad(sMask, a.mask + tile0, uint32_t(kTile), &sBar);
        if (!mbarWait(&sBar, 0, kLbSpinLimit)) {
            atomicOr(a.err, 2u);  // reported as a failed compaction; wait out the copy before going on
            (void)mbarWait(&sBar, 0, kLbSpinLimit);
        }
    } else {  // the last tile, or a mask not 16-byte aligned
#pragma unroll 1
        for (int q = 0; q < kRows; ++q)
            *reinterpret_cast<uint4*>(sMask + q * kRow + t * 16) =
                maskBytes16<Aligned>(a.mask, tile0 + int64_t(q) * kRow + int64_t(t) * 16, a.n);
    }
    uint32_t bits[kRows];
    uint64_t packed[kRows / 4] = {};  // row q's count in bits [16 (q % 4), + 16) of word q / 4
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
        const uint4 raw = *reinterpret_cast<const uint4*>(sMask + q * kRow + t * 16);
        bits[q] = keepOf16<Drop>(raw, tile0 + int64_t(q) * kRow + int64_t(t) * 16, a.n);
        packed[q / 4] |= uint64_t(__popc(bits[q])) << (16 * (q % 4));
    }
    // the thread's place in each row and each row's count, four rows to a 64-bit word
    uint64_t exclRows[kRows / 4], rowTotals[kRows / 4];
    uint32_t total = 0;
#pragma unroll
    for (int w = 0; w < kRows / 4; ++w) {
        exclRows[w] = blockExclusiveSum(packed[w], rowTotals[w], scan64);
#pragma unroll
        for (int q = 0; q < 4; ++q)
            total += uint32_t(rowTotals[w] >> (16 * q)) & 0xffffu;
    }
    uint32_t groups = 0;
    if constexpr (Trigger) {
        // a 32-sample group is two neighbouring threads of a row (rows start on a multiple of 32)
        uint32_t mine = 0;
#pragma unroll
        for (int q = 0; q < kRows; ++q) {
            const uint32_t pair = bits[q] | __shfl_xor_sync(kFull, bits[q], 1);
            mine += ((t & 1) == 0 && pair != 0) ? 1u : 0u;
        }
        blockExclusiveSum(mine, groups, scan);
    }
    const uint64_t payload = (uint64_t(groups) << 32) | uint64_t(total);
    if (t < 32) {
        uint64_t prefix = 0;
        if (tile == 0) {
            if (t == 0)
                lbPublish<PlainCodec>(a.status, tile, 0, kLbPrefix, payload);
        } else {
            if (t == 0)
                lbPublish<PlainCodec>(a.status, tile, 0, kLbAggregate, payload);
            prefix = lbExclusivePrefix<PlainCodec>(a.status, tile, 0, a.err, a.spinLimit);
            if (t == 0)
                lbPublish<PlainCodec>(a.status, tile, 0, kLbPrefix, prefix + payload);
        }
        if (t == 0)
            sPrefix = prefix;
    }
    __syncthreads();
    const uint64_t prefix = sPrefix;
    // the rows' kept indices gather in shared memory in output order; they are written
    // out whenever the next row would not fit (a sparse tile: once; a dense one: per row)
    uint32_t flushAt = uint32_t(prefix);  // the output index of stage[0]
    uint32_t fill = 0;                    // staged so far (uniform across the CTA)
    auto flush = [&]() {
        __syncthreads();
        for (uint32_t r = uint32_t(t); r < fill; r += kThreads) {
            const int32_t idx = stage[r];
            const size_t out = size_t(flushAt) + r;
            if (a.map != nullptr)
                a.map[out] = idx;
            if constexpr (Gather) {
                if (a.elemBytes == 8)
                    static_cast<uint64_t*>(a.outValues)[out] = static_cast<const uint64_t*>(a.values)[idx];
                else
                    static_cast<uint32_t*>(a.outValues)[out] = static_cast<const uint32_t*>(a.values)[idx];
            }
        }
        __syncthreads();
        flushAt += fill;
        fill = 0;
    };
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
        const uint32_t rowTotal = uint32_t(rowTotals[q / 4] >> (16 * (q % 4))) & 0xffffu;
        if (fill + rowTotal > kStage)
            flush();
        uint32_t k = fill + (uint32_t(exclRows[q / 4] >> (16 * (q % 4))) & 0xffffu);
        const int32_t i0 = int32_t(tile0 + int64_t(q) * kRow + int64_t(t) * 16);
        if (rowTotal > uint32_t(kRow / 4)) {  // a dense row (the choice is the CTA's): every bit, predicated
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if ((bits[q] >> j) & 1u)
                    stage[k++] = i0 + j;
        } else {
            for (uint32_t x = bits[q]; x != 0; x &= x - 1u)  // the set bits only
                stage[k++] = i0 + (__ffs(int(x)) - 1);
        }
        fill += rowTotal;
    }
    if (fill != 0)
        flush();
    if (tile == a.tiles - 1 && t == 0) {
        const uint32_t c = uint32_t(prefix) + total;
        const bool broken = *a.err != 0u;
        *a.count = broken ? 0xffffffffu : c;  // a count above n reports a failed compaction
        if constexpr (Trigger) {
            const uint32_t live32 = uint32_t(prefix >> 32) + groups;
            *a.live32 = live32;
            const uint32_t span = *a.span;
            const double limit = double(a.theta) * 32.0 * double(live32);
            *a.fire = (double(c) < limit && c < span && span >= 4096u) ? 1u : 0u;
        }
    }
}

__global__ void compactEmptyKernel(uint32_t* count, uint32_t* live32, uint32_t* fire)
{
    *count = 0u;
    if (live32 != nullptr) {
        *live32 = 0u;
        *fire = 0u;
    }
}

/** One CTA per tile (``grid`` fewer only when tiles are withheld on purpose). */
template <bool Drop, bool Trigger, bool Gather = false>
void launchCompact(const CompactArgs& a, bool aligned, cudaStream_t s, uint32_t grid = 0)
{
    const uint32_t g = grid != 0 ? grid : a.tiles;
    if (aligned)
        compactKernel<Drop, Trigger, true, Gather><<<g, kThreads, 0, s>>>(a);
    else
        compactKernel<Drop, Trigger, false, Gather><<<g, kThreads, 0, s>>>(a);
}

__global__ void setWordKernel(uint32_t* w, uint32_t value) { *w = value; }

constexpr size_t compactScratchBytes(int64_t n)
{
    const int64_t tiles = n > 0 ? (n + kTile - 1) / kTile : 1;
    const size_t bytes = size_t(tiles) * sizeof(uint64_t) + 2 * sizeof(uint32_t);
    return (bytes + 255) & ~size_t(255);
}

// ------------------------------------------------------------------- cell ops

__global__ void bumpKernel(uint32_t* cell) { cell[0] += 1u; }

/** ``cell += number of non-zero bytes``: 16 bytes per thread per step, one atomic per CTA. */
template <bool Aligned>
__global__ __launch_bounds__(256) void maskCountKernel(const uint8_t* __restrict__ mask, int64_t n, uint32_t* cell)
{
    __shared__ uint32_t part[8];
    uint32_t c = 0;
    const int64_t stride = int64_t(gridDim.x) * blockDim.x * 16;
    for (int64_t i = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * 16; i < n; i += stride) {
        if (Aligned && i + 16 <= n) {
            const uint4 w = __ldg(reinterpret_cast<const uint4*>(mask + i));
            c += __popc(__vcmpne4(w.x, 0u)) / 8 + __popc(__vcmpne4(w.y, 0u)) / 8 + __popc(__vcmpne4(w.z, 0u)) / 8
                + __popc(__vcmpne4(w.w, 0u)) / 8;
        } else {
            for (int j = 0; j < 16 && i + j < n; ++j)
                c += mask[i + j] != 0 ? 1u : 0u;
        }
    }
    c = warpSum(c);
    if ((threadIdx.x & 31) == 0)
        part[threadIdx.x >> 5] = c;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t s = 0;
        for (int w = 0; w < int(blockDim.x >> 5); ++w)
            s += part[w];
        if (s != 0)
            atomicAdd(cell, s);
    }
}

__global__ void identityKernel(int32_t* a, int64_t n)
{
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        a[i] = int32_t(i);
}

__global__ void countFiredKernel(const uint32_t* fire, uint32_t* reorders) { reorders[0] += fire[0] != 0u ? 1u : 0u; }

__global__ void groupAndKernel(const uint8_t* m, uint8_t* d, int64_t lanes, int group, int64_t groups)
{
    for (int64_t g = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; g < groups;
         g += int64_t(gridDim.x) * blockDim.x) {
        uint8_t all = 1;
        const int64_t s = g * group;
        for (int j = 0; j < group && s + j < lanes; ++j)
            all &= uint8_t(m[s + j] != 0);
        d[g] = all;
    }
}

__global__ void scaleCountKernel(const uint32_t* c, uint32_t* o, int group) { o[0] = c[0] * uint32_t(group); }

/** One step of the until-done band policy: eagle's POLICY cell op
 *  (python/src/plugin/eagle_cuda.cu:1990-2025; bandK of eagle/policy/Launch.h:184-190),
 *  the same expressions in the same order, so a host twin rounds identically. */
__global__ void policyKernel(const uint32_t* finished, const uint32_t* total, int64_t* cells, int64_t* word,
    uint32_t* go, int64_t* hist, int64_t kmin, int64_t kmax, int iK, int iFin, int iDone, int iCap, int iR,
    int iMapped, int scale)
{
    const int64_t fin = finished[0], all = total[0];
    const int64_t live = all - fin, newly = fin - cells[iFin];
    const int64_t done = cells[iDone] + word[0];
    cells[iMapped] += all - cells[iFin];
    cells[iFin] = fin;
    cells[iDone] = done;
    const int64_t k = cells[iK];
    const double rate = double(cells[iR]) / double(scale);
    int64_t kNext = k;
    if (newly <= 0) {
        kNext = kmax;
    } else {
        const double e2 = 2.0 * rate * double(live) * double(k) / double(newly);
        int64_t p = 1;
        while (p < (INT64_C(1) << 30) && e2 >= 2.0 * double(p) * double(p))
            p *= 2;
        kNext = p < kmin ? kmin : (p > kmax ? kmax : p);
    }
    cells[iK] = kNext;
    const int64_t left = cells[iCap] - done;
    const uint32_t g = (fin != all) && (left > 0);
    go[0] = g;
    if (g) {
        const int64_t w = kNext < left ? kNext : left;
        word[0] = w;
        hist[w] += 1;
    }
}

__global__ void resetKernel(int32_t* perm, int32_t* inv, int32_t* map, uint32_t* count, uint32_t* span, int64_t n)
{
    const int64_t i0 = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    for (int64_t i = i0; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        perm[i] = int32_t(i);
        inv[i] = int32_t(i);
        if (map != nullptr)
            map[i] = int32_t(i);
    }
    if (i0 == 0) {
        *count = uint32_t(n);
        *span = uint32_t(n);
    }
}

unsigned gridFor(int64_t n, int64_t perThread = 1)
{
    const int64_t threads = (n + perThread - 1) / perThread;
    const int64_t blocks = (threads + 255) / 256;
    const int64_t cap = int64_t(smCount()) * 16;
    return unsigned(std::max<int64_t>(1, std::min(blocks, cap)));
}

void need(const eagle_backend_cell_op_desc& d, int pointers, const char* who)
{
    for (int k = 0; k < pointers; ++k)
        if (d.p[k] == 0)
            invalid(std::string(who) + ": p" + std::to_string(k) + " must be a device address");
}

uint64_t firstPointer(const eagle_backend_cell_op_desc& d)
{
    for (uint64_t p : d.p)
        if (p != 0)
            return p;
    return 0;
}

}  // namespace

/** Enqueue ``cell[0] = number of set bytes of mask[0, n)`` (memset + count) on ``s``. */
void enqueueMaskCount(const uint8_t* mask, int64_t n, uint32_t* cell, cudaStream_t s, bool zeroFirst)
{
    if (zeroFirst)
        cudaCheck(cudaMemsetAsync(cell, 0, sizeof(uint32_t), s), "cudaMemsetAsync");
    if (n == 0)
        return;
    const bool aligned = (reinterpret_cast<uintptr_t>(mask) & 15u) == 0;
    if (aligned)
        maskCountKernel<true><<<gridFor(n, 16), 256, 0, s>>>(mask, n, cell);
    else
        maskCountKernel<false><<<gridFor(n, 16), 256, 0, s>>>(mask, n, cell);
    launchCheck("mask count");
}

}  // namespace eb

using namespace eb;

#define EB_API extern "C" __attribute__((visibility("default")))

namespace eb {
namespace {

/** compact_device's whole enqueue (after the query) over the scratch at ``scratch``
 *  (compactScratchBytes(n) bytes, zeroed here on the stream): shared by compact_device,
 *  the class trigger entry, the allocation-free entry and the wait check. The wait
 *  check passes ``withholdFirst``: the tile counter starts at 1, so no CTA takes
 *  tile 0 and every look-back that reaches it polls ``spinLimit`` times and gives up. */
void enqueueCompactOn(const eagle_backend_compact_desc& d, char* scratch, const char* who,
    uint32_t spinLimit = kLbSpinLimit, bool withholdFirst = false)
{
    if (d.count == 0 || (d.n > 0 && (d.mask == 0 || d.index_map == 0)))
        invalid(std::string(who) + ": mask, index_map and count must be device addresses");
    const bool trigger = d.live32 != 0;
    if (trigger) {
        if (d.span == 0 || d.fire == 0)
            invalid(std::string(who) + ": a trigger needs live32, span and fire");
        if (d.reserved2 != 0)
            invalid(std::string(who) + ": reserved2 must be zero");
        if (!(d.theta > 0.0f && d.theta < 1.0f))
            invalid(std::string(who) + ": the trigger's theta must lie in (0, 1)");
    }
    const cudaStream_t s = seamStream(d.stream);
    if (d.n == 0) {
        compactEmptyKernel<<<1, 1, 0, s>>>(reinterpret_cast<uint32_t*>(d.count),
            trigger ? reinterpret_cast<uint32_t*>(d.live32) : nullptr,
            trigger ? reinterpret_cast<uint32_t*>(d.fire) : nullptr);
        launchCheck(who);
        return;
    }
    CompactArgs a{};
    a.mask = reinterpret_cast<const uint8_t*>(d.mask);
    a.n = d.n;
    a.map = reinterpret_cast<int32_t*>(d.index_map);
    a.count = reinterpret_cast<uint32_t*>(d.count);
    a.tiles = uint32_t((d.n + kTile - 1) / kTile);
    a.status = reinterpret_cast<uint64_t*>(scratch);
    a.tileNext = reinterpret_cast<uint32_t*>(scratch + size_t(a.tiles) * sizeof(uint64_t));
    a.err = a.tileNext + 1;
    a.live32 = reinterpret_cast<uint32_t*>(d.live32);
    a.span = reinterpret_cast<const uint32_t*>(d.span);
    a.fire = reinterpret_cast<uint32_t*>(d.fire);
    a.theta = d.theta;
    a.spinLimit = spinLimit;
    // the status words, the tile counter and the error word start at zero on every call
    cudaCheck(cudaMemsetAsync(scratch, 0, compactScratchBytes(d.n), s), "cudaMemsetAsync");
    uint32_t grid = a.tiles;
    if (withholdFirst) {
        setWordKernel<<<1, 1, 0, s>>>(a.tileNext, 1u);
        launchCheck(who);
        grid = a.tiles - 1;
    }
    const bool aligned = (d.mask & 15u) == 0;
    const bool drop = (d.flags & EAGLE_BACKEND_COMPACT_MASK_IS_DROP) != 0;
    if (drop)
        trigger ? launchCompact<true, true>(a, aligned, s, grid) : launchCompact<true, false>(a, aligned, s, grid);
    else
        trigger ? launchCompact<false, true>(a, aligned, s, grid) : launchCompact<false, false>(a, aligned, s, grid);
    launchCheck(who);
}

void enqueueCompactDevice(const eagle_backend_compact_desc& d, const char* who)
{
    enqueueCompactOn(d, reinterpret_cast<char*>(d.scratch), who);
}

/** Per 32-slot group of [0, n): does it hold two or more live classes
 *  (ReorderClasses.h classMixed32)? One atomic per CTA. */
__global__ __launch_bounds__(256) void mixed32Kernel(const uint8_t* __restrict__ mask, const uint8_t* __restrict__ cls,
    uint32_t* mixed32, bool drop, int64_t n)
{
    __shared__ uint32_t part[8];
    uint32_t mine = 0;
    for (int64_t i0 = int64_t(blockIdx.x) * blockDim.x; i0 < n; i0 += int64_t(gridDim.x) * blockDim.x) {
        const int64_t i = i0 + threadIdx.x;
        bool live = false;
        unsigned c = 0u;
        if (i < n) {
            const bool set = mask[i] != 0;
            live = drop ? !set : set;
            c = cls[i];
        }
        unsigned lo = live ? c : 255u, hi = live ? c : 0u;
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
            lo = min(lo, __shfl_xor_sync(kFull, lo, d));
            hi = max(hi, __shfl_xor_sync(kFull, hi, d));
        }
        if ((threadIdx.x & 31u) == 0u && lo < hi)
            ++mine;
    }
    if ((threadIdx.x & 31u) == 0u)
        part[threadIdx.x >> 5] = mine;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t t = 0;
        for (int w = 0; w < int(blockDim.x >> 5); ++w)
            t += part[w];
        if (t != 0)
            atomicAdd(mixed32, t);
    }
}

/** ReorderClasses.h classTriggerFires: a mixing, a class drift or the liveness trigger. */
__global__ void classFireKernel(const uint32_t* count, const uint32_t* live32, const uint32_t* span,
    const uint32_t* mixed32, const uint32_t* stale, const uint32_t* liveFire, float classTheta, uint32_t* classFire)
{
    const uint32_t mixed = *mixed32;
    const bool warpMix = mixed > 0u && double(mixed) >= double(classTheta) * double(*live32) && *span >= 4096u;
    const bool drift = double(stale != nullptr ? *stale : 0u) > 0.05 * double(*count);
    *classFire = (warpMix || drift || (liveFire != nullptr && *liveFire != 0u)) ? 1u : 0u;
}

__global__ void zeroWordKernel(uint32_t* w) { *w = 0u; }

}  // namespace
}  // namespace eb

EB_API eagle_backend_status eagle_backend_compact_device(struct eagle_backend_compact_desc* desc)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_compact_device";
        const auto d = readDesc(desc, EAGLE_BACKEND_COMPACT_MASK_IS_DROP, who);
        if (d.n < 0)
            invalid(std::string(who) + ": n must be >= 0");
        if (d.n > INT64_C(2147483647))
            unsupported(std::string(who) + ": the int32 index map addresses at most 2^31-1 samples, got n = "
                + std::to_string(d.n));
        if (d.scratch == 0) {
            constexpr size_t end = offsetof(eagle_backend_compact_desc, scratch_bytes) + sizeof(int64_t);
            if (desc->struct_size < end)
                invalid(std::string(who) + ": the scratch query needs a desc carrying scratch_bytes");
            desc->scratch_bytes = int64_t(compactScratchBytes(d.n));
            return;
        }
        DeviceScope scope(resolveDevice(d.device, d.mask != 0 ? d.mask : d.count));
        enqueueCompactDevice(d, who);
    });
}

EB_API eagle_backend_status eagle_backend_x_b200_compact_wait_check(struct eagle_backend_compact_desc* desc,
    uint32_t spin_limit)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_b200_compact_wait_check";
        const auto d = readDesc(desc, EAGLE_BACKEND_COMPACT_MASK_IS_DROP, who);
        if (d.n <= kTile || d.n > INT64_C(2147483647))
            invalid(std::string(who) + ": n must lie in (" + std::to_string(kTile) + ", 2^31 - 1]: the check "
                "withholds the first tile and needs a later one to wait for it");
        if (spin_limit == 0 || spin_limit > kLbSpinLimit)
            invalid(std::string(who) + ": spin_limit must lie in [1, 2^22]");
        if (d.scratch == 0)
            invalid(std::string(who) + ": needs compact_device's scratch (query it there)");
        DeviceScope scope(resolveDevice(d.device, d.mask != 0 ? d.mask : d.count));
        enqueueCompactOn(d, reinterpret_cast<char*>(d.scratch), who, spin_limit, true);
    });
}

EB_API eagle_backend_status eagle_backend_compact_classes_device(struct eagle_backend_compact_classes_desc* desc)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_compact_classes_device";
        if (desc == nullptr)
            invalid(std::string(who) + ": null desc");
        constexpr size_t need = offsetof(eagle_backend_compact_classes_desc, reserved3) + sizeof(uint64_t);
        if (desc->struct_size < need)
            invalid(std::string(who) + ": the desc must carry the class fields");
        const auto d = readDesc(desc, EAGLE_BACKEND_COMPACT_MASK_IS_DROP, who);
        if (d.n < 0)
            invalid(std::string(who) + ": n must be >= 0");
        if (d.n > INT64_C(2147483647))
            unsupported(std::string(who) + ": the int32 index map addresses at most 2^31-1 samples, got n = "
                + std::to_string(d.n));
        if (d.scratch == 0) {
            desc->scratch_bytes = int64_t(compactScratchBytes(d.n));
            return;
        }
        if (d.live32 == 0 || d.span == 0 || d.fire == 0 || d.mixed32 == 0 || d.class_fire == 0
            || (d.n > 0 && d.class_plane == 0))
            invalid(std::string(who) + ": live32, span, fire, class_plane, mixed32 and class_fire are required");
        if (d.reserved2 != 0 || d.reserved3 != 0)
            invalid(std::string(who) + ": reserved fields must be zero");
        if (d.classes < 2 || d.classes > EAGLE_BACKEND_MAX_CLASSES)
            invalid(std::string(who) + ": classes must lie in [2, 255]");
        if (!(d.class_theta > 0.0f && d.class_theta < 1.0f))
            invalid(std::string(who) + ": class_theta must lie in (0, 1)");
        DeviceScope scope(resolveDevice(d.device, d.mask != 0 ? d.mask : d.count));
        eagle_backend_compact_desc base{};
        std::memcpy(&base, &d, sizeof base);  // the first block repeats compact_desc field for field
        base.struct_size = sizeof base;
        enqueueCompactDevice(base, who);
        const cudaStream_t s = seamStream(d.stream);
        auto* mixed = reinterpret_cast<uint32_t*>(d.mixed32);
        zeroWordKernel<<<1, 1, 0, s>>>(mixed);
        if (d.n > 0) {
            const int64_t blocks = std::min<int64_t>((d.n + 255) / 256, int64_t(smCount()) * 16);
            mixed32Kernel<<<unsigned(blocks), 256, 0, s>>>(reinterpret_cast<const uint8_t*>(d.mask),
                reinterpret_cast<const uint8_t*>(d.class_plane), mixed,
                (d.flags & EAGLE_BACKEND_COMPACT_MASK_IS_DROP) != 0, d.n);
        }
        classFireKernel<<<1, 1, 0, s>>>(reinterpret_cast<const uint32_t*>(d.count),
            reinterpret_cast<const uint32_t*>(d.live32), reinterpret_cast<const uint32_t*>(d.span), mixed,
            reinterpret_cast<const uint32_t*>(d.stale_count), reinterpret_cast<const uint32_t*>(d.fire), d.class_theta,
            reinterpret_cast<uint32_t*>(d.class_fire));
        launchCheck(who);
    });
}

EB_API eagle_backend_status eagle_backend_reset_device(struct eagle_backend_reorder_desc* desc)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_reset_device";
        const auto d = readDesc(desc, EAGLE_BACKEND_COMPACT_MASK_IS_DROP, who);
        if (d.n < 0 || d.n > INT64_C(2147483647))
            invalid(std::string(who) + ": n must lie in [0, 2^31 - 1]");
        if (d.perm == 0 || d.inv == 0 || d.count == 0 || d.span == 0)
            invalid(std::string(who) + ": perm, inv, count and span must be device addresses");
        DeviceScope scope(resolveDevice(d.device, d.perm));
        const cudaStream_t s = seamStream(d.stream);
        resetKernel<<<gridFor(std::max<int64_t>(d.n, 1)), 256, 0, s>>>(reinterpret_cast<int32_t*>(d.perm),
            reinterpret_cast<int32_t*>(d.inv), reinterpret_cast<int32_t*>(d.index_map),
            reinterpret_cast<uint32_t*>(d.count), reinterpret_cast<uint32_t*>(d.span), d.n);
        launchCheck(who);
    });
}

EB_API eagle_backend_status eagle_backend_cell_op(const struct eagle_backend_cell_op_desc* desc)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_cell_op";
        const auto d = readDesc(desc, 0u, who);
        if (d.n < 0)
            invalid(std::string(who) + ": n must be >= 0");
        if (d.op > EAGLE_BACKEND_CELL_SCALE_COUNT)
            unsupported(std::string(who) + ": op " + std::to_string(d.op)
                + " is an array op this backend does not carry (it serves the until-done loop's ops 0-6)");
        DeviceScope scope(resolveDevice(d.device, firstPointer(d)));
        const cudaStream_t s = seamStream(d.stream);
        switch (d.op) {
        case EAGLE_BACKEND_CELL_BUMP:
            need(d, 1, who);
            bumpKernel<<<1, 1, 0, s>>>(reinterpret_cast<uint32_t*>(d.p[0]));
            break;
        case EAGLE_BACKEND_CELL_MASK_COUNT:
            if (d.n == 0)
                return;
            need(d, 2, who);
            enqueueMaskCount(reinterpret_cast<const uint8_t*>(d.p[0]), d.n, reinterpret_cast<uint32_t*>(d.p[1]), s,
                false);
            break;
        case EAGLE_BACKEND_CELL_POLICY:
            need(d, 6, who);
            if (d.i[8] == 0)
                invalid(std::string(who) + ": POLICY rate scale (i8) must be non-zero");
            policyKernel<<<1, 1, 0, s>>>(reinterpret_cast<const uint32_t*>(d.p[0]),
                reinterpret_cast<const uint32_t*>(d.p[1]), reinterpret_cast<int64_t*>(d.p[2]),
                reinterpret_cast<int64_t*>(d.p[3]), reinterpret_cast<uint32_t*>(d.p[4]),
                reinterpret_cast<int64_t*>(d.p[5]), d.i[0], d.i[1], int(d.i[2]), int(d.i[3]), int(d.i[4]), int(d.i[5]),
                int(d.i[6]), int(d.i[7]), int(d.i[8]));
            break;
        case EAGLE_BACKEND_CELL_IDENTITY:
            if (d.n == 0)
                return;
            need(d, 1, who);
            identityKernel<<<gridFor(d.n), 256, 0, s>>>(reinterpret_cast<int32_t*>(d.p[0]), d.n);
            break;
        case EAGLE_BACKEND_CELL_COUNT_FIRED:
            need(d, 2, who);
            countFiredKernel<<<1, 1, 0, s>>>(reinterpret_cast<const uint32_t*>(d.p[0]),
                reinterpret_cast<uint32_t*>(d.p[1]));
            break;
        case EAGLE_BACKEND_CELL_GROUP_AND:
            if (d.n == 0)
                return;
            need(d, 2, who);
            if (d.i[1] < 1)
                invalid(std::string(who) + ": GROUP_AND group must be >= 1");
            groupAndKernel<<<gridFor(d.n), 256, 0, s>>>(reinterpret_cast<const uint8_t*>(d.p[0]),
                reinterpret_cast<uint8_t*>(d.p[1]), d.i[0], int(d.i[1]), d.n);
            break;
        default:  // SCALE_COUNT
            need(d, 2, who);
            scaleCountKernel<<<1, 1, 0, s>>>(reinterpret_cast<const uint32_t*>(d.p[0]),
                reinterpret_cast<uint32_t*>(d.p[1]), int(d.i[0]));
        }
        launchCheck(who);
    });
}

EB_API eagle_backend_status eagle_backend_x_b200_compact_gather(struct eagle_backend_compact_desc* desc,
    uint64_t values, uint64_t out_values, uint32_t elem_bytes)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_b200_compact_gather";
        const auto d = readDesc(desc, EAGLE_BACKEND_COMPACT_MASK_IS_DROP, who);
        if (d.n < 0)
            invalid(std::string(who) + ": n must be >= 0");
        if (d.n > INT64_C(2147483647))
            unsupported(std::string(who) + ": at most 2^31-1 samples, got n = " + std::to_string(d.n));
        if (elem_bytes != 4 && elem_bytes != 8)
            invalid(std::string(who) + ": elem_bytes must be 4 or 8");
        if (d.scratch == 0) {
            constexpr size_t end = offsetof(eagle_backend_compact_desc, scratch_bytes) + sizeof(int64_t);
            if (desc->struct_size < end)
                invalid(std::string(who) + ": the scratch query needs a desc carrying scratch_bytes");
            desc->scratch_bytes = int64_t(compactScratchBytes(d.n));
            return;
        }
        if (d.count == 0 || (d.n > 0 && (d.mask == 0 || values == 0 || out_values == 0)))
            invalid(std::string(who) + ": mask, values, out_values and count must be device addresses");
        if (d.live32 != 0)
            unsupported(std::string(who) + ": the reorder trigger is not offered with the value gather");
        const int dev = resolveDevice(d.device, d.mask != 0 ? d.mask : d.count);
        DeviceScope scope(dev);
        const cudaStream_t s = seamStream(d.stream);
        if (d.n == 0) {
            compactEmptyKernel<<<1, 1, 0, s>>>(reinterpret_cast<uint32_t*>(d.count), nullptr, nullptr);
            launchCheck(who);
            return;
        }
        CompactArgs a{};
        a.mask = reinterpret_cast<const uint8_t*>(d.mask);
        a.n = d.n;
        a.map = reinterpret_cast<int32_t*>(d.index_map);  // may be 0: no map written
        a.count = reinterpret_cast<uint32_t*>(d.count);
        a.tiles = uint32_t((d.n + kTile - 1) / kTile);
        a.status = reinterpret_cast<uint64_t*>(d.scratch);
        a.tileNext = reinterpret_cast<uint32_t*>(d.scratch + size_t(a.tiles) * sizeof(uint64_t));
        a.err = a.tileNext + 1;
        a.values = reinterpret_cast<const void*>(values);
        a.outValues = reinterpret_cast<void*>(out_values);
        a.elemBytes = elem_bytes;
        a.spinLimit = kLbSpinLimit;
        cudaCheck(cudaMemsetAsync(reinterpret_cast<void*>(d.scratch), 0, compactScratchBytes(d.n), s),
            "cudaMemsetAsync");
        const bool aligned = (d.mask & 15u) == 0;
        if (d.flags & EAGLE_BACKEND_COMPACT_MASK_IS_DROP)
            launchCompact<true, false, true>(a, aligned, s);
        else
            launchCompact<false, false, true>(a, aligned, s);
        launchCheck(who);
    });
}

// ---------------------------------------------------------- allocation-free form
//
// Some callers of the compaction cannot allocate device memory: code that runs
// where an allocation would break its guarantees (inside a latency-critical
// loop, where cudaMalloc may synchronise the device), bindings from a host
// language that has no handle on the process's CUDA allocator, or a runtime
// whose device memory is fixed at start-up. For them the scratch of one
// compaction lives in a file-scope device array instead of a caller buffer.

namespace eb {
namespace {

/** The largest batch the allocation-free compaction serves (2^28 samples). */
constexpr int64_t kNoAllocMaxSamples = INT64_C(1) << 28;
/** One status word per 32768-sample (kTile) tile, then the tile counter and the error word,
 *  rounded up to 256 bytes: compactScratchBytes of the largest batch. */
constexpr size_t kNoAllocScratchBytes = size_t(kNoAllocMaxSamples / kTile) * sizeof(uint64_t) + 256;

/** The scratch every allocation-free call shares (each device that loads this
 *  library holds its own copy until the process exits). Host code must not use
 *  this name as an address: see noAllocScratch. */
static __device__ __align__(256) unsigned char g_noAllocScratch[kNoAllocScratchBytes];
static_assert(compactScratchBytes(kNoAllocMaxSamples) <= kNoAllocScratchBytes,
    "the built-in scratch must hold the largest batch's status words, tile counter and error word");

/** The device address of g_noAllocScratch on ``device`` (current when called),
 *  looked up on the first call for that device and kept for the life of the
 *  process: a cudaDeviceReset of that device afterwards would leave the kept
 *  address stale, so the entry does not support one. */
void* noAllocScratch(int device)
{
    static std::mutex mu;
    static void* addr[256] = {};
    if (device < 0 || device >= 256)
        invalid("eagle_backend_x_b200_compact_device_noalloc: device ordinal out of range");
    std::lock_guard<std::mutex> lock(mu);
    if (addr[device] == nullptr) {
        void* p = nullptr;
        cudaCheck(cudaGetSymbolAddress(&p, g_noAllocScratch), "cudaGetSymbolAddress");
        addr[device] = p;
    }
    return addr[device];
}

}  // namespace
}  // namespace eb

EB_API eagle_backend_status eagle_backend_x_b200_compact_device_noalloc(struct eagle_backend_compact_desc* desc)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_b200_compact_device_noalloc";
        const auto d = readDesc(desc, EAGLE_BACKEND_COMPACT_MASK_IS_DROP, who);
        if (d.n < 0)
            invalid(std::string(who) + ": n must be >= 0");
        if (d.n > kNoAllocMaxSamples)
            unsupported(std::string(who) + ": n = " + std::to_string(d.n) + " exceeds the "
                + std::to_string(kNoAllocMaxSamples) + " samples its built-in scratch serves; use "
                "eagle_backend_compact_device with caller scratch");
        if (d.scratch != 0)
            invalid(std::string(who) + ": takes no scratch (leave the field 0)");
        if (d.count == 0 || (d.n > 0 && (d.mask == 0 || d.index_map == 0)))
            invalid(std::string(who) + ": mask, index_map and count must be device addresses");
        const int dev = resolveDevice(d.device, d.mask != 0 ? d.mask : d.count);
        DeviceScope scope(dev);
        char* scratch = d.n > 0 ? static_cast<char*>(noAllocScratch(dev)) : nullptr;
        enqueueCompactOn(d, scratch, who);
    });
}
