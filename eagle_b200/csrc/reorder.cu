// The physical reorder of the active set (eagle/filtering/Reorder.h; seam
// python/src/seam/eagle_backend.h:705-740) and its undo (x_restore_device,
// :855-859).
//
// reorder_device moves every plane IN PLACE over [0, *span) so that the samples
// the mask keeps fill [0, *count) in ascending sample order and the dropped ones
// follow, also in ascending order (a stable partition: slot i goes to
// incl(i) - 1 when kept, to count + i - incl(i) when dropped, incl being the
// inclusive kept count, Reorder.h reorderDst); perm moves with the planes, inv is
// rebuilt for the moved slots, index_map becomes the identity over [0, *count)
// and *span = *count. With a fire word, every kernel returns at once while
// *fire == 0, and the last one clears it, so the whole reorder can sit in a
// captured loop and run only when the reorder trigger fired.
//
// Here: ONE scan kernel (16 mask bytes per thread, CTA scan, decoupled look-back
// over 4096-slot tiles) records each tile's keep bits and its exclusive kept
// prefix in the scratch, since the mask itself is one of the planes that move.
// Each plane then takes two kernels. The place kernel reads a tile of the plane
// itself, orders it in shared memory (kept run first, dropped run after), writes
// the kept run straight to its final slots and the dropped run to the stage, both
// with coalesced stores; a copy then puts the staged dropped run at [count, span).
// In place works for the kept run because a kept slot only moves down (slot i to
// incl(i) - 1 <= i): a tile's kept run lands in its own slots or in the tiles just
// before it, and it waits only until those tiles have been read (a per-tile flag;
// tiles are claimed in order, and a tile's read never waits, so the wait always
// ends; it is bounded all the same). The plane is read once and written once, the
// dropped run twice more: (4 - 2p) element bytes a slot at keep fraction p where a
// copy of the whole span to the stage and a place back cost 4. Nothing reads
// *span or *fire on the host, so every launch is capturable.
#include "common.cuh"

#include <cstdlib>
#include <mutex>
#include <set>
#include <string>
#include <utility>
#include <vector>

#define EB_API extern "C" __attribute__((visibility("default")))

namespace eb {
namespace {

constexpr int kThreads = 256;
constexpr int kPer = 16;
constexpr int64_t kTile = int64_t(kThreads) * kPer;

struct alignas(16) Elem16 {
    uint64_t lo, hi;
};

/** The scratch layout of a reorder of n samples over ``planes`` planes whose
 *  widest moved element is ``elem`` bytes: tile status words, three counters, each
 *  tile's read flag, one tile counter per moved plane (perm included; all zeroed per
 *  call), tile prefixes, tile keep bits (one uint16 per thread), then the stage. */
struct Layout {
    size_t status, words, done, claims, prefix, bits, stage, total;
};

Layout layoutFor(int64_t n, uint32_t elem, size_t planes = 0)
{
    const size_t tiles = size_t(n > 0 ? (n + kTile - 1) / kTile : 1);
    auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
    Layout l{};
    l.status = 0;
    l.words = up(tiles * sizeof(uint64_t));
    l.done = l.words + 256;
    l.claims = up(l.done + tiles * sizeof(uint32_t));
    l.prefix = up(l.claims + (planes + 1) * sizeof(uint32_t));
    l.bits = up(l.prefix + tiles * sizeof(uint32_t));
    l.stage = up(l.bits + tiles * kThreads * sizeof(uint16_t));
    l.total = up(l.stage + size_t(n > 0 ? n : 1) * (elem > 4 ? elem : 4));
    return l;
}

struct ScanArgs {
    const uint8_t* mask;
    int64_t n;
    const uint32_t* span;
    const uint32_t* fire;
    uint64_t* status;
    uint32_t* tileNext;
    uint32_t* err;
    uint32_t* cnt;
    uint32_t* prefix;
    uint16_t* bits;
    uint32_t tiles;
};

__device__ __forceinline__ int64_t spanOf(const uint32_t* span, int64_t n)
{
    const int64_t s = int64_t(*span);
    return s < n ? s : n;
}

template <bool Drop>
__global__ __launch_bounds__(kThreads) void reorderScanKernel(ScanArgs a)
{
    if (a.fire != nullptr && *a.fire == 0u)
        return;
    __shared__ uint32_t sTile;
    __shared__ uint32_t scan[33];
    const int t = int(threadIdx.x);
    if (t == 0)
        sTile = atomicAdd(a.tileNext, 1u);
    __syncthreads();
    const uint32_t tile = sTile;
    const int64_t sp = spanOf(a.span, a.n);
    const int64_t i0 = int64_t(tile) * kTile + int64_t(t) * kPer;
    uint32_t keep = 0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int64_t i = i0 + j;
        if (i < sp) {
            const bool set = a.mask[i] != 0;
            keep |= uint32_t(set != Drop) << j;
        }
    }
    a.bits[size_t(tile) * kThreads + size_t(t)] = uint16_t(keep);
    uint32_t total = 0;
    blockExclusiveSum(uint32_t(__popc(keep)), total, scan);
    if (t < 32) {
        uint64_t prefix = 0;
        if (tile == 0) {
            if (t == 0)
                lbPublish<PlainCodec>(a.status, tile, 0, kLbPrefix, total);
        } else {
            if (t == 0)
                lbPublish<PlainCodec>(a.status, tile, 0, kLbAggregate, total);
            prefix = lbExclusivePrefix<PlainCodec>(a.status, tile, 0, a.err);
            if (t == 0)
                lbPublish<PlainCodec>(a.status, tile, 0, kLbPrefix, prefix + total);
        }
        if (t == 0) {
            a.prefix[tile] = uint32_t(prefix);
            if (tile == a.tiles - 1)
                *a.cnt = *a.err != 0u ? 0xffffffffu : uint32_t(prefix + total);
        }
    }
}

/** stage[i] = plane[i] over [0, *span) (or [0, n) without a span). */
template <class T>
__global__ __launch_bounds__(kThreads) void copySpanKernel(const T* __restrict__ src, T* __restrict__ dst,
    const uint32_t* span, const uint32_t* fire, int64_t n)
{
    if (fire != nullptr && *fire == 0u)
        return;
    const int64_t end = span != nullptr ? spanOf(span, n) : n;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < end; i += int64_t(gridDim.x) * blockDim.x)
        dst[i] = src[i];
}

struct InPlaceArgs {
    void* plane;
    void* stage;
    void* plane2;  // the second plane of a pair (G = 2), its dropped run staged at stage2
    void* stage2;
    const uint16_t* bits;
    const uint32_t* prefix;
    const uint32_t* cnt;
    const uint32_t* span;
    const uint32_t* fire;
    uint32_t* err;
    uint32_t* claim;     // this plane's tile counter (zero on entry)
    uint32_t* readDone;  // per tile: the epoch of the latest plane whose tile has been read
    int32_t* inv;        // Perm only
    int32_t* indexMap;   // Perm only
    int64_t n;
    uint32_t epoch, tiles;
};

__device__ __forceinline__ uint32_t readFlag(const uint32_t* readDone, int64_t w)
{
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(readDone + w) : "memory");
    return v;
}

/** Whether tile ``w`` of the plane with ``epoch`` has been read, polled at most
 *  kLbSpinLimit times (acquire: the tile's slots may be overwritten after it). */
__device__ __forceinline__ bool waitTileRead(const uint32_t* readDone, int64_t w, uint32_t epoch)
{
    for (uint32_t i = 0; i < kLbSpinLimit; ++i) {
        if (readFlag(readDone, w) >= epoch)
            return true;
        if (i > 32)
            __nanosleep(64);
    }
    return false;
}

/** 4096-slot tiles of ``G`` planes (1, or 2 of the same element size) moved in
 *  place, one CTA per resident slot: each tile (claimed in order; the next claim goes
 *  out while the tile is worked on) is read, ordered in shared memory and its read
 *  published, then its kept run written to [pre, pre + kept) once the earlier tiles
 *  that range covers have been read, and its dropped run to the stage at its rank
 *  among the dropped slots. Two planes share the tile's scan, read flag and wait.
 *  With ``Perm`` the plane is perm: inv[v] = the new slot of each moved value v (a
 *  dropped one's is count + its rank), and index_map is the identity over the
 *  tile's part of [0, count). A wait that gives up sets bit 2 of ``*err`` and
 *  leaves the tile's kept run unwritten: the count then reports the failure. No
 *  wait is on a tile whose read cannot finish: the lowest tile not yet read is being
 *  read (reads wait on nothing) or is claimed by a CTA writing an earlier tile, whose
 *  waits are on tiles lower still, all read. */
template <class T, bool Perm, int G>
__global__ __launch_bounds__(kThreads, sizeof(T) > 8 ? 2 : (sizeof(T) <= 2 && G == 1 ? 8 : 4)) void placeInPlaceKernel(
    InPlaceArgs a)
{
    static_assert(G == 1 || (G == 2 && !Perm), "perm moves alone");
    if (a.fire != nullptr && *a.fire == 0u)
        return;
    if (*a.err != 0u)
        return;  // the scan gave up (the planes stay as they were), or an earlier plane's wait did
    extern __shared__ __align__(16) unsigned char smem[];
    T* out = reinterpret_cast<T*>(smem);  // [G][kTile]
    __shared__ uint32_t scan[33];
    __shared__ uint16_t sKeep[kThreads];
    __shared__ uint32_t sExcl[kThreads];
    __shared__ uint32_t sTile;
    __shared__ int sOk;
    const int t = int(threadIdx.x);
    if (t == 0)
        sTile = atomicAdd(a.claim, 1u);
    __syncthreads();
    uint32_t tile = sTile;
    const int64_t sp = spanOf(a.span, a.n);
    const int64_t cnt = int64_t(*a.cnt);
    T* planes[G];
    T* stages[G];
    planes[0] = static_cast<T*>(a.plane);
    stages[0] = static_cast<T*>(a.stage);
    if constexpr (G == 2) {
        planes[1] = static_cast<T*>(a.plane2);
        stages[1] = static_cast<T*>(a.stage2);
    }
    constexpr bool kNarrow = sizeof(T) <= 2;
    bool vecOk = true;
#pragma unroll
    for (int g = 0; g < G; ++g)
        vecOk = vecOk && (reinterpret_cast<uintptr_t>(planes[g]) & 15u) == 0;
    while (tile < a.tiles) {
        const int64_t tile0 = int64_t(tile) * kTile;
        if (tile0 >= sp)
            break;  // nothing of this tile moves, nor of any later claim; no kept slot lands here
        const int64_t len = sp - tile0 < kTile ? sp - tile0 : kTile;
        // Elements 1 or 2 bytes wide: thread t takes the tile's elements [16 t, 16 t + 16)
        // -- exactly its own keep bits -- in one or two 16-byte loads. Wider ones: element
        // e is the (e % 16)-th of thread e / 16's keep bits, read coalesced
        // (lane-consecutive e). All loads go out before the keep counts are scanned.
        T v[G][kPer];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const T* plane = planes[g];
            if constexpr (kNarrow) {
                const int64_t e0 = int64_t(t) * kPer;
                if (vecOk && e0 + kPer <= len) {
                    union {
                        uint4 q[sizeof(T)];
                        T x[kPer];
                    } u;
#pragma unroll
                    for (int k = 0; k < int(sizeof(T)); ++k)
                        u.q[k] = reinterpret_cast<const uint4*>(plane + tile0 + e0)[k];
#pragma unroll
                    for (int j = 0; j < kPer; ++j)
                        v[g][j] = u.x[j];
                } else {
#pragma unroll
                    for (int j = 0; j < kPer; ++j)
                        v[g][j] = e0 + j < len ? plane[tile0 + e0 + j] : T{};
                }
            } else {
#pragma unroll
                for (int j = 0; j < kPer; ++j) {
                    const int e = t + j * kThreads;
                    v[g][j] = int64_t(e) < len ? plane[tile0 + e] : T{};
                }
            }
        }
        uint32_t next = 0;
        if (t == 0)
            next = atomicAdd(a.claim, 1u);  // used at the end of the tile
        const uint32_t keep = a.bits[size_t(tile) * kThreads + size_t(t)];
        const int64_t pre = int64_t(a.prefix[tile]);  // kept slots before the tile
        // the read flags of the (at most two) earlier tiles the kept run may land in,
        // fetched now so that the check after the scan seldom waits
        const int64_t first = pre / kTile;
        uint32_t seen = 0;
        if (t < 2 && first + t < int64_t(tile))
            seen = readFlag(a.readDone, first + t);
        uint32_t kept = 0;
        const uint32_t excl = blockExclusiveSum(uint32_t(__popc(keep)), kept, scan);
        if (t == 0)
            sOk = 1;
        if constexpr (kNarrow) {
#pragma unroll
            for (int j = 0; j < kPer; ++j) {
                const int64_t e = int64_t(t) * kPer + j;
                if (e < len) {
                    const uint32_t before = excl + __popc(keep & ((1u << j) - 1u));  // kept before e
                    const uint32_t pos = ((keep >> j) & 1u) ? before : kept + uint32_t(e) - before;
#pragma unroll
                    for (int g = 0; g < G; ++g)
                        out[g * kTile + pos] = v[g][j];
                }
            }
        } else {
            sKeep[t] = uint16_t(keep);
            sExcl[t] = excl;
            __syncthreads();
#pragma unroll
            for (int j = 0; j < kPer; ++j) {
                const int e = t + j * kThreads;
                if (int64_t(e) < len) {
                    const uint32_t kb = sKeep[e >> 4], bit = uint32_t(e & 15);
                    const uint32_t before = sExcl[e >> 4] + __popc(kb & ((1u << bit) - 1u));  // kept before e
                    const uint32_t pos = ((kb >> bit) & 1u) ? before : kept + uint32_t(e) - before;
#pragma unroll
                    for (int g = 0; g < G; ++g)
                        out[g * kTile + pos] = v[g][j];
                }
            }
        }
        __syncthreads();  // every load of the tile has landed (its value is in shared memory)
        if (t == 0)  // so its slots may be overwritten: reads that have returned need no fence
            asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(a.readDone + tile), "r"(a.epoch) : "memory");
        if (kept > 0) {
            // [pre, pre + kept) covers at most two tiles, the last of them this one at most
            const int64_t last = (pre + int64_t(kept) - 1) / kTile;
            if (t < 2) {
                const int64_t w = first + t;
                if (w <= last && w < int64_t(tile) && seen < a.epoch && !waitTileRead(a.readDone, w, a.epoch)) {
                    atomicOr(a.err, 4u);
                    sOk = 0;
                }
            }
            __syncthreads();
        }
        const int64_t dropBase = tile0 - pre;  // dropped slots before the tile
        const bool ok = sOk != 0;
        for (int q = t; q < int(len); q += kThreads) {
            if (q < int(kept)) {
                if (!ok)
                    continue;
                const int64_t d = pre + q;
#pragma unroll
                for (int g = 0; g < G; ++g)
                    planes[g][d] = out[g * kTile + q];
                if constexpr (Perm) {
                    const T x = out[q];
                    a.inv[static_cast<int32_t>(x)] = int32_t(d);
                    a.indexMap[d] = int32_t(d);
                }
            } else {
                const int64_t r = dropBase + (q - int(kept));
#pragma unroll
                for (int g = 0; g < G; ++g)
                    stages[g][r] = out[g * kTile + q];
                if constexpr (Perm)
                    a.inv[static_cast<int32_t>(out[q])] = int32_t(cnt + r);
            }
        }
        if (t == 0)
            sTile = next;
        __syncthreads();  // out, sKeep and sExcl are free again; sTile holds the next claim
        tile = sTile;
    }
}

/** plane[count + r] = stage[r] for the staged dropped run, r < span - count, and the
 *  same for a second plane (plane2, stage2) when it is not null. */
template <class T>
__global__ __launch_bounds__(kThreads) void dropBackKernel(const T* __restrict__ stage, T* __restrict__ plane,
    const T* __restrict__ stage2, T* __restrict__ plane2, const uint32_t* cnt, const uint32_t* span,
    const uint32_t* fire, const uint32_t* err, int64_t n)
{
    if (fire != nullptr && *fire == 0u)
        return;
    if (*err != 0u)
        return;
    const int64_t c = int64_t(*cnt);
    const int64_t end = spanOf(span, n) - c;
    for (int64_t r = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; r < end; r += int64_t(gridDim.x) * blockDim.x) {
        plane[c + r] = stage[r];
        if (plane2 != nullptr)
            plane2[c + r] = stage2[r];
    }
}

__global__ void reorderFinishKernel(const uint32_t* cnt, const uint32_t* err, uint32_t* count, uint32_t* span,
    uint32_t* fire)
{
    if (fire != nullptr && *fire == 0u)
        return;
    const uint32_t c = *err != 0u ? 0xffffffffu : *cnt;  // a count above n reports a failed reorder
    *count = c;
    if (*err == 0u)
        *span = c;
    if (fire != nullptr)
        *fire = 0u;
}

__global__ void reorderEmptyKernel(uint32_t* count, uint32_t* span, uint32_t* fire)
{
    if (fire != nullptr && *fire == 0u)
        return;
    *count = 0u;
    *span = 0u;
    if (fire != nullptr)
        *fire = 0u;
}

/** plane[perm[s]] = stage[s] over [0, n): back to sample order. */
template <class T>
__global__ __launch_bounds__(kThreads) void restoreScatterKernel(const T* __restrict__ stage, T* plane,
    const int32_t* __restrict__ perm, int64_t n)
{
    for (int64_t s = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; s < n; s += int64_t(gridDim.x) * blockDim.x)
        plane[perm[s]] = stage[s];
}

__global__ void identityPairKernel(int32_t* perm, int32_t* inv, int64_t n)
{
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        perm[i] = int32_t(i);
        inv[i] = int32_t(i);
    }
}

/** Opt the place kernel of ``kernel`` into ``bytes`` of dynamic shared memory, once
 *  per kernel and device (a function attribute, not a stream operation). */
void allowShared(const void* kernel, size_t bytes)
{
    static std::mutex mu;
    static std::set<std::pair<const void*, int>> done;
    int dev = 0;
    cudaCheck(cudaGetDevice(&dev), "cudaGetDevice");
    std::lock_guard<std::mutex> lock(mu);
    if (done.count({kernel, dev}) != 0)
        return;
    cudaCheck(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes)),
        "cudaFuncSetAttribute");
    done.insert({kernel, dev});
}

unsigned streamGrid(int64_t n)
{
    const int64_t want = (n + kThreads - 1) / kThreads;
    const int64_t cap = int64_t(smCount()) * 8;
    return unsigned(want < 1 ? 1 : (want < cap ? want : cap));
}

/** The in-place place kernel's grid for ``tiles`` tiles: one CTA per resident slot
 *  (the kernel's occupancy, looked up once per device), at most one per tile. Also
 *  opts the kernel into ``shared`` bytes of dynamic shared memory. */
template <class T, bool Perm, int G>
unsigned placeGrid(uint32_t tiles, size_t shared)
{
    static std::mutex mu;
    static int perSm[64] = {};
    const void* kernel = reinterpret_cast<const void*>(&placeInPlaceKernel<T, Perm, G>);
    allowShared(kernel, shared);
    int dev = 0;
    cudaCheck(cudaGetDevice(&dev), "cudaGetDevice");
    int occ = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (perSm[dev & 63] == 0) {
            cudaCheck(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&perSm[dev & 63], placeInPlaceKernel<T, Perm, G>,
                          kThreads, shared),
                "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
            if (perSm[dev & 63] < 1)
                perSm[dev & 63] = 1;
        }
        occ = perSm[dev & 63];
    }
    const int64_t slots = int64_t(occ) * smCount();
    return unsigned(int64_t(tiles) < slots ? int64_t(tiles) : slots);
}

template <class F>
void withElem(uint32_t bytes, F&& f)
{
    switch (bytes) {
    case 1: f(uint8_t{}); break;
    case 2: f(uint16_t{}); break;
    case 4: f(uint32_t{}); break;
    case 8: f(uint64_t{}); break;
    default: f(Elem16{}); break;
    }
}

/** One move of the reorder: a plane, or two planes of one element size (``second``
 *  nonzero) moved together. */
struct PlaneMove {
    uint64_t first, second;
    uint32_t elem;
};

uint32_t widestOf(const std::vector<eagle_backend_reorder_plane>& p);

/** The planes' moves: planes of one element size up to 4 bytes paired (in table
 *  order) when both fit the stage one after the other, which holds n x max(widest
 *  element, 4) bytes; the rest one by one. */
std::vector<PlaneMove> pairPlanes(const std::vector<eagle_backend_reorder_plane>& planes)
{
    const uint32_t stageWidth = std::max<uint32_t>(widestOf(planes), 4u);
    std::vector<bool> done(planes.size(), false);
    std::vector<PlaneMove> moves;
    for (size_t k = 0; k < planes.size(); ++k) {
        if (done[k])
            continue;
        done[k] = true;
        PlaneMove m{planes[k].data, 0, planes[k].elem_bytes};
        if (m.elem <= 4 && 2 * m.elem <= stageWidth)
            for (size_t q = k + 1; q < planes.size(); ++q)
                if (!done[q] && planes[q].elem_bytes == m.elem) {
                    m.second = planes[q].data;
                    done[q] = true;
                    break;
                }
        moves.push_back(m);
    }
    return moves;
}

/** The plane table, checked as eagle checks it (Reorder.h checkReorder). */
std::vector<eagle_backend_reorder_plane> planesOf(const eagle_backend_reorder_desc& d, const char* who,
    bool needMask)
{
    if (d.n_planes > 0 && d.planes == 0)
        invalid(std::string(who) + ": a null plane table");
    if (d.n_planes > 4096)
        invalid(std::string(who) + ": at most 4096 planes");
    std::vector<eagle_backend_reorder_plane> p(d.n_planes);
    if (d.n_planes > 0)
        std::memcpy(p.data(), reinterpret_cast<const void*>(d.planes), d.n_planes * sizeof p[0]);
    bool maskSeen = false;
    for (size_t k = 0; k < p.size(); ++k) {
        const uint32_t e = p[k].elem_bytes;
        if (e != 1 && e != 2 && e != 4 && e != 8 && e != 16)
            invalid(std::string(who) + ": plane " + std::to_string(k) + " has " + std::to_string(e)
                + "-byte elements; supported are 1, 2, 4, 8 and 16");
        if (d.n > 0 && p[k].data == 0)
            invalid(std::string(who) + ": plane " + std::to_string(k) + " is null");
        if (p[k].data % e != 0)
            invalid(std::string(who) + ": plane " + std::to_string(k) + " is not aligned to its element size");
        const uint64_t lo = p[k].data, hi = lo + uint64_t(d.n) * e;
        for (size_t q = 0; q < k; ++q) {
            const uint64_t qlo = p[q].data, qhi = qlo + uint64_t(d.n) * p[q].elem_bytes;
            if (d.n > 0 && lo < qhi && qlo < hi)
                invalid(std::string(who) + ": planes " + std::to_string(q) + " and " + std::to_string(k) + " overlap");
        }
        if (p[k].data == d.mask && e == 1)
            maskSeen = true;
    }
    if (needMask && d.n > 0 && !maskSeen)
        invalid(std::string(who) + ": the mask must be one of the planes (it moves with them)");
    return p;
}

uint32_t widestOf(const std::vector<eagle_backend_reorder_plane>& p)
{
    uint32_t w = 4;  // perm
    for (const auto& q : p)
        w = q.elem_bytes > w ? q.elem_bytes : w;
    return w;
}


// ------------------------------------------------------------------ K classes
//
// reorder_classes_device (ReorderClasses.h reorderClassesDevice; seam
// eagle_backend.h:793-824): a stable counting sort of the slots [0, lim) by key,
// key = class (clamped to K-1) for a live sample and K for a dead one (dead
// last), or by class alone over the live prefix with CLASSES_WITHIN_LIVE; lim is
// *span, or *count within the live prefix. A tile of 4096 slots is ranked by its
// 8 warps, 16 rounds of 32 consecutive slots each: __match_any_sync groups the
// round's lanes by key, a lane's rank is its peers below it plus its warp's count
// of that key so far, and a prefix over the warps gives each warp's start per key.
// The first kernel writes each tile's count per key (key-major) and the slots'
// keys (the mask and class planes move later); one look-back scan turns the
// counts into each (key, tile)'s first destination; then every plane is staged
// and placed (dst = base[key][tile] + warp start + rank).

constexpr int kWarps = kThreads / 32;
constexpr int kRounds = int(kTile) / kThreads;
constexpr uint32_t kNoKey = 0x100u;

__device__ __forceinline__ uint32_t classKeyOf(uint8_t m, uint8_t c, bool drop, bool within, uint32_t classes)
{
    const uint32_t cc = uint32_t(c) < classes ? uint32_t(c) : classes - 1u;
    if (within)
        return cc;
    const bool set = m != 0;
    return (drop ? !set : set) ? cc : classes;
}

struct ClassArgs {
    const uint8_t* mask;
    const uint8_t* cls;
    int64_t n;
    const uint32_t* lim;
    const uint32_t* fire;
    uint32_t classes, nKeys;
    int drop, within;
    uint8_t* keys;   // n: each slot's key, kept while the planes move
    uint16_t* rel;   // n: each slot's rank among its tile's slots of the same key
    uint32_t* hist;  // nKeys x tiles, key-major: counts, then the first destinations
    uint32_t tiles;
};

/** Per-warp counts of each key over the tile's rounds; a lane's round-r slot comes
 *  back in ``kr[r]`` as key << 16 | its rank among the warp's earlier slots of that
 *  key (kNoKey past lim). */
__device__ __forceinline__ void rankTile(const uint8_t* keys, int64_t tile0, int64_t lim, uint16_t (*cnt)[256],
    uint32_t (&kr)[kRounds])
{
    const unsigned lane = threadIdx.x & 31u, w = threadIdx.x >> 5;
#pragma unroll
    for (int r = 0; r < kRounds; ++r) {
        const int64_t i = tile0 + int64_t(w) * (kRounds * 32) + int64_t(r) * 32 + lane;
        const uint32_t k = i < lim ? uint32_t(keys[i]) : kNoKey;
        const unsigned peers = __match_any_sync(kFull, k);
        const uint32_t below = __popc(peers & ((1u << lane) - 1u));
        uint32_t base = 0;
        if (k != kNoKey)
            base = cnt[w][k];
        __syncwarp();
        if (k != kNoKey && below == 0)
            cnt[w][k] = uint16_t(base + __popc(peers));
        __syncwarp();
        kr[r] = (k << 16) | (base + below);
    }
}

__global__ __launch_bounds__(kThreads) void classHistKernel(ClassArgs a)
{
    if (a.fire != nullptr && *a.fire == 0u)
        return;
    __shared__ uint16_t cnt[kWarps][256];
    const int t = int(threadIdx.x);
    for (int q = t; q < kWarps * 256; q += kThreads)
        (&cnt[0][0])[q] = 0;
    __syncthreads();
    const int64_t lim = spanOf(a.lim, a.n);
    const int64_t tile0 = int64_t(blockIdx.x) * kTile;
    const unsigned lane = threadIdx.x & 31u, w = threadIdx.x >> 5;
    // the keys of the tile's slots, saved for the place kernels
#pragma unroll
    for (int r = 0; r < kRounds; ++r) {
        const int64_t i = tile0 + int64_t(w) * (kRounds * 32) + int64_t(r) * 32 + lane;
        if (i < lim)
            a.keys[i] = uint8_t(classKeyOf(a.mask[i], a.cls[i], a.drop != 0, a.within != 0, a.classes));
    }
    __syncwarp();
    uint32_t kr[kRounds];
    rankTile(a.keys, tile0, lim, cnt, kr);
    __syncthreads();
    // per key: each warp's first rank (the counts of the warps before it) and the total
    uint32_t total = 0;
#pragma unroll
    for (int q = 0; q < kWarps; ++q) {
        const uint32_t c = cnt[q][t];
        cnt[q][t] = uint16_t(total);
        total += c;
    }
    if (uint32_t(t) < a.nKeys)
        a.hist[size_t(t) * a.tiles + blockIdx.x] = total;
    __syncthreads();
    // each slot's rank within its key's run of the tile, for every plane's place
#pragma unroll
    for (int r = 0; r < kRounds; ++r) {
        const uint32_t k = kr[r] >> 16;
        if (k != kNoKey) {
            const int64_t i = tile0 + int64_t(w) * (kRounds * 32) + int64_t(r) * 32 + lane;
            a.rel[i] = uint16_t(cnt[w][k] + (kr[r] & 0xffffu));
        }
    }
}

struct ScanU32Args {
    uint32_t* data;  // in: counts; out: exclusive prefixes
    int64_t m;
    const uint32_t* fire;
    uint64_t* status;
    uint32_t* tileNext;
    uint32_t* err;
    uint32_t* total;
    uint32_t tiles;
};

/** Exclusive prefix sum of m uint32 counts in place: 16 per thread, CTA scan,
 *  decoupled look-back over 4096-element tiles. */
__global__ __launch_bounds__(kThreads) void scanU32Kernel(ScanU32Args a)
{
    if (a.fire != nullptr && *a.fire == 0u)
        return;
    __shared__ uint32_t sTile;
    __shared__ uint32_t scan[33];
    __shared__ uint64_t sPrefix;
    const int t = int(threadIdx.x);
    if (t == 0)
        sTile = atomicAdd(a.tileNext, 1u);
    __syncthreads();
    const uint32_t tile = sTile;
    const int64_t i0 = int64_t(tile) * kTile + int64_t(t) * kPer;
    uint32_t v[kPer];
    uint32_t sum = 0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        v[j] = i0 + j < a.m ? a.data[i0 + j] : 0u;
        sum += v[j];
    }
    uint32_t total = 0;
    const uint32_t excl = blockExclusiveSum(sum, total, scan);
    if (t < 32) {
        uint64_t prefix = 0;
        if (tile == 0) {
            if (t == 0)
                lbPublish<PlainCodec>(a.status, tile, 0, kLbPrefix, total);
        } else {
            if (t == 0)
                lbPublish<PlainCodec>(a.status, tile, 0, kLbAggregate, total);
            prefix = lbExclusivePrefix<PlainCodec>(a.status, tile, 0, a.err);
            if (t == 0)
                lbPublish<PlainCodec>(a.status, tile, 0, kLbPrefix, prefix + total);
        }
        if (t == 0) {
            sPrefix = prefix;
            if (tile == a.tiles - 1)
                *a.total = uint32_t(prefix + total);
        }
    }
    __syncthreads();
    uint32_t run = uint32_t(sPrefix) + excl;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        if (i0 + j < a.m)
            a.data[i0 + j] = run;
        run += v[j];
    }
}

struct ClassPlaceArgs {
    const void* stage;
    void* plane;
    const void* stage2;  // the second plane of a pair (G = 2) and its staged copy
    void* plane2;
    const uint8_t* keys;
    const uint16_t* rel;     // each slot's rank within its key's run of the tile
    const uint32_t* total;   // the count matrix's total (the entry after the last)
    uint32_t nKeys;
    const uint32_t* base;  // nKeys x tiles first destinations
    const uint32_t* lim;
    const uint32_t* fire;
    const uint32_t* err;
    int32_t* inv;  // Perm only
    int64_t n;
    uint32_t tiles;
};

/** One tile of ``G`` planes (1, or 2 of the same element size, sharing the tile's
 *  keys, ranks and scan) placed in key order: each slot to its key's run of the
 *  destination at its rank, the tile staged in shared memory in key order first so
 *  that each key's run is written with coalesced stores. With ``Perm`` the plane is
 *  perm and inv follows it. */
template <class T, bool Perm, int G>
__global__ __launch_bounds__(kThreads) void classPlaceKernel(ClassPlaceArgs a)
{
    static_assert(G == 1 || (G == 2 && !Perm), "perm moves alone");
    if (a.fire != nullptr && *a.fire == 0u)
        return;
    if (*a.err != 0u)
        return;
    extern __shared__ __align__(16) unsigned char smem[];
    T* out = reinterpret_cast<T*>(smem);                                         // [G][kTile], key order
    uint8_t* outKey = reinterpret_cast<uint8_t*>(smem + G * kTile * sizeof(T));  // each place's key
    __shared__ uint32_t sStart[256];
    __shared__ int64_t sShift[256];  // a key's first destination less its first place in the tile
    __shared__ uint32_t scan[33];
    const int t = int(threadIdx.x);
    const int64_t lim = spanOf(a.lim, a.n);
    const int64_t tile0 = int64_t(blockIdx.x) * kTile;
    if (tile0 >= lim)
        return;
    const int64_t len = lim - tile0 < kTile ? lim - tile0 : kTile;
    // each slot's value, key and rank among its key's slots (the histogram pass ranked
    // them): thread t takes slots t, t + 256, ..., all loads in flight while the tile's
    // key counts below are scanned
    const T* src[G];
    T* dst[G];
    src[0] = static_cast<const T*>(a.stage);
    dst[0] = static_cast<T*>(a.plane);
    if constexpr (G == 2) {
        src[1] = static_cast<const T*>(a.stage2);
        dst[1] = static_cast<T*>(a.plane2);
    }
    T v[G][kPer];
    uint32_t kr[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int64_t i = tile0 + t + int64_t(j) * kThreads;
        const bool in = i - tile0 < len;
#pragma unroll
        for (int g = 0; g < G; ++g)
            v[g][j] = in ? src[g][i] : T{};
        kr[j] = in ? (uint32_t(a.keys[i]) << 16) | uint32_t(a.rel[i]) : kNoKey << 16;
    }
    // the tile's count of each key, from the scanned key-major matrix: the next entry's
    // first destination (the next key's first tile, or the total after the last) less its own
    uint32_t c = 0, first = 0;
    if (uint32_t(t) < a.nKeys) {
        const size_t at = size_t(t) * a.tiles + blockIdx.x;
        const size_t m = size_t(a.nKeys) * a.tiles;
        first = a.base[at];
        c = (at + 1 < m ? a.base[at + 1] : *a.total) - first;
    }
    uint32_t all = 0;
    const uint32_t start = blockExclusiveSum(c, all, scan);  // the key's first place in the tile
    sStart[t] = start;
    sShift[t] = int64_t(first) - int64_t(start);
    __syncthreads();  // sStart, sShift
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const uint32_t k = kr[j] >> 16;
        if (k != kNoKey) {
            const uint32_t pos = sStart[k] + (kr[j] & 0xffffu);
#pragma unroll
            for (int g = 0; g < G; ++g)
                out[g * kTile + pos] = v[g][j];
            outKey[pos] = uint8_t(k);
        }
    }
    __syncthreads();
    // each key's run of the tile is contiguous in the plane: coalesced stores
    for (int q = t; q < int(len); q += kThreads) {
        const int64_t d = sShift[outKey[q]] + q;
#pragma unroll
        for (int g = 0; g < G; ++g)
            dst[g][d] = out[g * kTile + q];
        if constexpr (Perm)
            a.inv[static_cast<int32_t>(out[q])] = int32_t(d);
    }
}

__global__ void classIdentityKernel(int32_t* indexMap, const uint32_t* live, const uint32_t* fire, const uint32_t* err)
{
    if (fire != nullptr && *fire == 0u)
        return;
    if (*err != 0u)
        return;
    const int64_t end = int64_t(*live);
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < end; i += int64_t(gridDim.x) * blockDim.x)
        indexMap[i] = int32_t(i);
}

__global__ void classFinishKernel(const uint32_t* base, uint32_t tiles, uint32_t nKeys, const uint32_t* total,
    uint32_t classes, int within, const uint32_t* err, uint32_t* offsets, uint32_t* count, uint32_t* span,
    uint32_t* fire, uint32_t* classSorts)
{
    if (fire != nullptr && *fire == 0u)
        return;
    if (*err != 0u) {
        *count = 0xffffffffu;  // a count above n reports a failed sort
        return;
    }
    for (uint32_t c = 0; c <= classes; ++c)
        offsets[c] = c < nKeys ? base[size_t(c) * tiles] : *total;
    if (!within) {
        const uint32_t live = base[size_t(classes) * tiles];  // the dead key's first slot
        *count = live;
        *span = live;
    }
    if (fire != nullptr)
        *fire = 0u;
    *classSorts += 1u;
}

struct ClassLayout {
    size_t keys, rel, hist, status, words, stage, total;
};

ClassLayout classLayoutFor(int64_t n, uint32_t elem, uint32_t classes)
{
    const size_t m = size_t(n > 0 ? n : 1);
    const size_t tiles = (m + size_t(kTile) - 1) / size_t(kTile);
    const size_t histN = size_t(classes + 1) * tiles;
    const size_t scanTiles = (histN + size_t(kTile) - 1) / size_t(kTile);
    auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
    ClassLayout l{};
    l.keys = 0;
    l.rel = up(m);
    l.hist = up(l.rel + m * sizeof(uint16_t));
    l.status = up(l.hist + histN * sizeof(uint32_t));
    l.words = up(l.status + scanTiles * sizeof(uint64_t));
    l.stage = l.words + 256;
    l.total = up(l.stage + m * (elem > 4 ? elem : 4));
    return l;
}
}  // namespace
}  // namespace eb

using namespace eb;

EB_API eagle_backend_status eagle_backend_reorder_device(struct eagle_backend_reorder_desc* desc)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_reorder_device";
        const auto d = readDesc(desc, EAGLE_BACKEND_COMPACT_MASK_IS_DROP, who);
        if (d.n < 0)
            invalid(std::string(who) + ": n must be >= 0");
        if (d.n > INT64_C(2147483647))
            unsupported(std::string(who) + ": the int32 perm addresses at most 2^31-1 samples, got n = "
                + std::to_string(d.n));
        const auto planes = planesOf(d, who, true);
        const Layout l = layoutFor(d.n, widestOf(planes), planes.size());
        if (d.scratch == 0) {
            constexpr size_t end = offsetof(eagle_backend_reorder_desc, scratch_bytes) + sizeof(int64_t);
            if (desc->struct_size < end)
                invalid(std::string(who) + ": the scratch query needs a desc carrying scratch_bytes");
            desc->scratch_bytes = int64_t(l.total);
            return;
        }
        if (d.count == 0 || d.span == 0 || (d.n > 0 && (d.mask == 0 || d.perm == 0 || d.inv == 0 || d.index_map == 0)))
            invalid(std::string(who) + ": mask, perm, inv, index_map, count and span must be device addresses");
        DeviceScope scope(resolveDevice(d.device, d.n > 0 ? d.mask : d.count));
        const cudaStream_t s = seamStream(d.stream);
        auto* count = reinterpret_cast<uint32_t*>(d.count);
        auto* span = reinterpret_cast<uint32_t*>(d.span);
        auto* fire = reinterpret_cast<uint32_t*>(d.fire);
        if (d.n == 0) {
            reorderEmptyKernel<<<1, 1, 0, s>>>(count, span, fire);
            launchCheck(who);
            return;
        }
        char* base = reinterpret_cast<char*>(d.scratch);
        ScanArgs a{};
        a.mask = reinterpret_cast<const uint8_t*>(d.mask);
        a.n = d.n;
        a.span = span;
        a.fire = fire;
        a.tiles = uint32_t((d.n + kTile - 1) / kTile);
        a.status = reinterpret_cast<uint64_t*>(base + l.status);
        a.tileNext = reinterpret_cast<uint32_t*>(base + l.words);
        a.err = a.tileNext + 1;
        a.cnt = a.tileNext + 2;
        a.prefix = reinterpret_cast<uint32_t*>(base + l.prefix);
        a.bits = reinterpret_cast<uint16_t*>(base + l.bits);
        cudaCheck(cudaMemsetAsync(base, 0, l.prefix, s), "cudaMemsetAsync");  // status words and counters
        if (d.flags & EAGLE_BACKEND_COMPACT_MASK_IS_DROP)
            reorderScanKernel<true><<<a.tiles, kThreads, 0, s>>>(a);
        else
            reorderScanKernel<false><<<a.tiles, kThreads, 0, s>>>(a);
        launchCheck(who);
        InPlaceArgs p{};
        p.stage = base + l.stage;
        p.bits = a.bits;
        p.prefix = a.prefix;
        p.cnt = a.cnt;
        p.span = span;
        p.fire = fire;
        p.err = a.err;
        p.readDone = reinterpret_cast<uint32_t*>(base + l.done);
        p.n = d.n;
        p.tiles = a.tiles;
        uint32_t epoch = 0;
        // planes of one element size up to 4 bytes move two at a time when both dropped
        // runs fit the stage one after the other, sharing each tile's scan, read flag and
        // wait; perm moves alone (it also writes inv and index_map)
        char* stage = base + l.stage;
        auto move = [&](uint64_t data, uint64_t data2, uint32_t elem, bool perm) {
            p.claim = reinterpret_cast<uint32_t*>(base + l.claims) + epoch;
            ++epoch;
            p.epoch = epoch;
            withElem(elem, [&](auto tag) {
                using T = decltype(tag);
                p.plane = reinterpret_cast<void*>(data);
                p.stage = stage;
                p.plane2 = reinterpret_cast<void*>(data2);
                p.stage2 = stage + size_t(d.n) * sizeof(T);
                if (perm) {
                    const size_t shared = size_t(kTile) * sizeof(int32_t);
                    p.inv = reinterpret_cast<int32_t*>(d.inv);
                    p.indexMap = reinterpret_cast<int32_t*>(d.index_map);
                    placeInPlaceKernel<int32_t, true, 1>
                        <<<placeGrid<int32_t, true, 1>(a.tiles, shared), kThreads, shared, s>>>(p);
                } else if (data2 != 0) {
                    if constexpr (sizeof(T) <= 4) {
                        const size_t shared = 2 * size_t(kTile) * sizeof(T);
                        placeInPlaceKernel<T, false, 2><<<placeGrid<T, false, 2>(a.tiles, shared), kThreads, shared, s>>>(p);
                    }
                } else {
                    const size_t shared = size_t(kTile) * sizeof(T);
                    placeInPlaceKernel<T, false, 1><<<placeGrid<T, false, 1>(a.tiles, shared), kThreads, shared, s>>>(p);
                }
                launchCheck(who);
                dropBackKernel<T><<<streamGrid(d.n), kThreads, 0, s>>>(reinterpret_cast<const T*>(p.stage),
                    reinterpret_cast<T*>(data), reinterpret_cast<const T*>(p.stage2), reinterpret_cast<T*>(data2),
                    a.cnt, span, fire, a.err, d.n);
                launchCheck(who);
            });
        };
        for (const auto& m : pairPlanes(planes))
            move(m.first, m.second, m.elem, false);
        move(d.perm, 0, 4, true);
        reorderFinishKernel<<<1, 1, 0, s>>>(a.cnt, a.err, count, span, fire);
        launchCheck(who);
    });
}

EB_API eagle_backend_status eagle_backend_reorder_classes_device(struct eagle_backend_reorder_classes_desc* desc)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_reorder_classes_device";
        if (desc == nullptr)
            invalid(std::string(who) + ": null desc");
        constexpr size_t need = offsetof(eagle_backend_reorder_classes_desc, class_sorts) + sizeof(uint64_t);
        if (desc->struct_size < need)
            invalid(std::string(who) + ": the desc must carry the class fields");
        const auto d = readDesc(desc, EAGLE_BACKEND_COMPACT_MASK_IS_DROP | EAGLE_BACKEND_CLASSES_WITHIN_LIVE, who);
        if (d.classes < 2 || d.classes > EAGLE_BACKEND_MAX_CLASSES)
            invalid(std::string(who) + ": classes must lie in [2, 255]");
        if (d.reserved3 != 0)
            invalid(std::string(who) + ": reserved3 must be zero");
        if (d.n < 0)
            invalid(std::string(who) + ": n must be >= 0");
        if (d.n > INT64_C(2147483647))
            unsupported(std::string(who) + ": the int32 perm addresses at most 2^31-1 samples, got n = "
                + std::to_string(d.n));
        eagle_backend_reorder_desc base{};
        std::memcpy(&base, &d, sizeof base);
        const auto planes = planesOf(base, who, true);
        bool classSeen = false;
        for (const auto& q : planes)
            classSeen = classSeen || (q.data == d.class_plane && q.elem_bytes == 1);
        if (d.n > 0 && !classSeen)
            invalid(std::string(who) + ": the class plane must be one of the planes (it moves with them)");
        const ClassLayout l = classLayoutFor(d.n, widestOf(planes), d.classes);
        if (d.scratch == 0) {
            desc->scratch_bytes = int64_t(l.total);
            return;
        }
        if (d.n > 0
            && (d.mask == 0 || d.perm == 0 || d.inv == 0 || d.index_map == 0 || d.count == 0 || d.span == 0
                || d.class_plane == 0 || d.offsets == 0 || d.class_sorts == 0))
            invalid(std::string(who) + ": mask, perm, inv, index_map, count, span, class_plane, offsets and "
                                       "class_sorts must be device addresses");
        DeviceScope scope(resolveDevice(d.device, d.n > 0 ? d.mask : d.count));
        const cudaStream_t s = seamStream(d.stream);
        auto* count = reinterpret_cast<uint32_t*>(d.count);
        auto* span = reinterpret_cast<uint32_t*>(d.span);
        auto* fire = reinterpret_cast<uint32_t*>(d.fire);
        if (d.n == 0) {
            reorderEmptyKernel<<<1, 1, 0, s>>>(count, span, fire);
            launchCheck(who);
            return;
        }
        const bool within = (d.flags & EAGLE_BACKEND_CLASSES_WITHIN_LIVE) != 0;
        const uint32_t* lim = within ? count : span;
        char* raw = reinterpret_cast<char*>(d.scratch);
        ClassArgs c{};
        c.mask = reinterpret_cast<const uint8_t*>(d.mask);
        c.cls = reinterpret_cast<const uint8_t*>(d.class_plane);
        c.n = d.n;
        c.lim = lim;
        c.fire = fire;
        c.classes = d.classes;
        c.nKeys = within ? d.classes : d.classes + 1;
        c.drop = (d.flags & EAGLE_BACKEND_COMPACT_MASK_IS_DROP) != 0;
        c.within = within;
        c.keys = reinterpret_cast<uint8_t*>(raw + l.keys);
        c.rel = reinterpret_cast<uint16_t*>(raw + l.rel);
        c.hist = reinterpret_cast<uint32_t*>(raw + l.hist);
        c.tiles = uint32_t((d.n + kTile - 1) / kTile);
        ScanU32Args sa{};
        sa.data = c.hist;
        sa.m = int64_t(c.nKeys) * c.tiles;
        sa.fire = fire;
        sa.status = reinterpret_cast<uint64_t*>(raw + l.status);
        sa.tileNext = reinterpret_cast<uint32_t*>(raw + l.words);
        sa.err = sa.tileNext + 1;
        sa.total = sa.tileNext + 2;
        sa.tiles = uint32_t((sa.m + kTile - 1) / kTile);
        cudaCheck(cudaMemsetAsync(raw + l.status, 0, l.stage - l.status, s), "cudaMemsetAsync");
        // tiles past lim still write zero counts, so the whole count matrix is defined
        cudaCheck(cudaMemsetAsync(c.hist, 0, size_t(sa.m) * sizeof(uint32_t), s), "cudaMemsetAsync");
        classHistKernel<<<c.tiles, kThreads, 0, s>>>(c);
        launchCheck(who);
        scanU32Kernel<<<sa.tiles, kThreads, 0, s>>>(sa);
        launchCheck(who);
        ClassPlaceArgs p{};
        p.stage = raw + l.stage;
        p.keys = c.keys;
        p.rel = c.rel;
        p.total = sa.total;
        p.nKeys = c.nKeys;
        p.base = c.hist;
        p.lim = lim;
        p.fire = fire;
        p.err = sa.err;
        p.n = d.n;
        p.tiles = c.tiles;
        // planes of one element size up to 4 bytes move two at a time when both fit the
        // stage one after the other (they share the tile's keys, ranks and scan); perm
        // moves alone
        char* stage = raw + l.stage;
        auto move = [&](uint64_t data, uint64_t data2, uint32_t elem, bool perm) {
            withElem(elem, [&](auto tag) {
                using T = decltype(tag);
                T* st = reinterpret_cast<T*>(stage);
                T* st2 = st + d.n;
                copySpanKernel<T><<<streamGrid(d.n), kThreads, 0, s>>>(reinterpret_cast<const T*>(data), st, lim,
                    fire, d.n);
                launchCheck(who);
                if (data2 != 0) {
                    copySpanKernel<T><<<streamGrid(d.n), kThreads, 0, s>>>(reinterpret_cast<const T*>(data2), st2, lim,
                        fire, d.n);
                    launchCheck(who);
                }
                p.stage = st;
                p.plane = reinterpret_cast<void*>(data);
                p.stage2 = st2;
                p.plane2 = reinterpret_cast<void*>(data2);
                if (perm) {
                    const size_t shared = size_t(kTile) * (sizeof(int32_t) + 1);
                    p.inv = reinterpret_cast<int32_t*>(d.inv);
                    allowShared(reinterpret_cast<const void*>(&classPlaceKernel<int32_t, true, 1>), shared);
                    classPlaceKernel<int32_t, true, 1><<<c.tiles, kThreads, shared, s>>>(p);
                } else if (data2 != 0) {
                    if constexpr (sizeof(T) <= 4) {
                        const size_t shared = size_t(kTile) * (2 * sizeof(T) + 1);
                        allowShared(reinterpret_cast<const void*>(&classPlaceKernel<T, false, 2>), shared);
                        classPlaceKernel<T, false, 2><<<c.tiles, kThreads, shared, s>>>(p);
                    }
                } else {
                    const size_t shared = size_t(kTile) * (sizeof(T) + 1);
                    allowShared(reinterpret_cast<const void*>(&classPlaceKernel<T, false, 1>), shared);
                    classPlaceKernel<T, false, 1><<<c.tiles, kThreads, shared, s>>>(p);
                }
                launchCheck(who);
            });
        };
        for (const auto& m : pairPlanes(planes))
            move(m.first, m.second, m.elem, false);
        move(d.perm, 0, 4, true);
        // the live count: *count within the live prefix, else the dead key's first slot
        const uint32_t* live = within ? count : c.hist + size_t(d.classes) * c.tiles;
        classIdentityKernel<<<streamGrid(d.n), kThreads, 0, s>>>(reinterpret_cast<int32_t*>(d.index_map), live, fire,
            sa.err);
        launchCheck(who);
        classFinishKernel<<<1, 1, 0, s>>>(c.hist, c.tiles, c.nKeys, sa.total, d.classes, within ? 1 : 0, sa.err,
            reinterpret_cast<uint32_t*>(d.offsets), count, span, fire, reinterpret_cast<uint32_t*>(d.class_sorts));
        launchCheck(who);
    });
}

EB_API eagle_backend_status eagle_backend_x_restore_device(struct eagle_backend_reorder_desc* desc)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_restore_device";
        const auto d = readDesc(desc, EAGLE_BACKEND_COMPACT_MASK_IS_DROP, who);
        if (d.n < 0 || d.n > INT64_C(2147483647))
            invalid(std::string(who) + ": n must lie in [0, 2^31 - 1]");
        const auto planes = planesOf(d, who, false);
        const Layout l = layoutFor(d.n, widestOf(planes));
        if (d.scratch == 0) {
            constexpr size_t end = offsetof(eagle_backend_reorder_desc, scratch_bytes) + sizeof(int64_t);
            if (desc->struct_size < end)
                invalid(std::string(who) + ": the scratch query needs a desc carrying scratch_bytes");
            desc->scratch_bytes = int64_t(l.total);
            return;
        }
        if (d.n == 0)
            return;
        if (d.perm == 0 || d.inv == 0)
            invalid(std::string(who) + ": perm and inv must be device addresses");
        DeviceScope scope(resolveDevice(d.device, d.perm));
        const cudaStream_t s = seamStream(d.stream);
        char* stage = reinterpret_cast<char*>(d.scratch) + l.stage;
        const auto* perm = reinterpret_cast<const int32_t*>(d.perm);
        for (const auto& q : planes) {
            withElem(q.elem_bytes, [&](auto tag) {
                using T = decltype(tag);
                copySpanKernel<T><<<streamGrid(d.n), kThreads, 0, s>>>(reinterpret_cast<const T*>(q.data),
                    reinterpret_cast<T*>(stage), nullptr, nullptr, d.n);
                launchCheck(who);
                restoreScatterKernel<T><<<streamGrid(d.n), kThreads, 0, s>>>(reinterpret_cast<const T*>(stage),
                    reinterpret_cast<T*>(q.data), perm, d.n);
                launchCheck(who);
            });
        }
        identityPairKernel<<<streamGrid(d.n), kThreads, 0, s>>>(reinterpret_cast<int32_t*>(d.perm),
            reinterpret_cast<int32_t*>(d.inv), d.n);
        launchCheck(who);
    });
}

EB_API eagle_backend_status eagle_backend_pointer_residency(int32_t device, uint64_t ptr, int32_t* cls)
{
    return guarded([&] {
        if (cls == nullptr)
            invalid("eagle_backend_pointer_residency: null output");
        int dev = device;
        if (dev < 0 && cudaGetDevice(&dev) != cudaSuccess) {
            (void)cudaGetLastError();
            *cls = EAGLE_BACKEND_RESIDENCY_PAGEABLE;
            return;
        }
        cudaPointerAttributes at{};
        if (cudaPointerGetAttributes(&at, reinterpret_cast<const void*>(ptr)) != cudaSuccess) {
            (void)cudaGetLastError();
            *cls = EAGLE_BACKEND_RESIDENCY_PAGEABLE;
            return;
        }
        switch (at.type) {
        case cudaMemoryTypeDevice:
            *cls = at.device == dev ? EAGLE_BACKEND_RESIDENCY_DEVICE : EAGLE_BACKEND_RESIDENCY_OTHER_DEVICE;
            break;
        case cudaMemoryTypeManaged: *cls = EAGLE_BACKEND_RESIDENCY_MANAGED; break;
        case cudaMemoryTypeHost:
            *cls = at.devicePointer != nullptr ? EAGLE_BACKEND_RESIDENCY_MAPPED_HOST : EAGLE_BACKEND_RESIDENCY_PAGEABLE;
            break;
        default: *cls = EAGLE_BACKEND_RESIDENCY_PAGEABLE; break;
        }
    });
}
