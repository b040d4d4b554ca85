// Compact-then-sum without materialising the survivors.
//
// The canonical sum of the samples a mask keeps (eagle's ActiveSet.compact, then
// the ``ordered`` reduction over the compacted plane: python/eagle/_active_set.py:482-525,
// eagle/reduce/canonical.h:10-32) depends on each kept value's RANK among the
// survivors: leaf l holds ranks [4096 l, 4096 l + 4096), and slot t of a leaf folds
// its ranks t, t + 256, ..., in that order. Writing the survivors out and reading
// them back costs 16 bytes per survivor on top of the mask and the value sectors,
// the whole gap between a compaction and its roofline. Instead, after a 16-byte
// memset:
//
//   keepCountKernel   one 16384-sample tile per CTA (four coalesced rows of 4096 mask
//                     bytes): the keep bits go out as a bitmap (one bit per sample)
//                     and the tile's count as one word. No look-back: a tile never
//                     waits on another, so the pass streams.
//   tileScanKernel    one CTA: the exclusive scan of the tile counts, and the count.
//   leafStartKernel   a warp per tile: for every multiple of 4096 among the tile's
//                     ranks, the sample holding it (leafStart[l]), from the tile's
//                     512 bitmap words.
//   keptLeavesKernel  CTAs claim groups of 2^q consecutive leaves. Per leaf: the
//                     bitmap words over [leafStart[l], leafStart[l + 1]) are scanned
//                     across the CTA, the kept sample indices staged in shared memory
//                     by rank, then thread t loads the values of ranks t + 256 i,
//                     i = 0..15, together and folds them into slot t's partial in
//                     order -- the leaf walk, term by term -- before one warp runs the
//                     in-leaf tree. The next leaf's words are in flight meanwhile. A
//                     group's leaves join by the pairwise levels; the last CTA runs
//                     the remaining levels over the group partials.
//
// Traffic: the mask (n bytes), the bitmap written and read (n / 4 bytes), the value
// sectors holding a survivor; the bits are those of the two-kernel compaction +
// canonical sum, which the tests check against the oracle.
#include "canonical.cuh"

#include <mutex>

namespace eb {
namespace {

constexpr int kThreads = 256;
constexpr int kRows = 4;
constexpr int64_t kRow = int64_t(kThreads) * 16;  // 4096 samples: 16 mask bytes per thread
constexpr int64_t kTile = kRow * kRows;           // 16384 samples per keepCount CTA
constexpr int64_t kTileWords = kTile / 32;        // its bitmap words
constexpr int kScanThreads = 1024;
constexpr int kScanPer = 16;                      // tile counts per scan thread per round

using P = CompP<double>;

template <bool Drop, bool Aligned>
__global__ __launch_bounds__(kThreads) void keepCountKernel(const uint8_t* __restrict__ mask, int64_t n,
    uint32_t* __restrict__ bitmap, uint32_t* __restrict__ tileCount)
{
    __shared__ uint32_t part[kThreads / 32];
    const int t = int(threadIdx.x);
    const int64_t tile = blockIdx.x;
    const int64_t tile0 = tile * kTile;
    uint32_t bits[kRows];
    uint32_t c = 0;
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
        bits[q] = keepBits16<Drop, Aligned>(mask, tile0 + int64_t(q) * kRow + int64_t(t) * 16, n);
        c += uint32_t(__popc(bits[q]));
    }
    // threads 2u and 2u + 1 hold the low and high halves of one 32-sample word
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
        const uint32_t hi = __shfl_down_sync(kFull, bits[q], 1);
        if ((t & 1) == 0)
            bitmap[tile * kTileWords + q * (kRow / 32) + (t >> 1)] = bits[q] | (hi << 16);
    }
    c = warpSum(c);
    if ((t & 31) == 0)
        part[t >> 5] = c;
    __syncthreads();
    if (t == 0) {
        uint32_t s = 0;
#pragma unroll
        for (int w = 0; w < kThreads / 32; ++w)
            s += part[w];
        tileCount[tile] = s;
    }
}

/** tileOff[i] = the kept samples before tile i; ``*count`` = all of them. One CTA. */
__global__ __launch_bounds__(kScanThreads) void tileScanKernel(const uint32_t* __restrict__ tileCount,
    uint32_t* __restrict__ tileOff, int64_t tiles, uint32_t* count)
{
    __shared__ uint32_t scan[33];
    const int t = int(threadIdx.x);
    uint32_t carry = 0;
    for (int64_t r0 = 0; r0 < tiles; r0 += int64_t(kScanThreads) * kScanPer) {
        const int64_t i0 = r0 + int64_t(t) * kScanPer;
        uint32_t v[kScanPer];
        if (i0 + kScanPer <= tiles) {  // four 16-byte loads (the counts start 256-byte aligned)
#pragma unroll
            for (int k = 0; k < kScanPer / 4; ++k) {
                const uint4 x = reinterpret_cast<const uint4*>(tileCount + i0)[k];
                v[4 * k] = x.x;
                v[4 * k + 1] = x.y;
                v[4 * k + 2] = x.z;
                v[4 * k + 3] = x.w;
            }
        } else {
#pragma unroll
            for (int k = 0; k < kScanPer; ++k)
                v[k] = i0 + k < tiles ? tileCount[i0 + k] : 0u;
        }
        uint32_t mine = 0;
#pragma unroll
        for (int k = 0; k < kScanPer; ++k)
            mine += v[k];
        uint32_t total = 0;
        uint32_t run = carry + blockExclusiveSum(mine, total, scan);
#pragma unroll
        for (int k = 0; k < kScanPer; ++k) {
            if (i0 + k < tiles)
                tileOff[i0 + k] = run;
            run += v[k];
        }
        carry += total;
    }
    if (t == 0)
        *count = carry;
}

/** One warp per tile: every leaf whose first rank (a multiple of 4096) falls among
 *  the tile's kept samples gets that sample's index in ``leafStart``. Lane l holds
 *  the tile's words [16 l, 16 l + 16). */
__global__ __launch_bounds__(kThreads) void leafStartKernel(const uint32_t* __restrict__ bitmap,
    const uint32_t* __restrict__ tileCount, const uint32_t* __restrict__ tileOff, int64_t tiles,
    int32_t* __restrict__ leafStart)
{
    const int lane = int(threadIdx.x & 31);
    const int64_t warps = int64_t(gridDim.x) * (kThreads / 32);
    for (int64_t tile = int64_t(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5); tile < tiles; tile += warps) {
        const uint64_t o = tileOff[tile], c = tileCount[tile];
        const uint64_t b0 = (o + uint64_t(kLeaf) - 1) / uint64_t(kLeaf) * uint64_t(kLeaf);
        if (c == 0 || b0 >= o + c)
            continue;  // warp-uniform
        const uint4* src = reinterpret_cast<const uint4*>(bitmap + tile * kTileWords) + lane * 4;
        uint32_t w[16];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint4 x = src[k];
            w[4 * k] = x.x;
            w[4 * k + 1] = x.y;
            w[4 * k + 2] = x.z;
            w[4 * k + 3] = x.w;
        }
        uint32_t mine = 0;
#pragma unroll
        for (int k = 0; k < 16; ++k)
            mine += uint32_t(__popc(w[k]));
        const uint32_t excl = warpInclusiveSum(mine) - mine;
        for (uint64_t b = b0; b < o + c; b += uint64_t(kLeaf)) {
            const uint32_t r = uint32_t(b - o);  // the boundary's rank inside the tile
            if (r >= excl && r < excl + mine) {
                uint32_t rem = r - excl;
                int at = -1;
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    const uint32_t pc = uint32_t(__popc(w[k]));
                    if (at < 0) {
                        if (rem < pc) {
                            uint32_t x = w[k];
                            for (uint32_t d = rem; d > 0; --d)
                                x &= x - 1u;  // drop the lowest kept sample
                            at = (lane * 16 + k) * 32 + __ffs(int(x)) - 1;
                        } else {
                            rem -= pc;
                        }
                    }
                }
                leafStart[b / uint64_t(kLeaf)] = int32_t(tile * kTile + at);
            }
        }
    }
}


/** Pulls the values of samples [s0, s1) into L2 (128-byte lines spread over the
 *  warp) when the range is dense enough that nearly all of its sectors will be
 *  read: at most two samples per survivor. The lines stay inside the values. */
__device__ __forceinline__ void prefetchLeafWarp(const double* values, int64_t n, int64_t s0, int64_t s1, int cnt)
{
    if (s1 - s0 > 2 * int64_t(cnt))
        return;
    const uintptr_t lo = reinterpret_cast<uintptr_t>(values);
    const uintptr_t hi = lo + uintptr_t(n) * sizeof(double);
    uintptr_t p = reinterpret_cast<uintptr_t>(values + s0) & ~uintptr_t(127);
    const uintptr_t e = reinterpret_cast<uintptr_t>(values + s1);
    for (p += uintptr_t(threadIdx.x & 31) * 128; p < e; p += 32 * 128)
        if (p >= lo && p < hi)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

struct LeafArgs {
    const uint32_t* bitmap;
    const int32_t* leafStart;
    const uint32_t* count;
    const double* values;
    int64_t n;
    P* leafPart;          // one partial per leaf
    P* chunkPart;         // one per aligned chunk of kChunk leaves
    uint32_t* chunkDone;  // leaves finished per chunk, zero on entry
    uint32_t* topDone;    // chunks finished, zero on entry
    uint32_t* leafNext;   // the leaf claim counter, zero on entry
    uint32_t* err;        // zero on entry
    double* out;
    int pairOut;
};

constexpr int kLeafWarps = kThreads / 32;
constexpr int kRing = 512;      // a warp's staged values: under 256 waiting + 8 words' worth
constexpr int kBatchWords = 8;  // non-empty bitmap words whose values a lane loads together
constexpr int kSlotsPerLane = kSlots / 32;

/** Pairwise levels over ``m <= 512`` partials at ``in`` (an aligned 512-node
 *  subtree), by one warp: lane l takes nodes [16 l, 16 l + 16) and joins them in
 *  registers (offsets 1..8), then lanes pair up by shuffles (offsets 16..256): the
 *  pairs and order of ``levels``. Result in lane 0. Reads through L2, so partials
 *  that other CTAs published before their counter increment are seen. */
__device__ __forceinline__ P warpLevels(const P* in, int m)
{
    const int lane = int(threadIdx.x & 31);
    P x[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int i = lane * 16 + j;
        x[j] = i < m ? P{__ldcg(&in[i].h), __ldcg(&in[i].c)} : P{};
    }
#pragma unroll
    for (int off = 1; off < 16; off <<= 1)
#pragma unroll
        for (int j = 0; j < 16; j += 2 * off)
            if (lane * 16 + j + off < m)
                x[j] = P::join(x[j], x[j + off]);
    P q = x[0];
#pragma unroll
    for (int lo = 1; lo < 32; lo <<= 1) {
        const P o = q.shflDown(unsigned(lo));
        if ((lane & (2 * lo - 1)) == 0 && (lane + lo) * 16 < m)
            q = P::join(q, o);
    }
    return q;
}

/** One warp sums one leaf: the samples [s0, s1) hold its ``cnt`` survivors. Lane l
 *  owns slots l + 32 i (i < 8). The bitmap words go 32 at a time (one per lane); the
 *  non-empty ones 8 at a time, each lane loading the value of its bit in each (one
 *  coalesced 256-byte row per word), into a ring at the value's rank; every full
 *  row of 256 ranks is folded, slot by slot, in rank order. The fold skips the
 *  non-finite test of each step and applies it once at the end: once a slot's hi
 *  is infinite or NaN it stays so, and its comp ends zero either way; while hi is
 *  finite the comp of a join with (x, 0) is never -0, so adding that 0 is exact. */
__device__ __forceinline__ P sumLeaf(const LeafArgs& a, int64_t s0, int64_t s1, int cnt, double* ring)
{
    const int lane = int(threadIdx.x & 31);
    const uint32_t below = (1u << lane) - 1u;
    const int64_t w0 = s0 >> 5, wEnd = ((s1 - 1) >> 5) + 1;
    double h[kSlotsPerLane], c[kSlotsPerLane];
#pragma unroll
    for (int i = 0; i < kSlotsPerLane; ++i)
        h[i] = c[i] = 0.0;
    uint32_t have = 0, used = 0;  // ranks staged, ranks folded (warp-uniform)
    auto fold = [&](int live) {   // the row at ``used``: slots below ``live`` take a term
        const bool first = used == 0;
#pragma unroll
        for (int i = 0; i < kSlotsPerLane; ++i) {
            if (lane + 32 * i < live) {
                const double x = ring[(used + uint32_t(lane + 32 * i)) & (kRing - 1)];
                if (first) {
                    h[i] = x;
                } else {
                    const double sum = h[i] + x;
                    const double bb = sum - h[i];
                    const double e = (h[i] - (sum - bb)) + (x - bb);
                    c[i] = c[i] + e;
                    h[i] = sum;
                }
            }
        }
    };
    for (int64_t wb = w0; wb < wEnd; wb += 32) {
        uint32_t word = 0;
        const int64_t w = wb + lane;
        if (w < wEnd) {
            word = a.bitmap[w];
            if (w == w0)
                word &= ~0u << (s0 & 31);
            if (w == wEnd - 1) {
                const int e = int((s1 - 1) & 31);
                word &= e == 31 ? ~0u : ((2u << e) - 1u);
            }
        }
        uint32_t nz = __ballot_sync(kFull, word != 0);
        while (nz != 0) {
            double v[kBatchWords];
            uint32_t r[kBatchWords];
#pragma unroll
            for (int b = 0; b < kBatchWords; ++b) {
                const int src = nz != 0 ? __ffs(int(nz)) - 1 : 0;
                const uint32_t wd = __shfl_sync(kFull, word, src) & (nz != 0 ? ~0u : 0u);
                nz &= nz - 1u;
                const bool mine = (wd >> lane) & 1u;
                r[b] = mine ? have + uint32_t(__popc(wd & below)) : 0xffffffffu;
                v[b] = mine ? __ldg(a.values + (wb + src) * 32 + lane) : 0.0;
                have += uint32_t(__popc(wd));
            }
#pragma unroll
            for (int b = 0; b < kBatchWords; ++b)
                if (r[b] < uint32_t(kLeaf))
                    ring[r[b] & (kRing - 1)] = v[b];
            __syncwarp();
            while (have - used >= uint32_t(kSlots) && used < uint32_t(kLeaf)) {
                fold(kSlots);
                used += kSlots;
            }
            __syncwarp();
        }
    }
    if (have != uint32_t(cnt) && lane == 0)
        atomicOr(a.err, 2u);  // the bitmap and the leaf starts disagree
    if (have > used && used < uint32_t(kLeaf))
        fold(int(have - used));  // the last leaf's short row
    __syncwarp();
    // the in-leaf tree over slots l + 32 i: offsets 128, 64, 32 in registers, then shuffles
    const int live = cnt < kSlots ? cnt : kSlots;
    P x[kSlotsPerLane];
#pragma unroll
    for (int i = 0; i < kSlotsPerLane; ++i)
        x[i] = P{h[i], isfinite(h[i]) ? c[i] : 0.0};
#pragma unroll
    for (int i = 0; i < 4; ++i)
        if (lane + 32 * i + 128 < live)
            x[i] = P::join(x[i], x[i + 4]);
#pragma unroll
    for (int i = 0; i < 2; ++i)
        if (lane + 32 * i + 64 < live)
            x[i] = P::join(x[i], x[i + 2]);
    if (lane + 32 < live)
        x[0] = P::join(x[0], x[1]);
    P q = x[0];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const P o = q.shflDown(unsigned(off));
        if (lane < off && lane + off < live)
            q = P::join(q, o);
    }
    return q;
}

/** Warps claim leaves off a counter and sum each alone (no CTA barrier anywhere).
 *  A leaf's partial goes to leafPart; the warp that finishes the last leaf of an
 *  aligned chunk of 512 runs the chunk's pairwise levels, and the warp that
 *  finishes the last chunk the levels above, and stores the value. The next leaf's
 *  value range, when dense, is pulled toward L2 while the current one is summed. */
__global__ __launch_bounds__(kThreads, 3) void keptLeavesKernel(LeafArgs a)
{
    __shared__ double rings[kLeafWarps][kRing];
    const int lane = int(threadIdx.x & 31), warp = int(threadIdx.x >> 5);
    double* ring = rings[warp];
    const int64_t rows = int64_t(*a.count) > a.n ? 0 : int64_t(*a.count);
    const int64_t leaves = (rows + kLeaf - 1) / kLeaf;
    if (leaves == 0) {
        if (blockIdx.x == 0 && threadIdx.x == 0) {
            a.out[0] = 0.0;
            if (a.pairOut)
                a.out[1] = 0.0;
        }
        return;
    }
    const int64_t chunks = (leaves + kChunk - 1) / kChunk;
    auto range = [&](int64_t l, int64_t& s0, int64_t& s1) {
        // kept inside [0, n) whatever the starts hold, so a failed pass reads in bounds
        s0 = a.leafStart[l];
        s0 = s0 < 0 ? 0 : (s0 >= a.n ? a.n - 1 : s0);
        s1 = l + 1 < leaves ? int64_t(a.leafStart[l + 1]) : a.n;
        s1 = s1 <= s0 ? s0 + 1 : (s1 > a.n ? a.n : s1);
    };
    auto claim = [&]() -> int64_t {
        uint32_t l = 0;
        if (lane == 0)
            l = atomicAdd(a.leafNext, 1u);
        return int64_t(__shfl_sync(kFull, l, 0));
    };
    auto cntOf = [&](int64_t l) { return int(rows - l * kLeaf < kLeaf ? rows - l * kLeaf : kLeaf); };
    int64_t l = claim();
    if (l < leaves) {
        int64_t s0, s1;
        range(l, s0, s1);
        prefetchLeafWarp(a.values, a.n, s0, s1, cntOf(l));
    }
    while (l < leaves) {
        const int64_t next = claim();
        if (next < leaves) {
            int64_t n0, n1;
            range(next, n0, n1);
            prefetchLeafWarp(a.values, a.n, n0, n1, cntOf(next));
        }
        int64_t s0, s1;
        range(l, s0, s1);
        const P q = sumLeaf(a, s0, s1, cntOf(l), ring);
        const int64_t ch = l / kChunk;
        const int inChunk = int(leaves - ch * kChunk < kChunk ? leaves - ch * kChunk : kChunk);
        uint32_t last = 0;
        if (lane == 0) {
            a.leafPart[l] = q;
            __threadfence();
            last = atomicAdd(&a.chunkDone[ch], 1u) == uint32_t(inChunk - 1) ? 1u : 0u;
        }
        if (__shfl_sync(kFull, last, 0)) {
            __threadfence();
            const P cp = warpLevels(a.leafPart + ch * kChunk, inChunk);
            uint32_t top = 0;
            if (lane == 0) {
                a.chunkPart[ch] = cp;
                __threadfence();
                top = atomicAdd(a.topDone, 1u) == uint32_t(chunks - 1) ? 1u : 0u;
            }
            if (__shfl_sync(kFull, top, 0)) {
                __threadfence();
                // the levels above the chunks: aligned runs of 512, then the level above
                int64_t m = chunks;
                P* v = a.chunkPart;
                while (m > 1) {
                    const int64_t runs = (m + kChunk - 1) / kChunk;
                    for (int64_t rr = 0; rr < runs; ++rr) {
                        const int cnt = int(m - rr * kChunk < kChunk ? m - rr * kChunk : kChunk);
                        const P r = warpLevels(v + rr * kChunk, cnt);
                        __syncwarp();
                        if (lane == 0)
                            v[rr] = r;
                        __threadfence();
                        __syncwarp();
                    }
                    m = runs;
                }
                if (lane == 0) {
                    const P r{__ldcg(&v[0].h), __ldcg(&v[0].c)};
                    const bool failed = *reinterpret_cast<volatile uint32_t*>(a.err) != 0u;
                    const double nan = __longlong_as_double(0x7ff8000000000000ll);
                    if (a.pairOut) {
                        a.out[0] = failed ? nan : r.h;
                        a.out[1] = failed ? nan : (isfinite(r.h) ? r.c : 0.0);
                    } else {
                        a.out[0] = failed ? nan : r.value();
                    }
                    if (failed)
                        *const_cast<uint32_t*>(a.count) = 0xffffffffu;
                }
            }
        }
        l = next;
    }
}

__global__ void compactSumEmptyKernel(uint32_t* count, double* out, int pairOut)
{
    *count = 0u;
    out[0] = 0.0;
    if (pairOut)
        out[1] = 0.0;
}

/** Scratch of one call over n samples: [leaf claim, chunks finished, error, pad |
 *  leaves finished per chunk] (zeroed by the call's memset), then the tile counts
 *  and offsets, the bitmap, the leaf starts, the leaf partials and the chunk
 *  partials. */
struct SumLayout {
    int64_t tiles = 0;
    int64_t maxLeaves = 0, maxChunks = 0;
    size_t zeroed = 0, tileCount = 0, tileOff = 0, bitmap = 0, leafStart = 0, leafPart = 0, chunkPart = 0,
           total = 0;
};

size_t up(size_t x, size_t a) { return (x + a - 1) / a * a; }

int leavesGrid()
{
    static std::mutex mu;
    static int perSm[64] = {};
    int dev = 0;
    cudaCheck(cudaGetDevice(&dev), "cudaGetDevice");
    std::lock_guard<std::mutex> lock(mu);
    int& k = perSm[dev & 63];
    if (k == 0) {
        cudaCheck(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&k, keptLeavesKernel, kThreads, 0),
            "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
        if (k < 1)
            k = 1;
    }
    return k * smCount();
}

SumLayout sumLayout(int64_t n)
{
    SumLayout L;
    L.tiles = n > 0 ? (n + kTile - 1) / kTile : 1;
    L.maxLeaves = (n + kLeaf - 1) / kLeaf;
    L.maxChunks = (L.maxLeaves + kChunk - 1) / kChunk;
    L.zeroed = up(size_t(4 + L.maxChunks) * sizeof(uint32_t), 16);
    L.tileCount = up(L.zeroed, 256);
    L.tileOff = up(L.tileCount + size_t(L.tiles) * sizeof(uint32_t), 256);
    L.bitmap = up(L.tileOff + size_t(L.tiles) * sizeof(uint32_t), 256);
    L.leafStart = up(L.bitmap + size_t(L.tiles) * kTileWords * sizeof(uint32_t), 256);
    L.leafPart = up(L.leafStart + size_t(L.maxLeaves + 1) * sizeof(int32_t), 256);
    L.chunkPart = up(L.leafPart + size_t(L.maxLeaves > 0 ? L.maxLeaves : 1) * sizeof(P), 256);
    L.total = up(L.chunkPart + size_t(L.maxChunks > 0 ? L.maxChunks : 1) * sizeof(P), 256);
    return L;
}

}  // namespace
}  // namespace eb

using namespace eb;

#define EB_API extern "C" __attribute__((visibility("default")))

EB_API eagle_backend_status eagle_backend_x_b200_compact_sum(struct eagle_backend_compact_desc* desc,
    uint64_t values, uint64_t out, uint32_t flags)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_b200_compact_sum";
        const auto d = readDesc(desc, EAGLE_BACKEND_COMPACT_MASK_IS_DROP, who);
        if (d.n < 0)
            invalid(std::string(who) + ": n must be >= 0");
        if (d.n > INT64_C(2147483647))
            unsupported(std::string(who) + ": at most 2^31-1 samples, got n = " + std::to_string(d.n));
        if (flags & ~uint32_t(EAGLE_BACKEND_REDUCE_PAIR_OUT))
            unsupported(std::string(who) + ": unknown flag bits " + std::to_string(flags));
        if (d.index_map != 0)
            unsupported(std::string(who) + ": writes no index map (eagle_backend_compact_device does)");
        if (d.live32 != 0)
            unsupported(std::string(who) + ": the reorder trigger is not offered with the fused sum");
        const SumLayout L = sumLayout(d.n);
        if (d.scratch == 0) {
            constexpr size_t end = offsetof(eagle_backend_compact_desc, scratch_bytes) + sizeof(int64_t);
            if (desc->struct_size < end)
                invalid(std::string(who) + ": the scratch query needs a desc carrying scratch_bytes");
            desc->scratch_bytes = int64_t(L.total);
            return;
        }
        if (d.count == 0 || out == 0 || (d.n > 0 && (d.mask == 0 || values == 0)))
            invalid(std::string(who) + ": mask, values, out and count must be device addresses");
        if ((values & 7u) != 0 || (out & 7u) != 0)
            invalid(std::string(who) + ": values and out must be 8-byte aligned float64 arrays");
        if ((d.scratch & 255u) != 0)
            invalid(std::string(who) + ": scratch must be 256-byte aligned");
        const int dev = resolveDevice(d.device, d.mask != 0 ? d.mask : d.count);
        DeviceScope scope(dev);
        const cudaStream_t s = seamStream(d.stream);
        const int pairOut = (flags & EAGLE_BACKEND_REDUCE_PAIR_OUT) ? 1 : 0;
        if (d.n == 0) {
            compactSumEmptyKernel<<<1, 1, 0, s>>>(reinterpret_cast<uint32_t*>(d.count), reinterpret_cast<double*>(out),
                pairOut);
            launchCheck(who);
            return;
        }
        char* base = reinterpret_cast<char*>(d.scratch);
        uint32_t* words = reinterpret_cast<uint32_t*>(base);
        uint32_t* tileCount = reinterpret_cast<uint32_t*>(base + L.tileCount);
        uint32_t* tileOff = reinterpret_cast<uint32_t*>(base + L.tileOff);
        uint32_t* bitmap = reinterpret_cast<uint32_t*>(base + L.bitmap);
        int32_t* leafStart = reinterpret_cast<int32_t*>(base + L.leafStart);
        uint32_t* count = reinterpret_cast<uint32_t*>(d.count);
        LeafArgs la{};
        la.bitmap = bitmap;
        la.leafStart = leafStart;
        la.count = count;
        la.values = reinterpret_cast<const double*>(values);
        la.n = d.n;
        la.leafPart = reinterpret_cast<P*>(base + L.leafPart);
        la.chunkPart = reinterpret_cast<P*>(base + L.chunkPart);
        la.leafNext = words;
        la.topDone = words + 1;
        la.err = words + 2;
        la.chunkDone = words + 4;
        la.out = reinterpret_cast<double*>(out);
        la.pairOut = pairOut;
        cudaCheck(cudaMemsetAsync(base, 0, L.zeroed, s), "cudaMemsetAsync");
        const auto mask = reinterpret_cast<const uint8_t*>(d.mask);
        const unsigned tiles = unsigned(L.tiles);
        const bool aligned = (d.mask & 15u) == 0;
        if (d.flags & EAGLE_BACKEND_COMPACT_MASK_IS_DROP)
            aligned ? keepCountKernel<true, true><<<tiles, kThreads, 0, s>>>(mask, d.n, bitmap, tileCount)
                    : keepCountKernel<true, false><<<tiles, kThreads, 0, s>>>(mask, d.n, bitmap, tileCount);
        else
            aligned ? keepCountKernel<false, true><<<tiles, kThreads, 0, s>>>(mask, d.n, bitmap, tileCount)
                    : keepCountKernel<false, false><<<tiles, kThreads, 0, s>>>(mask, d.n, bitmap, tileCount);
        launchCheck(who);
        tileScanKernel<<<1, kScanThreads, 0, s>>>(tileCount, tileOff, L.tiles, count);
        launchCheck(who);
        const int64_t warpsPerCta = kThreads / 32;
        const int64_t startCtas = (L.tiles + warpsPerCta - 1) / warpsPerCta;
        const int64_t startCap = int64_t(smCount()) * 8;
        leafStartKernel<<<unsigned(startCtas < startCap ? startCtas : startCap), kThreads, 0, s>>>(bitmap, tileCount,
            tileOff, L.tiles, leafStart);
        launchCheck(who);
        keptLeavesKernel<<<unsigned(leavesGrid()), kThreads, 0, s>>>(la);
        launchCheck(who);
    });
}
