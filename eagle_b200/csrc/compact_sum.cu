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
constexpr int kMaxK = 4;                          // bitmap words per thread per chunk, at most
constexpr int kMaxGroup = 128;                    // leaves a group holds at most
constexpr int kGroupsPerCta = 8;                  // groups per CTA the claim aims at
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
        uint32_t mine = 0;
#pragma unroll
        for (int k = 0; k < kScanPer; ++k) {
            v[k] = i0 + k < tiles ? tileCount[i0 + k] : 0u;
            mine += v[k];
        }
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

struct LeafArgs {
    const uint32_t* bitmap;
    const int32_t* leafStart;
    const uint32_t* count;
    const double* values;
    int64_t n;
    P* partials;          // one per claimed group
    uint32_t groupCap;    // partials' capacity
    uint32_t* groupNext;  // zero on entry
    uint32_t* done;       // zero on entry
    uint32_t* err;        // zero on entry
    double* out;
    int pairOut;
};

/** Bitmap words [cw + t K, cw + t K + K) of a leaf whose samples are [s0, s1):
 *  bits outside the leaf cleared (they belong to its neighbours). */
__device__ __forceinline__ void leafWords(const uint32_t* __restrict__ bitmap, int64_t cw, int K, int64_t s0,
    int64_t s1, uint32_t (&wd)[kMaxK])
{
    const int64_t w0 = s0 >> 5, wEnd = ((s1 - 1) >> 5) + 1;
#pragma unroll
    for (int k = 0; k < kMaxK; ++k) {
        uint32_t x = 0;
        const int64_t w = cw + int64_t(threadIdx.x) * K + k;
        if (k < K && w < wEnd) {
            x = bitmap[w];
            if (w == w0)
                x &= ~0u << (s0 & 31);
            if (w == wEnd - 1) {
                const int e = int((s1 - 1) & 31);
                x &= e == 31 ? ~0u : ((2u << e) - 1u);
            }
        }
        wd[k] = x;
    }
}

/** Words per thread for a leaf over [s0, s1): one chunk of 256 K words covers it
 *  when K <= kMaxK does. */
__device__ __forceinline__ int wordsPerThread(int64_t s0, int64_t s1)
{
    const int64_t words = ((s1 - 1) >> 5) - (s0 >> 5) + 1;
    int K = 1;
    while (K < kMaxK && int64_t(K) * kThreads < words)
        K *= 2;
    return K;
}

__global__ __launch_bounds__(kThreads, 4) void keptLeavesKernel(LeafArgs a)
{
    __shared__ __align__(16) int32_t idx[kLeaf];  // the leaf's kept samples by rank; the final levels reuse it
    __shared__ P s[2][kSlots];      // the slot partials of the last two leaves
    __shared__ P group[kMaxGroup];
    __shared__ int32_t sStart[kMaxGroup + 1];
    __shared__ uint32_t scan[33];
    __shared__ uint32_t sGroup;
    __shared__ int amLast;
    const int t = int(threadIdx.x);
    const int64_t rows = int64_t(*a.count) > a.n ? 0 : int64_t(*a.count);
    const int64_t leaves = (rows + kLeaf - 1) / kLeaf;
    int64_t gl = 1;  // leaves per group: a power of two, so a group is a subtree of the levels
    while (gl < kMaxGroup && (leaves + gl - 1) / gl > int64_t(a.groupCap))
        gl *= 2;
    while (gl < kMaxGroup && (leaves + gl - 1) / gl > int64_t(gridDim.x) * kGroupsPerCta)
        gl *= 2;
    const int64_t groups = (leaves + gl - 1) / gl;
    int parity = 0;  // the slot buffer the next in-leaf tree takes
    for (;;) {
        if (t == 0)
            sGroup = atomicAdd(a.groupNext, 1u);
        __syncthreads();
        const int64_t g = int64_t(sGroup);
        if (g >= groups)
            break;
        const int64_t l0 = g * gl;
        const int64_t l1 = l0 + gl < leaves ? l0 + gl : leaves;
        // the group's leaf starts, kept inside [0, n] so that any start reads in bounds
        for (int64_t i = t; i <= l1 - l0; i += kThreads) {
            int64_t v = l0 + i < leaves ? int64_t(a.leafStart[l0 + i]) : a.n;
            v = v < 0 ? 0 : (v > a.n ? a.n : v);
            sStart[i] = int32_t(v);
        }
        __syncthreads();  // sStart is read below; sGroup is rewritten only after a later barrier
        uint32_t word[kMaxK];
        {
            const int64_t s0 = sStart[0] < a.n ? sStart[0] : a.n - 1;
            const int64_t s1 = sStart[1] > s0 ? sStart[1] : s0 + 1;
            leafWords(a.bitmap, s0 >> 5, wordsPerThread(s0, s1), s0, s1, word);
        }
        for (int64_t l = l0; l < l1; ++l) {
            const int64_t s0 = sStart[l - l0] < a.n ? sStart[l - l0] : a.n - 1;
            const int64_t s1 = sStart[l - l0 + 1] > s0 ? sStart[l - l0 + 1] : s0 + 1;
            const int cnt = int(rows - l * kLeaf < kLeaf ? rows - l * kLeaf : kLeaf);
            const int K = wordsPerThread(s0, s1);
            const int64_t wEnd = ((s1 - 1) >> 5) + 1;
            uint32_t base = 0;
            for (int64_t cw = s0 >> 5;;) {
                uint32_t mine = 0;
#pragma unroll
                for (int k = 0; k < kMaxK; ++k)
                    mine += uint32_t(__popc(word[k]));
                uint32_t total = 0;
                uint32_t r = base + blockExclusiveSum(mine, total, scan);
#pragma unroll
                for (int k = 0; k < kMaxK; ++k) {
                    uint32_t x = word[k];
                    const int64_t sample0 = (cw + int64_t(t) * K + k) * 32;
                    while (x != 0) {
                        if (r < uint32_t(kLeaf))
                            idx[r] = int32_t(sample0 + __ffs(int(x)) - 1);
                        x &= x - 1u;
                        ++r;
                    }
                }
                base += total;
                cw += int64_t(kThreads) * K;
                if (cw >= wEnd)
                    break;
                leafWords(a.bitmap, cw, K, s0, s1, word);  // a sparse leaf's next chunk
            }
            if (t == 0 && int(base) != cnt)
                atomicOr(a.err, 2u);  // the bitmap and the leaf starts disagree
            __syncthreads();          // idx holds the leaf
            if (l + 1 < l1) {         // the next leaf's first words go out now
                const int64_t n0 = sStart[l - l0 + 1] < a.n ? sStart[l - l0 + 1] : a.n - 1;
                const int64_t n1 = sStart[l - l0 + 2] > n0 ? sStart[l - l0 + 2] : n0 + 1;
                leafWords(a.bitmap, n0 >> 5, wordsPerThread(n0, n1), n0, n1, word);
            }
            double v[kTerms];
            if (cnt == int(kLeaf) && int(base) == cnt) {
#pragma unroll
                for (int i = 0; i < kTerms; ++i)
                    v[i] = __ldg(a.values + idx[t + i * kSlots]);
            } else {
                const int have = int(base) < cnt ? int(base) : cnt;  // staged entries only
#pragma unroll
                for (int i = 0; i < kTerms; ++i)
                    v[i] = t + i * kSlots < have ? __ldg(a.values + idx[t + i * kSlots]) : 0.0;
            }
            P slot = P::of(v[0]);
#pragma unroll
            for (int i = 1; i < kTerms; ++i)
                if (t + i * kSlots < cnt)
                    slot.add(v[i]);
            const P q = leafTreeWarp0(slot, cnt < kSlots ? cnt : kSlots, s[parity]);
            parity ^= 1;
            if (t == 0)
                group[l - l0] = q;
        }
        __syncthreads();
        levels(group, int(l1 - l0));
        if (t == 0)
            a.partials[g] = group[0];
    }
    if (t == 0) {
        __threadfence();
        amLast = atomicAdd(a.done, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!amLast)
        return;
    __threadfence();
    P* buf = reinterpret_cast<P*>(idx);
    P* v = a.partials;
    int64_t m = groups;
    while (m > 1) {
        const int64_t chunks = (m + kChunk - 1) / kChunk;
        for (int64_t cc = 0; cc < chunks; ++cc) {
            const int cnt = int(m - cc * kChunk < kChunk ? m - cc * kChunk : kChunk);
            for (int i = t; i < cnt; i += kThreads)
                buf[i] = v[cc * kChunk + i];
            __syncthreads();
            levels(buf, cnt);
            if (t == 0)
                v[cc] = buf[0];
            __syncthreads();
        }
        m = chunks;
    }
    if (t == 0) {
        const bool failed = *a.err != 0u;
        P r{0.0, 0.0};
        if (groups > 0)
            r = v[0];
        const double nan = __longlong_as_double(0x7ff8000000000000ll);
        if (a.pairOut) {
            a.out[0] = failed ? nan : r.h;
            a.out[1] = failed ? nan : (isfinite(r.h) ? r.c : 0.0);
        } else {
            a.out[0] = failed ? nan : (groups > 0 ? r.value() : 0.0);
        }
        if (failed)
            *const_cast<uint32_t*>(a.count) = 0xffffffffu;
        *a.groupNext = 0u;
        *a.done = 0u;
    }
}

__global__ void compactSumEmptyKernel(uint32_t* count, double* out, int pairOut)
{
    *count = 0u;
    out[0] = 0.0;
    if (pairOut)
        out[1] = 0.0;
}

/** Scratch of one call over n samples: [3 counter words | pad] (zeroed by the
 *  call's memset), then the tile counts and offsets, the bitmap, the leaf starts
 *  and the group partials. */
struct SumLayout {
    int64_t tiles = 0;
    int64_t maxLeaves = 0;
    uint32_t groupCap = 0;
    size_t zeroed = 0, tileCount = 0, tileOff = 0, bitmap = 0, leafStart = 0, partials = 0, total = 0;
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

SumLayout sumLayout(int64_t n, int grid)
{
    SumLayout L;
    L.tiles = n > 0 ? (n + kTile - 1) / kTile : 1;
    L.maxLeaves = (n + kLeaf - 1) / kLeaf;
    const int64_t byGroup = (L.maxLeaves + kMaxGroup - 1) / kMaxGroup;
    const int64_t target = int64_t(grid) * kGroupsPerCta;
    L.groupCap = uint32_t((byGroup > target ? byGroup : target) + 1);
    L.zeroed = 4 * sizeof(uint32_t);
    L.tileCount = 256;
    L.tileOff = up(L.tileCount + size_t(L.tiles) * sizeof(uint32_t), 256);
    L.bitmap = up(L.tileOff + size_t(L.tiles) * sizeof(uint32_t), 256);
    L.leafStart = up(L.bitmap + size_t(L.tiles) * kTileWords * sizeof(uint32_t), 256);
    L.partials = up(L.leafStart + size_t(L.maxLeaves + 1) * sizeof(int32_t), 256);
    L.total = up(L.partials + size_t(L.groupCap) * sizeof(P), 256);
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
        const int dev = resolveDevice(d.device, d.mask != 0 ? d.mask : (d.count != 0 ? d.count : out));
        DeviceScope scope(dev);
        const SumLayout L = sumLayout(d.n, leavesGrid());
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
        la.partials = reinterpret_cast<P*>(base + L.partials);
        la.groupCap = L.groupCap;
        la.groupNext = words;
        la.done = words + 1;
        la.err = words + 2;
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
