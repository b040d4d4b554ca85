// Compact-then-sum without materialising the survivors.
//
// The canonical sum of the samples a mask keeps (eagle's ActiveSet.compact, then
// the ``ordered`` reduction over the compacted plane: python/eagle/_active_set.py:482-525,
// eagle/reduce/canonical.h:10-32) depends on each kept value's RANK among the
// survivors: leaf l holds ranks [4096 l, 4096 l + 4096). Writing the survivors out
// and reading them back costs 16 bytes per survivor on top of the mask and the value
// sectors, the whole gap between a compaction and its roofline. Two kernels after
// one memset instead:
//
//   keepBitsKernel    one 16384-sample tile per CTA (four coalesced rows of 4096 mask
//                     bytes): the keep bits go out as a bitmap (one bit per sample),
//                     a decoupled look-back gives the tile's first rank, and the
//                     thread holding rank 4096 l writes leafStart[l], the sample where
//                     leaf l begins. The last tile writes the count.
//   keptLeavesKernel  CTAs claim groups of 2^q consecutive leaves. Per leaf: the
//                     bitmap words over [leafStart[l], leafStart[l + 1]) are scanned
//                     across the CTA, each warp reads 32 consecutive samples' values
//                     (one coalesced 256-byte row, a lane loading only where its bit
//                     is set) into a shared-memory stage at their in-leaf rank, and
//                     the stage goes through the same leaf walk as the reduction's.
//                     The group's leaves join by the pairwise levels; the last CTA
//                     runs the remaining levels over the group partials.
//
// Traffic: the mask (n bytes), the bitmap written and read (n / 4 bytes), the
// value sectors holding a survivor; the bits are those of the two-kernel
// compaction + canonical sum, which the tests check against the oracle.
#include "canonical.cuh"

#include <mutex>

namespace eb {
namespace {

constexpr int kThreads = 256;
constexpr int kRows = 4;
constexpr int64_t kRow = int64_t(kThreads) * 16;  // 4096 samples: 16 mask bytes per thread
constexpr int64_t kTile = kRow * kRows;           // 16384 samples per keepBits CTA
constexpr int64_t kTileWords = kTile / 32;        // its bitmap words
constexpr int kMaxK = 4;                          // bitmap words per thread per chunk, at most
constexpr int kCap = 8192;                        // kept sample indices one pass stages
constexpr int kMaxGroup = 128;                    // leaves a group holds at most
constexpr int kGroupsPerCta = 8;                  // groups per CTA the claim aims at

using P = CompP<double>;

struct KeepArgs {
    const uint8_t* mask;
    int64_t n;
    uint32_t tiles;
    uint32_t* bitmap;    // tiles * kTileWords words; bit j of word w: sample 32 w + j is kept
    int32_t* leafStart;  // leafStart[l]: the sample holding kept rank 4096 l
    uint32_t* count;
    uint64_t* status;    // one look-back word per tile, zero on entry
    uint32_t* tileNext;  // zero on entry
    uint32_t* err;       // zero on entry
};

template <bool Drop, bool Aligned>
__global__ __launch_bounds__(kThreads) void keepBitsKernel(KeepArgs a)
{
    __shared__ uint32_t sTile;
    __shared__ uint64_t scan64[33];
    __shared__ uint32_t firstOf[32];
    const int t = int(threadIdx.x);
    if (t == 0)
        sTile = atomicAdd(a.tileNext, 1u);
    __syncthreads();
    const uint32_t tile = sTile;
    const int64_t tile0 = int64_t(tile) * kTile;
    uint32_t bits[kRows];
    uint64_t packed = 0;  // row q's count in bits [16q, 16q + 16)
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
        bits[q] = keepBits16<Drop, Aligned>(a.mask, tile0 + int64_t(q) * kRow + int64_t(t) * 16, a.n);
        packed |= uint64_t(__popc(bits[q])) << (16 * q);
    }
    // threads 2u and 2u + 1 hold the low and high halves of one 32-sample word
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
        const uint32_t hi = __shfl_down_sync(kFull, bits[q], 1);
        if ((t & 1) == 0)
            a.bitmap[int64_t(tile) * kTileWords + q * (kRow / 32) + (t >> 1)] = bits[q] | (hi << 16);
    }
    uint64_t rowTotals = 0;
    const uint64_t excl = blockExclusiveSum(packed, rowTotals, scan64);
    uint32_t total = 0;
#pragma unroll
    for (int q = 0; q < kRows; ++q)
        total += uint32_t(rowTotals >> (16 * q)) & 0xffffu;
    uint64_t prefix = 0;
    if (tile == 0) {
        if (t == 0)
            lbPublish<PlainCodec>(a.status, tile, 0, kLbPrefix, total);
    } else {
        if (t == 0)
            lbPublish<PlainCodec>(a.status, tile, 0, kLbAggregate, total);
        prefix = lbExclusivePrefixBlock<PlainCodec>(a.status, tile, 0, a.err, firstOf, scan64);
        if (t == 0)
            lbPublish<PlainCodec>(a.status, tile, 0, kLbPrefix, prefix + total);
    }
    // a leaf starts at every kept rank that is a multiple of 4096; a thread's 16
    // samples of a row hold at most one such rank
    uint64_t rowBase = prefix;
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
        const uint32_t c = uint32_t(__popc(bits[q]));
        const uint64_t g0 = rowBase + ((excl >> (16 * q)) & 0xffffu);
        const uint64_t b = (g0 + uint64_t(kLeaf) - 1) / uint64_t(kLeaf) * uint64_t(kLeaf);
        if (c != 0 && b < g0 + c) {
            uint32_t w = bits[q];
            for (uint64_t r = b - g0; r > 0; --r)
                w &= w - 1u;  // drop the lowest kept sample
            const int j = __ffs(int(w)) - 1;
            a.leafStart[b / uint64_t(kLeaf)] = int32_t(tile0 + int64_t(q) * kRow + int64_t(t) * 16 + j);
        }
        rowBase += (rowTotals >> (16 * q)) & 0xffffu;
    }
    if (tile == a.tiles - 1 && t == 0)
        *a.count = *a.err != 0u ? 0xffffffffu : uint32_t(prefix) + total;  // above n: a failed pass
}

struct LeafArgs {
    const uint32_t* bitmap;
    const int32_t* leafStart;
    const uint32_t* count;
    const double* values;
    int64_t n;
    P* partials;         // one per claimed group
    uint32_t groupCap;   // partials' capacity
    uint32_t* groupNext; // zero on entry
    uint32_t* done;      // zero on entry
    uint32_t* err;
    double* out;
    int pairOut;
};

/** Bitmap words [cw + t K, cw + t K + K) of a group whose samples are [s0, s1):
 *  bits outside the group cleared (they belong to the leaves on either side). */
__device__ __forceinline__ void groupWords(const uint32_t* __restrict__ bitmap, int64_t cw, int K, int64_t s0,
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

/** CTAs claim groups of 2^q consecutive leaves off a counter. A group's survivors
 *  are one stream: positions 0, 1, ... in rank order, leaf = position / 4096, row =
 *  position / 256, slot = position % 256, so thread t owns slot t of every row and
 *  folds its values into its slot's partial in row order -- the leaf walk, term by
 *  term, with no value ever staged. Per chunk of 256 K bitmap words (K grows as the
 *  group thins out, so a chunk holds about 8192 survivors): a CTA scan of the
 *  words' counts, the kept sample indices staged in shared memory by rank, then
 *  rows in batches of 16, each thread loading its slot's value of every row
 *  together (consecutive threads, consecutive survivors: coalesced where the mask
 *  is dense). A row that ends a leaf runs the in-leaf tree. The next chunk's words
 *  are in flight while the current one is summed. */
__global__ __launch_bounds__(kThreads, 4) void keptLeavesKernel(LeafArgs a)
{
    __shared__ int32_t idx[kCap];  // a pass's kept samples by rank; the final levels reuse it
    __shared__ P s[2][kSlots];     // the slot partials of the last two leaves
    __shared__ P group[kMaxGroup];
    __shared__ uint32_t scan[33];
    __shared__ uint32_t sGroup;
    __shared__ int amLast;
    const int t = int(threadIdx.x);
    const uint32_t c = *a.count;
    const int64_t rows = int64_t(c) > a.n ? 0 : int64_t(c);
    const int64_t leaves = (rows + kLeaf - 1) / kLeaf;
    int64_t gl = 1;  // leaves per group: a power of two, so a group is a subtree of the levels
    while (gl < kMaxGroup && (leaves + gl - 1) / gl > int64_t(a.groupCap))
        gl *= 2;
    while (gl < kMaxGroup && (leaves + gl - 1) / gl > int64_t(gridDim.x) * kGroupsPerCta)
        gl *= 2;
    const int64_t groups = (leaves + gl - 1) / gl;
    for (;;) {
        if (t == 0)
            sGroup = atomicAdd(a.groupNext, 1u);
        __syncthreads();
        const int64_t g = int64_t(sGroup);
        __syncthreads();
        if (g >= groups)
            break;
        const int64_t l0 = g * gl;
        const int64_t l1 = l0 + gl < leaves ? l0 + gl : leaves;
        const int64_t want = rows - l0 * kLeaf < (l1 - l0) * kLeaf ? rows - l0 * kLeaf : (l1 - l0) * kLeaf;
        // kept inside [0, n) whatever the starts hold, so a failed pass reads in bounds
        int64_t s0 = a.leafStart[l0];
        s0 = s0 < 0 ? 0 : (s0 >= a.n ? a.n - 1 : s0);
        int64_t s1 = l1 < leaves ? int64_t(a.leafStart[l1]) : a.n;
        s1 = s1 <= s0 ? s0 + 1 : (s1 > a.n ? a.n : s1);
        const int64_t w0 = s0 >> 5, wEnd = ((s1 - 1) >> 5) + 1;
        int K = 1;
        while (K < kMaxK && int64_t(2 * K) * want <= s1 - s0)
            K *= 2;
        const int64_t chunkWords = int64_t(kThreads) * K;
        P slot{};
        int parity = 0;        // the slot buffer the next in-leaf tree takes
        int done = 0;          // survivors of the group folded so far (at most 128 leaves' worth)
        int64_t leaf = l0;     // the leaf being folded
        uint32_t word[kMaxK];
        groupWords(a.bitmap, w0, K, s0, s1, word);
        for (int64_t cw = w0; cw < wEnd; cw += chunkWords) {
            uint32_t next[kMaxK];
            groupWords(a.bitmap, cw + chunkWords, K, s0, s1, next);
            uint32_t mine = 0;
#pragma unroll
            for (int k = 0; k < kMaxK; ++k)
                mine += uint32_t(__popc(word[k]));
            uint32_t total = 0;
            const uint32_t base = blockExclusiveSum(mine, total, scan);
            for (uint32_t p0 = 0; p0 < total; p0 += kCap) {
                if (mine != 0 && base < p0 + kCap && base + mine > p0) {
                    uint32_t r = base;
#pragma unroll
                    for (int k = 0; k < kMaxK; ++k) {
                        uint32_t x = word[k];
                        const int64_t sample0 = (cw + int64_t(t) * K + k) * 32;
                        while (x != 0) {
                            const int j = __ffs(int(x)) - 1;
                            x &= x - 1u;
                            if (r >= p0 && r < p0 + kCap)
                                idx[r - p0] = int32_t(sample0 + j);
                            ++r;
                        }
                    }
                }
                __syncthreads();
                const int m = total - p0 < uint32_t(kCap) ? int(total - p0) : kCap;
                const int rowEnd = (done + m - 1) / kSlots;  // the last row this pass touches
                // one leaf's 16 rows per batch (a group starts on a leaf), so only the
                // batch's last row can end a leaf
                for (int rowA = (done / kSlots) & ~(kTerms - 1); rowA <= rowEnd; rowA += kTerms) {
                    double v[kTerms];
                    const int first = rowA * kSlots + t - done;  // this thread's value of row rowA, by pass rank
#pragma unroll
                    for (int i = 0; i < kTerms; ++i) {
                        const int local = first + i * kSlots;
                        v[i] = (local >= 0 && local < m) ? __ldg(a.values + idx[local]) : 0.0;
                    }
#pragma unroll
                    for (int i = 0; i < kTerms; ++i) {
                        const int local = first + i * kSlots;
                        if (local >= 0 && local < m) {
                            if (i == 0)
                                slot = P::of(v[i]);
                            else
                                slot.add(v[i]);
                        }
                    }
                    if ((rowA + kTerms) * kSlots <= done + m) {  // the leaf's last row is in
                        const P q = leafTreeWarp0(slot, kSlots, s[parity]);
                        parity ^= 1;
                        if (t == 0 && leaf < l1)
                            group[leaf - l0] = q;
                        ++leaf;
                    }
                }
                done += m;
                __syncthreads();  // idx is rewritten by the next pass
            }
#pragma unroll
            for (int k = 0; k < kMaxK; ++k)
                word[k] = next[k];
        }
        if (want % kLeaf != 0) {  // the last leaf of all, short of 4096
            const int cnt = int(want % kLeaf);
            const P q = leafTreeWarp0(slot, cnt < kSlots ? int(cnt) : kSlots, s[parity]);
            parity ^= 1;
            if (t == 0 && leaf < l1)
                group[leaf - l0] = q;
            ++leaf;
        }
        if (t == 0 && (done != want || leaf != l1))
            atomicOr(a.err, 2u);  // the bitmap and the leaf starts disagree
        __syncthreads();
        levels(group, int(l1 - l0));
        if (t == 0)
            a.partials[g] = group[0];
        __syncthreads();
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
        const bool failed = int64_t(c) > a.n || *a.err != 0u;
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

/** Scratch of one call over n samples: [status words | 4 counters] (zeroed by the
 *  call's memset), then the bitmap, the leaf starts and the group partials. */
struct SumLayout {
    uint32_t tiles = 0;
    int64_t maxLeaves = 0;
    uint32_t groupCap = 0;
    size_t zeroed = 0, bitmap = 0, leafStart = 0, partials = 0, total = 0;
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
    L.tiles = uint32_t(n > 0 ? (n + kTile - 1) / kTile : 1);
    L.maxLeaves = (n + kLeaf - 1) / kLeaf;
    const int64_t byGroup = (L.maxLeaves + kMaxGroup - 1) / kMaxGroup;
    const int64_t target = int64_t(grid) * kGroupsPerCta;
    L.groupCap = uint32_t((byGroup > target ? byGroup : target) + 1);
    L.zeroed = size_t(L.tiles) * sizeof(uint64_t) + 4 * sizeof(uint32_t);
    L.bitmap = up(L.zeroed, 256);
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
        uint32_t* words = reinterpret_cast<uint32_t*>(base + size_t(L.tiles) * sizeof(uint64_t));
        KeepArgs k{};
        k.mask = reinterpret_cast<const uint8_t*>(d.mask);
        k.n = d.n;
        k.tiles = L.tiles;
        k.bitmap = reinterpret_cast<uint32_t*>(base + L.bitmap);
        k.leafStart = reinterpret_cast<int32_t*>(base + L.leafStart);
        k.count = reinterpret_cast<uint32_t*>(d.count);
        k.status = reinterpret_cast<uint64_t*>(base);
        k.tileNext = words;
        k.err = words + 1;
        LeafArgs la{};
        la.bitmap = k.bitmap;
        la.leafStart = k.leafStart;
        la.count = k.count;
        la.values = reinterpret_cast<const double*>(values);
        la.n = d.n;
        la.partials = reinterpret_cast<P*>(base + L.partials);
        la.groupCap = L.groupCap;
        la.groupNext = words + 2;
        la.done = words + 3;
        la.err = words + 1;
        la.out = reinterpret_cast<double*>(out);
        la.pairOut = pairOut;
        cudaCheck(cudaMemsetAsync(base, 0, L.zeroed, s), "cudaMemsetAsync");
        const bool aligned = (d.mask & 15u) == 0;
        const bool drop = (d.flags & EAGLE_BACKEND_COMPACT_MASK_IS_DROP) != 0;
        if (drop)
            aligned ? keepBitsKernel<true, true><<<L.tiles, kThreads, 0, s>>>(k)
                    : keepBitsKernel<true, false><<<L.tiles, kThreads, 0, s>>>(k);
        else
            aligned ? keepBitsKernel<false, true><<<L.tiles, kThreads, 0, s>>>(k)
                    : keepBitsKernel<false, false><<<L.tiles, kThreads, 0, s>>>(k);
        launchCheck(who);
        keptLeavesKernel<<<unsigned(leavesGrid()), kThreads, 0, s>>>(la);
        launchCheck(who);
    });
}
