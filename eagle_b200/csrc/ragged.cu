// The canonical sum of a compaction's survivors spread over several ranks, with no
// host round trip.
//
// After a compaction on every rank, rank r holds c_r survivors in sample order; the
// survivors of all ranks, concatenated in rank order, are the one-device compaction
// of the whole batch, and its canonical sum is the pairwise tree over 4096-survivor
// leaves of that concatenation (eagle/reduce/canonical.h:10-32). Rank r starts at
// o_r = c_0 + ... + c_{r-1}, which no rank knows before the counts are exchanged, so
// a rank's leaves are not aligned to its own survivors. The exchange here is two
// fixed-size all-gathers -- every rank's head block (its first 4095 survivors and its
// count), then its partial block (its leaf partials and their number) -- around
// kernels that read the gathered blocks on the device:
//
//   raggedHeadKernel    this rank's head block from its survivors;
//   raggedLeavesKernel  one CTA per leaf that STARTS in this rank's part: the leaf's
//                       survivors come from this rank, and past its end from the
//                       next ranks' gathered heads (a leaf that starts here ends
//                       within 4095 survivors of this rank's end);
//   raggedChunkKernel   every rank's leaf partials, in rank order (the order of the
//   raggedTopKernel     leaves), through the pairwise levels: aligned chunks of 512
//                       leaves by one CTA each, then the levels above by one CTA.
//
// Every rank runs the same fold over the same gathered partials, so every rank gets
// the bits of the one-device compact-then-sum, at any rank count.
#include "canonical.cuh"

#define EB_API extern "C" __attribute__((visibility("default")))

namespace eb {
namespace {

struct RaggedLeavesArgs {
    const double* kept;    // this rank's survivors, sample order
    const double* blocks;  // every rank's head block (gathered), [world][kHeadBlock]
    int32_t rank, world;
    double* partials;      // out: this rank's partial block (partialBlock(cap) doubles)
    int64_t cap;           // leaves the partial block holds
};

/** This rank's head block: its first min(count, kHead) survivors and its count. */
__global__ __launch_bounds__(256) void raggedHeadKernel(const double* __restrict__ kept,
    const uint32_t* __restrict__ count, double* __restrict__ block)
{
    const uint32_t c = *count;
    const int64_t len = int64_t(c) < kHead ? int64_t(c) : kHead;
    for (int64_t i = threadIdx.x; i < len; i += blockDim.x)
        block[i] = kept[i];
    if (threadIdx.x == 0)
        block[kHead] = countSlot(c);
}

__global__ __launch_bounds__(kSlots) void raggedLeavesKernel(RaggedLeavesArgs a)
{
    __shared__ int64_t sOff[kMaxRanks + 1];  // sOff[q] = first survivor of rank q; sOff[world] = total
    __shared__ CompP<double> s[kSlots];
    if (threadIdx.x == 0) {
        int64_t o = 0;
        for (int q = 0; q < a.world; ++q) {
            sOff[q] = o;
            o += int64_t(blockCount(a.blocks, q));
        }
        sOff[a.world] = o;
    }
    __syncthreads();
    const int64_t mine = sOff[a.rank], end = sOff[a.rank + 1], total = sOff[a.world];
    const int64_t first = (mine + kLeaf - 1) / kLeaf;  // the first leaf starting at or after ``mine``
    const int64_t leaves = end > first * kLeaf ? (end - first * kLeaf + kLeaf - 1) / kLeaf : 0;
    if (blockIdx.x == 0 && threadIdx.x == 0)
        a.partials[2 * a.cap] = countSlot(uint32_t(leaves));  // above cap: the fold reports the overflow
    const int64_t k = blockIdx.x;
    if (k >= leaves || k >= a.cap)
        return;
    const int64_t start = (first + k) * kLeaf;  // global position of the leaf's first survivor
    const int64_t cnt = total - start < kLeaf ? total - start : kLeaf;
    const double* blocks = a.blocks;
    const int32_t rank = a.rank, world = a.world;
    CompP<double> p;
    if (start + cnt <= end) {  // the whole leaf is this rank's (every leaf but the last)
        const double* mineLeaf = a.kept + (start - mine);
        p = leafPartialAt<CompP<double>, double>([&](int64_t i) { return mineLeaf[i]; }, cnt, s);
    } else {
        const double* kept = a.kept;
        auto at = [&](int64_t i) -> double {
            const int64_t g = start + i;
            if (g < end)
                return kept[g - mine];
            int q = rank + 1;  // a later rank's head: g - sOff[q] < kHead for the rank holding g
            while (q + 1 < world && g >= sOff[q + 1])
                ++q;
            return blockHead(blocks, q, g - sOff[q]);
        };
        p = leafPartialAt<CompP<double>, double>(at, cnt, s);
    }
    if (threadIdx.x == 0) {
        a.partials[2 * k] = p.h;
        a.partials[2 * k + 1] = p.c;
    }
}

/** Rank q's leaf count from the gathered partial blocks. */
__device__ __forceinline__ int64_t leafCountOf(const double* __restrict__ gathered, int q, int64_t cap)
{
    return int64_t(uint32_t(__double_as_longlong(gathered[int64_t(q) * partialBlock(cap) + 2 * cap])));
}

/** Rank q's first leaf in the whole order (sFirst[q]; sFirst[world] = all leaves) and
 *  whether some rank formed more leaves than ``cap`` holds, in shared memory. */
__device__ __forceinline__ void leafOrigins(const double* __restrict__ gathered, int32_t world, int64_t cap,
    int64_t* sFirst, int* sOver)
{
    if (threadIdx.x == 0) {
        int64_t o = 0;
        int over = 0;
        for (int q = 0; q < world; ++q) {
            const int64_t k = leafCountOf(gathered, q, cap);
            sFirst[q] = o;
            o += k;
            over |= k > cap ? 1 : 0;
        }
        sFirst[world] = o;
        *sOver = over;
    }
    __syncthreads();
}

/** The first level of the fold: CTA c joins leaves [512 c, 512 c + 512) of the whole
 *  order (rank q's partials lead its block at ``gathered + partialBlock(cap) q``) by
 *  the pairwise levels into work[2 c, 2 c + 1]. */
__global__ __launch_bounds__(kSlots) void raggedChunkKernel(const double* __restrict__ gathered, int32_t world,
    int64_t cap, double* __restrict__ work)
{
    __shared__ CompP<double> v[kChunk];
    __shared__ int64_t sFirst[kMaxRanks + 1];
    __shared__ int sOver;
    leafOrigins(gathered, world, cap, sFirst, &sOver);
    const int64_t count = sFirst[world];
    const int64_t c = blockIdx.x;
    if (sOver != 0 || c * kChunk >= count)
        return;
    const int cnt = int(count - c * kChunk < kChunk ? count - c * kChunk : kChunk);
    for (int i = int(threadIdx.x); i < cnt; i += int(blockDim.x)) {
        const int64_t j = c * kChunk + i;
        int q = 0;  // the rank whose leaves hold j
        while (q + 1 < world && j >= sFirst[q + 1])
            ++q;
        const double* src = gathered + partialBlock(cap) * q + 2 * (j - sFirst[q]);
        v[i] = CompP<double>{src[0], src[1]};
    }
    __syncthreads();
    levels(v, cnt);
    if (threadIdx.x == 0) {
        work[2 * c] = v[0].h;
        work[2 * c + 1] = v[0].c;
    }
}

/** The levels above the chunks, one CTA: out = {hi, comp, value}; no leaves: zeros;
 *  some rank's leaves past ``cap``: NaN. */
__global__ __launch_bounds__(kSlots) void raggedTopKernel(const double* __restrict__ gathered, int32_t world,
    int64_t cap, double* __restrict__ work, double* __restrict__ out)
{
    __shared__ CompP<double> v[kChunk];
    __shared__ int64_t sFirst[kMaxRanks + 1];
    __shared__ int sOver;
    leafOrigins(gathered, world, cap, sFirst, &sOver);
    if (sOver != 0) {  // some rank formed more leaves than ``cap`` holds: no valid sum
        if (threadIdx.x == 0)
            out[0] = out[1] = out[2] = __longlong_as_double(0x7ff8000000000000ll);
        return;
    }
    if (sFirst[world] == 0) {
        if (threadIdx.x == 0)
            out[0] = out[1] = out[2] = 0.0;
        return;
    }
    int64_t count = (sFirst[world] + kChunk - 1) / kChunk;  // the chunk partials
    while (count > 1) {
        const int64_t chunks = (count + kChunk - 1) / kChunk;
        for (int64_t c = 0; c < chunks; ++c) {
            const int cnt = int(count - c * kChunk < kChunk ? count - c * kChunk : kChunk);
            for (int i = int(threadIdx.x); i < cnt; i += int(blockDim.x))
                v[i] = CompP<double>{work[2 * (c * kChunk + i)], work[2 * (c * kChunk + i) + 1]};
            __syncthreads();
            levels(v, cnt);
            if (threadIdx.x == 0) {
                work[2 * c] = v[0].h;
                work[2 * c + 1] = v[0].c;
            }
            __syncthreads();
        }
        count = chunks;
    }
    if (threadIdx.x == 0) {
        const CompP<double> r{work[0], work[1]};
        out[0] = r.h;
        out[1] = r.c;
        out[2] = r.value();
    }
}

}  // namespace
}  // namespace eb

using namespace eb;

EB_API eagle_backend_status eagle_backend_x_b200_ragged_head(uint64_t kept, uint64_t count, uint64_t block,
    uint64_t stream)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_b200_ragged_head";
        if (count == 0 || block == 0)
            invalid(std::string(who) + ": count and block must be device addresses");
        if ((kept & 7u) != 0 || (block & 7u) != 0)
            invalid(std::string(who) + ": kept and block must be 8-byte aligned float64 arrays");
        raggedHeadKernel<<<1, 256, 0, seamStream(stream)>>>(reinterpret_cast<const double*>(kept),
            reinterpret_cast<const uint32_t*>(count), reinterpret_cast<double*>(block));
        launchCheck(who);
    });
}

EB_API eagle_backend_status eagle_backend_x_b200_ragged_leaves(uint64_t kept, uint64_t blocks, int32_t rank,
    int32_t world, uint64_t partials, int64_t cap, uint64_t stream)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_b200_ragged_leaves";
        if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
            invalid(std::string(who) + ": need 0 <= rank < world <= 256");
        if (cap < 1 || cap > (INT64_C(1) << 31))
            invalid(std::string(who) + ": cap must lie in [1, 2^31]");
        if (blocks == 0 || partials == 0)
            invalid(std::string(who) + ": blocks and partials must be device addresses");
        RaggedLeavesArgs a{};
        a.kept = reinterpret_cast<const double*>(kept);
        a.blocks = reinterpret_cast<const double*>(blocks);
        a.rank = rank;
        a.world = world;
        a.partials = reinterpret_cast<double*>(partials);
        a.cap = cap;
        raggedLeavesKernel<<<unsigned(cap), kSlots, 0, seamStream(stream)>>>(a);
        launchCheck(who);
    });
}

EB_API eagle_backend_status eagle_backend_x_b200_ragged_fold(uint64_t gathered, int32_t world, int64_t cap,
    uint64_t work, uint64_t out, uint64_t stream)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_b200_ragged_fold";
        if (world < 1 || world > kMaxRanks)
            invalid(std::string(who) + ": world must lie in [1, 256]");
        if (cap < 1)
            invalid(std::string(who) + ": cap must be >= 1");
        if (gathered == 0 || work == 0 || out == 0)
            invalid(std::string(who) + ": gathered, work and out must be device addresses");
        const cudaStream_t s = seamStream(stream);
        const int64_t chunks = (int64_t(world) * cap + kChunk - 1) / kChunk;  // at most; idle CTAs leave at once
        raggedChunkKernel<<<unsigned(chunks), kSlots, 0, s>>>(reinterpret_cast<const double*>(gathered), world, cap,
            reinterpret_cast<double*>(work));
        launchCheck(who);
        raggedTopKernel<<<1, kSlots, 0, s>>>(reinterpret_cast<const double*>(gathered), world, cap,
            reinterpret_cast<double*>(work), reinterpret_cast<double*>(out));
        launchCheck(who);
    });
}
