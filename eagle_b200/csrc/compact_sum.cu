// Compact-then-sum without materialising the survivors.
//
// The canonical sum of the samples a mask keeps (eagle's ActiveSet.compact, then
// the ``ordered`` reduction over the compacted plane: python/eagle/_active_set.py:482-525,
// eagle/reduce/canonical.h:10-32) depends on each kept value's RANK among the
// survivors: leaf l holds ranks [4096 l, 4096 l + 4096), and slot t of a leaf folds
// its ranks t, t + 256, ..., in that order. Writing the survivors out and reading
// them back costs 16 bytes per survivor on top of the mask and the value sectors,
// the whole gap between a compaction and its roofline. Instead, after a memset of
// the claim and chunk counters:
//
//   keepCountKernel   (tiles.cuh) one 16384-sample tile per CTA (four coalesced rows of 4096 mask
//                     bytes): the keep bits go out as a bitmap (one bit per sample)
//                     and the tile's count as one word. No look-back: a tile never
//                     waits on another, so the pass streams.
//   tileScanKernel    (tiles.cuh) one CTA: the exclusive scan of the tile counts, and the count.
//   leafStartKernel   a warp per tile: for every multiple of 4096 among the tile's
//                     ranks, the sample holding it (leafStart[l]), from the tile's
//                     512 bitmap words.
//   keptDenseKernel   warps claim leaves. A leaf spanning at most 4 samples per
//                     survivor is summed by the one warp: bitmap words 32 at a time,
//                     each kept value copied by cp.async straight into a per-warp
//                     ring at its rank (three batches in flight, no register held),
//                     every full row of 256 ranks folded slot by slot in rank order,
//                     and the in-leaf tree in registers and shuffles. Sparser leaves
//                     go on a list.
//   keptSparseKernel  CTAs take the listed leaves one at a time: the survivors
//                     staged in shared memory by rank (a leaf over many bitmap tiles
//                     by its tiles spread over the warps, each tile ranked from its
//                     scanned offset; a denser one by a CTA scan of its bitmap words),
//                     each thread loading its slot's 16 values together, one warp
//                     running the in-leaf tree.
//   The warp that finishes the last leaf of an aligned chunk of 512 joins the
//   chunk's leaves by the pairwise levels; the one that finishes the last chunk,
//   the chunks, and stores the value. No CTA ever waits on another.
//
// Traffic: the mask (n bytes), the bitmap written and read (n / 4 bytes), the value
// sectors holding a survivor; the bits are those of the two-kernel compaction +
// canonical sum, which the tests check against the oracle.
#include "canonical.cuh"
#include "tiles.cuh"

#include <mutex>

namespace eb {
namespace {

constexpr int kThreads = 256;
constexpr int kRows = 4;
constexpr int64_t kRow = int64_t(kThreads) * 16;  // 4096 samples: 16 mask bytes per thread
constexpr int64_t kTile = kRow * kRows;           // 16384 samples per keepCount CTA
constexpr int64_t kTileWords = kTile / 32;        // its bitmap words

using P = CompP<double>;

/** The position of the ``r``-th set bit (from 0) of ``x``, which has more than r:
 *  five halvings, each keeping the half the bit lies in. */
__device__ __forceinline__ int selectBit(uint32_t x, uint32_t r)
{
    int pos = 0;
#pragma unroll
    for (int w = 16; w > 0; w >>= 1) {
        const uint32_t lo = x & ((1u << w) - 1u);
        const uint32_t c = uint32_t(__popc(lo));
        if (r >= c) {
            r -= c;
            x >>= w;
            pos += w;
        } else {
            x = lo;
        }
    }
    return pos;
}

/** One rank's share of the leaves of the concatenation of every rank's survivors
 *  (compact-then-sum across ranks), formed on the device from the gathered counts.
 *  This rank's survivors are ranks [offset, offset + count) of the concatenation;
 *  counting ``shift`` = offset mod 4096 phantom survivors in front of them makes the
 *  concatenation's leaves this rank's leaves of shifted ranks (leaf L: shifted ranks
 *  [4096 L, 4096 L + 4096), local ranks from 4096 L - shift). Leaves [first, full)
 *  start and end here; with ``straddle`` the leaf starting at local rank
 *  ``tailStart`` runs on into the later ranks (or to the end of all survivors). */
struct RaggedPlan {
    int64_t offset, total, count, shift;
    int64_t first, full;
    int64_t tailStart, tailLen, headLen;
    int32_t straddle, pad;
};

/** One warp per tile: every leaf whose first rank (a multiple of 4096) falls among
 *  the tile's kept samples gets that sample's index in ``leafStart``. Lane l holds
 *  the tile's words [16 l, 16 l + 16). */
__global__ __launch_bounds__(kThreads, 4) void leafStartKernel(const uint32_t* __restrict__ bitmap,
    const uint32_t* __restrict__ tileCount, const uint32_t* __restrict__ tileOff, int64_t tiles,
    int32_t* __restrict__ leafStart, const RaggedPlan* __restrict__ plan)
{
    const int lane = int(threadIdx.x & 31);
    const int64_t warps = int64_t(gridDim.x) * (kThreads / 32);
    const uint64_t shift = plan != nullptr ? uint64_t(plan->shift) : 0u;  // ranks counted as shifted ones
    for (int64_t tile = int64_t(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5); tile < tiles; tile += warps) {
        const uint64_t o = tileOff[tile] + shift, c = tileCount[tile];
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
                // the word holding the boundary, then its bit (one select, not one per word)
                uint32_t rem = r - excl, wd = 0;
                int at = -1;
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    const uint32_t pc = uint32_t(__popc(w[k]));
                    if (at < 0) {
                        if (rem < pc) {
                            at = k;
                            wd = w[k];
                        } else {
                            rem -= pc;
                        }
                    }
                }
                leafStart[b / uint64_t(kLeaf)] = int32_t(tile * kTile + (lane * 16 + at) * 32 + selectBit(wd, rem));
            }
        }
    }
}


struct LeafArgs {
    const uint32_t* bitmap;
    const uint32_t* tileOff;  // the survivors before each bitmap tile
    const int32_t* leafStart;
    const uint32_t* count;
    const double* values;
    int64_t n;
    P* leafPart;           // one partial per leaf
    P* chunkPart;          // one per aligned chunk of kChunk leaves
    uint32_t* chunkDone;   // leaves finished per chunk, zero on entry
    uint32_t* topDone;     // chunks finished, zero on entry
    uint32_t* leafNext;    // the dense pass's claim counter over all leaves, zero on entry
    int32_t* sparseList;   // the leaves the dense pass hands on
    uint32_t* sparseCount; // zero on entry
    uint32_t* sparseNext;  // the sparse pass's claim counter, zero on entry
    uint32_t* err;         // zero on entry
    double* out;
    int pairOut;
    const RaggedPlan* plan;  // null: one device's sum; else this rank's leaves of the concatenation
    double* partOut;         // with a plan: (hi, comp) of leaves [first, full), from index 0
};

/** The leaves a pass walks: shifted survivor count, all leaves, and the range to sum. */
struct LeafSpan {
    int64_t rows, leaves, first, end, shift;
};

__device__ __forceinline__ LeafSpan leafSpan(const LeafArgs& a)
{
    LeafSpan sp;
    const int64_t c = int64_t(*a.count) > a.n ? 0 : int64_t(*a.count);
    sp.shift = a.plan != nullptr ? a.plan->shift : 0;
    sp.rows = c + sp.shift;
    sp.leaves = (sp.rows + kLeaf - 1) / kLeaf;
    sp.first = a.plan != nullptr ? a.plan->first : 0;
    sp.end = a.plan != nullptr ? a.plan->full : sp.leaves;
    return sp;
}

constexpr int kDenseThreads = 128;          // four warps, one leaf each
constexpr int kDenseWarps = kDenseThreads / 32;
constexpr int kRing = 1024;                 // a warp's staged values (see sumDenseLeaf)
constexpr int kBatchWords = 8;              // non-empty bitmap words per async batch
constexpr int kInflight = 3;                // async batches a warp keeps in flight (land0..2)
constexpr int kSlotsPerLane = kSlots / 32;
constexpr int kMaxK = 4;                    // bitmap words per thread per chunk (sparse pass)
constexpr int64_t kDenseSpan = 4;           // a leaf goes to a warp when it spans at most 4 samples per survivor

/** ``cp.async`` of one float64 from global to shared memory when ``pred`` (the
 *  copy lands asynchronously; cpWait orders it). */
__device__ __forceinline__ void cpAsync8(double* dst, const double* src, bool pred)
{
    const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %2, 0;\n @p cp.async.ca.shared.global [%0], [%1], 8;\n}\n" ::"r"(d),
        "l"(src), "r"(int(pred))
        : "memory");
}
__device__ __forceinline__ void cpCommit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
/** Waits until at most ``pending`` of this thread's committed groups are in flight. */
__device__ __forceinline__ void cpWait(int pending)
{
    if (pending <= 0)
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    else if (pending == 1)
        asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    else
        asm volatile("cp.async.wait_group 2;\n" ::: "memory");
}

/** One slot's fold of term ``x``: the join with (x, 0) without its non-finite test,
 *  which the caller applies once at the end (hi, once infinite or NaN, stays so and
 *  the comp ends zero; while hi is finite the comp is never -0, so the join's
 *  ``comp + 0`` is exact and dropped). ``first`` starts the slot at (x, 0). */
__device__ __forceinline__ void foldTerm(double& h, double& c, double x, bool first)
{
    if (first) {
        h = x;
        c = 0.0;
    } else {
        const double sum = h + x;
        const double bb = sum - h;
        const double e = (h - (sum - bb)) + (x - bb);
        c = c + e;
        h = sum;
    }
}

/** Bitmap word ``w`` of a leaf whose samples are [s0, s1) (0 outside [w0, wEnd)),
 *  its bits outside the leaf cleared: they belong to its neighbours. */
__device__ __forceinline__ uint32_t leafWord(const uint32_t* __restrict__ bitmap, int64_t w, int64_t s0, int64_t s1)
{
    const int64_t w0 = s0 >> 5, wEnd = ((s1 - 1) >> 5) + 1;
    uint32_t x = 0;
    if (w >= w0 && w < wEnd) {
        x = bitmap[w];
        if (w == w0)
            x &= ~0u << (s0 & 31);
        if (w == wEnd - 1) {
            const int e = int((s1 - 1) & 31);
            x &= e == 31 ? ~0u : ((2u << e) - 1u);
        }
    }
    return x;
}

/** A leaf's sample range, kept inside [0, n) whatever the starts hold, so that a
 *  failed pass still reads in bounds. */
__device__ __forceinline__ void leafRange(const LeafArgs& a, int64_t l, int64_t leaves, int64_t& s0, int64_t& s1)
{
    s0 = a.leafStart[l];
    s0 = s0 < 0 ? 0 : (s0 >= a.n ? a.n - 1 : s0);
    s1 = l + 1 < leaves ? int64_t(a.leafStart[l + 1]) : a.n;
    s1 = s1 <= s0 ? s0 + 1 : (s1 > a.n ? a.n : s1);
}

/** Pairwise levels over ``m <= 512`` partials at ``in`` (an aligned 512-node
 *  subtree), by one warp: lane l takes nodes [16 l, 16 l + 16) as two runs of 8,
 *  joins each run in registers (offsets 1, 2, 4) and the two runs (offset 8), then
 *  lanes pair up by shuffles (offsets 16..256): the pairs and order of ``levels``.
 *  Result in lane 0. Reads through L2, so partials other CTAs published before
 *  their counter increment are seen. */
__device__ __forceinline__ P warpLevels(const P* in, int m)
{
    const int lane = int(threadIdx.x & 31);
    P run[2];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const int i0 = lane * 16 + half * 8;
        P x[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            x[j] = i0 + j < m ? P{__ldcg(&in[i0 + j].h), __ldcg(&in[i0 + j].c)} : P{};
#pragma unroll
        for (int off = 1; off < 8; off <<= 1)
#pragma unroll
            for (int j = 0; j < 8; j += 2 * off)
                if (i0 + j + off < m)
                    x[j] = P::join(x[j], x[j + off]);
        run[half] = x[0];
    }
    P q = lane * 16 + 8 < m ? P::join(run[0], run[1]) : run[0];
#pragma unroll
    for (int lo = 1; lo < 32; lo <<= 1) {
        const P o = q.shflDown(unsigned(lo));
        if ((lane & (2 * lo - 1)) == 0 && (lane + lo) * 16 < m)
            q = P::join(q, o);
    }
    return q;
}

/** Called by one whole warp once leaf ``l``'s partial ``q`` (valid in lane 0) is
 *  known: stores it, and the warp that finishes the last leaf of an aligned chunk
 *  of 512 runs that chunk's pairwise levels; the warp that finishes the last chunk
 *  runs the levels above and stores the value. Counters are bumped after a
 *  __threadfence and partials read through L2, so either pass may finish a chunk. */
__device__ __forceinline__ void finishLeaf(const LeafArgs& a, int64_t l, int64_t leaves, const P& q)
{
    const int lane = int(threadIdx.x & 31);
    if (a.plan != nullptr) {  // one rank's leaves: stored for the exchange, joined elsewhere
        if (lane == 0) {
            a.partOut[2 * (l - a.plan->first)] = q.h;
            a.partOut[2 * (l - a.plan->first) + 1] = q.c;
        }
        return;
    }
    const int64_t chunks = (leaves + kChunk - 1) / kChunk;
    const int64_t ch = l / kChunk;
    const int inChunk = int(leaves - ch * kChunk < kChunk ? leaves - ch * kChunk : kChunk);
    uint32_t last = 0;
    if (lane == 0) {
        a.leafPart[l] = q;
        __threadfence();
        last = atomicAdd(&a.chunkDone[ch], 1u) == uint32_t(inChunk - 1) ? 1u : 0u;
    }
    if (!__shfl_sync(kFull, last, 0))
        return;
    __threadfence();
    const P cp = warpLevels(a.leafPart + ch * kChunk, inChunk);
    uint32_t top = 0;
    if (lane == 0) {
        a.chunkPart[ch] = cp;
        __threadfence();
        top = atomicAdd(a.topDone, 1u) == uint32_t(chunks - 1) ? 1u : 0u;
    }
    if (!__shfl_sync(kFull, top, 0))
        return;
    __threadfence();
    int64_t m = chunks;  // the levels above the chunks: aligned runs of 512, then the level above
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

/** The in-leaf tree over the slots a warp holds in registers (lane l: slots
 *  l + 32 i, i < 8): offsets 128, 64, 32 inside each lane, then shuffles 16..1 --
 *  the pairs and order of leafTree. Result in lane 0. */
__device__ __forceinline__ P warpLeafTree(const double (&h)[kSlotsPerLane], const double (&c)[kSlotsPerLane], int live)
{
    const int lane = int(threadIdx.x & 31);
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

/** One warp sums one leaf (samples [s0, s1) holding its ``cnt`` survivors). The
 *  bitmap words go 32 at a time, one per lane, the next two blocks already in
 *  flight. Each kept value is copied with cp.async straight into a ring at its
 *  rank -- no register holds a value in flight, so a warp keeps three batches of
 *  at most 256 values under way. A block holding at most 256 survivors is one
 *  batch, each lane walking its own word's bits; a fuller block is walked word by
 *  word, lane l copying bit l of each (one coalesced row of 32 samples per word),
 *  in batches of 8 words. When the oldest batch has landed, every full row of 256
 *  ranks below it is folded: lane l folds slots l + 32 i in rank order. The ring
 *  holds under 256 ranks waiting plus three batches of at most 256, so 1024
 *  entries never wrap onto a live one. */
__device__ __forceinline__ P sumDenseLeaf(const LeafArgs& a, int64_t s0, int64_t s1, int cnt, double* ring)
{
    const int lane = int(threadIdx.x & 31);
    const uint32_t below = (1u << lane) - 1u;
    const int64_t w0 = s0 >> 5, wEnd = ((s1 - 1) >> 5) + 1;
    double h[kSlotsPerLane], c[kSlotsPerLane];
#pragma unroll
    for (int i = 0; i < kSlotsPerLane; ++i)
        h[i] = c[i] = 0.0;
    uint32_t have = 0, used = 0;                // ranks issued, ranks folded (warp-uniform)
    uint32_t land0 = 0, land1 = 0, land2 = 0;  // ``have`` after each batch in flight, oldest first
    int inflight = 0;
    auto foldRows = [&](uint32_t limit) {  // every full row below ``limit``
        while (used + uint32_t(kSlots) <= limit && used < uint32_t(kLeaf)) {
            const double* row = ring + (used & (kRing - 1)) + lane;
            if (used == 0) {
#pragma unroll
                for (int i = 0; i < kSlotsPerLane; ++i)
                    foldTerm(h[i], c[i], row[32 * i], true);
            } else {
#pragma unroll
                for (int i = 0; i < kSlotsPerLane; ++i)
                    foldTerm(h[i], c[i], row[32 * i], false);
            }
            used += uint32_t(kSlots);
        }
    };
    auto batchDone = [&]() {  // after each commit: fold below the oldest batch once three are out
        cpCommit();
        if (inflight == 0)
            land0 = have;
        else if (inflight == 1)
            land1 = have;
        else
            land2 = have;
        if (++inflight == kInflight) {
            cpWait(kInflight - 1);
            __syncwarp();
            foldRows(land0);
            land0 = land1;
            land1 = land2;
            --inflight;
            __syncwarp();
        }
    };
    uint32_t word = leafWord(a.bitmap, w0 + lane, s0, s1);
    uint32_t next1 = leafWord(a.bitmap, w0 + 32 + lane, s0, s1);
    for (int64_t wb = w0; wb < wEnd; wb += 32) {
        const uint32_t next2 = leafWord(a.bitmap, wb + 64 + lane, s0, s1);  // two blocks ahead
        const uint32_t pc = uint32_t(__popc(word));
        const uint32_t incl = warpInclusiveSum(pc);
        const uint32_t total = __shfl_sync(kFull, incl, 31);
        if (total <= uint32_t(kSlots)) {
            // a thin block: each lane walks its own word's bits (one batch of at most 256)
            uint32_t r = have + incl - pc;
            const double* src = a.values + (wb + lane) * 32;
            for (uint32_t x = word; x != 0; x &= x - 1u, ++r)
                cpAsync8(ring + (r & (kRing - 1)), src + (__ffs(int(x)) - 1), r < uint32_t(kLeaf));
            __syncwarp();
            have += total;
            batchDone();
        } else {
            // a full block: the warp walks the words in order, lane l taking bit l
            const double* src = a.values + wb * 32 + lane;
#pragma unroll
            for (int k0 = 0; k0 < 32; k0 += kBatchWords) {
#pragma unroll
                for (int k = k0; k < k0 + kBatchWords; ++k) {
                    const uint32_t wd = __shfl_sync(kFull, word, k);
                    const uint32_t r = have + uint32_t(__popc(wd & below));
                    cpAsync8(ring + (r & (kRing - 1)), src + k * 32,
                        ((wd >> lane) & 1u) != 0u && r < uint32_t(kLeaf));
                    have += uint32_t(__popc(wd));
                }
                batchDone();
            }
        }
        word = next1;
        next1 = next2;
    }
    cpWait(0);
    __syncwarp();
    foldRows(have);
    if (have > used && used < uint32_t(kLeaf)) {  // the last leaf's short row
        const int live = int(have - used);
        const double* row = ring + (used & (kRing - 1)) + lane;
#pragma unroll
        for (int i = 0; i < kSlotsPerLane; ++i)
            if (lane + 32 * i < live)
                foldTerm(h[i], c[i], row[32 * i], used == 0);
    }
    if (have != uint32_t(cnt) && lane == 0)
        atomicOr(a.err, 2u);  // the bitmap and the leaf starts disagree
    __syncwarp();             // the ring is rewritten by the next leaf
    return warpLeafTree(h, c, cnt < kSlots ? cnt : kSlots);
}

/** The dense pass: warps claim leaves off a counter over all leaves; a leaf
 *  spanning more than kDenseSpan samples per survivor goes on the sparse list for
 *  the CTA pass, the others are summed here by one warp each. */
__global__ __launch_bounds__(kDenseThreads, 6) void keptDenseKernel(LeafArgs a)
{
    __shared__ __align__(16) double rings[kDenseWarps][kRing];
    const int lane = int(threadIdx.x & 31);
    double* ring = rings[threadIdx.x >> 5];
    const LeafSpan sp = leafSpan(a);
    const int64_t rows = sp.rows, leaves = sp.leaves;
    if (leaves == 0 && a.plan == nullptr) {
        if (blockIdx.x == 0 && threadIdx.x == 0) {
            a.out[0] = 0.0;
            if (a.pairOut)
                a.out[1] = 0.0;
        }
        return;
    }
    auto claim = [&]() -> int64_t {
        uint32_t l = 0;
        if (lane == 0)
            l = atomicAdd(a.leafNext, 1u);
        return int64_t(__shfl_sync(kFull, l, 0));
    };
    int64_t next = sp.first + claim();
    while (next < sp.end) {
        const int64_t l = next;
        next = sp.first + claim();  // the next claim's round trip overlaps this leaf
        int64_t s0, s1;
        leafRange(a, l, leaves, s0, s1);
        const int cnt = int(rows - l * kLeaf < kLeaf ? rows - l * kLeaf : kLeaf);
        if (s1 - s0 > kDenseSpan * int64_t(cnt)) {
            if (lane == 0)
                a.sparseList[atomicAdd(a.sparseCount, 1u)] = int32_t(l);
            continue;
        }
        const P q = sumDenseLeaf(a, s0, s1, cnt, ring);
        finishLeaf(a, l, leaves, q);
    }
}

/** Words per thread for a sparse leaf over [s0, s1): the smallest power of two up
 *  to kMaxK whose chunk of 256 K words covers the leaf. */
__device__ __forceinline__ int wordsPerThread(int64_t s0, int64_t s1)
{
    const int64_t words = ((s1 - 1) >> 5) - (s0 >> 5) + 1;
    int K = 1;
    while (K < kMaxK && int64_t(K) * kThreads < words)
        K *= 2;
    return K;
}

/** The sparse pass: CTAs take the leaves the dense pass listed, one leaf per CTA at
 *  a time, and stage its survivors' sample indices in shared memory by rank. A leaf
 *  over at least eight 16384-sample bitmap tiles spreads them over the CTA's warps:
 *  the front end's scanned tile offset gives the rank of a tile's first survivor, so
 *  a warp stages its tiles' survivors (those ranked inside the leaf) with no wait on
 *  the other warps. A denser leaf is walked in chunks of 256 K bitmap words, a CTA
 *  scan of each chunk's counts giving the ranks. Then thread t loads the values
 *  of ranks t + 256 i, i < 16, together (each in its own sector: the leaf is
 *  sparse; every staged index is a bitmap position, so below n) and folds them
 *  into slot t in order; one warp runs the in-leaf tree and finishes the leaf. */
__global__ __launch_bounds__(kThreads, 3) void keptSparseKernel(LeafArgs a)
{
    __shared__ __align__(16) int32_t idx[kLeaf];
    __shared__ P s[2][kSlots];
    __shared__ uint32_t scan[33], sHits[kThreads / 32];
    __shared__ int64_t sClaim[2][3];  // a claimed leaf and its sample range, two deep
    const int t = int(threadIdx.x);
    const LeafSpan sp = leafSpan(a);
    const int64_t rows = sp.rows, leaves = sp.leaves;
    if (sp.end <= sp.first)
        return;
    const uint32_t listed = *a.sparseCount;
    auto claimInto = [&](int b) {  // one thread: the next listed leaf, or -1
        const uint32_t i = atomicAdd(a.sparseNext, 1u);
        int64_t l = i < listed ? int64_t(a.sparseList[i]) : -1;
        l = l >= sp.end ? -1 : l;
        int64_t s0 = 0, s1 = 1;
        if (l >= 0)
            leafRange(a, l, leaves, s0, s1);
        sClaim[b][0] = l;
        sClaim[b][1] = s0;
        sClaim[b][2] = s1;
    };
    if (t == 0)
        claimInto(0);
    __syncthreads();
    int parity = 0;  // the slot buffer the next in-leaf tree takes
    for (int cur = 0;; cur ^= 1) {
        const int64_t l = sClaim[cur][0];
        if (l < 0)
            break;
        const int64_t s0 = sClaim[cur][1], s1 = sClaim[cur][2];
        if (t == 32)
            claimInto(cur ^ 1);  // the next claim's round trips overlap this leaf
        const int cnt = int(rows - l * kLeaf < kLeaf ? rows - l * kLeaf : kLeaf);
        const int64_t tileEnd = (s1 - 1) / kTile + 1;
        uint32_t staged = 0;
        if (tileEnd - s0 / kTile >= kThreads / 32) {
            // a leaf over at least one tile per warp (under ~3 % kept): the tiles go to the
            // warps in turn, and a tile's scanned offset gives the rank of its first survivor,
            // so each warp stages its tiles' survivors ranked inside the leaf with no wait on
            // the others (lane l holds the tile's words [16 l, 16 l + 16))
            const int warp = t >> 5, lane = t & 31;
            const int64_t rank0 = l * int64_t(kLeaf) - sp.shift;  // the leaf's first survivor's local rank
            uint32_t hits = 0;
            for (int64_t tile = s0 / kTile + warp; tile < tileEnd; tile += kThreads / 32) {
                const uint4* src = reinterpret_cast<const uint4*>(a.bitmap + tile * kTileWords) + lane * 4;
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
                int64_t r = int64_t(a.tileOff[tile]) + int64_t(excl) - rank0;  // the lane's first rank in the leaf
                if (r < int64_t(cnt) && r + int64_t(mine) > 0) {
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        const int32_t sample0 = int32_t((tile * kTileWords + lane * 16 + k) * 32);
                        for (uint32_t x = w[k]; x != 0; x &= x - 1u, ++r)
                            if (r >= 0 && r < int64_t(cnt)) {
                                idx[r] = sample0 + (__ffs(int(x)) - 1);
                                ++hits;
                            }
                    }
                }
            }
            hits = warpSum(hits);
            if (lane == 0)
                sHits[warp] = hits;
            __syncthreads();
#pragma unroll
            for (int k = 0; k < kThreads / 32; ++k)
                staged += sHits[k];
        } else {
            // a denser leaf: chunks of 256 K bitmap words (the next chunk's words in flight),
            // a CTA scan of each chunk's counts giving the ranks
            const int K = wordsPerThread(s0, s1);
            const int64_t wEnd = ((s1 - 1) >> 5) + 1;
            uint32_t word[kMaxK];
#pragma unroll
            for (int k = 0; k < kMaxK; ++k)
                word[k] = k < K ? leafWord(a.bitmap, (s0 >> 5) + int64_t(t) * K + k, s0, s1) : 0u;
            for (int64_t cw = s0 >> 5; cw < wEnd; cw += int64_t(kThreads) * K) {
                uint32_t next[kMaxK];
#pragma unroll
                for (int k = 0; k < kMaxK; ++k)
                    next[k] = k < K ? leafWord(a.bitmap, cw + int64_t(kThreads) * K + int64_t(t) * K + k, s0, s1)
                                    : 0u;
                uint32_t mine = 0;
#pragma unroll
                for (int k = 0; k < kMaxK; ++k)
                    mine += uint32_t(__popc(word[k]));
                uint32_t total = 0;
                uint32_t r = staged + blockExclusiveSum(mine, total, scan);
#pragma unroll
                for (int k = 0; k < kMaxK; ++k) {
                    const int32_t sample0 = int32_t((cw + int64_t(t) * K + k) * 32);
                    for (uint32_t x = word[k]; x != 0; x &= x - 1u, ++r)
                        if (r < uint32_t(cnt))
                            idx[r] = sample0 + (__ffs(int(x)) - 1);
                }
                staged += total;
#pragma unroll
                for (int k = 0; k < kMaxK; ++k)
                    word[k] = next[k];
            }
        }
        if (t == 0 && staged != uint32_t(cnt))
            atomicOr(a.err, 2u);  // the bitmap, the tile offsets and the leaf starts disagree
        __syncthreads();          // idx holds the leaf
        const int have = staged == uint32_t(cnt) ? cnt : 0;  // a failed leaf reads nothing
        double v[kTerms];
#pragma unroll
        for (int i = 0; i < kTerms; ++i)
            v[i] = t + i * kSlots < have ? __ldg(a.values + idx[t + i * kSlots]) : 0.0;
        double h = 0.0, c = 0.0;
#pragma unroll
        for (int i = 0; i < kTerms; ++i)
            if (t + i * kSlots < cnt)
                foldTerm(h, c, v[i], i == 0);
        const P q = leafTreeWarp0(P{h, isfinite(h) ? c : 0.0}, cnt < kSlots ? cnt : kSlots, s[parity]);
        parity ^= 1;
        if ((t >> 5) == 0)
            finishLeaf(a, l, leaves, q);
        __syncthreads();  // the next claim is visible; this one is rewritten a leaf later
    }
}

__global__ void compactSumEmptyKernel(uint32_t* count, double* out, int pairOut)
{
    *count = 0u;
    out[0] = 0.0;
    if (pairOut)
        out[1] = 0.0;
}

/** Scratch of one call over n samples: [dense claim, chunks finished, error,
 *  sparse listed, sparse claim, pad | leaves finished per chunk] (zeroed by the
 *  call's memset), then the tile counts and offsets, the bitmap, the leaf starts,
 *  the sparse list, the leaf partials and the chunk partials. */
struct SumLayout {
    int64_t maxLeaves = 0, maxChunks = 0;
    tiles::TileLayout t;
    size_t zeroed = 0, leafStart = 0, sparseList = 0, leafPart = 0, chunkPart = 0, plan = 0, tail = 0, total = 0;
};

size_t up(size_t x, size_t a) { return (x + a - 1) / a * a; }

/** Resident CTAs of the dense (which = 0) or sparse (1) pass on the current device:
 *  both passes are persistent grids that claim their leaves. */
int passGrid(int which)
{
    static std::mutex mu;
    static int perSm[64][2] = {};
    int dev = 0;
    cudaCheck(cudaGetDevice(&dev), "cudaGetDevice");
    std::lock_guard<std::mutex> lock(mu);
    int& k = perSm[dev & 63][which];
    if (k == 0) {
        if (which == 0)
            cudaCheck(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&k, keptDenseKernel, kDenseThreads, 0),
                "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
        else
            cudaCheck(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&k, keptSparseKernel, kThreads, 0),
                "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
        if (k < 1)
            k = 1;
    }
    return k * smCount();
}

SumLayout sumLayout(int64_t n)
{
    SumLayout L;
    L.maxLeaves = (n + kLeaf - 1) / kLeaf;
    L.maxChunks = (L.maxLeaves + kChunk - 1) / kChunk;
    L.zeroed = up(size_t(8 + L.maxChunks) * sizeof(uint32_t), 16);
    L.t = tiles::tileLayout(n, L.zeroed);
    L.leafStart = up(L.t.end, 256);
    L.sparseList = up(L.leafStart + size_t(L.maxLeaves + 1) * sizeof(int32_t), 256);
    L.leafPart = up(L.sparseList + size_t(L.maxLeaves + 1) * sizeof(int32_t), 256);
    L.chunkPart = up(L.leafPart + size_t(L.maxLeaves > 0 ? L.maxLeaves : 1) * sizeof(P), 256);
    L.plan = up(L.chunkPart + size_t(L.maxChunks > 0 ? L.maxChunks : 1) * sizeof(P), 256);
    L.tail = up(L.plan + sizeof(RaggedPlan), 256);
    L.total = up(L.tail + size_t(kLeaf) * sizeof(double), 256);
    return L;
}

// ------------------------------------------------- the same leaves across ranks

/** This rank's survivor count as its passes read it (a count above n: a failed scan, none). */
__device__ __forceinline__ int64_t ownCount(const uint32_t* count, int64_t n)
{
    return int64_t(*count) > n ? 0 : int64_t(*count);
}

/** One thread: the head's length in ``plan`` (the rest of the plan needs every
 *  rank's count) and this rank's count in its head block. */
__global__ void headPlanKernel(const uint32_t* __restrict__ count, int64_t n, RaggedPlan* plan, double* block)
{
    const int64_t c = ownCount(count, n);
    plan->headLen = c < kHead ? c : kHead;
    block[kHead] = countSlot(uint32_t(c));
}

/** One thread: this rank's RaggedPlan from every rank's gathered head block. */
__global__ void raggedPlanKernel(const double* __restrict__ blocks, int32_t rank, int32_t world,
    const uint32_t* __restrict__ count, int64_t n, RaggedPlan* plan)
{
    int64_t o = 0, total = 0;
    for (int q = 0; q < world; ++q) {
        if (q < rank)
            o += int64_t(blockCount(blocks, q));
        total += int64_t(blockCount(blocks, q));
    }
    const int64_t c = ownCount(count, n);
    RaggedPlan r{};
    r.offset = o;
    r.total = total;
    r.count = c;
    r.shift = o % kLeaf;
    r.first = r.shift > 0 ? 1 : 0;
    r.full = (c + r.shift) / kLeaf;  // leaf L ends by local rank 4096 (L + 1) - shift <= c
    if (r.full < r.first)
        r.full = r.first;
    const int64_t s0 = r.full * kLeaf - r.shift;  // where the next leaf would start
    r.straddle = (s0 >= 0 && s0 < c) ? 1 : 0;
    r.tailStart = r.straddle ? s0 : c;
    r.tailLen = r.straddle ? c - s0 : 0;
    r.headLen = c < kHead ? c : kHead;
    *plan = r;
}

constexpr int kSelectCtas = 32;  // CTAs of rankSelectKernel: a sparse range's tiles in one round

/** The values of this rank's survivors of local ranks [r0, r1) (at most 4096) into
 *  ``out[0, r1 - r0)``: the head (``tail`` false: ranks [0, headLen)) or the
 *  straddling leaf's part here (ranks [tailStart, count)). The first tile holding
 *  rank r0 is found by a binary search over the scanned tile offsets; CTA b then
 *  takes that tile + b, + b + kSelectCtas, ... while the tile starts below r1. In a
 *  tile, thread t holds bitmap words 2t and 2t + 1 (64 samples), ranks them by a CTA
 *  scan from the tile's offset, and loads each word's survivors in the range with 32
 *  predicated loads issued together. */
__global__ __launch_bounds__(kThreads) void rankSelectKernel(const uint32_t* __restrict__ bitmap,
    const uint32_t* __restrict__ tileOff, int64_t tiles, const double* __restrict__ values,
    const RaggedPlan* __restrict__ plan, const uint32_t* __restrict__ count, int64_t n, bool tail,
    double* __restrict__ out)
{
    static_assert(kTileWords == 2 * kThreads, "two bitmap words per thread cover a tile");
    __shared__ int64_t sLo, sHi;
    __shared__ int sBest;
    __shared__ uint32_t scan[33];
    const int t = int(threadIdx.x);
    int64_t r0 = 0, r1 = 0;
    if (tail) {
        r0 = plan->tailStart;
        r1 = plan->tailStart + plan->tailLen;
    } else {  // the head block: its length from the count, and the count into its slot
        const int64_t c = ownCount(count, n);
        r1 = c < kHead ? c : kHead;
        if (blockIdx.x == 0 && t == 0)
            out[kHead] = countSlot(uint32_t(c));
    }
    if (r1 <= r0)
        return;
    // the last tile whose first survivor's rank is <= r0 (tile 0's is 0): kThreads probes
    // per round over [lo, hi], each round narrowing it to one stride. The head (r0 = 0)
    // starts at tile 0: any empty tiles before its first survivor are passed over below.
    if (t == 0) {
        sLo = 0;
        sHi = r0 == 0 ? 0 : tiles - 1;
    }
    __syncthreads();
    while (sHi > sLo) {
        const int64_t lo = sLo, hi = sHi;
        const int64_t step = (hi - lo + kThreads) / kThreads;  // ceil((hi - lo + 1) / kThreads)
        if (t == 0)
            sBest = 0;
        __syncthreads();
        const int64_t at = lo + int64_t(t) * step;
        if (t > 0 && at <= hi && int64_t(tileOff[at]) <= r0)
            atomicMax(&sBest, t);
        __syncthreads();
        if (t == 0) {
            sLo = lo + int64_t(sBest) * step;
            sHi = sLo + step - 1 < hi ? sLo + step - 1 : hi;
        }
        __syncthreads();
    }
    const int64_t first = sLo;
    for (int64_t tile = first + blockIdx.x; tile < tiles && int64_t(tileOff[tile]) < r1; tile += gridDim.x) {
        const uint2 w = reinterpret_cast<const uint2*>(bitmap + tile * kTileWords)[t];
        const uint32_t mine = uint32_t(__popc(w.x) + __popc(w.y));
        uint32_t total = 0;
        const uint32_t excl = blockExclusiveSum(mine, total, scan);
        int64_t r = int64_t(tileOff[tile]) + int64_t(excl);  // the thread's first survivor's rank
        if (r >= r1 || r + int64_t(mine) <= r0)
            continue;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const uint32_t x = k == 0 ? w.x : w.y;
            const int64_t sample0 = (tile * kTileWords + 2 * t + k) * 32;
            double v[32];
#pragma unroll
            for (int b = 0; b < 32; ++b) {
                const int64_t rb = r + __popc(x & ((1u << b) - 1u));
                v[b] = ((x >> b) & 1u) && rb >= r0 && rb < r1 ? values[sample0 + b] : 0.0;
            }
#pragma unroll
            for (int b = 0; b < 32; ++b) {
                const int64_t rb = r + __popc(x & ((1u << b) - 1u));
                if (((x >> b) & 1u) && rb >= r0 && rb < r1)
                    out[rb - r0] = v[b];
            }
            r += __popc(x);
        }
    }
}

/** One CTA: the leaf that starts here and runs into the later ranks, from this
 *  rank's part (``tail``) and the later ranks' gathered head blocks, at partials
 *  index full - first; then this rank's leaf count into the partial block's count
 *  slot (all of 0xffffffff when a pass reported an error, so that the fold gives
 *  NaN). */
__global__ __launch_bounds__(kSlots) void straddleKernel(const RaggedPlan* __restrict__ plan,
    const double* __restrict__ blocks, int32_t rank, int32_t world, const double* __restrict__ tail,
    const uint32_t* __restrict__ err, double* __restrict__ partials, int64_t cap)
{
    __shared__ int64_t sOff[kMaxRanks + 1];
    __shared__ P s[kSlots];
    if (threadIdx.x == 0) {
        int64_t o = 0;
        for (int q = 0; q < world; ++q) {
            sOff[q] = o;
            o += int64_t(blockCount(blocks, q));
        }
        sOff[world] = o;
    }
    __syncthreads();
    const RaggedPlan r = *plan;
    const int64_t own = r.full - r.first;
    if (r.straddle) {
        const int64_t start = r.offset + r.tailStart;  // the leaf's first survivor in the concatenation
        const int64_t cnt = r.total - start < kLeaf ? r.total - start : kLeaf;
        auto at = [&](int64_t i) -> double {
            if (i < r.tailLen)
                return tail[i];
            const int64_t g = start + i;
            int q = rank + 1;  // the later rank holding g: g - sOff[q] < kHead
            while (q + 1 < world && g >= sOff[q + 1])
                ++q;
            return blockHead(blocks, q, g - sOff[q]);
        };
        const P q = leafPartialAt<P, double>(at, cnt, s);
        if (threadIdx.x == 0) {
            partials[2 * own] = q.h;
            partials[2 * own + 1] = q.c;
        }
    }
    if (threadIdx.x == 0)
        partials[2 * cap] = countSlot(*err != 0u ? 0xffffffffu : uint32_t(own + r.straddle));
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
        uint32_t* tileCount = reinterpret_cast<uint32_t*>(base + L.t.count);
        uint32_t* tileOff = reinterpret_cast<uint32_t*>(base + L.t.off);
        uint32_t* bitmap = reinterpret_cast<uint32_t*>(base + L.t.bitmap);
        int32_t* leafStart = reinterpret_cast<int32_t*>(base + L.leafStart);
        uint32_t* count = reinterpret_cast<uint32_t*>(d.count);
        LeafArgs la{};
        la.bitmap = bitmap;
        la.tileOff = tileOff;
        la.leafStart = leafStart;
        la.count = count;
        la.values = reinterpret_cast<const double*>(values);
        la.n = d.n;
        la.leafPart = reinterpret_cast<P*>(base + L.leafPart);
        la.chunkPart = reinterpret_cast<P*>(base + L.chunkPart);
        la.leafNext = words;
        la.topDone = words + 1;
        la.err = words + 2;
        la.sparseCount = words + 3;
        la.sparseNext = words + 4;
        la.chunkDone = words + 8;
        la.sparseList = reinterpret_cast<int32_t*>(base + L.sparseList);
        la.out = reinterpret_cast<double*>(out);
        la.pairOut = pairOut;
        cudaCheck(cudaMemsetAsync(base, 0, L.zeroed, s), "cudaMemsetAsync");
        tiles::enqueueTiles(reinterpret_cast<const uint8_t*>(d.mask), d.n,
            (d.flags & EAGLE_BACKEND_COMPACT_MASK_IS_DROP) != 0, base, L.t, count, tiles::ScanTrigger{}, s, who);
        const int64_t warpsPerCta = kThreads / 32;
        const int64_t startCtas = (L.t.tiles + warpsPerCta - 1) / warpsPerCta;
        const int64_t startCap = int64_t(smCount()) * 8;
        leafStartKernel<<<unsigned(startCtas < startCap ? startCtas : startCap), kThreads, 0, s>>>(bitmap, tileCount,
            tileOff, L.t.tiles, leafStart, nullptr);
        launchCheck(who);
        keptDenseKernel<<<unsigned(passGrid(0)), kDenseThreads, 0, s>>>(la);
        launchCheck(who);
        keptSparseKernel<<<unsigned(passGrid(1)), kThreads, 0, s>>>(la);
        launchCheck(who);
    });
}

// ---------------------------------------------- compact-then-sum across ranks
//
// The one-device call above, cut where the ranks must exchange: _count runs the
// front end (keep bitmap, tile counts and offsets, this rank's count); _head writes
// this rank's head block (its first 4095 survivors, selected by a CTA per bitmap tile,
// and its count); the caller all-gathers the head blocks; _leaves forms this rank's
// plan from the gathered counts on the device, places the leaf starts in the
// concatenation's leaves, sums every leaf that starts and ends here with the same
// dense and sparse passes (their partials written out, not joined) and selects the
// part of the leaf that straddles into the next ranks; _straddle sums that leaf from
// its part here and the later ranks' heads and closes the partial block with the leaf
// count. The caller all-gathers the partial blocks, and eagle_backend_x_b200_ragged_fold
// joins them. The kept values are never written out, as in the one-device call.

namespace eb {
namespace {

/** The split entries' common checks (the desc is compact_sum's, with its scratch). */
SumLayout checkSplit(const eagle_backend_compact_desc& d, const char* who)
{
    if (d.n < 0)
        invalid(std::string(who) + ": n must be >= 0");
    if (d.n > INT64_C(2147483647))
        unsupported(std::string(who) + ": at most 2^31-1 samples, got n = " + std::to_string(d.n));
    if (d.index_map != 0 || d.live32 != 0)
        unsupported(std::string(who) + ": writes no index map and offers no trigger");
    if (d.scratch == 0 || d.count == 0 || (d.n > 0 && d.mask == 0))
        invalid(std::string(who) + ": mask, count and scratch (queried from compact_sum) must be device addresses");
    if ((d.scratch & 255u) != 0)
        invalid(std::string(who) + ": scratch must be 256-byte aligned");
    return sumLayout(d.n);
}

}  // namespace
}  // namespace eb

EB_API eagle_backend_status eagle_backend_x_b200_compact_sum_count(struct eagle_backend_compact_desc* desc)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_b200_compact_sum_count";
        const auto d = readDesc(desc, EAGLE_BACKEND_COMPACT_MASK_IS_DROP, who);
        const SumLayout L = checkSplit(d, who);
        DeviceScope scope(resolveDevice(d.device, d.mask != 0 ? d.mask : d.count));
        const cudaStream_t s = seamStream(d.stream);
        char* base = reinterpret_cast<char*>(d.scratch);
        cudaCheck(cudaMemsetAsync(base, 0, L.zeroed, s), "cudaMemsetAsync");
        if (d.n == 0) {
            cudaCheck(cudaMemsetAsync(reinterpret_cast<void*>(d.count), 0, sizeof(uint32_t), s), "cudaMemsetAsync");
            return;
        }
        tiles::enqueueTiles(reinterpret_cast<const uint8_t*>(d.mask), d.n,
            (d.flags & EAGLE_BACKEND_COMPACT_MASK_IS_DROP) != 0, base, L.t, reinterpret_cast<uint32_t*>(d.count),
            tiles::ScanTrigger{}, s, who);
    });
}

EB_API eagle_backend_status eagle_backend_x_b200_compact_sum_head(struct eagle_backend_compact_desc* desc,
    uint64_t values, uint64_t block)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_b200_compact_sum_head";
        const auto d = readDesc(desc, EAGLE_BACKEND_COMPACT_MASK_IS_DROP, who);
        const SumLayout L = checkSplit(d, who);
        if (block == 0 || (d.n > 0 && values == 0))
            invalid(std::string(who) + ": values and block must be device addresses");
        if ((values & 7u) != 0 || (block & 7u) != 0)
            invalid(std::string(who) + ": values and block must be 8-byte aligned float64 arrays");
        DeviceScope scope(resolveDevice(d.device, d.mask != 0 ? d.mask : d.count));
        const cudaStream_t s = seamStream(d.stream);
        char* base = reinterpret_cast<char*>(d.scratch);
        auto* plan = reinterpret_cast<RaggedPlan*>(base + L.plan);
        if (d.n == 0) {
            headPlanKernel<<<1, 1, 0, s>>>(reinterpret_cast<const uint32_t*>(d.count), d.n, plan,
                reinterpret_cast<double*>(block));
            launchCheck(who);
            return;
        }
        rankSelectKernel<<<kSelectCtas, kThreads, 0, s>>>(reinterpret_cast<const uint32_t*>(base + L.t.bitmap),
            reinterpret_cast<const uint32_t*>(base + L.t.off), L.t.tiles, reinterpret_cast<const double*>(values),
            plan, reinterpret_cast<const uint32_t*>(d.count), d.n, false, reinterpret_cast<double*>(block));
        launchCheck(who);
    });
}

EB_API eagle_backend_status eagle_backend_x_b200_compact_sum_leaves(struct eagle_backend_compact_desc* desc,
    uint64_t values, uint64_t blocks, int32_t rank, int32_t world, uint64_t partials, int64_t cap)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_b200_compact_sum_leaves";
        const auto d = readDesc(desc, EAGLE_BACKEND_COMPACT_MASK_IS_DROP, who);
        const SumLayout L = checkSplit(d, who);
        if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
            invalid(std::string(who) + ": need 0 <= rank < world <= 256");
        if (blocks == 0 || partials == 0 || (d.n > 0 && values == 0))
            invalid(std::string(who) + ": values, blocks and partials must be device addresses");
        if ((values & 7u) != 0)
            invalid(std::string(who) + ": values must be an 8-byte aligned float64 array");
        if (cap < L.maxLeaves + 1)
            invalid(std::string(who) + ": cap must be at least ceil(n / 4096) + 1 leaves");
        DeviceScope scope(resolveDevice(d.device, d.mask != 0 ? d.mask : d.count));
        const cudaStream_t s = seamStream(d.stream);
        char* base = reinterpret_cast<char*>(d.scratch);
        auto* plan = reinterpret_cast<RaggedPlan*>(base + L.plan);
        raggedPlanKernel<<<1, 1, 0, s>>>(reinterpret_cast<const double*>(blocks), rank, world,
            reinterpret_cast<const uint32_t*>(d.count), d.n, plan);
        launchCheck(who);
        if (d.n == 0)
            return;
        uint32_t* words = reinterpret_cast<uint32_t*>(base);
        const uint32_t* tileCount = reinterpret_cast<const uint32_t*>(base + L.t.count);
        const uint32_t* tileOff = reinterpret_cast<const uint32_t*>(base + L.t.off);
        const uint32_t* bitmap = reinterpret_cast<const uint32_t*>(base + L.t.bitmap);
        int32_t* leafStart = reinterpret_cast<int32_t*>(base + L.leafStart);
        LeafArgs la{};
        la.bitmap = bitmap;
        la.tileOff = tileOff;
        la.leafStart = leafStart;
        la.count = reinterpret_cast<const uint32_t*>(d.count);
        la.values = reinterpret_cast<const double*>(values);
        la.n = d.n;
        la.leafPart = reinterpret_cast<P*>(base + L.leafPart);
        la.chunkPart = reinterpret_cast<P*>(base + L.chunkPart);
        la.leafNext = words;
        la.topDone = words + 1;
        la.err = words + 2;
        la.sparseCount = words + 3;
        la.sparseNext = words + 4;
        la.chunkDone = words + 8;
        la.sparseList = reinterpret_cast<int32_t*>(base + L.sparseList);
        la.out = nullptr;
        la.plan = plan;
        la.partOut = reinterpret_cast<double*>(partials);
        const int64_t warpsPerCta = kThreads / 32;
        const int64_t startCtas = (L.t.tiles + warpsPerCta - 1) / warpsPerCta;
        const int64_t startCap = int64_t(smCount()) * 8;
        leafStartKernel<<<unsigned(startCtas < startCap ? startCtas : startCap), kThreads, 0, s>>>(bitmap, tileCount,
            tileOff, L.t.tiles, leafStart, plan);
        launchCheck(who);
        keptDenseKernel<<<unsigned(passGrid(0)), kDenseThreads, 0, s>>>(la);
        launchCheck(who);
        keptSparseKernel<<<unsigned(passGrid(1)), kThreads, 0, s>>>(la);
        launchCheck(who);
        rankSelectKernel<<<kSelectCtas, kThreads, 0, s>>>(bitmap, tileOff, L.t.tiles,
            reinterpret_cast<const double*>(values), plan, la.count, d.n, true,
            reinterpret_cast<double*>(base + L.tail));
        launchCheck(who);
    });
}

EB_API eagle_backend_status eagle_backend_x_b200_compact_sum_straddle(struct eagle_backend_compact_desc* desc,
    uint64_t blocks, int32_t rank, int32_t world, uint64_t partials, int64_t cap)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_b200_compact_sum_straddle";
        const auto d = readDesc(desc, EAGLE_BACKEND_COMPACT_MASK_IS_DROP, who);
        const SumLayout L = checkSplit(d, who);
        if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
            invalid(std::string(who) + ": need 0 <= rank < world <= 256");
        if (blocks == 0 || partials == 0)
            invalid(std::string(who) + ": blocks and partials must be device addresses");
        if (cap < L.maxLeaves + 1)
            invalid(std::string(who) + ": cap must be at least ceil(n / 4096) + 1 leaves");
        DeviceScope scope(resolveDevice(d.device, d.mask != 0 ? d.mask : d.count));
        const cudaStream_t s = seamStream(d.stream);
        char* base = reinterpret_cast<char*>(d.scratch);
        straddleKernel<<<1, kSlots, 0, s>>>(reinterpret_cast<const RaggedPlan*>(base + L.plan),
            reinterpret_cast<const double*>(blocks), rank, world, reinterpret_cast<const double*>(base + L.tail),
            reinterpret_cast<const uint32_t*>(base) + 2, reinterpret_cast<double*>(partials), cap);
        launchCheck(who);
    });
}
