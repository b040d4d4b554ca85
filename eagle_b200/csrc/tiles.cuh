// The reduce-then-scan front end of the fused compact-then-sum (and of any pass
// that wants a keep bitmap with tile offsets): a mask becomes a keep bitmap plus per-tile counts in one
// streaming pass (no tile ever waits on another), and one CTA scans the counts.
//
//   keepCountKernel  one 16384-sample tile per CTA, four coalesced rows of 4096
//                    mask bytes (16 per thread per row): the keep bits go out as a
//                    bitmap (bit j of word w: sample 32 w + j is kept; a tile is 512
//                    words), the tile's kept count as one word and, when asked, the
//                    number of its 32-sample groups holding a kept sample (eagle's
//                    live32, eagle/filtering/Compact.h:113-118).
//   tileScanKernel   one CTA: tileOff[i] = the kept samples before tile i, the count,
//                    and, for a trigger, live32 and the fire decision.
#pragma once

#include "common.cuh"

namespace eb {
namespace {
namespace tiles {

constexpr int kThreads = 256;
constexpr int kRows = 4;
constexpr int64_t kRow = int64_t(kThreads) * 16;  // 4096 samples: 16 mask bytes per thread
constexpr int64_t kTile = kRow * kRows;           // 16384 samples per CTA
constexpr int64_t kWords = kTile / 32;            // a tile's bitmap words
constexpr int kScanThreads = 1024;
constexpr int kScanRound = kScanThreads * 8;     // tile counts per scan round (8 per thread)

/** One 16384-sample tile per CTA (a CTA looping over several tiles held more
 *  registers and measured slower: 72-79 against 67 us for 2^28 samples). */
template <bool Drop, bool Aligned>
__global__ __launch_bounds__(kThreads) void keepCountKernel(const uint8_t* __restrict__ mask, int64_t n,
    uint32_t* __restrict__ bitmap, uint32_t* __restrict__ tileCount, uint32_t* __restrict__ tileLive)
{
    __shared__ uint32_t part[kThreads / 32], partLive[kThreads / 32];
    const int t = int(threadIdx.x);
    const int64_t tile = blockIdx.x;
    const int64_t tile0 = tile * kTile;
    uint32_t bits[kRows];
    uint32_t c = 0, live = 0;
    uint4 raw[kRows];
#pragma unroll
    for (int q = 0; q < kRows; ++q)  // every row's load in flight before the first is used
        raw[q] = maskBytes16<Aligned>(mask, tile0 + int64_t(q) * kRow + int64_t(t) * 16, n);
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
        bits[q] = keepOf16<Drop>(raw[q], tile0 + int64_t(q) * kRow + int64_t(t) * 16, n);
        c += uint32_t(__popc(bits[q]));
    }
    // threads 2u and 2u + 1 hold the low and high halves of one 32-sample word
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
        const uint32_t hi = __shfl_down_sync(kFull, bits[q], 1);
        if ((t & 1) == 0) {
            const uint32_t w = bits[q] | (hi << 16);
            bitmap[tile * kWords + q * (kRow / 32) + (t >> 1)] = w;
            live += w != 0 ? 1u : 0u;
        }
    }
    c = warpSum(c);
    live = warpSum(live);
    if ((t & 31) == 0) {
        part[t >> 5] = c;
        partLive[t >> 5] = live;
    }
    __syncthreads();
    if (t == 0) {
        uint32_t s = 0, l = 0;
#pragma unroll
        for (int w = 0; w < kThreads / 32; ++w) {
            s += part[w];
            l += partLive[w];
        }
        tileCount[tile] = s;
        if (tileLive != nullptr)
            tileLive[tile] = l;
    }
}

/** A compaction's reorder trigger (Compact.h:113-118): fire when the count is under
 *  theta of the slots its live 32-groups span and under the span (of at least 4096). */
struct ScanTrigger {
    const uint32_t* tileLive;  // null: no trigger
    uint32_t* live32;
    const uint32_t* span;
    uint32_t* fire;
    float theta;
};

/** tileOff[i] = the kept samples before tile i; ``*count`` = all of them; with a
 *  trigger, live32 and fire as the one-pass compaction writes them. One CTA, in
 *  rounds of 8192 counts: the counts come in and the offsets go out as coalesced
 *  16-byte rows through shared memory, where thread t scans its 8 neighbours (16
 *  scattered 4-byte stores per thread throttled the load-store queue). */
__global__ __launch_bounds__(kScanThreads) void tileScanKernel(const uint32_t* __restrict__ tileCount,
    uint32_t* __restrict__ tileOff, int64_t tiles, uint32_t* count, ScanTrigger trig)
{
    __shared__ __align__(16) uint32_t buf[kScanRound];
    __shared__ uint32_t scan[33];
    const int t = int(threadIdx.x);
    uint32_t carry = 0, liveSum = 0;
    for (int64_t r0 = 0; r0 < tiles; r0 += kScanRound) {
        // coalesced rows in: thread t takes rows t and t + kScanThreads of four counts
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int row = t + h * kScanThreads;
            const int64_t i = r0 + int64_t(row) * 4;
            uint4 x;
            if (i + 4 <= tiles) {  // the counts start 256-byte aligned
                x = *reinterpret_cast<const uint4*>(tileCount + i);
            } else {
                x.x = i < tiles ? tileCount[i] : 0u;
                x.y = i + 1 < tiles ? tileCount[i + 1] : 0u;
                x.z = i + 2 < tiles ? tileCount[i + 2] : 0u;
                x.w = i + 3 < tiles ? tileCount[i + 3] : 0u;
            }
            reinterpret_cast<uint4*>(buf)[row] = x;
        }
        __syncthreads();
        // thread t scans counts [8 t, 8 t + 8) of the round
        uint4 lo = reinterpret_cast<const uint4*>(buf)[2 * t], hi = reinterpret_cast<const uint4*>(buf)[2 * t + 1];
        const uint32_t mine = lo.x + lo.y + lo.z + lo.w + hi.x + hi.y + hi.z + hi.w;
        uint32_t total = 0;
        uint32_t run = carry + blockExclusiveSum(mine, total, scan);  // its barriers order buf's reads
        uint4 olo, ohi;
        olo.x = run;
        run += lo.x;
        olo.y = run;
        run += lo.y;
        olo.z = run;
        run += lo.z;
        olo.w = run;
        run += lo.w;
        ohi.x = run;
        run += hi.x;
        ohi.y = run;
        run += hi.y;
        ohi.z = run;
        run += hi.z;
        ohi.w = run;
        reinterpret_cast<uint4*>(buf)[2 * t] = olo;
        reinterpret_cast<uint4*>(buf)[2 * t + 1] = ohi;
        carry += total;
        __syncthreads();
        // coalesced rows out
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int row = t + h * kScanThreads;
            const int64_t i = r0 + int64_t(row) * 4;
            const uint4 x = reinterpret_cast<const uint4*>(buf)[row];
            if (i + 4 <= tiles) {
                *reinterpret_cast<uint4*>(tileOff + i) = x;
            } else {
                if (i < tiles)
                    tileOff[i] = x.x;
                if (i + 1 < tiles)
                    tileOff[i + 1] = x.y;
                if (i + 2 < tiles)
                    tileOff[i + 2] = x.z;
                if (i + 3 < tiles)
                    tileOff[i + 3] = x.w;
            }
        }
        if (trig.tileLive != nullptr) {
            uint32_t l = 0;
            for (int64_t i = r0 + t; i < r0 + kScanRound && i < tiles; i += kScanThreads)
                l += trig.tileLive[i];
            uint32_t lt = 0;
            blockExclusiveSum(l, lt, scan);
            liveSum += lt;
        }
        __syncthreads();  // buf is rewritten by the next round
    }
    if (t == 0) {
        *count = carry;
        if (trig.tileLive != nullptr) {
            *trig.live32 = liveSum;
            const uint32_t span = *trig.span;
            const double limit = double(trig.theta) * 32.0 * double(liveSum);
            *trig.fire = (double(carry) < limit && carry < span && span >= 4096u) ? 1u : 0u;
        }
    }
}

/** The offsets of one tile's scratch arrays for n samples: [tile counts | tile
 *  offsets | tile live groups | bitmap], each 256-byte aligned. */
struct TileLayout {
    int64_t tiles = 0;
    size_t count = 0, off = 0, live = 0, bitmap = 0, end = 0;
};

inline size_t up256(size_t x) { return (x + 255) / 256 * 256; }

inline TileLayout tileLayout(int64_t n, size_t at)
{
    TileLayout L;
    L.tiles = n > 0 ? (n + kTile - 1) / kTile : 1;
    L.count = up256(at);
    L.off = up256(L.count + size_t(L.tiles) * sizeof(uint32_t));
    L.live = up256(L.off + size_t(L.tiles) * sizeof(uint32_t));
    L.bitmap = up256(L.live + size_t(L.tiles) * sizeof(uint32_t));
    L.end = up256(L.bitmap + size_t(L.tiles) * kWords * sizeof(uint32_t));
    return L;
}

/** Enqueues keepCountKernel and tileScanKernel over ``scratch`` laid out by
 *  tileLayout(n, at). */
inline void enqueueTiles(const uint8_t* mask, int64_t n, bool drop, char* scratch, const TileLayout& L,
    uint32_t* count, ScanTrigger trig, cudaStream_t s, const char* who)
{
    auto* bitmap = reinterpret_cast<uint32_t*>(scratch + L.bitmap);
    auto* tileCount = reinterpret_cast<uint32_t*>(scratch + L.count);
    auto* tileOff = reinterpret_cast<uint32_t*>(scratch + L.off);
    uint32_t* tileLive = trig.live32 != nullptr ? reinterpret_cast<uint32_t*>(scratch + L.live) : nullptr;
    // one tile per CTA measured faster for this pass than fewer CTAs looping (67 against 72 us
    // for 2^28 samples): its tiles are independent and short, so the launch keeps them all in flight
    const unsigned grid = unsigned(L.tiles);
    const bool aligned = (reinterpret_cast<uintptr_t>(mask) & 15u) == 0;
    if (drop)
        aligned ? keepCountKernel<true, true><<<grid, kThreads, 0, s>>>(mask, n, bitmap, tileCount, tileLive)
                : keepCountKernel<true, false><<<grid, kThreads, 0, s>>>(mask, n, bitmap, tileCount, tileLive);
    else
        aligned ? keepCountKernel<false, true><<<grid, kThreads, 0, s>>>(mask, n, bitmap, tileCount, tileLive)
                : keepCountKernel<false, false><<<grid, kThreads, 0, s>>>(mask, n, bitmap, tileCount, tileLive);
    launchCheck(who);
    trig.tileLive = tileLive;
    tileScanKernel<<<1, kScanThreads, 0, s>>>(tileCount, tileOff, L.tiles, count, trig);
    launchCheck(who);
}

}  // namespace tiles
}  // namespace
}  // namespace eb
