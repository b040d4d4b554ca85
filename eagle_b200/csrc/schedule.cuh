// The schedules a step model runs under, shared by the built-in models: the
// per-block flush of the run counters, one lane per sample over a contiguous range
// (the plain / _range entries), and persistent lanes claiming samples off a counter
// (the _persist entry). A model M provides ``Sample``, ``load(i)``, ``store(i, s)``,
// ``prepare(s)``, ``run(s, budget, fin)`` and its ``term`` mask plane.
#pragma once

#include "models.cuh"

namespace eb {

/** Flush a thread's run counters with one atomic per block and counter:
 *  finished count (u32), longest steps (u32 max) and executed steps (u64 sum);
 *  a null cell is skipped. Every thread of the block calls it. */
__device__ __forceinline__ void blockFlush(uint32_t fin, uint32_t longest, unsigned long long sum,
    uint32_t* finished, uint32_t* steps, unsigned long long* stepsum)
{
    __shared__ uint32_t sFin[32], sMax[32];
    __shared__ unsigned long long sSum[32];
    fin = warpSum(fin);
    longest = warpMax(longest);
    sum = warpSum(sum);
    const unsigned lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    if (lane == 0) {
        sFin[warp] = fin;
        sMax[warp] = longest;
        sSum[warp] = sum;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t f = 0, m = 0;
        unsigned long long u = 0;
        for (unsigned w = 0; w < (blockDim.x + 31) / 32; ++w) {
            f += sFin[w];
            m = sMax[w] > m ? sMax[w] : m;
            u += sSum[w];
        }
        if (finished != nullptr && f != 0)
            atomicAdd(finished, f);
        if (steps != nullptr && m != 0)
            atomicMax(steps, m);
        if (stepsum != nullptr && u != 0)
            atomicAdd(stepsum, u);
    }
}

/** One lane per sample of [base, base + count): a live sample runs up to ``budget``
 *  steps (its mask set if it terminates); counters flushed per block. */
template <class M>
__device__ __forceinline__ void rangeLoop(const M& m, int64_t base, int64_t count, int64_t budget,
    uint32_t* finished, uint32_t* steps, unsigned long long* stepsum)
{
    const int64_t j = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t i = base + j;
    int64_t taken = 0;
    bool fin = false;
    if (j < count && m.term[i] == 0) {
        auto s = m.load(i);
        m.prepare(s);
        while (taken < budget && !fin) {
            const int64_t left = budget - taken;
            taken += m.run(s, left < (INT64_C(1) << 30) ? int(left) : (1 << 30), fin);
        }
        m.store(i, s);
        if (fin)
            m.term[i] = 1;
    }
    blockFlush(fin ? 1u : 0u, uint32_t(taken), (unsigned long long)taken, finished, steps, stepsum);
}

/** Persistent lanes: each lane holds its current sample and, one chunk ahead, the
 *  next one; at each chunk head the lanes lacking a next sample claim the following
 *  indices together off ``next`` (one atomic per warp) and issue its loads, which
 *  complete while the chunk runs. A claimed sample already terminated is skipped;
 *  a lane whose sample ends mid-chunk waits, masked, for the next head. */
template <class M>
__device__ __forceinline__ void persistLoop(const M& m, int64_t base, int64_t count, int64_t budget, int chunk,
    uint32_t* next, unsigned long long* util, uint32_t* finished, uint32_t* steps, unsigned long long* stepsum)
{
    const unsigned lane = threadIdx.x & 31u;
    typename M::Sample cur{}, nxt{};
    int64_t i = -1, ni = -1;
    uint8_t nterm = 0;
    int64_t taken = 0;
    bool exhausted = false;
    uint32_t finCount = 0, longest = 0;
    unsigned long long ranSum = 0, slots = 0;
    auto prefetch = [&]() {
        const bool needs = ni < 0 && !exhausted;
        const unsigned want = __ballot_sync(kFull, needs);
        if (want == 0)
            return;
        const unsigned leader = __ffs(want) - 1;
        uint32_t first = 0;
        if (lane == leader)
            first = atomicAdd(next, uint32_t(__popc(want)));
        first = __shfl_sync(kFull, first, leader);
        if (needs) {
            const int64_t k = int64_t(first) + __popc(want & ((1u << lane) - 1u));
            if (k >= count) {
                exhausted = true;
            } else {
                ni = base + k;
                nterm = m.term[ni];
                nxt = m.load(ni);
            }
        }
    };
    auto swap = [&]() {
        if (i < 0 && ni >= 0) {
            if (nterm == 0) {
                cur = nxt;
                m.prepare(cur);
                i = ni;
                taken = 0;
            }
            ni = -1;
        }
    };
    prefetch();
    for (;;) {
        swap();
        prefetch();
        const bool active = i >= 0;
        if (__ballot_sync(kFull, active || ni >= 0) == 0)
            break;
        int ran = 0;
        bool fin = false;
        if (active) {
            const int64_t room = budget - taken;
            ran = m.run(cur, int(room < chunk ? room : chunk), fin);
            taken += ran;
        }
        ranSum += (unsigned long long)ran;
        slots += (unsigned long long)chunk;
        if (active && (fin || taken >= budget)) {
            m.store(i, cur);
            if (fin) {
                m.term[i] = 1;
                ++finCount;
            }
            longest = uint32_t(taken) > longest ? uint32_t(taken) : longest;
            i = -1;
        }
    }
    blockFlush(finCount, longest, ranSum, finished, steps, stepsum);
    if (util != nullptr) {
        const unsigned long long r = warpSum(ranSum), sl = warpSum(slots);
        if (lane == 0) {
            atomicAdd(&util[0], r);
            atomicAdd(&util[1], sl);
        }
    }
}

}  // namespace eb
