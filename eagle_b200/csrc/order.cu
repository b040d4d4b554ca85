// The longest-first claim order of the persistent oscillator.
//
// A persistent warp runs its 32 lanes' samples in lockstep, 512 steps per claim
// head: a lane whose sample stops early idles until the head, and a batch with
// t_end log-uniform over three decades leaves a lane idle about a fifth of the
// time when samples are claimed in index order. The oscillator's stop step is
// known before it steps (about (t_end - t) / dt), so the engine first sorts the
// samples by it, longest first, and the lanes claim them in that order: a warp's
// lanes then hold samples of like length, and the long ones start first, which
// also shortens the launch's tail. Only the claim order changes -- every sample
// takes the same steps in the same order, so every plane, the mask and the run
// counters keep their bits.
//
// The sort is local: each run of 32768 consecutive samples (fewer for a small batch,
// down to 4096) is ordered within its own range by a counting sort over at most
// kBuckets buckets of ``width`` steps (the budget spread over them), longest first,
// samples already terminated last. Two launches: stopKeyKernel streams the mask,
// t_end and t (17 bytes a sample) near the rate of a copy and writes each sample's
// 2-byte bucket; stopSortKernel then sorts each run in one CTA, all in shared
// memory, from keys that are still in L2, builds the run's order in shared memory
// and writes it out coalesced, and counts the run's terminated samples for the run
// report (so the launch needs no mask count of its own). At 2^24 samples: 58 + 44
// us, where one kernel doing both per run (its loads, then its scattered 4-byte
// order stores) took 149 us and the mask count 6.5 more.
//
// The lanes claim the runs one after another, so a claim's loads and its results'
// stores stay inside a few runs at a time: the gathered planes are read once from
// DRAM and their partly written sectors merge in L2 (a global sort made every access a random one: 5.9 ms against 5.3 ms in index
// order, where the same samples moved into sorted order beforehand took 3.6 ms).
#include "common.cuh"

#include <mutex>

namespace eb {
namespace {

constexpr int kThreads = 1024;
constexpr int64_t kTile = 32768;  // samples per run (and per CTA), at most
constexpr int64_t kMinRun = 4096;  // the shortest run a small batch is cut into
constexpr int kBuckets = 2048;    // step buckets; bucket kBuckets: terminated
constexpr int kSlots = kBuckets + 1;
constexpr int kSubs = 4;          // copies of the histogram
constexpr int kPerScan = (kSlots + kThreads - 1) / kThreads;
constexpr size_t kSmem = size_t(kSubs) * kSlots * sizeof(uint32_t) + size_t(kTile) * sizeof(uint16_t);

constexpr int kKeyThreads = 256;
constexpr int kKeyPer = 8;  // samples per thread of the key pass, their loads issued together
constexpr int kVecPer = int(kTile / 8 / kThreads);  // 16-byte key loads per thread of a full run

struct StopKeyArgs {
    const double* tEnd;  // null: ``tEndU`` for every sample
    double tEndU;
    const double* t;
    const uint8_t* term;
    int64_t n;
    double dt, perDt;  // perDt = 1 / dt
    int64_t budget;
    int64_t width;  // steps per bucket
    int64_t run;    // samples per run, a power of two in [kMinRun, kTile]
    int64_t woven;  // runs whose claims are interleaved (the full runs, or 0: runs claimed one after another)
    uint16_t* keys;  // n bucket keys, 16-byte aligned
    int32_t* order;
    uint32_t* finished;  // += the samples already terminated (the mask's set bytes, counted by the sort); null: not counted
};

constexpr int64_t kWeave = 32;  // claims a run gives before the next run's turn (one warp's worth)

/** The claim index of place ``pos`` of run ``r`` (the runs' own longest-first order):
 *  run after run, or -- over the first ``woven`` runs -- kWeave places of every run in
 *  turn, so that the longest samples of all those runs are claimed first. */
__device__ __forceinline__ int64_t claimOf(const StopKeyArgs& a, int64_t r, int64_t pos)
{
    if (r >= a.woven)
        return r * a.run + pos;
    return (pos / kWeave) * (kWeave * a.woven) + r * kWeave + pos % kWeave;
}

/** Sample i's bucket from its mask byte, t_end and t: its estimated steps this run,
 *  ceil((t_end - t) / dt) kept in [1, budget] (the budget for a non-finite estimate
 *  or dt not above zero), over ``width``, counted from the longest (bucket 0) down;
 *  kBuckets for a terminated sample. */
__device__ __forceinline__ uint32_t stopKeyOf(const StopKeyArgs& a, uint8_t done, double te, double t0)
{
    if (done != 0)
        return kBuckets;
    const double d = (te - t0) * a.perDt;  // an estimate: only the order depends on it
    int64_t steps = a.budget;
    if (a.dt > 0.0 && d < double(a.budget))  // false for NaN
        steps = d <= 1.0 ? 1 : int64_t(ceil(d));
    steps = steps < 1 ? 1 : (steps > a.budget ? a.budget : steps);
    const int64_t k = (steps - 1) / a.width;
    return uint32_t(kBuckets - 1) - uint32_t(k < kBuckets ? k : kBuckets - 1);
}

/** Sample i's bucket key for every i < n: the mask byte, t_end and t of kKeyPer
 *  samples a thread (a stride of kKeyThreads apart, so every load is coalesced), all
 *  loads out before any key is formed. */
__global__ __launch_bounds__(kKeyThreads) void stopKeyKernel(StopKeyArgs a)
{
    const int64_t i0 = int64_t(blockIdx.x) * (kKeyThreads * kKeyPer) + threadIdx.x;
    uint8_t done[kKeyPer];
    double te[kKeyPer], t0[kKeyPer];
#pragma unroll
    for (int r = 0; r < kKeyPer; ++r) {
        const int64_t i = i0 + int64_t(r) * kKeyThreads;
        const int64_t at = i < a.n ? i : 0;
        done[r] = a.term[at];
        te[r] = a.tEnd != nullptr ? a.tEnd[at] : a.tEndU;
        t0[r] = a.t[at];
    }
#pragma unroll
    for (int r = 0; r < kKeyPer; ++r) {
        const int64_t i = i0 + int64_t(r) * kKeyThreads;
        if (i < a.n)
            a.keys[i] = uint16_t(stopKeyOf(a, done[r], te[r], t0[r]));
    }
}

/** The histogram copy that sample j of a run counts into: copies alternate every 8
 *  samples, so the lanes of one shared-memory atomic (8 or 32 samples apart) spread
 *  over all kSubs copies and the many samples of a crowded bucket (short stops)
 *  collide kSubs times less. */
__device__ __forceinline__ int subOf(int j) { return (j >> 3) & (kSubs - 1); }

/** The run's keys of whole 16-byte groups (8 keys each) that thread t takes: group
 *  t + q kThreads, zeros past ``vecs``; the loads all go out together. */
__device__ __forceinline__ void loadKeyGroups(const uint4* src, int vecs, uint4 (&w)[kVecPer])
{
#pragma unroll
    for (int q = 0; q < kVecPer; ++q) {
        const int v = int(threadIdx.x) + q * kThreads;
        w[q] = v < vecs ? src[v] : make_uint4(0u, 0u, 0u, 0u);
    }
}

__device__ __forceinline__ uint32_t keyAt(const uint4& w, int e)
{
    const uint32_t word = e < 2 ? w.x : e < 4 ? w.y : e < 6 ? w.z : w.w;
    return (word >> (16 * (e & 1))) & 0xffffu;
}

/** One CTA per run of ``a.run`` samples, from the keys the key pass left in L2: a
 *  histogram of the run's keys, the buckets' starts by a CTA scan, then each sample's
 *  place in its bucket (in no particular order within it) taken by a shared-memory
 *  atomic. The run's order is built in shared memory (2-byte offsets into the run)
 *  and written out in place order, coalesced: writing each sample's claim straight
 *  to global memory scattered 4-byte stores over the run's 128 KB, one L1 wavefront
 *  per lane (104 us at 2^24 against about 30). Each of the kSubs histogram copies
 *  gets its own range inside the bucket. */
__global__ __launch_bounds__(kThreads, 2) void stopSortKernel(StopKeyArgs a)
{
    extern __shared__ __align__(16) uint32_t smem[];
    uint32_t* cnt = smem;                                                  // [kSubs][kSlots]
    uint16_t* ord = reinterpret_cast<uint16_t*>(smem + kSubs * kSlots);   // [kTile]: place -> offset
    __shared__ uint32_t scan[33];
    const int t = int(threadIdx.x);
    const int64_t i0 = int64_t(blockIdx.x) * a.run;
    const int live = int(a.n - i0 < a.run ? a.n - i0 : a.run);
    const int vecs = live / 8;  // whole 16-byte groups of keys (i0 is a multiple of 8)
    const uint4* src = reinterpret_cast<const uint4*>(a.keys + i0);
    uint4 w[kVecPer];
    loadKeyGroups(src, vecs, w);
    for (int b = t; b < kSubs * kSlots; b += kThreads)
        cnt[b] = 0;
    __syncthreads();
#pragma unroll
    for (int q = 0; q < kVecPer; ++q) {
        const int v = t + q * kThreads;
        if (v < vecs) {
#pragma unroll
            for (int e = 0; e < 8; ++e)
                atomicAdd(&cnt[subOf(v * 8 + e) * kSlots + int(keyAt(w[q], e))], 1u);
        }
    }
    for (int j = vecs * 8 + t; j < live; j += kThreads)  // the last run's ragged end
        atomicAdd(&cnt[subOf(j) * kSlots + int(a.keys[i0 + j])], 1u);
    __syncthreads();
    if (a.finished != nullptr && t == kThreads - 1) {  // the run's terminated samples: bucket kBuckets
        uint32_t c = 0;
#pragma unroll
        for (int q = 0; q < kSubs; ++q)
            c += cnt[q * kSlots + kBuckets];
        if (c != 0)
            atomicAdd(a.finished, c);
    }
    // positions run bucket by bucket (longest first), and inside a bucket copy by copy:
    // thread t owns buckets [kPerScan t, kPerScan t + kPerScan)
    uint32_t mine = 0;
#pragma unroll
    for (int q = 0; q < kPerScan; ++q) {
        const int b = t * kPerScan + q;
#pragma unroll
        for (int c = 0; c < kSubs; ++c)
            mine += b < kSlots ? cnt[c * kSlots + b] : 0u;
    }
    uint32_t total = 0;
    uint32_t run = blockExclusiveSum(mine, total, scan);
#pragma unroll
    for (int q = 0; q < kPerScan; ++q) {
        const int b = t * kPerScan + q;
#pragma unroll
        for (int c = 0; c < kSubs; ++c)
            if (b < kSlots) {
                const uint32_t here = cnt[c * kSlots + b];
                cnt[c * kSlots + b] = run;  // now the copy's next position in the bucket
                run += here;
            }
    }
    __syncthreads();
    loadKeyGroups(src, vecs, w);  // again from L2: holding them through the scan costs a CTA per SM
#pragma unroll
    for (int q = 0; q < kVecPer; ++q) {
        const int v = t + q * kThreads;
        if (v < vecs) {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int j = v * 8 + e;
                ord[atomicAdd(&cnt[subOf(j) * kSlots + int(keyAt(w[q], e))], 1u)] = uint16_t(j);
            }
        }
    }
    for (int j = vecs * 8 + t; j < live; j += kThreads)
        ord[atomicAdd(&cnt[subOf(j) * kSlots + int(a.keys[i0 + j])], 1u)] = uint16_t(j);
    __syncthreads();
    for (int p = t; p < live; p += kThreads)
        a.order[claimOf(a, blockIdx.x, p)] = int32_t(i0 + int64_t(ord[p]));
}

}  // namespace

namespace {

/** The current device's L2 size in bytes, looked up once per device. */
int l2Bytes()
{
    static std::mutex mu;
    static int bytes[64] = {};
    int dev = 0;
    cudaCheck(cudaGetDevice(&dev), "cudaGetDevice");
    std::lock_guard<std::mutex> lock(mu);
    int& b = bytes[dev & 63];
    if (b == 0)
        cudaCheck(cudaDeviceGetAttribute(&b, cudaDevAttrL2CacheSize, dev), "cudaDeviceGetAttribute");
    return b;
}

}  // namespace

/** Bytes of the claim order proper (n int32), rounded to 256. */
size_t orderPart(int64_t n) { return (size_t(n) * sizeof(int32_t) + 255) / 256 * 256; }

/** Device bytes of the claim order over n samples: the order, then the n 2-byte
 *  bucket keys the sort reads. */
size_t stopOrderBytes(int64_t n) { return orderPart(n) + (size_t(n) * sizeof(uint16_t) + 255) / 256 * 256; }

/** Raise the sort kernel's dynamic shared-memory limit on the current device, once
 *  per device (the engine calls it at create, outside any stream capture). */
void prepareStopOrder()
{
    static std::mutex mu;
    static bool raised[64] = {};
    int dev = 0;
    cudaCheck(cudaGetDevice(&dev), "cudaGetDevice");
    std::lock_guard<std::mutex> lock(mu);
    if (!raised[dev & 63]) {
        cudaCheck(cudaFuncSetAttribute(stopSortKernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmem)),
            "cudaFuncSetAttribute");
        raised[dev & 63] = true;
    }
}

/** Enqueue the claim order of samples [0, n) into ``order`` (stopOrderBytes(n)
 *  bytes, 16-byte aligned): each run of up to 32768 samples longest first, t_end
 *  from ``tEnd`` (null: ``tEndU`` for all), t from ``t``, the mask ``term``; stop
 *  steps estimated against ``budget``. The mask's set bytes are added to
 *  ``finished`` unless it is null. */
void enqueueStopOrder(const double* tEnd, double tEndU, const double* t, const uint8_t* term, int64_t n, double dt,
    int64_t budget, int32_t* order, uint32_t* finished, cudaStream_t s)
{
    if (n <= 0)
        return;
    StopKeyArgs a{};
    a.tEnd = tEnd;
    a.tEndU = tEndU;
    a.t = t;
    a.term = term;
    a.n = n;
    a.dt = dt;
    a.perDt = 1.0 / dt;
    a.budget = budget > 0 ? budget : 1;
    a.width = (a.budget + kBuckets - 1) / kBuckets;
    a.order = order;
    a.keys = reinterpret_cast<uint16_t*>(reinterpret_cast<char*>(order) + orderPart(n));
    a.finished = finished;
    // A run's sort takes one CTA the same time whatever else runs, so a batch too small
    // to give every SM two runs of kTile is cut into shorter runs (down to kMinRun):
    // the order then groups lengths a little less finely, but its launch no longer
    // outlasts the batch's own steps at a few million samples (a shard of the
    // multi-GPU split).
    const int64_t fill = int64_t(2) * smCount();
    a.run = kTile;
    while (a.run > kMinRun && (n + a.run - 1) / a.run < fill)
        a.run /= 2;
    // Interleave the full runs' claims when the batch's planes (40 bytes a sample, the
    // mask and the order entry: 48 bytes to spare) fit in L2: then the claims'
    // scattered loads and stores cost no extra DRAM traffic, and the longest samples of
    // every run start first instead of the last runs' longest starting last, which
    // cuts the launch's tail (2^21 samples: 0.554 against 0.609 ms per launch). Past
    // L2 the scattered accesses cost more than the tail (2^22: 1.063 against 1.049 ms;
    // 2^24: 5.71 against 3.64 ms), so larger batches claim run after run.
    a.woven = n * 48 <= int64_t(l2Bytes()) ? n / a.run : 0;
    prepareStopOrder();
    stopKeyKernel<<<unsigned((n + kKeyThreads * kKeyPer - 1) / (kKeyThreads * kKeyPer)), kKeyThreads, 0, s>>>(a);
    launchCheck("stop order");
    stopSortKernel<<<unsigned((n + a.run - 1) / a.run), kThreads, kSmem, s>>>(a);
    launchCheck("stop order");
}

}  // namespace eb
