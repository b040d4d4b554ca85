// The oscillator's step entries in the hawk kernel ABI, so eagle's own launch
// path (run_device, launch_raw, BoundPlan.launch/_range/_persist) can drive them.
//
// Argument order: the role arguments of the kernel's arg_spec, packed as eagle's
// registry packs them (plugin/plugin_registry/registry.h:605-710): a 32-byte
// handle per per-sample / terminated / mutable / lookup plane, float64 uniforms
// by value. The arg_spec of the oscillator (README.md:89-97 plus the two planes
// a finishing, automatic kernel binds, python/eagle/_until_done.py:58-66):
//
//   ("per_sample", "omega"), ("uniform", "t_end"), ("uniform", "dt"),
//   ("terminated", "terminated"), ("mutable", "x"), ("mutable", "v"),
//   ("mutable", "t"), ("lookup", "finished_count"), ("lookup", "fused_steps")
//
// (the "_spread" entries take t_end as ("per_sample", "t_end") instead). Then the
// partition triple ``int64 base, count, nSamples`` (eagle/exec/DeviceKernel.h:47-84),
// then the fast-entry tails of python/eagle/_plan_binding.py:455-460 / :582-591:
//   _range:   uint32* hawk_steps, uint64* hawk_stepsum
//   _persist: uint32* hawk_next, uint64* hawk_util, uint32* hawk_steps,
//             uint64* hawk_stepsum, uint32 hawk_chunk
// ``fused_steps`` (int64) is the steps one launch may take per sample.
#include "schedule.cuh"

#include <map>
#include <mutex>
#include <string>

namespace eb {

/** t_end as a Param (by value) or a per-sample plane (a handle). */
template <bool Spread>
struct TEnd;
template <>
struct TEnd<false> {
    double v;
    __device__ __forceinline__ double at(int64_t) const { return v; }
};
template <>
struct TEnd<true> {
    ScalarHandle h;
    __device__ __forceinline__ double at(int64_t i) const { return static_cast<const double*>(h.data)[i]; }
};

__device__ __forceinline__ double* dplane(const ScalarHandle& h) { return static_cast<double*>(h.data); }

/** The plain and range entries: one lane per sample of [base, base + count). */
template <bool Fma, bool Spread>
__device__ __forceinline__ void rangeBody(const ScalarHandle& omega, const TEnd<Spread>& tEnd, double dt,
    const ScalarHandle& terminated, const ScalarHandle& x, const ScalarHandle& v, const ScalarHandle& t,
    const ScalarHandle& finished, const ScalarHandle& fused, int64_t base, int64_t count, uint32_t* steps,
    unsigned long long* stepsum)
{
    const int64_t j = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t i = base + j;
    uint8_t* term = static_cast<uint8_t*>(terminated.data);
    const int64_t budget = *static_cast<const int64_t*>(fused.data);
    int64_t taken = 0;
    bool fin = false;
    if (j < count && term[i] == 0) {
        Oscillator<Fma> s;
        s.x = dplane(x)[i];
        s.v = dplane(v)[i];
        s.t = dplane(t)[i];
        s.c = Oscillator<Fma>::coeff(dt, static_cast<const double*>(omega.data)[i]);
        s.te = tEnd.at(i);
        taken = s.runLong(dt, budget, fin);
        dplane(x)[i] = s.x;
        dplane(v)[i] = s.v;
        dplane(t)[i] = s.t;
        if (fin)
            term[i] = 1;
    }
    blockFlush(fin ? 1u : 0u, uint32_t(taken), (unsigned long long)taken, static_cast<uint32_t*>(finished.data),
        steps, stepsum);
}

#define EB_OSC_ROLES(TEND_T)                                                                                  \
    ScalarHandle omega, TEND_T tEnd, double dt, ScalarHandle terminated, ScalarHandle x, ScalarHandle v,     \
        ScalarHandle t, ScalarHandle finished, ScalarHandle fused, int64_t base, int64_t count, int64_t nSamples

template <bool Fma, bool Spread>
__global__ __launch_bounds__(256) void oscillatorPlain(EB_OSC_ROLES(TEnd<Spread>))
{
    (void)nSamples;
    rangeBody<Fma, Spread>(omega, tEnd, dt, terminated, x, v, t, finished, fused, base, count, nullptr, nullptr);
}

template <bool Fma, bool Spread>
__global__ __launch_bounds__(256) void oscillatorRange(EB_OSC_ROLES(TEnd<Spread>), uint32_t* hawkSteps,
    unsigned long long* hawkStepsum)
{
    (void)nSamples;
    rangeBody<Fma, Spread>(omega, tEnd, dt, terminated, x, v, t, finished, fused, base, count, hawkSteps,
        hawkStepsum);
}

/** t after k steps of a sample that starts at t = +0: T[0] = +0, T[k + 1] = T[k] + dt,
 *  rounded -- one sequence for every such sample, since dt is a Param. A CTA keeps
 *  every S-th term (S a power of two, at most kTCoarse + 1 terms) in shared memory;
 *  a sample then finds the step it stops at (the first k >= 1 with T[k] >= t_end,
 *  the model's step-then-test) by a binary search of the coarse terms and at most S
 *  additions from the one below, instead of adding dt and testing at every step. The
 *  terms are the very additions the sample's own steps would make, so its t, its
 *  stop step and its x, v are those of the step-by-step run, bit for bit. */
constexpr int kTCoarse = 5120;          // coarse terms a CTA keeps (40 KB of shared memory)
constexpr int64_t kTMaxBudget = 65536;  // longer runs keep the step-by-step test

struct TTable {
    const double* c;  // c[j] = T[j * stride], j <= budget / stride
    int stride;       // 0: no table (dt negative, infinite or NaN, or a budget too long)
    int64_t budget;
    double perTerm;   // 1 / (dt * stride): the coarse index of a t, roughly (T[k] is close to k dt)
};

/** Terms between kept ones for a run of ``budget`` steps: a power of two keeping at
 *  most kTCoarse + 1 of them. */
__device__ __forceinline__ int tStride(int64_t budget)
{
    int stride = 1;
    while (int64_t(stride) * kTCoarse < budget)
        stride *= 2;
    return stride;
}

/** Built by thread 0 of the CTA; the others wait at the barrier that follows. */
__device__ __forceinline__ int buildTTable(double* c, double dt, int64_t budget)
{
    if (!(dt >= 0.0 && dt <= 1.7976931348623157e308) || budget < 1 || budget > kTMaxBudget)
        return 0;
    const int stride = tStride(budget);
    const int last = int(budget / stride);
    double tt = 0.0;
    c[0] = 0.0;
    for (int j = 1; j <= last; ++j) {  // stride additions per kept term, no index arithmetic in between
        for (int r = 0; r < stride; ++r)
            tt = __dadd_rn(tt, dt);
        c[j] = tt;
    }
    return stride;
}

/** One t sequence per device, kept across launches: the first launch that finds the
 *  slot empty claims it (state 0 -> 1), builds its sequence in shared memory as
 *  usual, publishes it with its key (dt's bits, budget) and sets state 2; a later
 *  launch with the same key copies it instead of building (a chunked run launches the
 *  same sequence many times). A launch finding another key, or the slot being
 *  built, builds its own; the slot is never rewritten once published, so no launch
 *  ever reads a sequence that is changing. */
__device__ double g_tSeq[kTCoarse + 1];
__device__ unsigned long long g_tKey[2];
__device__ int g_tState;

/** Thread 0: whether the cached sequence for (dt, budget) can be copied (its stride in
 *  ``stride``); otherwise builds into ``c`` and, when it claimed the slot, publishes. */
__device__ __forceinline__ bool cachedTTable(double* c, double dt, int64_t budget, int& stride)
{
    const unsigned long long key0 = (unsigned long long)__double_as_longlong(dt), key1 = (unsigned long long)budget;
    const int state = *reinterpret_cast<volatile int*>(&g_tState);
    if (state == 2) {
        __threadfence();
        if (__ldcg(&g_tKey[0]) == key0 && __ldcg(&g_tKey[1]) == key1) {
            stride = tStride(budget);
            return true;
        }
    }
    stride = buildTTable(c, dt, budget);
    if (stride != 0 && state == 0 && atomicCAS(&g_tState, 0, 1) == 0) {
        const int64_t last = budget / stride;
        for (int64_t j = 0; j <= last; ++j)
            g_tSeq[j] = c[j];
        g_tKey[0] = key0;
        g_tKey[1] = key1;
        __threadfence();
        atomicExch(&g_tState, 2);
    }
    return false;
}

/** For a sample at t = +0 with end ``te``: the steps it runs within ``budget``
 *  (``target``), whether it stops on the last of them, and its t after them. The
 *  first coarse term at or past te is guessed from te / (dt stride) and confirmed by
 *  its neighbour (a binary search when the guess misses by more than one), then at
 *  most ``stride`` additions find the step. */
__device__ __forceinline__ void tTarget(const TTable& T, double dt, double te, int64_t& target, bool& stops,
    double& tAfter)
{
    const int64_t last = T.budget / T.stride;  // coarse terms 0..last
    // j: the first index >= 1 with c[j] >= te, or last + 1
    int64_t g = 1;
    if (te > 0.0) {
        const double e = te * T.perTerm;
        g = e < double(last) ? int64_t(e) : last;
        g = g < 1 ? 1 : g;
    }
    int64_t j;
    if (T.c[g] >= te) {
        if (g == 1 || T.c[g - 1] < te) {
            j = g;
        } else {
            int64_t lo = 1, hi = g - 1;
            while (lo < hi) {
                const int64_t mid = (lo + hi) >> 1;
                if (T.c[mid] >= te)
                    hi = mid;
                else
                    lo = mid + 1;
            }
            j = lo;
        }
    } else if (g == last || T.c[g + 1] >= te) {
        j = g + 1;
    } else {
        int64_t lo = g + 2, hi = last + 1;
        while (lo < hi) {
            const int64_t mid = (lo + hi) >> 1;
            if (T.c[mid] >= te)
                hi = mid;
            else
                lo = mid + 1;
        }
        j = lo;
    }
    int64_t k = (j - 1) * T.stride;
    double tt = T.c[j - 1];
    stops = false;
    while (k < T.budget) {
        ++k;
        tt = __dadd_rn(tt, dt);
        if (tt >= te) {
            stops = true;
            break;
        }
    }
    target = k;
    tAfter = tt;
}

/** The persistent entry. Every lane holds its current sample and, one chunk
 *  ahead, the NEXT one: at each chunk head the lanes of a warp lacking a next
 *  sample claim the following indices together off ``hawk_next`` (one atomic per
 *  warp) and issue its loads, which complete while the chunk runs; a lane whose
 *  sample ended takes its prefetched one without waiting. A claimed sample
 *  already terminated is skipped (python/eagle/_plan_binding.py:431-446). Each
 *  lane runs up to ``chunk`` steps of its sample per head, within the budget; a
 *  lane whose sample ends mid-chunk waits, masked, for the next head. */
template <bool Fma, bool Spread>
__device__ __forceinline__ void persistBody(EB_OSC_ROLES(TEnd<Spread>), uint32_t* hawkNext,
    unsigned long long* hawkUtil, uint32_t* hawkSteps, unsigned long long* hawkStepsum, uint32_t hawkChunk,
    const int32_t* __restrict__ order)
{
    (void)nSamples;
    const unsigned lane = threadIdx.x & 31u;
    uint8_t* term = static_cast<uint8_t*>(terminated.data);
    const double* om = static_cast<const double*>(omega.data);
    const int64_t budget = *static_cast<const int64_t*>(fused.data);
    const int chunk = hawkChunk == 0 ? 32 : int(hawkChunk < (1u << 20) ? hawkChunk : (1u << 20));
    uint32_t* finished_ = static_cast<uint32_t*>(finished.data);
    __shared__ double sT[kTCoarse + 1];
    __shared__ int sStride, sCached;
    if (threadIdx.x == 0) {
        int stride = 0;
        sCached = cachedTTable(sT, dt, budget, stride) ? 1 : 0;
        sStride = stride;
    }
    __syncthreads();
    if (sCached != 0) {  // copy the device's sequence in
        const int64_t last = budget / sStride;
        for (int64_t j = threadIdx.x; j <= last; j += blockDim.x)
            sT[j] = __ldcg(&g_tSeq[j]);
        __syncthreads();
    }
    const TTable table{sT, sStride, budget, sStride != 0 ? 1.0 / (dt * double(sStride)) : 0.0};
    Oscillator<Fma> cur{}, nxt{};
    int64_t i = -1, ni = -1;  // the lane's current and prefetched samples (-1: none)
    bool fast = false;        // the current sample started at t = +0: its stop is known
    int64_t target = 0;       // fast: the steps it runs in this launch
    bool stops = false;       // fast: it terminates on the last of them
    double tAfter = 0.0;      // fast: its t after them
    uint8_t nterm = 0;        // the prefetched sample's mask byte
    int64_t taken = 0;        // steps of the current sample so far
    bool exhausted = false;
    uint32_t finCount = 0, longest = 0;  // the lane's run counters, flushed once at the end
    unsigned long long ranSum = 0, slots = 0;

    // lanes without a next sample claim one and issue its loads (no wait here)
    auto prefetch = [&]() {
        const bool needs = ni < 0 && !exhausted;
        const unsigned want = __ballot_sync(kFull, needs);
        if (want == 0)
            return;
        const unsigned leader = __ffs(want) - 1;
        uint32_t first = 0;
        if (lane == leader)
            first = atomicAdd(hawkNext, uint32_t(__popc(want)));
        first = __shfl_sync(kFull, first, leader);
        if (needs) {
            const int64_t k = int64_t(first) + __popc(want & ((1u << lane) - 1u));
            if (k >= count) {
                exhausted = true;
            } else {
                ni = order != nullptr ? int64_t(__ldg(order + k)) : base + k;  // the claim's sample
                nterm = term[ni];
                nxt.x = dplane(x)[ni];
                nxt.v = dplane(v)[ni];
                nxt.t = dplane(t)[ni];
                nxt.c = om[ni];  // the coefficient is formed at the swap
                nxt.te = tEnd.at(ni);
            }
        }
    };
    // lanes without a current sample take the prefetched one (a terminated one is skipped)
    auto swap = [&]() {
        if (i < 0 && ni >= 0) {
            if (nterm == 0) {
                cur = nxt;
                cur.c = Oscillator<Fma>::coeff(dt, nxt.c);
                i = ni;
                taken = 0;
                fast = table.stride != 0 && __double_as_longlong(cur.t) == 0;
                if (fast)
                    tTarget(table, dt, cur.te, target, stops, tAfter);
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
            if (fast) {
                const int64_t room = target - taken;
                ran = int(room < chunk ? room : chunk);
                cur.stepsXV(dt, ran);
                taken += ran;
                if (taken == target) {
                    cur.t = tAfter;
                    fin = stops;
                }
            } else {
                const int64_t room = budget - taken;
                ran = cur.run(dt, int(room < chunk ? room : chunk), fin);
                taken += ran;
            }
        }
        ranSum += (unsigned long long)ran;
        slots += (unsigned long long)chunk;
        if (active && (fin || taken >= budget)) {
            dplane(x)[i] = cur.x;
            dplane(v)[i] = cur.v;
            dplane(t)[i] = cur.t;
            if (fin) {
                term[i] = 1;
                ++finCount;
            }
            longest = uint32_t(taken) > longest ? uint32_t(taken) : longest;
            i = -1;
        }
    }
    blockFlush(finCount, longest, ranSum, finished_, hawkSteps, hawkStepsum);
    if (hawkUtil != nullptr) {
        const unsigned long long r = warpSum(ranSum), sl = warpSum(slots);
        if (lane == 0) {
            atomicAdd(&hawkUtil[0], r);
            atomicAdd(&hawkUtil[1], sl);
        }
    }
}

template <bool Fma, bool Spread>
__global__ __launch_bounds__(256, 4) void oscillatorPersist(EB_OSC_ROLES(TEnd<Spread>), uint32_t* hawkNext,
    unsigned long long* hawkUtil, uint32_t* hawkSteps, unsigned long long* hawkStepsum, uint32_t hawkChunk)
{
    persistBody<Fma, Spread>(omega, tEnd, dt, terminated, x, v, t, finished, fused, base, count, nSamples,
        hawkNext, hawkUtil, hawkSteps, hawkStepsum, hawkChunk, nullptr);
}

/** The persistent entry with the claims taken through ``order``: claim k runs sample
 *  order[k] (a permutation of [0, count) with base 0), so that an order grouping
 *  samples of like length keeps a warp's lanes busy together. The engine's persist
 *  mode launches it behind its longest-first order (order.cu). */
template <bool Fma, bool Spread>
__global__ __launch_bounds__(256, 4) void oscillatorPersistOrdered(EB_OSC_ROLES(TEnd<Spread>), uint32_t* hawkNext,
    unsigned long long* hawkUtil, uint32_t* hawkSteps, unsigned long long* hawkStepsum, uint32_t hawkChunk,
    const int32_t* order)
{
    persistBody<Fma, Spread>(omega, tEnd, dt, terminated, x, v, t, finished, fused, base, count, nSamples,
        hawkNext, hawkUtil, hawkSteps, hawkStepsum, hawkChunk, order);
}

void addGamblerEntries(std::map<std::string, const void*>& m);  // walks.cu
void addLorenzEntries(std::map<std::string, const void*>& m);   // lorenz.cu

namespace {

template <bool Fma, bool Spread>
void addEntries(std::map<std::string, const void*>& m, const std::string& stem)
{
    const std::string suffix = Fma ? "_fma" : "";
    m[stem + suffix] = reinterpret_cast<const void*>(&oscillatorPlain<Fma, Spread>);
    m[stem + "_range" + suffix] = reinterpret_cast<const void*>(&oscillatorRange<Fma, Spread>);
    m[stem + "_persist" + suffix] = reinterpret_cast<const void*>(&oscillatorPersist<Fma, Spread>);
}

const std::map<std::string, const void*>& entryTable()
{
    static const std::map<std::string, const void*> table = [] {
        std::map<std::string, const void*> m;
        addEntries<false, false>(m, "oscillator");
        addEntries<true, false>(m, "oscillator");
        addEntries<false, true>(m, "oscillator_spread");
        addEntries<true, true>(m, "oscillator_spread");
        addGamblerEntries(m);
        addLorenzEntries(m);
        return m;
    }();
    return table;
}

}  // namespace

/** The host stub of a built-in entry by name (nullptr if unknown). */
const void* entryStub(const std::string& name)
{
    const auto& t = entryTable();
    const auto it = t.find(name);
    return it == t.end() ? nullptr : it->second;
}

/** The ordered persistent oscillator entry (the engine's; not in the name table). */
const void* orderedPersistStub(bool fma, bool spread)
{
    if (fma)
        return spread ? reinterpret_cast<const void*>(&oscillatorPersistOrdered<true, true>)
                      : reinterpret_cast<const void*>(&oscillatorPersistOrdered<true, false>);
    return spread ? reinterpret_cast<const void*>(&oscillatorPersistOrdered<false, true>)
                  : reinterpret_cast<const void*>(&oscillatorPersistOrdered<false, false>);
}

}  // namespace eb

using namespace eb;

extern "C" __attribute__((visibility("default"))) eagle_backend_status eagle_backend_x_b200_entry(
    const char* name, int32_t device, uint64_t* function)
{
    return guarded([&] {
        if (name == nullptr || function == nullptr)
            invalid("eagle_backend_x_b200_entry: null name or output");
        const void* stub = entryStub(name);
        if (stub == nullptr)
            fail(EAGLE_BACKEND_INDEX, std::string("eagle_backend_x_b200_entry: no built-in entry named '") + name + "'");
        DeviceScope scope(resolveDevice(device, 0));
        cudaFunction_t f = nullptr;
        cudaCheck(cudaGetFuncBySymbol(&f, stub), "cudaGetFuncBySymbol");
        *function = reinterpret_cast<uint64_t>(f);
    });
}
