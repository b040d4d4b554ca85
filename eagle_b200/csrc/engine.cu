// The until-done engine: eagle's until-done loop (python/eagle/_until_done.py:528-1845)
// for one built-in model, as one B200-native unit.
//
// BAND mode (the loop eagle captures as a WHILE graph over step launch,
// compaction and policy, _until_done.py:844-985) is here ONE kernel per pass
// inside one CUDA graph with a conditional WHILE node:
//
//   pass p:  each CTA takes 256-sample tiles off a counter; a thread loads its
//            sample's state (pass 0: straight from the planes, skipping set mask
//            bytes; later passes: from the compacted state of pass p-1, a dense SoA
//            copy, so every load and store is coalesced), runs the pass's ``word``
//            steps with the state in registers, writes a sample that terminated
//            (or every sample, on the pass that reaches max_steps) back to its
//            planes and mask, and appends the survivors, in sample order, to the
//            other compacted buffer: a CTA-wide scan plus a decoupled look-back
//            over the earlier tiles gives each tile its offset. The last CTA to
//            finish runs the band policy (eagle/policy/Launch.h:184-190's bandK,
//            with R priced for this pass) and sets the WHILE condition on the
//            device, so a replay never returns to the host.
//
// PERSIST mode is one launch of the persistent entry (lanes claim samples off a
// counter, _plan_binding.py:431-476); FUSED mode one launch of the range entry
// with the whole budget (_until_done.py:1016-1135's "fused_one"). All three leave
// the same bits in every plane: each sample takes the same steps in the same
// order; only the schedule differs.
#include "models.cuh"

#include <algorithm>
#include <vector>

namespace eb {

// defined in compact.cu, entries.cu and order.cu
void enqueueMaskCount(const uint8_t* mask, int64_t n, uint32_t* cell, cudaStream_t s, bool zeroFirst);
const void* entryStub(const std::string& name);
const void* orderedPersistStub(bool fma, bool spread);
size_t stopOrderBytes(int64_t n);
void prepareStopOrder();
void enqueueStopOrder(const double* tEnd, double tEndU, const double* t, const uint8_t* term, int64_t n, double dt,
    int64_t budget, int32_t* order, uint32_t* finished, cudaStream_t s);

namespace {

constexpr int kBandThreads = 256;

/** The engine's device cells: the loop state one pass hands the next. */
struct Cells {
    unsigned long long epoch;    // look-back epoch: bumped per pass, never reset
    unsigned long long longest;  // the longest sample's steps in this run
    unsigned long long stepsum;  // steps executed in this run
    int64_t k, word, done, cap;  // band K, this pass's steps, steps run, max_steps
    int64_t kFirst, kMin, kMax;
    double overheadSteps, intervalSteps;
    int64_t budget;              // the persist / fused entries' fused_steps word
    uint32_t iter;               // passes run in this run
    uint32_t go;
    uint32_t live;               // samples in the compacted input of the next pass
    uint32_t liveNext;           // written by the pass's last tile
    uint32_t tileNext, ctasDone;
    uint32_t finished;           // set mask bytes
    uint32_t newly;              // samples finished in the current pass
    uint32_t err;
    uint32_t total;
    uint32_t next;               // persist: the claim counter
    uint32_t steps32;            // persist / fused: the longest sample's steps
    unsigned long long stepsum64;
    unsigned long long guard;    // band: passes started in this run (the runaway guard)
};

struct BandArgs {
    Cells* cells;
    uint64_t* status;
    const double* omega;
    const double* tend;
    double tendU, dt;
    double* x;
    double* v;
    double* t;
    uint8_t* term;
    double* rc[2];
    double* rte[2];
    double* rx[2];
    double* rv[2];
    double* rt[2];
    int32_t* ridx[2];
    int64_t n;
    cudaGraphConditionalHandle cond;
};

__device__ __forceinline__ int64_t bandK(double rate, int64_t newly, int64_t live, int64_t k, int64_t kMax,
    int64_t kMin)
{
    if (newly <= 0)
        return kMax;
    const double e2 = 2.0 * rate * double(live) * double(k) / double(newly);
    int64_t p = 1;
    while (p < (INT64_C(1) << 30) && e2 >= 2.0 * double(p) * double(p))
        p *= 2;
    return p < kMin ? kMin : (p > kMax ? kMax : p);
}

template <bool Fma, bool Spread, bool Graph>
__global__ __launch_bounds__(kBandThreads, 6) void bandKernel(BandArgs a)
{
    __shared__ uint32_t sTile;
    __shared__ uint32_t scan[33];
    __shared__ uint32_t sPrefix;
    __shared__ uint32_t sLast;
    __shared__ uint32_t sPre[kBandThreads / 32], sNew[kBandThreads / 32];
    __shared__ unsigned long long sLong[kBandThreads / 32], sSum[kBandThreads / 32];
    Cells* c = a.cells;
    const int tid = int(threadIdx.x);
    if (blockIdx.x == 0 && tid == 0) {
        // every pass takes at least one step, so a run never needs more than
        // max_steps passes: past that the loop is stopped here, whatever else happens
        const unsigned long long started = atomicAdd(&c->guard, 1ull) + 1ull;
        if (started > (unsigned long long)c->cap + 1ull) {
            atomicOr(&c->err, 2u);
            c->go = 0;
            if constexpr (Graph)
                cudaGraphSetConditional(a.cond, 0u);
        }
    }
    const uint32_t iter = c->iter;
    const uint32_t epoch = uint32_t(c->epoch);
    const int64_t word = c->word;
    const int64_t doneBefore = c->done;
    const bool last = word >= c->cap - doneBefore;  // this pass reaches max_steps
    const bool dense = iter == 0;
    const int64_t inCount = dense ? a.n : int64_t(c->live);
    const int src = int((iter + 1) & 1), dst = int(iter & 1);
    const uint32_t tiles = uint32_t((inCount + kBandThreads - 1) / kBandThreads);
    uint32_t pre = 0, newly = 0;
    unsigned long long longest = 0, stepsum = 0;
    for (;;) {
        if (tid == 0)
            sTile = atomicAdd(&c->tileNext, 1u);
        __syncthreads();
        const uint32_t tile = sTile;
        __syncthreads();
        if (tile >= tiles)
            break;
        const int64_t j = int64_t(tile) * kBandThreads + tid;
        bool valid = j < inCount;
        int64_t idx = 0;
        Oscillator<Fma> s{};
        if (valid) {
            if (dense) {
                idx = j;
                if (a.term[idx] != 0) {
                    valid = false;
                    ++pre;
                } else {
                    s.x = a.x[idx];
                    s.v = a.v[idx];
                    s.t = a.t[idx];
                    s.c = Oscillator<Fma>::coeff(a.dt, a.omega[idx]);
                    s.te = Spread ? a.tend[idx] : a.tendU;
                }
            } else {
                idx = a.ridx[src][j];
                s.x = a.rx[src][j];
                s.v = a.rv[src][j];
                s.t = a.rt[src][j];
                s.c = a.rc[src][j];
                s.te = Spread ? a.rte[src][j] : a.tendU;
            }
        }
        int64_t taken = 0;
        bool fin = false;
        if (valid)
            taken = s.run(a.dt, int(word), fin);
        bool keep = valid && !fin;
        if (valid && (fin || last)) {
            // a sample leaving the loop: its state goes home
            a.x[idx] = s.x;
            a.v[idx] = s.v;
            a.t[idx] = s.t;
            if (fin) {
                a.term[idx] = 1;
                ++newly;
            }
            const unsigned long long steps = (unsigned long long)(doneBefore + taken);
            longest = steps > longest ? steps : longest;
            keep = false;
        }
        stepsum += (unsigned long long)taken;
        uint32_t total = 0;
        const uint32_t excl = blockExclusiveSum(keep ? 1u : 0u, total, scan);
        if (tid < 32) {
            uint32_t prefix = 0;
            if (tile == 0) {
                if (tid == 0)
                    lbPublish<EpochCodec>(a.status, tile, epoch, kLbPrefix, total);
            } else {
                if (tid == 0)
                    lbPublish<EpochCodec>(a.status, tile, epoch, kLbAggregate, total);
                prefix = uint32_t(lbExclusivePrefix<EpochCodec>(a.status, tile, epoch, &c->err));
                if (tid == 0)
                    lbPublish<EpochCodec>(a.status, tile, epoch, kLbPrefix, uint64_t(prefix) + total);
            }
            if (tid == 0) {
                sPrefix = prefix;
                if (tile == tiles - 1)
                    c->liveNext = prefix + total;
            }
        }
        __syncthreads();
        if (keep) {
            const int64_t o = int64_t(sPrefix) + excl;
            a.ridx[dst][o] = int32_t(idx);
            a.rx[dst][o] = s.x;
            a.rv[dst][o] = s.v;
            a.rt[dst][o] = s.t;
            a.rc[dst][o] = s.c;
            if constexpr (Spread)
                a.rte[dst][o] = s.te;
        }
    }
    // flush the run counters: one atomic per CTA and counter
    {
        const uint32_t wp = warpSum(pre), wn = warpSum(newly);
        const unsigned long long wl = warpMax(longest), ws = warpSum(stepsum);
        if ((tid & 31) == 0) {
            sPre[tid >> 5] = wp;
            sNew[tid >> 5] = wn;
            sLong[tid >> 5] = wl;
            sSum[tid >> 5] = ws;
        }
        __syncthreads();
        if (tid == 0) {
            uint32_t p = 0, nw = 0;
            unsigned long long l = 0, u = 0;
            for (int w = 0; w < kBandThreads / 32; ++w) {
                p += sPre[w];
                nw += sNew[w];
                l = sLong[w] > l ? sLong[w] : l;
                u += sSum[w];
            }
            if (p + nw != 0)
                atomicAdd(&c->finished, p + nw);
            if (nw != 0)
                atomicAdd(&c->newly, nw);
            if (l != 0)
                atomicMax(&c->longest, l);
            if (u != 0)
                atomicAdd(&c->stepsum, u);
            __threadfence();
            sLast = atomicAdd(&c->ctasDone, 1u) == gridDim.x - 1 ? 1u : 0u;
        }
        __syncthreads();
    }
    if (sLast == 0 || tid != 0)
        return;
    // the last CTA: close the pass and decide the next one
    __threadfence();
    const uint32_t live = tiles > 0 ? *reinterpret_cast<volatile uint32_t*>(&c->liveNext) : 0u;
    const uint32_t newlyPass = *reinterpret_cast<volatile uint32_t*>(&c->newly);
    const int64_t done = doneBefore + word;
    c->done = done;
    c->live = live;
    c->iter = iter + 1;
    c->epoch = c->epoch + 1;
    const double rate = c->overheadSteps / double(live > 0 ? live : 1u) + c->intervalSteps;
    const int64_t kNext = bandK(rate, int64_t(newlyPass), int64_t(live), c->k, c->kMax, c->kMin);
    const int64_t left = c->cap - done;
    const uint32_t go = (live > 0 && left > 0) ? 1u : 0u;
    c->k = kNext;
    c->word = kNext < left ? kNext : left;
    c->go = go;
    c->newly = 0;
    c->tileNext = 0;
    c->ctasDone = 0;
    __threadfence();
    if constexpr (Graph)
        cudaGraphSetConditional(a.cond, go);
}

/** Reset the run cells and arm the WHILE condition (one thread). */
template <bool Graph>
__global__ void bandInitKernel(Cells* c, int64_t n, cudaGraphConditionalHandle cond)
{
    c->iter = 0;
    c->done = 0;
    c->k = c->kFirst;
    c->word = c->kFirst < c->cap ? c->kFirst : c->cap;
    c->finished = 0;
    c->newly = 0;
    c->live = 0;
    c->liveNext = 0;
    c->longest = 0;
    c->stepsum = 0;
    c->tileNext = 0;
    c->ctasDone = 0;
    c->err = 0;
    c->guard = 0;
    c->epoch = c->epoch + 1;
    const uint32_t go = (c->cap > 0 && n > 0) ? 1u : 0u;
    c->go = go;
    if constexpr (Graph)
        cudaGraphSetConditional(cond, go);
}

/** After the loop: a run that took no pass still reports its mask count. */
__global__ __launch_bounds__(256) void bandFinishKernel(Cells* c, const uint8_t* term, int64_t n)
{
    if (c->iter != 0)
        return;
    uint32_t cnt = 0;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        cnt += term[i] != 0 ? 1u : 0u;
    cnt = warpSum(cnt);
    if ((threadIdx.x & 31) == 0 && cnt != 0)
        atomicAdd(&c->finished, cnt);
}

struct Engine {
    int device = 0;
    uint32_t model = 0, mode = 0, flags = 0;
    int64_t n = 0, maxSteps = 0;
    uint64_t planes[8] = {};
    double uniforms[4] = {};
    int64_t iuniforms[4] = {};
    double uext[4] = {};
    uint8_t* term = nullptr;
    Cells* cells = nullptr;
    Cells* host = nullptr;  // pinned mirror for the report
    uint64_t* status = nullptr;
    void* records = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    BandArgs band{};
    uint32_t* goHost = nullptr;  // pinned: the eager band loop's condition word
    int32_t* order = nullptr;  // persist oscillator: the claim order, each run longest first (order.cu)
    int bandGrid = 0, persistGrid = 0;
    uint32_t chunk = 32, block = 256;
    bool fma = false, spread = false;
    // armed by engine_time_kernel: events recorded around the main kernel of the next launches
    std::vector<cudaEvent_t> evStart, evStop;
    size_t evUsed = 0;
};

/** Record the next armed start (``stop`` false) or stop event of ``e`` on ``s``. */
void markKernel(Engine& e, cudaStream_t s, bool stop)
{
    if (e.evUsed >= e.evStart.size())
        return;
    if (!stop) {
        cudaCheck(cudaEventRecord(e.evStart[e.evUsed], s), "cudaEventRecord");
        return;
    }
    cudaCheck(cudaEventRecord(e.evStop[e.evUsed], s), "cudaEventRecord");
    ++e.evUsed;
}

void releaseTimers(Engine& e)
{
    for (cudaEvent_t ev : e.evStart)
        (void)cudaEventDestroy(ev);
    for (cudaEvent_t ev : e.evStop)
        (void)cudaEventDestroy(ev);
    e.evStart.clear();
    e.evStop.clear();
    e.evUsed = 0;
}

template <bool Fma, bool Spread, bool Graph>
void* bandKernelPtr()
{
    return reinterpret_cast<void*>(&bandKernel<Fma, Spread, Graph>);
}

void* pickBand(bool fma, bool spread, bool graph = true)
{
    if (graph) {
        if (fma)
            return spread ? bandKernelPtr<true, true, true>() : bandKernelPtr<true, false, true>();
        return spread ? bandKernelPtr<false, true, true>() : bandKernelPtr<false, false, true>();
    }
    if (fma)
        return spread ? bandKernelPtr<true, true, false>() : bandKernelPtr<true, false, false>();
    return spread ? bandKernelPtr<false, true, false>() : bandKernelPtr<false, false, false>();
}

void buildBandGraph(Engine& e, BandArgs& args)
{
    cudaCheck(cudaGraphCreate(&e.graph, 0), "cudaGraphCreate");
    cudaGraphConditionalHandle cond{};
    cudaCheck(cudaGraphConditionalHandleCreate(&cond, e.graph, 0, 0), "cudaGraphConditionalHandleCreate");
    args.cond = cond;

    cudaGraphNode_t init = nullptr, loop = nullptr, band = nullptr, finish = nullptr;
    {
        int64_t n = e.n;
        void* params[] = {&e.cells, &n, &cond};
        cudaKernelNodeParams p{};
        p.func = reinterpret_cast<void*>(&bandInitKernel<true>);
        p.gridDim = dim3(1);
        p.blockDim = dim3(1);
        p.kernelParams = params;
        cudaCheck(cudaGraphAddKernelNode(&init, e.graph, nullptr, 0, &p), "cudaGraphAddKernelNode(init)");
    }
    cudaGraphNodeParams cp{};
    cp.type = cudaGraphNodeTypeConditional;
    cp.conditional.handle = cond;
    cp.conditional.type = cudaGraphCondTypeWhile;
    cp.conditional.size = 1;
    cudaCheck(cudaGraphAddNode(&loop, e.graph, &init, 1, &cp), "cudaGraphAddNode(while)");
    cudaGraph_t body = cp.conditional.phGraph_out[0];
    {
        void* params[] = {&args};
        cudaKernelNodeParams p{};
        p.func = pickBand(e.fma, e.spread);
        p.gridDim = dim3(unsigned(e.bandGrid));
        p.blockDim = dim3(kBandThreads);
        p.kernelParams = params;
        cudaCheck(cudaGraphAddKernelNode(&band, body, nullptr, 0, &p), "cudaGraphAddKernelNode(band)");
    }
    {
        const uint8_t* term = e.term;
        int64_t n = e.n;
        void* params[] = {&e.cells, &term, &n};
        cudaKernelNodeParams p{};
        p.func = reinterpret_cast<void*>(&bandFinishKernel);
        p.gridDim = dim3(unsigned(std::max(1, smCount())));
        p.blockDim = dim3(256);
        p.kernelParams = params;
        cudaCheck(cudaGraphAddKernelNode(&finish, e.graph, &loop, 1, &p), "cudaGraphAddKernelNode(finish)");
    }
    cudaCheck(cudaGraphInstantiate(&e.exec, e.graph, 0), "cudaGraphInstantiate");
}

/** The built-in entry a persist / fused engine launches. */
std::string entryName(const Engine& e, bool persist)
{
    const std::string stem = e.model == EAGLE_B200_MODEL_GAMBLER ? "gambler"
        : e.model == EAGLE_B200_MODEL_LORENZ ? "lorenz"
        : (e.spread ? "oscillator_spread" : "oscillator");
    const bool oscillator = e.model == EAGLE_B200_MODEL_OSCILLATOR || e.model == EAGLE_B200_MODEL_OSCILLATOR_SPREAD;
    const std::string fma = (e.fma && oscillator) ? "_fma" : "";
    return stem + (persist ? "_persist" : "_range") + fma;
}

ScalarHandle handle(uint64_t p, int64_t n, int dev)
{
    return ScalarHandle{reinterpret_cast<void*>(p), uint64_t(n), 1, 2, dev};
}

void launchEngine(Engine& e, cudaStream_t s)
{
    if (e.mode == EAGLE_B200_MODE_BAND) {
        markKernel(e, s, false);
        cudaCheck(cudaGraphLaunch(e.exec, s), "cudaGraphLaunch");
        markKernel(e, s, true);
        return;
    }
    if (e.mode == EAGLE_B200_MODE_BAND_EAGER) {
        // the same passes, driven from the host: one condition read per pass
        bandInitKernel<false><<<1, 1, 0, s>>>(e.cells, e.n, cudaGraphConditionalHandle{});
        launchCheck("band init");
        void* pass = pickBand(e.fma, e.spread, false);
        for (;;) {
            cudaCheck(cudaMemcpyAsync(e.goHost, &e.cells->go, sizeof(uint32_t), cudaMemcpyDeviceToHost, s),
                "cudaMemcpyAsync");
            cudaCheck(cudaStreamSynchronize(s), "cudaStreamSynchronize");
            if (*e.goHost == 0)
                break;
            void* params[] = {&e.band};
            cudaCheck(cudaLaunchKernel(pass, dim3(unsigned(e.bandGrid)), dim3(kBandThreads), params, 0, s),
                "cudaLaunchKernel");
        }
        bandFinishKernel<<<unsigned(std::max(1, smCount())), 256, 0, s>>>(e.cells, e.term, e.n);
        launchCheck("band finish");
        return;
    }
    // persist / fused: zero the run words, count the mask, one launch
    Cells* c = e.cells;
    // one memset from finished through stepsum64 (newly, err and total between them are
    // the band schedule's; the persist and fused report reads none of them)
    static_assert(offsetof(Cells, finished) < offsetof(Cells, next), "finished precedes the run words");
    cudaCheck(cudaMemsetAsync(&c->finished, 0,
                  offsetof(Cells, stepsum64) + sizeof(c->stepsum64) - offsetof(Cells, finished), s),
        "cudaMemsetAsync");
    const bool persist = e.mode == EAGLE_B200_MODE_PERSIST;
    // the ordered persist launch counts the mask in its claim order's key pass
    const bool ordered = persist && e.order != nullptr && e.n > 0 && e.maxSteps > 0;
    if (!ordered)
        enqueueMaskCount(e.term, e.n, &c->finished, s, false);
    if (e.n == 0 || e.maxSteps == 0)
        return;
    const std::string name = entryName(e, persist);
    const void* stub = entryStub(name);
    const int dev = e.device;
    // role arguments in the arg_spec order, then the partition triple and the tail
    ScalarHandle h[8];
    double du[4];
    int64_t iu[4];
    std::vector<void*> args;
    ScalarHandle term = handle(reinterpret_cast<uint64_t>(e.term), e.n, dev);
    ScalarHandle fin = handle(reinterpret_cast<uint64_t>(&c->finished), 1, dev);
    ScalarHandle fused = handle(reinterpret_cast<uint64_t>(&c->budget), 1, dev);
    if (e.model == EAGLE_B200_MODEL_LORENZ) {
        for (int k = 0; k < 8; ++k)
            h[k] = handle(e.planes[k], e.n, dev);  // rho, x, y, z, t, h, n_acc, n_rej
        for (int k = 0; k < 4; ++k)
            du[k] = e.uniforms[k];  // sigma, beta, t_final, rtol
        args.push_back(&h[0]);
        for (int k = 0; k < 4; ++k)
            args.push_back(&du[k]);
        args.push_back(&e.uext[0]);  // atol
        args.push_back(&term);
        for (int k = 1; k < 8; ++k)
            args.push_back(&h[k]);
    } else if (e.model == EAGLE_B200_MODEL_GAMBLER) {
        h[0] = handle(e.planes[0], e.n, dev);  // pos
        h[1] = handle(e.planes[1], e.n, dev);  // time
        iu[0] = e.iuniforms[0];
        iu[1] = e.iuniforms[1];
        for (void* p : {static_cast<void*>(&h[0]), static_cast<void*>(&h[1]), static_cast<void*>(&term),
                 static_cast<void*>(&iu[0]), static_cast<void*>(&iu[1])})
            args.push_back(p);
    } else if (e.spread) {
        for (int k = 0; k < 5; ++k)
            h[k] = handle(e.planes[k], e.n, dev);  // omega, t_end, x, v, t
        du[0] = e.uniforms[0];
        for (void* p : {static_cast<void*>(&h[0]), static_cast<void*>(&h[1]), static_cast<void*>(&du[0]),
                 static_cast<void*>(&term), static_cast<void*>(&h[2]), static_cast<void*>(&h[3]),
                 static_cast<void*>(&h[4])})
            args.push_back(p);
    } else {
        for (int k = 0; k < 4; ++k)
            h[k] = handle(e.planes[k], e.n, dev);  // omega, x, v, t
        du[0] = e.uniforms[0];
        du[1] = e.uniforms[1];
        for (void* p : {static_cast<void*>(&h[0]), static_cast<void*>(&du[0]), static_cast<void*>(&du[1]),
                 static_cast<void*>(&term), static_cast<void*>(&h[1]), static_cast<void*>(&h[2]),
                 static_cast<void*>(&h[3])})
            args.push_back(p);
    }
    int64_t base = 0, count = e.n, nSamples = e.n;
    uint32_t* next = &c->next;
    unsigned long long* util = nullptr;
    uint32_t* steps = &c->steps32;
    unsigned long long* stepsum = &c->stepsum64;
    uint32_t chunk = e.chunk;
    for (void* p : {static_cast<void*>(&fin), static_cast<void*>(&fused), static_cast<void*>(&base),
             static_cast<void*>(&count), static_cast<void*>(&nSamples)})
        args.push_back(p);
    unsigned grid = 0;
    const int32_t* order = nullptr;
    if (persist) {
        for (void* p : {static_cast<void*>(&next), static_cast<void*>(&util), static_cast<void*>(&steps),
                 static_cast<void*>(&stepsum), static_cast<void*>(&chunk)})
            args.push_back(p);
        grid = unsigned(e.persistGrid);
        if (e.order != nullptr) {
            // claims longest first (order.cu): the same samples, the same steps, fuller warps
            const double* tEnd = e.spread ? reinterpret_cast<const double*>(e.planes[1]) : nullptr;
            const double* tPlane = reinterpret_cast<const double*>(e.planes[e.spread ? 4 : 3]);
            const double dt = e.spread ? e.uniforms[0] : e.uniforms[1];
            order = e.order;
            enqueueStopOrder(tEnd, e.spread ? 0.0 : e.uniforms[0], tPlane, e.term, e.n, dt, e.maxSteps, e.order,
                &c->finished, s);
            args.push_back(&order);
            stub = orderedPersistStub(e.fma, e.spread);
        }
    } else {
        args.push_back(&steps);
        args.push_back(&stepsum);
        grid = unsigned((e.n + e.block - 1) / e.block);
    }
    markKernel(e, s, false);
    cudaCheck(cudaLaunchKernel(stub, dim3(grid), dim3(e.block), args.data(), 0, s), "cudaLaunchKernel");
    markKernel(e, s, true);
}

/** The report from the host copy of the cells (already landed). */
void fillReport(const Engine& e, eagle_b200_report* out)
{
    const Cells& c = *e.host;
    eagle_b200_report r{};
    r.struct_size = sizeof r;
    r.n = e.n;
    r.finished = c.finished;
    r.done = uint32_t(int64_t(c.finished) == e.n);
    r.mode = e.mode;
    r.report_bytes = uint32_t(sizeof(Cells));
    if (e.mode == EAGLE_B200_MODE_BAND || e.mode == EAGLE_B200_MODE_BAND_EAGER) {
        r.steps = int64_t(c.longest);
        r.launches = c.iter;
        r.compactions = c.iter;
        r.step_sum = c.stepsum;
        r.error = c.err;
    } else {
        r.steps = int64_t(c.steps32);
        r.launches = (e.n > 0 && e.maxSteps > 0) ? 1 : 0;
        r.compactions = 0;
        r.step_sum = c.stepsum64;
        r.error = 0;
    }
    const uint32_t size = out->struct_size < sizeof r ? out->struct_size : uint32_t(sizeof r);
    std::memcpy(out, &r, size);
    out->struct_size = size;
}

void readReport(Engine& e, cudaStream_t s, eagle_b200_report* out)
{
    cudaCheck(cudaMemcpyAsync(e.host, e.cells, sizeof(Cells), cudaMemcpyDeviceToHost, s), "cudaMemcpyAsync");
    cudaCheck(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    fillReport(e, out);
}

void destroy(Engine* e)
{
    if (e == nullptr)
        return;
    int prev = 0;
    (void)cudaGetDevice(&prev);
    (void)cudaSetDevice(e->device);
    if (e->exec)
        (void)cudaGraphExecDestroy(e->exec);
    if (e->graph)
        (void)cudaGraphDestroy(e->graph);
    (void)cudaFree(e->cells);
    (void)cudaFree(e->status);
    (void)cudaFree(e->records);
    (void)cudaFreeHost(e->host);
    (void)cudaFreeHost(e->goHost);
    (void)cudaFree(e->order);
    releaseTimers(*e);
    (void)cudaSetDevice(prev);
    delete e;
}

}  // namespace
}  // namespace eb

using namespace eb;

#define EB_API extern "C" __attribute__((visibility("default")))

EB_API eagle_backend_status eagle_backend_x_b200_engine_create(const struct eagle_b200_engine_desc* desc,
    eagle_b200_engine* out)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_b200_engine_create";
        const auto d = readDesc(desc, EAGLE_B200_FLAG_FMA | EAGLE_B200_FLAG_INDEX_ORDER, who);
        if (out == nullptr)
            invalid(std::string(who) + ": null output");
        if (d.model > EAGLE_B200_MODEL_LORENZ)
            unsupported(std::string(who) + ": unknown model " + std::to_string(d.model));
        if ((d.model == EAGLE_B200_MODEL_GAMBLER || d.model == EAGLE_B200_MODEL_LORENZ)
            && (d.mode == EAGLE_B200_MODE_BAND || d.mode == EAGLE_B200_MODE_BAND_EAGER))
            unsupported(std::string(who) + ": the band schedule is built for the oscillator only; use persist or fused");
        if (d.mode > EAGLE_B200_MODE_BAND_EAGER)
            unsupported(std::string(who) + ": unknown mode " + std::to_string(d.mode));
        if (d.n < 0 || d.n > INT64_C(2147483647))
            unsupported(std::string(who) + ": n must lie in [0, 2^31 - 1]");
        if (d.max_steps < 0)
            invalid(std::string(who) + ": max_steps must be >= 0");
        if ((d.mode == EAGLE_B200_MODE_PERSIST || d.mode == EAGLE_B200_MODE_FUSED) && d.max_steps > INT64_C(4294967295))
            unsupported(std::string(who) + ": the persist and fused entries count steps in 32 bits");
        const bool spread = d.model == EAGLE_B200_MODEL_OSCILLATOR_SPREAD;
        const int nPlanes = d.model == EAGLE_B200_MODEL_LORENZ ? 8
            : d.model == EAGLE_B200_MODEL_GAMBLER ? 2 : (spread ? 5 : 4);
        if (d.n > 0) {
            for (int i = 0; i < nPlanes; ++i)
                if (d.planes[i] == 0)
                    invalid(std::string(who) + ": plane " + std::to_string(i) + " must be a device address");
            if (d.terminated == 0)
                invalid(std::string(who) + ": terminated must be a device address");
        }
        if (d.chunk != 0 && (d.chunk & (d.chunk - 1)) != 0)
            invalid(std::string(who) + ": chunk must be a power of two");
        auto* e = new Engine();
        try {
            e->device = resolveDevice(d.device, d.n > 0 ? d.planes[0] : 0);
            DeviceScope scope(e->device);
            e->model = d.model;
            e->mode = d.mode;
            e->flags = d.flags;
            e->fma = (d.flags & EAGLE_B200_FLAG_FMA) != 0;
            e->spread = spread;
            e->n = d.n;
            e->maxSteps = d.max_steps;
            std::memcpy(e->planes, d.planes, sizeof e->planes);
            std::memcpy(e->uniforms, d.uniforms, sizeof e->uniforms);
            std::memcpy(e->iuniforms, d.iuniforms, sizeof e->iuniforms);
            std::memcpy(e->uext, d.uniforms_ext, sizeof e->uext);
            e->term = reinterpret_cast<uint8_t*>(d.terminated);
            // steps per claim head: an oscillator lane idles from its sample's end to the next
            // head, a head costs a claim and a swap. Claimed in index order, 512 measured best
            // (5.74 against 5.90 ms at 256 and 6.32 ms at 1024 for 2^24 heterogeneous stops);
            // claimed longest first, a warp's lanes end together, so the heads only cost:
            // 3.84 ms at 4096 against 3.86 / 3.89 / 4.02 / 4.28 ms at 2048 / 1024 / 512 / 256
            const bool ordered = d.mode == EAGLE_B200_MODE_PERSIST && (d.flags & EAGLE_B200_FLAG_INDEX_ORDER) == 0
                && (d.model == EAGLE_B200_MODEL_OSCILLATOR || spread);
            e->chunk = d.chunk != 0 ? d.chunk
                : d.model == EAGLE_B200_MODEL_LORENZ ? 8u
                : d.model == EAGLE_B200_MODEL_GAMBLER ? 256u
                : ordered                             ? 4096u
                                                      : 512u;
            e->block = d.model == EAGLE_B200_MODEL_LORENZ ? 128u : 256u;
            cudaCheck(cudaMalloc(&e->cells, sizeof(Cells)), "cudaMalloc");
            cudaCheck(cudaMallocHost(&e->host, sizeof(Cells)), "cudaMallocHost");
            Cells init{};
            init.cap = d.max_steps;
            init.kFirst = d.k_first > 0 ? d.k_first : 16;
            init.kMin = d.k_min > 0 ? d.k_min : 8;
            init.kMax = d.k_max > 0 ? std::min<int64_t>(d.k_max, INT64_C(1) << 30) : 4096;
            init.overheadSteps = d.overhead_steps > 0 ? d.overhead_steps : 2.0e7;
            init.intervalSteps = d.interval_steps > 0 ? d.interval_steps : 16.0;
            init.budget = d.max_steps;
            init.total = uint32_t(d.n);
            cudaCheck(cudaMemcpy(e->cells, &init, sizeof init, cudaMemcpyHostToDevice), "cudaMemcpy");
            int occ = 0;
            const bool band = e->mode == EAGLE_B200_MODE_BAND || e->mode == EAGLE_B200_MODE_BAND_EAGER;
            if (band) {
                cudaCheck(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ,
                              pickBand(e->fma, spread, e->mode == EAGLE_B200_MODE_BAND), kBandThreads, 0),
                    "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
                e->bandGrid = std::max(1, occ) * smCount();
                const int64_t tiles = std::max<int64_t>(1, (d.n + kBandThreads - 1) / kBandThreads);
                cudaCheck(cudaMalloc(&e->status, size_t(tiles) * sizeof(uint64_t)), "cudaMalloc");
                cudaCheck(cudaMemset(e->status, 0, size_t(tiles) * sizeof(uint64_t)), "cudaMemset");
                // two compacted copies of the live state: c, te, x, v, t (f64) and the index (i32)
                const int64_t cap = std::max<int64_t>(d.n, 1);
                const int doubles = spread ? 5 : 4;
                const size_t perCopy = (size_t(cap) * (size_t(doubles) * 8 + 4) + 255) & ~size_t(255);
                cudaCheck(cudaMalloc(&e->records, 2 * perCopy + 256), "cudaMalloc");
                BandArgs args{};
                args.cells = e->cells;
                args.status = e->status;
                args.n = d.n;
                if (spread) {
                    args.omega = reinterpret_cast<const double*>(d.planes[0]);
                    args.tend = reinterpret_cast<const double*>(d.planes[1]);
                    args.x = reinterpret_cast<double*>(d.planes[2]);
                    args.v = reinterpret_cast<double*>(d.planes[3]);
                    args.t = reinterpret_cast<double*>(d.planes[4]);
                    args.dt = d.uniforms[0];
                } else {
                    args.omega = reinterpret_cast<const double*>(d.planes[0]);
                    args.x = reinterpret_cast<double*>(d.planes[1]);
                    args.v = reinterpret_cast<double*>(d.planes[2]);
                    args.t = reinterpret_cast<double*>(d.planes[3]);
                    args.tendU = d.uniforms[0];
                    args.dt = d.uniforms[1];
                }
                args.term = e->term;
                char* base = static_cast<char*>(e->records);
                for (int b = 0; b < 2; ++b) {
                    double* p = reinterpret_cast<double*>(base + size_t(b) * perCopy);
                    args.rx[b] = p;
                    args.rv[b] = p + cap;
                    args.rt[b] = p + 2 * cap;
                    args.rc[b] = p + 3 * cap;
                    args.rte[b] = spread ? p + 4 * cap : nullptr;
                    args.ridx[b] = reinterpret_cast<int32_t*>(p + size_t(doubles) * size_t(cap));
                }
                e->band = args;
                if (e->mode == EAGLE_B200_MODE_BAND)
                    buildBandGraph(*e, e->band);
                else
                    cudaCheck(cudaMallocHost(&e->goHost, sizeof(uint32_t)), "cudaMallocHost");
            } else {
                const void* stub = entryStub(entryName(*e, true));
                cudaCheck(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, stub, int(e->block), 0),
                    "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
                const int perSm = d.ctas_per_sm > 0 ? std::min(int(d.ctas_per_sm), std::max(1, occ)) : std::max(1, occ);
                e->persistGrid = perSm * smCount();
                if (ordered && d.n > 0) {
                    cudaCheck(cudaMalloc(&e->order, stopOrderBytes(d.n)), "cudaMalloc");
                    prepareStopOrder();
                }
            }
        } catch (...) {
            destroy(e);
            throw;
        }
        *out = reinterpret_cast<eagle_b200_engine>(e);
    });
}

EB_API eagle_backend_status eagle_backend_x_b200_engine_launch(eagle_b200_engine h, uint64_t stream)
{
    return guarded([&] {
        if (h == nullptr)
            fail(EAGLE_BACKEND_BAD_HANDLE, "eagle_backend_x_b200_engine_launch: null handle");
        auto* e = reinterpret_cast<Engine*>(h);
        DeviceScope scope(e->device);
        launchEngine(*e, seamStream(stream));
    });
}

EB_API eagle_backend_status eagle_backend_x_b200_engine_report(eagle_b200_engine h, uint64_t stream,
    struct eagle_b200_report* report)
{
    return guarded([&] {
        if (h == nullptr)
            fail(EAGLE_BACKEND_BAD_HANDLE, "eagle_backend_x_b200_engine_report: null handle");
        if (report == nullptr || report->struct_size < 8)
            invalid("eagle_backend_x_b200_engine_report: null or short report");
        auto* e = reinterpret_cast<Engine*>(h);
        DeviceScope scope(e->device);
        readReport(*e, seamStream(stream), report);
        if (report->struct_size >= offsetof(eagle_b200_report, error) + sizeof(uint32_t) && report->error != 0)
            fail(EAGLE_BACKEND_ERROR, "eagle_b200 engine: a device-side wait gave up (error word "
                + std::to_string(report->error) + "); the run's results are not valid");
    });
}

EB_API eagle_backend_status eagle_backend_x_b200_engine_report_enqueue(eagle_b200_engine h, uint64_t stream)
{
    return guarded([&] {
        if (h == nullptr)
            fail(EAGLE_BACKEND_BAD_HANDLE, "eagle_backend_x_b200_engine_report_enqueue: null handle");
        auto* e = reinterpret_cast<Engine*>(h);
        DeviceScope scope(e->device);
        cudaCheck(cudaMemcpyAsync(e->host, e->cells, sizeof(Cells), cudaMemcpyDeviceToHost, seamStream(stream)),
            "cudaMemcpyAsync");
    });
}

EB_API eagle_backend_status eagle_backend_x_b200_engine_report_read(eagle_b200_engine h,
    struct eagle_b200_report* report)
{
    return guarded([&] {
        if (h == nullptr)
            fail(EAGLE_BACKEND_BAD_HANDLE, "eagle_backend_x_b200_engine_report_read: null handle");
        if (report == nullptr || report->struct_size < 8)
            invalid("eagle_backend_x_b200_engine_report_read: null or short report");
        const auto* e = reinterpret_cast<const Engine*>(h);
        fillReport(*e, report);
        if (report->struct_size >= offsetof(eagle_b200_report, error) + sizeof(uint32_t) && report->error != 0)
            fail(EAGLE_BACKEND_ERROR, "eagle_b200 engine: a device-side wait gave up (error word "
                + std::to_string(report->error) + "); the run's results are not valid");
    });
}

EB_API eagle_backend_status eagle_backend_x_b200_engine_run(eagle_b200_engine h, uint64_t stream,
    struct eagle_b200_report* report)
{
    const eagle_backend_status s = eagle_backend_x_b200_engine_launch(h, stream);
    if (s != EAGLE_BACKEND_OK)
        return s;
    return eagle_backend_x_b200_engine_report(h, stream, report);
}

EB_API eagle_backend_status eagle_backend_x_b200_engine_time_kernel(eagle_b200_engine h, int32_t launches)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_b200_engine_time_kernel";
        if (h == nullptr)
            fail(EAGLE_BACKEND_BAD_HANDLE, std::string(who) + ": null handle");
        if (launches < 0 || launches > 65536)
            invalid(std::string(who) + ": launches must lie in [0, 65536]");
        auto* e = reinterpret_cast<Engine*>(h);
        DeviceScope scope(e->device);
        releaseTimers(*e);
        for (int32_t i = 0; i < launches; ++i) {
            cudaEvent_t a = nullptr, b = nullptr;
            cudaCheck(cudaEventCreate(&a), "cudaEventCreate");
            e->evStart.push_back(a);
            cudaCheck(cudaEventCreate(&b), "cudaEventCreate");
            e->evStop.push_back(b);
        }
    });
}

EB_API eagle_backend_status eagle_backend_x_b200_engine_kernel_ms(eagle_b200_engine h, float* ms, int32_t cap,
    int32_t* count)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_b200_engine_kernel_ms";
        if (h == nullptr)
            fail(EAGLE_BACKEND_BAD_HANDLE, std::string(who) + ": null handle");
        if (count == nullptr || cap < 0 || (cap > 0 && ms == nullptr))
            invalid(std::string(who) + ": null output");
        auto* e = reinterpret_cast<Engine*>(h);
        DeviceScope scope(e->device);
        const size_t m = std::min(e->evUsed, size_t(cap));
        for (size_t i = 0; i < m; ++i) {
            cudaCheck(cudaEventSynchronize(e->evStop[i]), "cudaEventSynchronize");
            cudaCheck(cudaEventElapsedTime(&ms[i], e->evStart[i], e->evStop[i]), "cudaEventElapsedTime");
        }
        *count = int32_t(e->evUsed);
    });
}

EB_API void eagle_backend_x_b200_engine_release(eagle_b200_engine h)
{
    destroy(reinterpret_cast<Engine*>(h));
}
