// The canonical ``ordered`` reduction on B200: one kernel per call.
//
// The tree is eagle's (eagle/reduce/canonical.h:10-32): leaves of 256 slots x 16
// terms, slot t folding samples t, t+256, ... of its leaf (a Neumaier walk for a
// floating sum), the in-leaf tree at offsets 128, 64, ..., 1 with an absent partner
// carried, then level-by-level pairwise over the leaf partials with an odd last
// node carried. The bits are a function of the values in sample order only.
//
// B200 mapping. A CTA of 256 threads owns an aligned group of 2^q consecutive
// leaves: thread t holds slot t (its 16 loads issued together, each a coalesced
// 2 KB row across the CTA), the offsets 128..32 go through shared memory and
// 16..1 through warp shuffles inside warp 0, and the group's leaf partials are
// joined by the same pairwise levels (an aligned group is a subtree of them).
// The last CTA to finish (a device-scope counter) runs the remaining levels over
// the group partials in aligned chunks of 512 and stores the value. One memset
// node zeroes the counters before the launch, so the call stays capturable.
#include "canonical.cuh"

#include <cmath>
#include <mutex>

namespace eb {
namespace {

constexpr int kMaxGroupLeaves = 64;  // leaves one CTA owns at most

// ------------------------------------------------------------------- partials

template <class T>
struct SumOp {
    __device__ __forceinline__ T operator()(T a, T b) const
    {
        if constexpr (std::is_integral_v<T>) {
            using U = std::make_unsigned_t<T>;
            return T(U(a) + U(b));
        } else {
            return a + b;
        }
    }
};
template <class T>
struct MaxOp {
    __device__ __forceinline__ T operator()(T a, T b) const { return a > b ? a : b; }
};
template <class T>
struct MinOp {
    __device__ __forceinline__ T operator()(T a, T b) const { return a < b ? a : b; }
};
struct AllOp {
    __device__ __forceinline__ uint8_t operator()(uint8_t a, uint8_t b) const { return uint8_t(a != 0 && b != 0); }
};

template <class T, class Op>
struct PlainP {  // the partial of an exact operator: one value
    T h;
    static __device__ __forceinline__ PlainP of(T x) { return {x}; }
    static __device__ __forceinline__ PlainP of(T x, T) { return {x}; }
    static __device__ __forceinline__ PlainP join(const PlainP& a, const PlainP& b) { return {Op{}(a.h, b.h)}; }
    __device__ __forceinline__ void add(T x) { h = Op{}(h, x); }
    __device__ __forceinline__ void add(T x, T) { add(x); }
    __device__ __forceinline__ T value() const { return h; }
    __device__ __forceinline__ PlainP shflDown(unsigned off) const
    {
        if constexpr (sizeof(T) < 4)
            return {T(__shfl_down_sync(kFull, int(h), off))};
        else
            return {__shfl_down_sync(kFull, h, off)};
    }
};

template <class P>
struct IsComp : std::false_type {};
template <class T>
struct IsComp<CompP<T>> : std::true_type {};

// ------------------------------------------------------------------- kernels

struct ReduceArgs {
    const void* in;
    const void* comp;
    int64_t rows, cols, col0;
    int64_t leaves, groupLeaves, groups;
    void* partials;      // cols * groups partials
    uint32_t* counters;  // cols words, zero on entry
    void* out;
    int pairOut;
};

/** Column ``col``'s result from its root partial: the value, or with PAIR_OUT the
 *  (hi, comp) pair (hi at ``col``, comp at ``cols + col``). */
template <class P, class T>
__device__ __forceinline__ void writeResult(const ReduceArgs& a, const P& r, int64_t col)
{
    T* out = static_cast<T*>(a.out);
    if constexpr (IsComp<P>::value) {
        if (a.pairOut) {
            out[col] = r.h;
            out[a.cols + col] = isfinite(r.h) ? r.c : T(0);
        } else {
            out[col] = r.value();
        }
    } else {
        out[col] = r.value();
    }
}

template <class P, class T, bool HasComp>
__global__ __launch_bounds__(kSlots) void canonicalKernel(ReduceArgs a)
{
    __shared__ P s[kSlots];
    __shared__ P group[kChunk > kMaxGroupLeaves ? kChunk : kMaxGroupLeaves];
    __shared__ int amLast;
    const T* in = static_cast<const T*>(a.in);
    const T* comp = static_cast<const T*>(a.comp);
    P* partials = static_cast<P*>(a.partials);
    const int64_t col = a.col0 + int64_t(blockIdx.y);
    const int64_t g = int64_t(blockIdx.x);
    const int64_t l0 = g * a.groupLeaves;
    const int64_t l1 = l0 + a.groupLeaves < a.leaves ? l0 + a.groupLeaves : a.leaves;
    for (int64_t l = l0; l < l1; ++l) {
        const int64_t base = l * kLeaf;
        const int64_t cnt = a.rows - base < kLeaf ? a.rows - base : kLeaf;
        const P p = leafPartial<P, T, HasComp>(in, comp, a.cols, col, base, cnt, s);
        if (threadIdx.x == 0)
            group[l - l0] = p;
    }
    __syncthreads();
    levels(group, int(l1 - l0));
    if (threadIdx.x == 0) {
        partials[col * a.groups + g] = group[0];
        __threadfence();
        amLast = atomicAdd(&a.counters[col], 1u) == uint32_t(a.groups - 1);
    }
    __syncthreads();
    if (!amLast)
        return;
    __threadfence();
    // the last CTA of this column: the remaining levels over the group partials,
    // in aligned chunks of kChunk nodes, written back in place
    P* v = partials + col * a.groups;
    int64_t m = a.groups;
    while (m > 1) {
        const int64_t chunks = (m + kChunk - 1) / kChunk;
        for (int64_t c = 0; c < chunks; ++c) {
            const int cnt = int(m - c * kChunk < kChunk ? m - c * kChunk : kChunk);
            for (int i = int(threadIdx.x); i < cnt; i += int(blockDim.x))
                group[i] = v[c * kChunk + i];
            __syncthreads();
            levels(group, cnt);
            if (threadIdx.x == 0)
                v[c] = group[0];
            __syncthreads();
        }
        m = chunks;
    }
    if (threadIdx.x == 0) {
        writeResult<P, T>(a, v[0], col);
        a.counters[col] = 0u;  // ready for a replay
    }
}

/** canonicalKernel for one column, one leaf at a time: persistent CTAs (one per
 *  resident slot) take leaf blockIdx.x first, then claim the leaves after the first
 *  gridDim.x in order off a counter (the next claim in flight while a leaf is folded),
 *  and write each leaf's partial; the CTA that completes an aligned chunk of
 *  kChunk leaves joins it by the pairwise levels, and the one that completes the last
 *  chunk joins the chunk partials (in aligned chunks of kChunk, level over level)
 *  into the result. Aligned chunks are subtrees of the canonical tree, so the bits
 *  are canonicalKernel's; no CTA waits on another. ``partials`` holds ``leaves`` leaf
 *  partials then one per chunk; ``counters`` = {leaves claimed past the first
 *  gridDim.x, chunks done, one count per chunk}, zero on entry. Claiming in order lets
 *  chunks complete, and their levels run, while later leaves are still folded. */
template <class P, class T, bool HasComp>
__global__ __launch_bounds__(kSlots) void canonicalLeafKernel(ReduceArgs a)
{
    __shared__ P s[kSlots];
    __shared__ P group[kChunk];
    __shared__ int64_t sLeaf;
    __shared__ int sFold, sTop;
    const T* in = static_cast<const T*>(a.in);
    const T* comp = static_cast<const T*>(a.comp);
    P* leafPart = static_cast<P*>(a.partials);
    const int64_t leaves = a.leaves;
    const int64_t chunks = (leaves + kChunk - 1) / kChunk;
    P* chunkPart = leafPart + leaves;
    uint32_t* leafNext = a.counters;
    uint32_t* chunksDone = a.counters + 1;
    uint32_t* chunkDone = a.counters + 2;
    const int t = int(threadIdx.x);
    int64_t leaf = blockIdx.x;
    while (leaf < leaves) {
        int64_t next = 0;
        if (t == 0)
            next = int64_t(gridDim.x) + int64_t(atomicAdd(leafNext, 1u));  // used after this leaf
        const int64_t base = leaf * kLeaf;
        const int64_t cnt = a.rows - base < kLeaf ? a.rows - base : kLeaf;
        const P p = leafPartial<P, T, HasComp>(in, comp, 1, 0, base, cnt, s);
        const int64_t c = leaf / kChunk;
        const int64_t inChunk = leaves - c * kChunk < kChunk ? leaves - c * kChunk : kChunk;
        if (t == 0) {
            leafPart[leaf] = p;
            __threadfence();
            sFold = atomicAdd(&chunkDone[c], 1u) == uint32_t(inChunk - 1) ? 1 : 0;
            sLeaf = next;
        }
        __syncthreads();
        if (sFold) {  // this CTA completed chunk c: its leaves' levels
            __threadfence();
            for (int i = t; i < int(inChunk); i += kSlots)
                group[i] = leafPart[c * kChunk + i];
            __syncthreads();
            levels(group, int(inChunk));
            if (t == 0) {
                chunkPart[c] = group[0];
                __threadfence();
                sTop = atomicAdd(chunksDone, 1u) == uint32_t(chunks - 1) ? 1 : 0;
            }
            __syncthreads();
            if (sTop) {  // and the last chunk: the levels above, in place over chunkPart
                __threadfence();
                int64_t m = chunks;
                while (m > 1) {
                    const int64_t up = (m + kChunk - 1) / kChunk;
                    for (int64_t u = 0; u < up; ++u) {
                        const int n = int(m - u * kChunk < kChunk ? m - u * kChunk : kChunk);
                        for (int i = t; i < n; i += kSlots)
                            group[i] = chunkPart[u * kChunk + i];
                        __syncthreads();
                        levels(group, n);
                        if (t == 0)
                            chunkPart[u] = group[0];
                        __syncthreads();
                    }
                    m = up;
                }
                if (t == 0)
                    writeResult<P, T>(a, chunkPart[0], 0);
            }
        }
        leaf = sLeaf;
        __syncthreads();  // sLeaf, sFold and group are reused by the next leaf
    }
}

/** Leaves per CTA for ``leaves`` leaves: a power of two keeping the group count at
 *  most ``target`` (any aligned power-of-two grouping gives the same bits). */
__device__ __forceinline__ int64_t groupLeavesDevice(int64_t leaves, int64_t target)
{
    int64_t g = 1;
    while (g < kMaxGroupLeaves && (leaves + g - 1) / g > target)
        g *= 2;
    return g;
}

/** The canonical reduction of the first ``*count`` elements of ``in`` (at most
 *  ``a.rows``): the element count is read on the device, so a reduction can follow
 *  a compaction with no host round trip. One column. ``gridDim.x`` CTAs (the group
 *  target); CTAs past the groups the count needs only take part in the last-CTA
 *  count. An empty input stores the operator's identity (0 for a sum). */
template <class P, class T>
__global__ __launch_bounds__(kSlots) void canonicalCountedKernel(ReduceArgs a, const uint32_t* count)
{
    __shared__ P s[kSlots];
    __shared__ P group[kChunk > kMaxGroupLeaves ? kChunk : kMaxGroupLeaves];
    __shared__ int amLast;
    const T* in = static_cast<const T*>(a.in);
    P* partials = static_cast<P*>(a.partials);
    const int64_t cap = a.rows;
    const int64_t c = int64_t(*count);
    const int64_t rows = c < cap ? c : cap;
    const int64_t leaves = (rows + kLeaf - 1) / kLeaf;
    const int64_t gl = groupLeavesDevice(leaves, int64_t(gridDim.x));
    const int64_t groups = (leaves + gl - 1) / gl;
    const int64_t g = int64_t(blockIdx.x);
    if (g < groups) {
        const int64_t l0 = g * gl;
        const int64_t l1 = l0 + gl < leaves ? l0 + gl : leaves;
        for (int64_t l = l0; l < l1; ++l) {
            const int64_t base = l * kLeaf;
            const int64_t cnt = rows - base < kLeaf ? rows - base : kLeaf;
            const P p = leafPartial<P, T, false>(in, nullptr, 1, 0, base, cnt, s);
            if (threadIdx.x == 0)
                group[l - l0] = p;
        }
        __syncthreads();
        levels(group, int(l1 - l0));
    }
    if (threadIdx.x == 0) {
        if (g < groups)
            partials[g] = group[0];
        __threadfence();
        amLast = atomicAdd(&a.counters[0], 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!amLast)
        return;
    __threadfence();
    P* v = partials;
    int64_t m = groups;
    while (m > 1) {
        const int64_t chunks = (m + kChunk - 1) / kChunk;
        for (int64_t cc = 0; cc < chunks; ++cc) {
            const int cnt = int(m - cc * kChunk < kChunk ? m - cc * kChunk : kChunk);
            for (int i = int(threadIdx.x); i < cnt; i += int(blockDim.x))
                group[i] = v[cc * kChunk + i];
            __syncthreads();
            levels(group, cnt);
            if (threadIdx.x == 0)
                v[cc] = group[0];
            __syncthreads();
        }
        m = chunks;
    }
    if (threadIdx.x == 0) {
        T* out = static_cast<T*>(a.out);
        if (groups == 0) {
            out[0] = T(0);
            if constexpr (IsComp<P>::value) {
                if (a.pairOut)
                    out[1] = T(0);
            }
        } else {
            const P r = v[0];
            if constexpr (IsComp<P>::value) {
                if (a.pairOut) {
                    out[0] = r.h;
                    out[1] = isfinite(r.h) ? r.c : T(0);
                } else {
                    out[0] = r.value();
                }
            } else {
                out[0] = r.value();
            }
        }
        a.counters[0] = 0u;
    }
}

/** Pairwise levels over m (hi, comp) partials -- chunk results in chunk order,
 *  e.g. one per rank -- into out = {hi, comp, value}. One CTA. */
__global__ __launch_bounds__(kSlots) void combinePairsKernel(const double* __restrict__ hc, int64_t m,
    double* __restrict__ work, double* __restrict__ out)
{
    __shared__ CompP<double> v[kChunk];
    const double* src = hc;
    int64_t count = m;
    while (count > 1) {
        const int64_t chunks = (count + kChunk - 1) / kChunk;
        for (int64_t c = 0; c < chunks; ++c) {
            const int cnt = int(count - c * kChunk < kChunk ? count - c * kChunk : kChunk);
            for (int i = int(threadIdx.x); i < cnt; i += int(blockDim.x))
                v[i] = CompP<double>{src[2 * (c * kChunk + i)], src[2 * (c * kChunk + i) + 1]};
            __syncthreads();
            levels(v, cnt);
            if (threadIdx.x == 0) {
                work[2 * c] = v[0].h;
                work[2 * c + 1] = v[0].c;
            }
            __syncthreads();
        }
        src = work;
        count = chunks;
    }
    if (threadIdx.x == 0) {
        const CompP<double> r{src[0], src[1]};
        out[0] = r.h;
        out[1] = r.c;
        out[2] = r.value();
    }
}

/** Every leaf's (hi, comp) partial of a float64 sum, leaf order, one CTA per leaf
 *  (the last leaf over the remainder): the leaves of the canonical tree
 *  (canonical.h:340-353), for callers that join leaves from several places. */
__global__ __launch_bounds__(kSlots) void leafPartialsKernel(const double* __restrict__ in, int64_t n,
    double* __restrict__ out)
{
    __shared__ CompP<double> s[kSlots];
    const int64_t l = blockIdx.x;
    const int64_t base = l * kLeaf;
    const int64_t cnt = n - base < kLeaf ? n - base : kLeaf;
    const CompP<double> p = leafPartial<CompP<double>, double, false>(in, nullptr, 1, 0, base, cnt, s);
    if (threadIdx.x == 0) {
        out[2 * l] = p.h;
        out[2 * l + 1] = p.c;
    }
}

// ------------------------------------------------------------------- host side

int64_t leafCount(int64_t rows) { return (rows + kLeaf - 1) / kLeaf; }

/** Leaves per CTA: a power of two that keeps about eight CTAs per SM busy. */
int64_t groupLeavesFor(int64_t leaves, int sms)
{
    const int64_t target = int64_t(sms) * 8;
    int64_t g = 1;
    while (g < kMaxGroupLeaves && (leaves + g - 1) / g > target)
        g *= 2;
    return g;
}

template <class P, class T>
int64_t workElemsFor(int64_t rows, int64_t cols, int sms)
{
    const int64_t leaves = leafCount(rows);
    const int64_t groups = (leaves + groupLeavesFor(leaves, sms) - 1) / groupLeavesFor(leaves, sms);
    const int64_t partialBytes = groups * cols * int64_t(sizeof(P));
    const int64_t counterBytes = cols * int64_t(sizeof(uint32_t));
    const int64_t need = (std::max(partialBytes, counterBytes) + int64_t(sizeof(T)) - 1) / int64_t(sizeof(T));
    // never less than eagle's own formula (3 elements per leaf and column), so a
    // caller that sized its buffers by it stays valid
    return std::max(need, 3 * leaves * cols);
}

/** canonicalLeafKernel<P, T, HasComp>'s CTAs resident per SM on the current device,
 *  looked up once per device. */
template <class P, class T, bool HasComp>
int leafKernelSlots()
{
    static std::mutex mu;
    static int perSm[64] = {};
    int dev = 0;
    cudaCheck(cudaGetDevice(&dev), "cudaGetDevice");
    std::lock_guard<std::mutex> lock(mu);
    int& k = perSm[dev & 63];
    if (k == 0) {
        cudaCheck(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&k, canonicalLeafKernel<P, T, HasComp>, kSlots, 0),
            "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
        if (k < 1)
            k = 1;
    }
    return k;
}

template <class P, class T, bool HasComp>
void launchLeafKernel(const ReduceArgs& a, int sms, cudaStream_t stream)
{
    const int64_t slots = int64_t(leafKernelSlots<P, T, HasComp>()) * sms;
    canonicalLeafKernel<P, T, HasComp><<<unsigned(a.leaves < slots ? a.leaves : slots), kSlots, 0, stream>>>(a);
    launchCheck("eagle_backend_x_reduce_canonical");
}

template <class P, class T>
void enqueueReduce(const eagle_backend_reduce_desc& d, int64_t cols, int pairOut, cudaStream_t stream)
{
    const int sms = smCount();
    ReduceArgs a{};
    a.in = reinterpret_cast<const void*>(d.in);
    a.rows = d.n;
    a.cols = cols;
    a.leaves = leafCount(d.n);
    a.groupLeaves = groupLeavesFor(a.leaves, sms);
    a.groups = (a.leaves + a.groupLeaves - 1) / a.groupLeaves;
    a.partials = reinterpret_cast<void*>(d.work_a);
    a.counters = reinterpret_cast<uint32_t*>(d.work_b);
    a.out = reinterpret_cast<void*>(d.out);
    a.pairOut = pairOut;
    const bool hasComp = d.comp_in != 0;
    a.comp = reinterpret_cast<const void*>(d.comp_in);
    // One column with more leaves than the device holds CTAs of the per-leaf kernel:
    // leaf by leaf over persistent CTAs (2^24 float64: 47 against 53 us; 2^27: 240
    // against 262), when a partial per leaf, one per 512-leaf chunk and the chunk
    // counters fit the room eagle's own formula gives each work buffer (3 elements per
    // leaf), so that a caller sizing by it stays valid. Up to one leaf per resident CTA
    // the grouped kernel is as fast or faster (2^20: 14 against 16 us).
    const int64_t chunks = (a.leaves + kChunk - 1) / kChunk;
    const int64_t room = 3 * a.leaves * int64_t(sizeof(T));
    const bool perLeaf = cols == 1 && int64_t(sizeof(P)) * (a.leaves + chunks) <= room
        && int64_t(sizeof(uint32_t)) * (2 + chunks) <= room
        && a.leaves > int64_t(leafKernelSlots<P, T, false>()) * sms;
    if (perLeaf) {
        cudaCheck(cudaMemsetAsync(a.counters, 0, size_t(2 + chunks) * sizeof(uint32_t), stream), "cudaMemsetAsync");
        a.col0 = 0;
        if constexpr (IsComp<P>::value) {
            if (hasComp) {
                launchLeafKernel<P, T, true>(a, sms, stream);
                return;
            }
        }
        launchLeafKernel<P, T, false>(a, sms, stream);
        return;
    }
    cudaCheck(cudaMemsetAsync(a.counters, 0, size_t(cols) * sizeof(uint32_t), stream), "cudaMemsetAsync");
    if (a.groups > INT64_C(2147483647))
        unsupported("eagle_backend_x_reduce_canonical: too many leaf groups");
    for (int64_t c0 = 0; c0 < cols; c0 += 65535) {
        a.col0 = c0;
        const dim3 grid(unsigned(a.groups), unsigned(std::min<int64_t>(cols - c0, 65535)));
        if constexpr (IsComp<P>::value || std::is_same_v<P, FixedP>) {
            if (hasComp)
                canonicalKernel<P, T, true><<<grid, kSlots, 0, stream>>>(a);
            else
                canonicalKernel<P, T, false><<<grid, kSlots, 0, stream>>>(a);
        } else {
            canonicalKernel<P, T, false><<<grid, kSlots, 0, stream>>>(a);
        }
        launchCheck("eagle_backend_x_reduce_canonical");
    }
}

/** Whether ``dev`` runs float64 at 1/8 of the float32 rate or slower, where eagle
 *  sums float64 on the fixed-point leaf (canonical.h:304-313, fixedLeafDevice :599-607). */
bool slowFp64(int dev)
{
    int ratio = 0;
    if (cudaDeviceGetAttribute(&ratio, cudaDevAttrSingleToDoublePrecisionPerfRatio, dev) != cudaSuccess) {
        (void)cudaGetLastError();
        return false;
    }
    return ratio >= 8;
}

template <class T>
void dispatchOp(const eagle_backend_reduce_desc& d, int64_t cols, int pairOut, cudaStream_t stream, bool query,
    int64_t* workElems)
{
    switch (d.op) {
    case EAGLE_BACKEND_REDUCE_OP_SUM:
        if constexpr (std::is_floating_point_v<T>) {
            if (query)
                *workElems = workElemsFor<CompP<T>, T>(d.n, cols, smCount());
            else
                enqueueReduce<CompP<T>, T>(d, cols, pairOut, stream);
        } else {
            if (query)
                *workElems = workElemsFor<PlainP<T, SumOp<T>>, T>(d.n, cols, smCount());
            else
                enqueueReduce<PlainP<T, SumOp<T>>, T>(d, cols, pairOut, stream);
        }
        break;
    case EAGLE_BACKEND_REDUCE_OP_MAX:
        if (query)
            *workElems = workElemsFor<PlainP<T, MaxOp<T>>, T>(d.n, cols, smCount());
        else
            enqueueReduce<PlainP<T, MaxOp<T>>, T>(d, cols, pairOut, stream);
        break;
    default:
        if (query)
            *workElems = workElemsFor<PlainP<T, MinOp<T>>, T>(d.n, cols, smCount());
        else
            enqueueReduce<PlainP<T, MinOp<T>>, T>(d, cols, pairOut, stream);
    }
}

}  // namespace
}  // namespace eb

using namespace eb;

extern "C" __attribute__((visibility("default"))) eagle_backend_status eagle_backend_x_reduce_canonical(
    struct eagle_backend_reduce_desc* desc)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_reduce_canonical";
        constexpr size_t base = offsetof(eagle_backend_reduce_desc, work_elems) + sizeof(int64_t);
        if (desc == nullptr || desc->struct_size < base)
            invalid(std::string(who) + ": null desc or struct_size too small");
        eagle_backend_reduce_desc d{};
        std::memcpy(&d, desc, std::min<size_t>(desc->struct_size, sizeof d));
        const bool ext = desc->struct_size >= offsetof(eagle_backend_reduce_desc, comp_in) + sizeof(uint64_t);
        if (!ext) {
            d.policy = EAGLE_BACKEND_REDUCE_ORDERED;
            d.flags = 0;
            d.columns = 1;
            d.comp_in = 0;
        }
        if (d.n < 1)
            invalid(std::string(who) + ": n must be >= 1");
        if (d.op > EAGLE_BACKEND_REDUCE_OP_MIN || d.dtype > EAGLE_BACKEND_REDUCE_U8)
            invalid(std::string(who) + ": unknown dtype or op");
        const bool all = d.op == EAGLE_BACKEND_REDUCE_OP_ALL;
        if (all != (d.dtype == EAGLE_BACKEND_REDUCE_U8))
            invalid(std::string(who) + ": the U8 element type goes with OP_ALL, and only with it");
        if (d.columns < 1 || d.policy > EAGLE_BACKEND_REDUCE_AUTO || d.flags > EAGLE_BACKEND_REDUCE_PAIR_OUT)
            invalid(std::string(who) + ": columns must be >= 1; unknown policy or flags");
        const bool fsum = d.op == EAGLE_BACKEND_REDUCE_OP_SUM
            && (d.dtype == EAGLE_BACKEND_REDUCE_F32 || d.dtype == EAGLE_BACKEND_REDUCE_F64);
        if ((d.comp_in != 0 || d.flags != 0) && !fsum)
            invalid(std::string(who) + ": comp_in and PAIR_OUT take a float32/float64 sum");
        const bool query = d.work_a == 0;
        if (!query && (d.in == 0 || d.out == 0 || d.work_b == 0))
            invalid(std::string(who) + ": in, out, work_a and work_b must be device addresses");
        const int dev = resolveDevice(d.device, query ? 0 : d.in);
        DeviceScope scope(dev);
        const cudaStream_t stream = seamStream(d.stream);
        const int pairOut = (d.flags & EAGLE_BACKEND_REDUCE_PAIR_OUT) != 0;
        int64_t workElems = 0;
        if (d.dtype == EAGLE_BACKEND_REDUCE_F64 && d.op == EAGLE_BACKEND_REDUCE_OP_SUM && d.flags == 0
            && slowFp64(dev)) {
            // a float64 sum without PAIR_OUT on a slow-FP64 device takes the fixed-point
            // leaf under every policy, as eagle does (eagle_backend.h:896-906, canonical.h:304-313)
            if (query)
                desc->work_elems = workElemsFor<FixedP, double>(d.n, d.columns, smCount());
            else
                enqueueReduce<FixedP, double>(d, d.columns, 0, stream);
            return;
        }
        switch (d.dtype) {
        case EAGLE_BACKEND_REDUCE_F32: dispatchOp<float>(d, d.columns, pairOut, stream, query, &workElems); break;
        case EAGLE_BACKEND_REDUCE_F64: dispatchOp<double>(d, d.columns, pairOut, stream, query, &workElems); break;
        case EAGLE_BACKEND_REDUCE_I32: dispatchOp<int32_t>(d, d.columns, pairOut, stream, query, &workElems); break;
        case EAGLE_BACKEND_REDUCE_I64: dispatchOp<int64_t>(d, d.columns, pairOut, stream, query, &workElems); break;
        default:
            if (query)
                workElems = workElemsFor<PlainP<uint8_t, AllOp>, uint8_t>(d.n, d.columns, smCount());
            else
                enqueueReduce<PlainP<uint8_t, AllOp>, uint8_t>(d, d.columns, 0, stream);
        }
        if (query)
            desc->work_elems = workElems;
    });
}

extern "C" __attribute__((visibility("default"))) eagle_backend_status eagle_backend_x_b200_reduce_fixed(
    struct eagle_backend_reduce_desc* desc)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_b200_reduce_fixed";
        constexpr size_t base = offsetof(eagle_backend_reduce_desc, work_elems) + sizeof(int64_t);
        if (desc == nullptr || desc->struct_size < base)
            invalid(std::string(who) + ": null desc or struct_size too small");
        eagle_backend_reduce_desc d{};
        std::memcpy(&d, desc, std::min<size_t>(desc->struct_size, sizeof d));
        const bool ext = desc->struct_size >= offsetof(eagle_backend_reduce_desc, comp_in) + sizeof(uint64_t);
        if (!ext) {
            d.policy = EAGLE_BACKEND_REDUCE_ORDERED;
            d.flags = 0;
            d.columns = 1;
            d.comp_in = 0;
        }
        if (d.n < 1)
            invalid(std::string(who) + ": n must be >= 1");
        if (d.dtype != EAGLE_BACKEND_REDUCE_F64 || d.op != EAGLE_BACKEND_REDUCE_OP_SUM)
            invalid(std::string(who) + ": the fixed-point leaf sums float64 (dtype F64, op SUM)");
        if (d.flags != 0)
            unsupported(std::string(who) + ": the fixed-point sum has no (hi, comp) pair to write (PAIR_OUT)");
        if (d.columns < 1 || d.policy > EAGLE_BACKEND_REDUCE_AUTO)
            invalid(std::string(who) + ": columns must be >= 1; unknown policy");
        const bool query = d.work_a == 0;
        if (!query && (d.in == 0 || d.out == 0 || d.work_b == 0))
            invalid(std::string(who) + ": in, out, work_a and work_b must be device addresses");
        DeviceScope scope(resolveDevice(d.device, query ? 0 : d.in));
        if (query)
            desc->work_elems = workElemsFor<FixedP, double>(d.n, d.columns, smCount());
        else
            enqueueReduce<FixedP, double>(d, d.columns, 0, seamStream(d.stream));
    });
}

extern "C" __attribute__((visibility("default"))) eagle_backend_status eagle_backend_x_b200_combine_partials(
    uint64_t hc, int64_t m, uint64_t work, uint64_t out, uint64_t stream)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_b200_combine_partials";
        if (m < 1)
            invalid(std::string(who) + ": m must be >= 1");
        if (hc == 0 || out == 0 || (m > 1 && work == 0))
            invalid(std::string(who) + ": hc, out and (for m > 1) work must be device addresses");
        DeviceScope scope(resolveDevice(-1, hc));
        combinePairsKernel<<<1, kSlots, 0, seamStream(stream)>>>(reinterpret_cast<const double*>(hc), m,
            reinterpret_cast<double*>(work), reinterpret_cast<double*>(out));
        launchCheck(who);
    });
}

namespace eb {
namespace {

/** CTAs of a counted reduction of up to ``capacity`` elements: about eight per SM,
 *  and never fewer than the groups the largest count needs. */
int64_t countedGrid(int64_t capacity)
{
    const int64_t leaves = (capacity + kLeaf - 1) / kLeaf;
    return std::max<int64_t>(int64_t(smCount()) * 8, (leaves + kMaxGroupLeaves - 1) / kMaxGroupLeaves);
}

template <class P, class T>
void enqueueCounted(const eagle_backend_reduce_desc& d, const uint32_t* count, int pairOut, cudaStream_t stream)
{
    const int64_t target = countedGrid(d.n);
    ReduceArgs a{};
    a.in = reinterpret_cast<const void*>(d.in);
    a.rows = d.n;
    a.cols = 1;
    a.partials = reinterpret_cast<void*>(d.work_a);
    a.counters = reinterpret_cast<uint32_t*>(d.work_b);
    a.out = reinterpret_cast<void*>(d.out);
    a.pairOut = pairOut;
    cudaCheck(cudaMemsetAsync(a.counters, 0, sizeof(uint32_t), stream), "cudaMemsetAsync");
    canonicalCountedKernel<P, T><<<unsigned(target), kSlots, 0, stream>>>(a, count);
    launchCheck("eagle_backend_x_b200_reduce_counted");
}

}  // namespace
}  // namespace eb

extern "C" __attribute__((visibility("default"))) eagle_backend_status eagle_backend_x_b200_reduce_counted(
    struct eagle_backend_reduce_desc* desc, uint64_t count)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_b200_reduce_counted";
        constexpr size_t base = offsetof(eagle_backend_reduce_desc, work_elems) + sizeof(int64_t);
        if (desc == nullptr || desc->struct_size < base)
            invalid(std::string(who) + ": null desc or struct_size too small");
        eagle_backend_reduce_desc d{};
        std::memcpy(&d, desc, std::min<size_t>(desc->struct_size, sizeof d));
        if (desc->struct_size < offsetof(eagle_backend_reduce_desc, comp_in) + sizeof(uint64_t)) {
            d.policy = EAGLE_BACKEND_REDUCE_ORDERED;
            d.flags = 0;
            d.columns = 1;
            d.comp_in = 0;
        }
        if (d.n < 1)
            invalid(std::string(who) + ": n (the capacity) must be >= 1");
        if (d.op != EAGLE_BACKEND_REDUCE_OP_SUM || d.dtype > EAGLE_BACKEND_REDUCE_I64)
            unsupported(std::string(who) + ": sums of F32 / F64 / I32 / I64 only");
        if (d.columns != 1 || d.comp_in != 0 || d.flags > EAGLE_BACKEND_REDUCE_PAIR_OUT)
            unsupported(std::string(who) + ": one column, no companion input");
        const bool fsum = d.dtype == EAGLE_BACKEND_REDUCE_F32 || d.dtype == EAGLE_BACKEND_REDUCE_F64;
        if (d.flags != 0 && !fsum)
            invalid(std::string(who) + ": PAIR_OUT takes a float sum");
        const int dev = resolveDevice(d.device, d.work_a == 0 ? 0 : d.in);
        DeviceScope scope(dev);
        const int64_t target = countedGrid(d.n);
        if (d.work_a == 0) {
            // partials: one per group (at most target of them); the counter word
            const int64_t elemBytes = (d.dtype == EAGLE_BACKEND_REDUCE_F32 || d.dtype == EAGLE_BACKEND_REDUCE_I32) ? 4 : 8;
            const int64_t partialBytes = target * 2 * elemBytes;
            desc->work_elems = std::max<int64_t>((partialBytes + elemBytes - 1) / elemBytes, 4);
            return;
        }
        if (d.in == 0 || d.out == 0 || d.work_b == 0 || count == 0)
            invalid(std::string(who) + ": in, out, work_a, work_b and count must be device addresses");
        const cudaStream_t stream = seamStream(d.stream);
        const uint32_t* cnt = reinterpret_cast<const uint32_t*>(count);
        const int pairOut = d.flags != 0;
        switch (d.dtype) {
        case EAGLE_BACKEND_REDUCE_F32: enqueueCounted<CompP<float>, float>(d, cnt, pairOut, stream); break;
        case EAGLE_BACKEND_REDUCE_F64: enqueueCounted<CompP<double>, double>(d, cnt, pairOut, stream); break;
        case EAGLE_BACKEND_REDUCE_I32: enqueueCounted<PlainP<int32_t, SumOp<int32_t>>, int32_t>(d, cnt, 0, stream); break;
        default: enqueueCounted<PlainP<int64_t, SumOp<int64_t>>, int64_t>(d, cnt, 0, stream);
        }
    });
}

extern "C" __attribute__((visibility("default"))) eagle_backend_status eagle_backend_x_b200_leaf_partials(
    uint64_t in, int64_t n, uint64_t out, uint64_t stream)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_b200_leaf_partials";
        if (n < 0)
            invalid(std::string(who) + ": n must be >= 0");
        if (n == 0)
            return;
        if (in == 0 || out == 0)
            invalid(std::string(who) + ": in and out must be device addresses");
        const int64_t leaves = (n + kLeaf - 1) / kLeaf;
        if (leaves > INT64_C(2147483647))
            unsupported(std::string(who) + ": too many leaves for one grid");
        DeviceScope scope(resolveDevice(-1, in));
        leafPartialsKernel<<<unsigned(leaves), kSlots, 0, seamStream(stream)>>>(reinterpret_cast<const double*>(in), n,
            reinterpret_cast<double*>(out));
        launchCheck(who);
    });
}
