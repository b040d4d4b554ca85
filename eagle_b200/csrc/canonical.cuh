// The canonical ``ordered`` tree's device pieces shared by the reduction kernels:
// eagle's leaf of 256 slots x 16 strided terms (eagle/reduce/canonical.h:10-32,
// leaf :340-353), its (hi, comp) partial with the Neumaier join of
// canonical.h:130-151 (bitwise the independent oracle of
// tests/CanonicalReduceCases.h:73-78), and the pairwise levels with an odd last
// node carried (canonical.h:358-381).
#pragma once

#include "common.cuh"

#include <cmath>

namespace eb {
namespace {

constexpr int kSlots = 256;
constexpr int kTerms = 16;
constexpr int64_t kLeaf = int64_t(kSlots) * kTerms;
constexpr int kChunk = 512;         // nodes one pass of the final levels joins
template <class T>
struct CompP {  // a floating-point sum's partial (hi, comp)
    T h, c;
    static __device__ __forceinline__ CompP of(T x) { return {x, T(0)}; }
    static __device__ __forceinline__ CompP of(T x, T xc) { return {x, isfinite(x) ? xc : T(0)}; }
    static __device__ __forceinline__ CompP join(const CompP& a, const CompP& b)
    {
        const T s = a.h + b.h;
        const T bb = s - a.h;
        const T e = (a.h - (s - bb)) + (b.h - bb);
        return {s, isfinite(s) ? (a.c + b.c) + e : T(0)};
    }
    __device__ __forceinline__ void add(T x) { *this = join(*this, CompP{x, T(0)}); }
    __device__ __forceinline__ void add(T x, T xc)
    {
        add(x);
        c = isfinite(h) ? c + xc : T(0);
    }
    __device__ __forceinline__ T value() const { return isfinite(h) ? h + c : h; }
    __device__ __forceinline__ CompP shflDown(unsigned off) const
    {
        return {__shfl_down_sync(kFull, h, off), __shfl_down_sync(kFull, c, off)};
    }
};

/** eagle's exact fixed-point partial of a float64 sum: the leaf eagle takes on a
 *  device whose FP32:FP64 throughput ratio is 8 or worse (canonical.h:153-313). It
 *  stands for A * 2^unit, A a signed 128-bit integer held as two 64-bit words. The
 *  rules that decide its bits are eagle's (its tests pin them through exact known
 *  sums):
 *   (1) before any finite non-zero term: A = 0 and unit = kNoTerm, below every real
 *       unit;
 *   (2) a finite non-zero term (-1)^s * m * 2^e (m its integer significand, at most
 *       53 bits; e the weight of m's last bit): when unit < e - 53 the unit rises to
 *       e - 53 and A is divided by 2^(the rise), rounding toward -infinity; then
 *       A += (-1)^s * floor(m * 2^(e - unit));
 *   (3) a join lifts the lower unit to the higher as in (2); if either accumulator
 *       then lies outside [-2^125, 2^125), both are halved toward -infinity and the
 *       unit rises by one; then the accumulators add and the flags combine;
 *   (4) an infinity or NaN only sets a sticky flag: NaN, or infinities of both
 *       signs, make the value NaN; infinities of one sign make it that infinity.
 *  A stays below 2^127 in magnitude: a leaf folds at most 32 terms of at most 2^106
 *  units each, and (3) keeps a join's sum below 2^127. value() rounds A * 2^unit
 *  once to the nearest double, ties to even, subnormals included. */
struct FixedP {
    using I = __int128;
    using U = unsigned __int128;
    static constexpr int32_t kNoTerm = -100000;
    static constexpr int32_t kInfUp = 1, kInfDown = 2, kNaN = 4;
    uint64_t accLo;  // A, low word
    int64_t accHi;   // A, high word (carries the sign)
    int32_t unit;
    int32_t sticky;  // kInfUp | kInfDown | kNaN

    __device__ __forceinline__ I acc() const { return I((U(uint64_t(accHi)) << 64) | U(accLo)); }
    __device__ __forceinline__ void store(I a)
    {
        accLo = uint64_t(U(a));
        accHi = int64_t(a >> 64);
    }
    /** floor(a / 2^k) for any k >= 0: the arithmetic shift, whose result is already 0
     *  or -1 for every 128-bit a once k reaches 127. */
    static __device__ __forceinline__ I floorDiv2k(I a, int32_t k) { return a >> (k < 127 ? k : 127); }
    static __device__ __forceinline__ bool outside125(I a)
    {
        const I lim = I(1) << 125;
        return a < -lim || a >= lim;
    }
    static __device__ __forceinline__ FixedP none() { return FixedP{0ull, 0ll, kNoTerm, 0}; }
    static __device__ __forceinline__ FixedP of(double x)
    {
        FixedP p = none();
        p.add(x);
        return p;
    }
    static __device__ __forceinline__ FixedP of(double x, double xc)
    {
        FixedP p = none();
        p.add(x);
        p.add(xc);
        return p;
    }
    __device__ __forceinline__ void add(double x, double xc)
    {
        add(x);
        add(xc);
    }
    /** Rule (2), or (4) for a non-finite term. */
    __device__ __forceinline__ void add(double x)
    {
        const uint64_t w = uint64_t(__double_as_longlong(x));
        const uint32_t field = uint32_t(w >> 52) & 0x7ffu;
        const bool minus = (w >> 63) != 0;
        uint64_t m = w & ((1ull << 52) - 1);
        if (field == 0x7ffu) {
            sticky |= m != 0 ? kNaN : (minus ? kInfDown : kInfUp);
            return;
        }
        int32_t e;  // the weight of m's last bit
        if (field == 0) {
            if (m == 0)
                return;  // a signed zero adds nothing
            e = -1074;
        } else {
            m |= 1ull << 52;
            e = int32_t(field) - 1075;
        }
        I a = acc();
        if (unit < e - 53) {
            a = floorDiv2k(a, e - 53 - unit);
            unit = e - 53;
        }
        const int32_t lift = e - unit;  // at most 53
        const U term = lift >= 0 ? U(m) << lift : (lift > -64 ? U(m >> -lift) : U(0));
        store(minus ? a - I(term) : a + I(term));
    }
    /** Rule (3); the flags of either side carry over. */
    static __device__ __forceinline__ FixedP join(const FixedP& p, const FixedP& q)
    {
        int32_t unit = p.unit > q.unit ? p.unit : q.unit;
        I a = floorDiv2k(p.acc(), unit - p.unit);
        I b = floorDiv2k(q.acc(), unit - q.unit);
        if (outside125(a) || outside125(b)) {
            a >>= 1;
            b >>= 1;
            ++unit;
        }
        FixedP r;
        r.store(a + b);
        r.unit = unit;
        r.sticky = p.sticky | q.sticky;
        return r;
    }
    /** A * 2^unit to the nearest double (ties to even). |A| is cut to its top 64 bits
     *  plus a sticky bit for everything below them; those 64 bits hold the 53 the
     *  double keeps (fewer for a subnormal) and at least 11 below, so one
     *  round-to-nearest-even on them, with the sticky bit breaking a tie, is the
     *  correctly rounded result. */
    __device__ __forceinline__ double value() const
    {
        if (sticky != 0) {
            if ((sticky & kNaN) != 0 || (sticky & (kInfUp | kInfDown)) == (kInfUp | kInfDown))
                return __longlong_as_double(0x7ff8000000000000ll);
            return (sticky & kInfUp) != 0 ? __longlong_as_double(0x7ff0000000000000ll)
                                          : __longlong_as_double(int64_t(0xfff0000000000000ull));
        }
        const I a = acc();
        if (a == 0)
            return 0.0;
        const bool minus = a < 0;
        const U mag = minus ? U(0) - U(a) : U(a);
        const uint64_t w1 = uint64_t(mag >> 64), w0 = uint64_t(mag);
        uint64_t top;  // |A|'s leading 64 bits, its highest set bit at bit 63
        bool below;    // any set bit of |A| under them
        int32_t len;   // |A|'s bit length
        if (w1 != 0) {
            const int32_t z = __clzll(int64_t(w1));
            len = 128 - z;
            top = z == 0 ? w1 : (w1 << z) | (w0 >> (64 - z));
            below = (z == 0 ? w0 : w0 << z) != 0;
        } else {
            const int32_t z = __clzll(int64_t(w0));
            len = 64 - z;
            top = w0 << z;
            below = false;
        }
        const int32_t lead = unit + len - 1;  // the weight of the leading bit
        // bits at weights >= 2^-1074 survive: 53 for a normal result, fewer for a subnormal
        const int32_t keep = lead + 1075 < 53 ? lead + 1075 : 53;
        double r;
        if (keep <= 0) {
            // under the smallest subnormal 2^-1074: above its half (2^-1075) rounds up to it,
            // exactly its half ties to the even 0, anything smaller is 0
            r = (keep == 0 && (below || top != (1ull << 63))) ? __longlong_as_double(1ll) : 0.0;
        } else {
            const int32_t cut = 64 - keep;  // 11..63 low bits of top go
            uint64_t q = top >> cut;
            const uint64_t rest = top & ((1ull << cut) - 1);
            const uint64_t half = 1ull << (cut - 1);
            if (rest > half || (rest == half && (below || (q & 1) != 0)))
                ++q;  // a carry to 2^keep is still exact in a double
            r = ldexp(double(q), lead - keep + 1);
        }
        return minus ? -r : r;
    }
    __device__ __forceinline__ FixedP shflDown(unsigned off) const
    {
        return {__shfl_down_sync(kFull, accLo, off), __shfl_down_sync(kFull, accHi, off),
            __shfl_down_sync(kFull, unit, off), __shfl_down_sync(kFull, sticky, off)};
    }
};

/** The in-leaf tree over the slot partials (thread t < ``live`` holds slot t in
 *  ``mine``): offsets 128..32 through shared memory, 16..1 by warp shuffles, an
 *  absent partner carried. The leaf's partial is valid in thread 0. */
template <class P>
__device__ __forceinline__ P leafTree(const P& mine, int live, P* s)
{
    const int t = int(threadIdx.x);
    if (t < live)
        s[t] = mine;
    __syncthreads();
#pragma unroll
    for (int off = kSlots / 2; off >= 32; off >>= 1) {
        if (t < off && t + off < live)
            s[t] = P::join(s[t], s[t + off]);
        __syncthreads();
    }
    P q{};
    if (t < 32) {
        q = s[t];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const P o = q.shflDown(unsigned(off));
            if (t < off && t + off < live)
                q = P::join(q, o);
        }
    }
    __syncthreads();  // s is reused by the next leaf
    return q;
}

/** leafTree with one barrier: every thread stores its slot, then warp 0 alone runs
 *  the offsets 128, 64 and 32 (lane t joins slots t + 32 i in registers, the same
 *  pairs in the same order) and the shuffles, while the other warps go on. ``s``
 *  must not be written again before the CTA's next barrier after this call:
 *  callers alternate two buffers. The leaf's partial is valid in thread 0. */
template <class P>
__device__ __forceinline__ P leafTreeWarp0(const P& mine, int live, P* s)
{
    const int t = int(threadIdx.x);
    if (t < live)
        s[t] = mine;
    __syncthreads();
    P q{};
    if (t < 32) {
        P x[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int j = t + 32 * i;
            x[i] = j < live ? s[j] : P{};
            if (j + 128 < live)
                x[i] = P::join(x[i], s[j + 128]);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i)
            if (t + 32 * i + 64 < live)
                x[i] = P::join(x[i], x[i + 2]);
        if (t + 32 < live)
            x[0] = P::join(x[0], x[1]);
        q = x[0];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const P o = q.shflDown(unsigned(off));
            if (t < off && t + off < live)
                q = P::join(q, o);
        }
    }
    return q;
}

/** One leaf's partial (valid in thread 0): the slot walk, then the in-leaf tree. */
template <class P, class T, bool HasComp>
__device__ __forceinline__ P leafPartial(const T* __restrict__ in, const T* __restrict__ comp, int64_t cols,
    int64_t col, int64_t base, int64_t cnt, P* s)
{
    const int t = int(threadIdx.x);
    const int live = cnt < kSlots ? int(cnt) : kSlots;
    P p{};
    if (t < live) {
        T v[kTerms];
        T vc[HasComp ? kTerms : 1];
#pragma unroll
        for (int k = 0; k < kTerms; ++k) {
            const int64_t i = int64_t(t) + int64_t(k) * kSlots;
            v[k] = i < cnt ? in[(base + i) * cols + col] : T(0);
            if constexpr (HasComp)
                vc[k] = i < cnt ? comp[(base + i) * cols + col] : T(0);
        }
        if constexpr (HasComp)
            p = P::of(v[0], vc[0]);
        else
            p = P::of(v[0]);
#pragma unroll
        for (int k = 1; k < kTerms; ++k) {
            if (int64_t(t) + int64_t(k) * kSlots < cnt) {
                if constexpr (HasComp)
                    p.add(v[k], vc[k]);
                else
                    p.add(v[k]);
            }
        }
    }
    return leafTree(p, live, s);
}

/** leafPartial of a leaf whose i-th element (i < ``cnt``) is ``at(i)``, for leaves
 *  whose elements do not sit in one plane; the same slots, terms and order, so the
 *  same bits as leafPartial over those elements. No companion. */
template <class P, class T, class At>
__device__ __forceinline__ P leafPartialAt(At at, int64_t cnt, P* s)
{
    const int t = int(threadIdx.x);
    const int live = cnt < kSlots ? int(cnt) : kSlots;
    P p{};
    if (t < live) {
        T v[kTerms];
#pragma unroll
        for (int k = 0; k < kTerms; ++k) {
            const int64_t i = int64_t(t) + int64_t(k) * kSlots;
            v[k] = i < cnt ? at(i) : T(0);
        }
        p = P::of(v[0]);
#pragma unroll
        for (int k = 1; k < kTerms; ++k)
            if (int64_t(t) + int64_t(k) * kSlots < cnt)
                p.add(v[k]);
    }
    return leafTree(p, live, s);
}

// ------------------------------------------------ exchange blocks across ranks
//
// A sum over survivors spread across ranks exchanges two fixed-size blocks per rank,
// each in one all-gather:
//   the head block, kLeaf doubles: the rank's first min(count, kHead) survivors at
//     [0, kHead), its survivor count in the low 32 bits of slot kHead;
//   the partial block, 2 cap + 2 doubles: (hi, comp) of each leaf starting in the
//     rank's part at [2 k, 2 k + 1], the number of those leaves in the low 32 bits of
//     slot 2 cap (all ones: a pass failed), slot 2 cap + 1 unused.

constexpr int kMaxRanks = 256;
constexpr int64_t kHead = kLeaf - 1;   // survivors a rank shares with the earlier ranks
constexpr int64_t kHeadBlock = kLeaf;  // doubles per head block

__device__ __forceinline__ uint32_t blockCount(const double* __restrict__ blocks, int q)
{
    return uint32_t(__double_as_longlong(blocks[int64_t(q) * kHeadBlock + kHead]));
}

__device__ __forceinline__ double blockHead(const double* __restrict__ blocks, int q, int64_t i)
{
    return blocks[int64_t(q) * kHeadBlock + i];
}

__device__ __forceinline__ double countSlot(uint32_t c)
{
    return __longlong_as_double(static_cast<long long>(c));
}

__host__ __device__ __forceinline__ int64_t partialBlock(int64_t cap) { return 2 * cap + 2; }

/** Pairwise levels over ``v[0, m)`` in shared memory (an aligned subtree): node i
 *  of level L sits at i * 2^L; its right child, if present, at + 2^(L-1). */
template <class P>
__device__ __forceinline__ void levels(P* v, int m)
{
    for (int off = 1; off < m; off <<= 1) {
        for (int i = int(threadIdx.x) * 2 * off; i < m; i += int(blockDim.x) * 2 * off)
            if (i + off < m)
                v[i] = P::join(v[i], v[i + off]);
        __syncthreads();
    }
}

}  // namespace
}  // namespace eb
