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

/** eagle's fixed-point partial of a float64 sum (canonical.h:153-302), the leaf it
 *  takes on a device whose FP32:FP64 throughput ratio is 8 or worse (:304-313):
 *  the value is v * 2^u, v a signed 128-bit integer held as (lo, hi). A term's
 *  last mantissa bit lands at most 53 bits above the unit, kept 106 bits below the
 *  largest term seen; a join aligns the units (floor shifts) and halves both sides
 *  when either reaches 2^125. Infinities and NaN set sticky flags; value() rounds
 *  once to nearest-even. All integer arithmetic: the bits do not depend on order of
 *  evaluation beyond the tree's. */
struct FixedP {
    using I = __int128;
    using U = unsigned __int128;
    static constexpr int32_t kEmpty = -100000;  // the unit of a partial that saw no term
    static constexpr int32_t kPosInf = 1, kNegInf = 2, kNan = 4;
    uint64_t lo;
    int64_t hi;
    int32_t u, fl;

    __device__ __forceinline__ I get() const { return I((U(uint64_t(hi)) << 64) | U(lo)); }
    __device__ __forceinline__ void set(I v)
    {
        lo = uint64_t(U(v));
        hi = int64_t(v >> 64);
    }
    static __device__ __forceinline__ I shr(I v, int32_t d) { return v >> (d < 127 ? d : 127); }
    static __device__ __forceinline__ FixedP empty() { return FixedP{0, 0, kEmpty, 0}; }
    static __device__ __forceinline__ FixedP of(double x)
    {
        FixedP p = empty();
        p.add(x);
        return p;
    }
    static __device__ __forceinline__ FixedP of(double x, double xc)
    {
        FixedP p = empty();
        p.add(x);
        p.add(xc);
        return p;
    }
    __device__ __forceinline__ void add(double x, double xc)
    {
        add(x);
        add(xc);
    }
    __device__ __forceinline__ void add(double x)
    {
        const uint64_t b = uint64_t(__double_as_longlong(x));
        const int32_t e = int32_t((b >> 52) & 0x7ff);
        if (e == 0x7ff) {
            fl |= (b << 12) != 0 ? kNan : ((b >> 63) != 0 ? kNegInf : kPosInf);
            return;
        }
        const uint64_t m = (b & 0xfffffffffffffull) | (e != 0 ? (1ull << 52) : 0ull);
        if (m == 0)
            return;
        const int32_t ex = (e != 0 ? e : 1) - 1075;  // the weight of m's last bit
        I v = get();
        if (ex - 53 > u) {
            v = shr(v, ex - 53 - u);
            u = ex - 53;
        }
        const int32_t sh = ex - u;  // at most 53
        const I t = sh >= 0 ? I(U(m) << sh) : (-sh < 64 ? I(m >> -sh) : I(0));
        set((b >> 63) != 0 ? v - t : v + t);
    }
    static __device__ __forceinline__ bool wide(I z)
    {
        const I top = z >> 125;
        return top != 0 && top != -1;
    }
    static __device__ __forceinline__ FixedP join(const FixedP& a, const FixedP& b)
    {
        I x = a.get(), y = b.get();
        int32_t un = a.u;
        if (b.u > un) {
            x = shr(x, b.u - un);
            un = b.u;
        } else {
            y = shr(y, un - b.u);
        }
        if (wide(x) || wide(y)) {
            x >>= 1;
            y >>= 1;
            ++un;
        }
        FixedP o;
        o.set(x + y);
        o.u = un;
        o.fl = a.fl | b.fl;
        return o;
    }
    __device__ __forceinline__ double value() const
    {
        if (fl != 0) {
            if ((fl & kNan) != 0 || (fl & (kPosInf | kNegInf)) == (kPosInf | kNegInf))
                return __longlong_as_double(0x7ff8000000000000ll);
            return __longlong_as_double((fl & kPosInf) != 0 ? 0x7ff0000000000000ll : int64_t(0xfff0000000000000ull));
        }
        const I v = get();
        if (v == 0)
            return 0.0;
        const bool neg = v < 0;
        const U mag = neg ? U(0) - U(v) : U(v);
        const uint64_t mh = uint64_t(mag >> 64), ml = uint64_t(mag);
        const int32_t lz = mh != 0 ? __clzll(int64_t(mh)) : 64 + __clzll(int64_t(ml));
        const int32_t len = 128 - lz;
        const int32_t sub = len + u + 1074;  // the bits of weight 2^-1074 and up
        const int32_t keep = sub < 53 ? sub : 53;
        const int32_t drop = len - keep;
        double r;
        if (drop <= 0) {
            r = ldexp(double(uint64_t(mag)), u);
        } else {
            U q = drop < 128 ? mag >> drop : U(0);
            const U rem = drop < 128 ? mag - (q << drop) : mag;
            if (drop <= 128) {
                const U half = U(1) << (drop - 1);
                if (rem > half || (rem == half && (q & 1) != 0))
                    ++q;
            }
            r = ldexp(double(uint64_t(q)), u + drop);
        }
        return neg ? -r : r;
    }
    __device__ __forceinline__ FixedP shflDown(unsigned off) const
    {
        return {__shfl_down_sync(kFull, lo, off), __shfl_down_sync(kFull, hi, off), __shfl_down_sync(kFull, u, off),
            __shfl_down_sync(kFull, fl, off)};
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
