// Test infrastructure: the CPU restatement of eagle's until-done hot path that the
// parity tests check the CUDA engine against. Nothing in the product links or calls
// this file; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg do.
//
// What it restates (paths relative to the eagle source tree):
//   * the canonical ``ordered`` reduction tree: eagle/reduce/canonical.h:10-32
//     (definition), :115-151 (Partial: of / add / join / value), :340-353 (leaf),
//     :358-381 (pairwise), :397-408 (partialRange). The join arithmetic is the one
//     the reference's own independent test oracle pins, tests/CanonicalReduceCases.h:73-78
//     ("a Neumaier step is a join with (x, 0)", :94); MinOp is canonical.h:110-113.
//   * active-set compaction: eagle/filtering/Compact.h:23-47 (ascending map of the
//     kept samples, count), :113-118 (reorder trigger), :233-236 (n == 0).
//   * the band policy: eagle/policy/Launch.h:184-190 (bandK) and the POLICY cell op,
//     python/src/plugin/eagle_cuda.cu:1990-2025.
//   * the until-done semantics of a finishing step kernel:
//     docs/content/modules/filtering/run_until_done.rst:4-24,36-75 (a live sample steps,
//     assigns ``terminated``, stops and is counted once when it is set); the fast-path
//     step count (python/eagle/_until_done.py:1345-1352: the longest sample's steps);
//     the Euler oscillator body of README.md:89-97 in its written expression order.
//   * the host twin's team schedule: python/eagle/_host_loop.py:400-455 (tiles of
//     contiguous samples, each run to completion), eagle/exec/HostTeam.h:23-27.
//
// Built with -ffp-contract=off: every floating-point operation below rounds once,
// exactly as written. The ``fma`` variants call std::fma explicitly where the device
// compiler would contract a multiply-add (x0 + dt*v0, v0 - c*x0).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <vector>

#include <omp.h>
#include <random>

#include "oracle.h"

namespace {

// ---------------------------------------------------------------- canonical tree

constexpr int64_t kSlots = 256;
constexpr int64_t kTerms = 16;
constexpr int64_t kLeaf = kSlots * kTerms;

template <class T>
struct Comp {  // a floating-point sum's partial: (hi, comp)
    T h, c;
    static Comp of(T x) { return {x, T(0)}; }
    static Comp join(const Comp& a, const Comp& b)
    {
        const T s = a.h + b.h;
        const T bb = s - a.h;
        const T e = (a.h - (s - bb)) + (b.h - bb);
        return {s, std::isfinite(s) ? (a.c + b.c) + e : T(0)};
    }
    // a Neumaier step is a join with (x, 0)
    void add(T x) { *this = join(*this, Comp{x, T(0)}); }
    // a term with a companion: canonical.h:139-143 (Neumaier step, then the companion)
    void add(T x, T xc)
    {
        add(x);
        c = std::isfinite(h) ? c + xc : T(0);
    }
    static Comp of(T x, T xc) { return {x, std::isfinite(x) ? xc : T(0)}; }
    T value() const { return std::isfinite(h) ? h + c : h; }
};

template <class T, class Op>
struct Plain {  // every exact operator folds plainly
    T h;
    static Plain of(T x) { return {x}; }
    static Plain of(T x, T) { return {x}; }
    static Plain join(const Plain& a, const Plain& b) { return {Op{}(a.h, b.h)}; }
    void add(T x) { h = Op{}(h, x); }
    void add(T x, T) { add(x); }
    T value() const { return h; }
};

template <class T>
struct SumOp {
    T operator()(T a, T b) const
    {
        if constexpr (std::is_integral_v<T>) {
            using U = std::make_unsigned_t<T>;
            return T(U(a) + U(b));  // two's-complement wrap, as the device adds
        } else {
            return a + b;
        }
    }
};
template <class T>
struct MaxOp {
    T operator()(T a, T b) const { return a > b ? a : b; }
};
template <class T>
struct MinOp {
    T operator()(T a, T b) const { return a < b ? a : b; }
};
struct AllOp {
    uint8_t operator()(uint8_t a, uint8_t b) const { return uint8_t((a != 0) && (b != 0)); }
};

// A column of a row-major (rows, cols) plane, with an optional companion plane.
template <class T>
struct ColumnIn {
    const T* in;
    const T* comp;
    int64_t cols, col;
    T x(int64_t i) const { return in[i * cols + col]; }
    T xc(int64_t i) const { return comp[i * cols + col]; }
};

template <class P, class T>
P leaf(const ColumnIn<T>& in, int64_t base, int64_t cnt)
{
    const int64_t live = std::min(cnt, kSlots);
    P s[kSlots];
    for (int64_t t = 0; t < live; ++t) {
        for (int64_t k = t; k < cnt; k += kSlots) {
            if (in.comp == nullptr) {
                if (k == t)
                    s[t] = P::of(in.x(base + k));
                else
                    s[t].add(in.x(base + k));
            } else {
                if (k == t)
                    s[t] = P::of(in.x(base + k), in.xc(base + k));
                else
                    s[t].add(in.x(base + k), in.xc(base + k));
            }
        }
    }
    for (int64_t off = kSlots / 2; off > 0; off >>= 1)
        for (int64_t t = 0; t < off; ++t)
            if (t + off < live)
                s[t] = P::join(s[t], s[t + off]);
    return s[0];
}

// Level-by-level pairwise reduction of v[0, m), an odd last node carried.
template <class P>
P pairwise(std::vector<P>& v)
{
    int64_t m = int64_t(v.size());
    while (m > 1) {
        const int64_t pairs = m / 2;
        for (int64_t i = 0; i < pairs; ++i)
            v[i] = P::join(v[2 * i], v[2 * i + 1]);
        if (m & 1)
            v[pairs] = v[m - 1];
        m = (m + 1) / 2;
    }
    return v[0];
}

template <class P, class T>
std::vector<P> leafPartials(const ColumnIn<T>& in, int64_t rows)
{
    const int64_t nl = (rows + kLeaf - 1) / kLeaf;
    std::vector<P> parts(static_cast<size_t>(nl));
#pragma omp parallel for schedule(static)
    for (int64_t l = 0; l < nl; ++l)
        parts[size_t(l)] = leaf<P>(in, l * kLeaf, std::min(kLeaf, rows - l * kLeaf));
    return parts;
}

template <class P, class T>
P reduceColumn(const ColumnIn<T>& in, int64_t rows)
{
    auto parts = leafPartials<P>(in, rows);
    return pairwise(parts);
}

// The fixed-point partial of a float64 sum that eagle takes on devices whose
// FP32:FP64 throughput ratio is 8 or worse (canonical.h:153-313, the rule :304-313):
// the value is v * 2^u with v a signed 128-bit integer. A term's last mantissa bit
// lands at most 53 bits above the unit, which is kept 106 bits below the largest
// term seen (a term, or an aligned partial, loses at most one unit); a join halves
// both sides and raises the unit when either reaches 2^125. Infinities and NaN set
// sticky flags; value() rounds once to nearest-even, subnormals included.
struct Fixed {
    using I = __int128;
    using U = unsigned __int128;
    static constexpr int32_t kEmpty = -100000;  // the unit of a partial that saw no term
    static constexpr int32_t kPosInf = 1, kNegInf = 2, kNan = 4;
    I v = 0;
    int32_t u = kEmpty, fl = 0;

    static I shr(I x, int32_t d) { return x >> (d < 127 ? d : 127); }  // floor, any d >= 0
    static Fixed of(double x)
    {
        Fixed p;
        p.add(x);
        return p;
    }
    static Fixed of(double x, double xc)
    {
        Fixed p;
        p.add(x);
        p.add(xc);
        return p;
    }
    void add(double x, double xc)
    {
        add(x);
        add(xc);
    }
    void add(double x)
    {
        uint64_t b;
        std::memcpy(&b, &x, sizeof b);
        const int32_t e = int32_t((b >> 52) & 0x7ff);
        if (e == 0x7ff) {
            fl |= (b << 12) != 0 ? kNan : ((b >> 63) != 0 ? kNegInf : kPosInf);
            return;
        }
        const uint64_t m = (b & 0xfffffffffffffull) | (e != 0 ? (1ull << 52) : 0ull);
        if (m == 0)
            return;
        const int32_t ex = (e != 0 ? e : 1) - 1075;  // the weight of m's last bit
        if (ex - 53 > u) {
            v = shr(v, ex - 53 - u);
            u = ex - 53;
        }
        const int32_t sh = ex - u;  // at most 53
        const I t = sh >= 0 ? I(U(m) << sh) : (-sh < 64 ? I(m >> -sh) : I(0));
        v = (b >> 63) != 0 ? v - t : v + t;
    }
    static Fixed join(const Fixed& a, const Fixed& b)
    {
        I x = a.v, y = b.v;
        int32_t u = a.u;
        if (b.u > u) {
            x = shr(x, b.u - u);
            u = b.u;
        } else {
            y = shr(y, u - b.u);
        }
        const auto wide = [](I z) { const I top = z >> 125; return top != 0 && top != -1; };
        if (wide(x) || wide(y)) {
            x >>= 1;
            y >>= 1;
            ++u;
        }
        Fixed o;
        o.v = x + y;
        o.u = u;
        o.fl = a.fl | b.fl;
        return o;
    }
    double value() const
    {
        if (fl != 0) {
            if ((fl & kNan) != 0 || (fl & (kPosInf | kNegInf)) == (kPosInf | kNegInf))
                return std::numeric_limits<double>::quiet_NaN();
            return (fl & kPosInf) != 0 ? std::numeric_limits<double>::infinity()
                                       : -std::numeric_limits<double>::infinity();
        }
        if (v == 0)
            return 0.0;
        const bool neg = v < 0;
        const U mag = neg ? U(0) - U(v) : U(v);
        int len = 0;
        for (U z = mag; z != 0; z >>= 1)
            ++len;
        const int32_t sub = len + u + 1074;  // the bits of weight 2^-1074 and up
        const int32_t keep = sub < 53 ? sub : 53;
        const int32_t drop = len - keep;
        double r;
        if (drop <= 0) {
            r = std::ldexp(double(uint64_t(mag)), u);
        } else {
            U q = drop < 128 ? mag >> drop : U(0);
            const U rem = drop < 128 ? mag - (q << drop) : mag;
            if (drop <= 128) {
                const U half = U(1) << (drop - 1);
                if (rem > half || (rem == half && (q & 1) != 0))
                    ++q;
            }
            r = std::ldexp(double(uint64_t(q)), u + drop);
        }
        return neg ? -r : r;
    }
};

template <class T, class Op>
int reducePlainTyped(const void* in, int64_t n, int64_t cols, void* out)
{
    auto* o = static_cast<T*>(out);
    for (int64_t j = 0; j < cols; ++j) {
        ColumnIn<T> ci{static_cast<const T*>(in), nullptr, cols, j};
        o[j] = reduceColumn<Plain<T, Op>>(ci, n).value();
    }
    return 0;
}

template <class T>
int reduceSumFloat(const void* in, int64_t n, int64_t cols, const void* comp, void* out, int pairOut)
{
    auto* o = static_cast<T*>(out);
    for (int64_t j = 0; j < cols; ++j) {
        ColumnIn<T> ci{static_cast<const T*>(in), static_cast<const T*>(comp), cols, j};
        const Comp<T> r = reduceColumn<Comp<T>>(ci, n);
        if (pairOut) {
            o[j] = r.h;
            o[cols + j] = std::isfinite(r.h) ? r.c : T(0);
        } else {
            o[j] = r.value();
        }
    }
    return 0;
}

// the exact-sum fixture of tests/CanonicalReduceCases.h:141-176 (used below)
template <class T>
double fixtureOf(int64_t n, double kappa, T* x, double* reached)
{
    std::mt19937_64 rng{static_cast<uint64_t>(n)};
    std::uniform_int_distribution<int> unit(1, 8);
    std::uniform_real_distribution<double> mag(1.0, 2.0);
    std::vector<double> big(static_cast<size_t>(n));
    long long units = 0;
    int64_t nbig = 0;
    for (int64_t i = 0; i < n; ++i) {
        const int64_t j = std::min(i, n - 1 - i);
        big[size_t(j)] = mag(rng);
        if (j % 4 == 0 || i == n - 1 - i) {
            const int u = unit(rng);
            units += u;
            x[i] = T(std::ldexp(double(u), -10));
        } else {
            ++nbig;
        }
    }
    const double exact = std::ldexp(double(units), -10);
    const double scale = kappa * exact / (1.5 * double(std::max<int64_t>(nbig, 1)));
    double abs = 0;
    for (int64_t i = 0; i < n; ++i) {
        const int64_t j = std::min(i, n - 1 - i);
        if (!(j % 4 == 0 || i == n - 1 - i))
            x[i] = (i < n - 1 - i) ? T(big[size_t(j)] * scale) : -T(big[size_t(j)] * scale);
        abs += std::fabs(double(x[i]));
    }
    *reached = abs / exact;
    return exact;
}

}  // namespace

extern "C" {

int oracle_threads(int threads)
{
    if (threads > 0)
        omp_set_num_threads(threads);
    return omp_get_max_threads();
}

int oracle_reduce(const void* in, int64_t n, int64_t cols, int dtype, int op, const void* comp_in,
    void* out, int pair_out)
{
    if (n < 1 || cols < 1 || in == nullptr || out == nullptr)
        return 2;
    const bool fsum = op == ORACLE_OP_SUM && (dtype == ORACLE_F32 || dtype == ORACLE_F64);
    if ((comp_in != nullptr || pair_out) && !fsum)
        return 2;
    if ((op == ORACLE_OP_ALL) != (dtype == ORACLE_U8))
        return 2;
    switch (dtype) {
    case ORACLE_F32:
        if (op == ORACLE_OP_SUM)
            return reduceSumFloat<float>(in, n, cols, comp_in, out, pair_out);
        if (op == ORACLE_OP_MAX)
            return reducePlainTyped<float, MaxOp<float>>(in, n, cols, out);
        return reducePlainTyped<float, MinOp<float>>(in, n, cols, out);
    case ORACLE_F64:
        if (op == ORACLE_OP_SUM)
            return reduceSumFloat<double>(in, n, cols, comp_in, out, pair_out);
        if (op == ORACLE_OP_MAX)
            return reducePlainTyped<double, MaxOp<double>>(in, n, cols, out);
        return reducePlainTyped<double, MinOp<double>>(in, n, cols, out);
    case ORACLE_I32:
        if (op == ORACLE_OP_SUM)
            return reducePlainTyped<int32_t, SumOp<int32_t>>(in, n, cols, out);
        if (op == ORACLE_OP_MAX)
            return reducePlainTyped<int32_t, MaxOp<int32_t>>(in, n, cols, out);
        return reducePlainTyped<int32_t, MinOp<int32_t>>(in, n, cols, out);
    case ORACLE_I64:
        if (op == ORACLE_OP_SUM)
            return reducePlainTyped<int64_t, SumOp<int64_t>>(in, n, cols, out);
        if (op == ORACLE_OP_MAX)
            return reducePlainTyped<int64_t, MaxOp<int64_t>>(in, n, cols, out);
        return reducePlainTyped<int64_t, MinOp<int64_t>>(in, n, cols, out);
    case ORACLE_U8:
        return reducePlainTyped<uint8_t, AllOp>(in, n, cols, out);
    default:
        return 2;
    }
}

int oracle_reduce_fixed(const double* in, int64_t n, int64_t cols, const double* comp_in, double* out)
{
    if (n < 1 || cols < 1 || in == nullptr || out == nullptr)
        return 2;
    for (int64_t j = 0; j < cols; ++j) {
        ColumnIn<double> ci{in, comp_in, cols, j};
        out[j] = reduceColumn<Fixed>(ci, n).value();
    }
    return 0;
}

// The cancellation ladder of eagle's fixed-point tests (tests/test_CanonicalReduce.cu:88-119):
// x at r and exactly -x at n-1-r, |x| a full 52-bit mantissa times 2^e, e uniform in
// [G - ER, G + ER]; a quarter of the pairs (and the middle) carry v * 2^-10 on both
// partners instead. ``units`` = the exact sum in units of 2^-10.
void oracle_ladder(int64_t n, int ER, int G, double* x, long long* units)
{
    const auto mix = [](uint64_t z) {
        z += 0x9E3779B97F4A7C15ull;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    };
    long long total = 0;
    for (int64_t r = 0; r < n; ++r) {
        const int64_t m = n - 1 - r, j = std::min(r, m);
        const uint64_t h = mix(uint64_t(j) * 0x100000001B3ull ^ mix(7));
        if (j == 0 || m == r || (h & 3) == 0) {
            const long long v = 1 + (long long)((h >> 8) % 4096);
            x[r] = std::ldexp(double(v), -10);
            total += v;
        } else {
            const uint64_t h2 = mix(h), h3 = mix(h2);
            const double mant = 1.0 + double(h2 & ((1ull << 52) - 1)) / double(1ull << 52);
            const double v = std::ldexp(mant, int((h3 >> 1) % uint64_t(2 * ER + 1)) - ER + G);
            x[r] = ((h3 & 1) != 0) == (r < m) ? -v : v;
        }
    }
    *units = total;
}

int64_t oracle_leaf_partials_f64(const double* x, int64_t n, double* hc)
{
    if (n < 1)
        return 0;
    ColumnIn<double> ci{x, nullptr, 1, 0};
    const auto parts = leafPartials<Comp<double>>(ci, n);
    for (size_t i = 0; i < parts.size(); ++i) {
        hc[2 * i] = parts[i].h;
        hc[2 * i + 1] = parts[i].c;
    }
    return int64_t(parts.size());
}

void oracle_pairwise_f64(const double* hc, int64_t m, double* root_hc)
{
    std::vector<Comp<double>> v(static_cast<size_t>(m));
    for (int64_t i = 0; i < m; ++i)
        v[size_t(i)] = {hc[2 * i], hc[2 * i + 1]};
    const auto r = pairwise(v);
    root_hc[0] = r.h;
    root_hc[1] = r.c;
}

double oracle_partial_value_f64(double h, double c)
{
    return std::isfinite(h) ? h + c : h;
}

// ------------------------------------------------------------------- compaction

int oracle_compact(const uint8_t* mask, int64_t n, uint32_t flags, int32_t* index_map, uint32_t* count,
    uint32_t span, float theta, uint32_t* live32, uint32_t* fire)
{
    if (n < 0 || n > INT64_C(2147483647))
        return 8;
    const bool drop = (flags & ORACLE_MASK_IS_DROP) != 0;
    uint32_t c = 0, groups = 0;
    for (int64_t g = 0; g * 32 < n; ++g) {
        bool any = false;
        for (int64_t i = g * 32; i < std::min<int64_t>(n, (g + 1) * 32); ++i) {
            const bool set = mask[i] != 0;
            if (drop ? !set : set) {
                index_map[c++] = int32_t(i);
                any = true;
            }
        }
        groups += any ? 1u : 0u;
    }
    *count = c;
    if (live32 != nullptr) {
        *live32 = groups;
        const double limit = double(theta) * 32.0 * double(groups);
        *fire = (double(c) < limit && c < span && span >= 4096u) ? 1u : 0u;
    }
    return 0;
}

uint32_t oracle_mask_count(const uint8_t* mask, int64_t n)
{
    uint32_t c = 0;
    for (int64_t i = 0; i < n; ++i)
        c += mask[i] != 0 ? 1u : 0u;
    return c;
}

// ----------------------------------------------------------------------- policy

int64_t oracle_band_k(double rate, int64_t newly, int64_t live, int64_t k, int64_t k_max, int64_t k_min)
{
    if (newly <= 0)
        return k_max;
    const double e2 = 2.0 * rate * double(live) * double(k) / double(newly);
    int64_t p = 1;
    while (p < (INT64_C(1) << 30) && e2 >= 2.0 * double(p) * double(p))
        p *= 2;
    return std::min(std::max(p, k_min), k_max);
}

void oracle_policy_step(uint32_t finished, uint32_t total, int64_t* cells, int64_t* word, uint32_t* go,
    int64_t* hist, int64_t k_min, int64_t k_max, int iK, int iFin, int iDone, int iCap, int iR, int iMapped,
    int scale)
{
    const int64_t fin = finished, all = total;
    const int64_t live = all - fin, newly = fin - cells[iFin];
    const int64_t done = cells[iDone] + word[0];
    cells[iMapped] += all - cells[iFin];
    cells[iFin] = fin;
    cells[iDone] = done;
    const int64_t k = cells[iK];
    const double rate = double(cells[iR]) / double(scale);
    const int64_t k_next = oracle_band_k(rate, newly, live, k, k_max, k_min);
    cells[iK] = k_next;
    const int64_t left = cells[iCap] - done;
    const uint32_t g = (fin != all) && (left > 0);
    go[0] = g;
    if (g) {
        const int64_t w = k_next < left ? k_next : left;
        word[0] = w;
        hist[w] += 1;
    }
}

// ------------------------------------------------------------ Euler oscillator

// One sample of the README oscillator run until it terminates or has taken
// ``max_steps`` steps in this run; returns the steps taken.
static inline int64_t oscillatorSample(double omega, double t_end, double dt, double& x, double& v, double& t,
    uint8_t& term, int64_t max_steps, bool fused)
{
    if (term != 0)
        return 0;
    const double c = (dt * omega) * omega;  // ((dt*omega)*omega), hoisted: the same product every step
    double x0 = x, v0 = v, tt = t;
    int64_t s = 0;
    while (s < max_steps) {
        double x1, v1;
        if (fused) {
            x1 = std::fma(dt, v0, x0);
            v1 = std::fma(-c, x0, v0);
        } else {
            x1 = x0 + dt * v0;
            v1 = v0 - c * x0;
        }
        x0 = x1;
        v0 = v1;
        tt = tt + dt;
        ++s;
        if (tt >= t_end) {
            term = 1;
            break;
        }
    }
    x = x0;
    v = v0;
    t = tt;
    return s;
}

int oracle_oscillator_run(int64_t n, const double* omega, const double* t_end, double t_end_uniform, double dt,
    double* x, double* v, double* t, uint8_t* term, int32_t* steps_out, int64_t max_steps, int fused,
    int64_t tile, int64_t* stats)
{
    if (n < 0 || max_steps < 0)
        return 2;
    if (tile <= 0)
        tile = 1024;
    const int64_t tiles = (n + tile - 1) / tile;
    int64_t finished = 0, longest = 0, total = 0;
#pragma omp parallel for schedule(dynamic, 1) reduction(+ : finished, total) reduction(max : longest)
    for (int64_t b = 0; b < tiles; ++b) {
        const int64_t end = std::min(n, (b + 1) * tile);
        for (int64_t i = b * tile; i < end; ++i) {
            const double te = t_end != nullptr ? t_end[i] : t_end_uniform;
            const int64_t s = oscillatorSample(omega[i], te, dt, x[i], v[i], t[i], term[i], max_steps, fused != 0);
            if (steps_out != nullptr)
                steps_out[i] = int32_t(s);
            finished += term[i] != 0 ? 1 : 0;
            longest = std::max(longest, s);
            total += s;
        }
    }
    if (stats != nullptr) {
        stats[0] = finished;
        stats[1] = longest;
        stats[2] = total;
    }
    return 0;
}

// ------------------------------------------------------------ gambler's ruin
//
// The random-walk configuration: a position in (0, 100) moves +1 or -1 per step
// and the sample stops when it reaches 0 or 100; the output is its absorption
// time. eagle has no code for it (its random numbers come from the absent aether
// library), so the random stream is this build's definition: Philox-4x32-10
// (Salmon, Moraes, Dror and Shaw, "Parallel random numbers: as easy as 1, 2, 3",
// SC'11) with key = the 64-bit seed and counter = (step / 128, sample id), both as
// two 32-bit words, low word first; step s of a sample (0-based, counted over its
// whole life) moves +1 when bit (s mod 128) of the 128-bit output (word s/32 mod 4,
// bit s mod 32) is set, else -1.

static inline void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1)
{
    for (int r = 0; r < 10; ++r) {
        if (r > 0) {
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
        const uint64_t p0 = uint64_t(0xD2511F53u) * c[0];
        const uint64_t p1 = uint64_t(0xCD9E8D57u) * c[2];
        const uint32_t hi0 = uint32_t(p0 >> 32), lo0 = uint32_t(p0);
        const uint32_t hi1 = uint32_t(p1 >> 32), lo1 = uint32_t(p1);
        const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
        c[0] = n0;
        c[1] = lo1;
        c[2] = n2;
        c[3] = lo0;
    }
}

void oracle_philox4x32_10(const uint32_t counter[4], uint64_t seed, uint32_t out[4])
{
    uint32_t c[4] = {counter[0], counter[1], counter[2], counter[3]};
    philox4x32_10(c, uint32_t(seed), uint32_t(seed >> 32));
    for (int q = 0; q < 4; ++q)
        out[q] = c[q];
}

int oracle_gambler_run(int64_t n, int32_t* pos, int64_t* time, uint8_t* term, int64_t id_base, uint64_t seed,
    int64_t max_steps, int64_t* stats)
{
    if (n < 0 || max_steps < 0)
        return 2;
    int64_t finished = 0, longest = 0, total = 0;
#pragma omp parallel for schedule(dynamic, 1024) reduction(+ : finished, total) reduction(max : longest)
    for (int64_t i = 0; i < n; ++i) {
        int64_t s = 0;
        if (term[i] == 0) {
            const uint64_t id = uint64_t(id_base + i);
            int32_t p = pos[i];
            int64_t tm = time[i];
            uint32_t block[4] = {0, 0, 0, 0};
            int64_t have = -1;  // the 128-step block held in ``block``
            while (s < max_steps) {
                const int64_t blk = tm >> 7;
                if (blk != have) {
                    uint32_t c[4] = {uint32_t(uint64_t(blk)), uint32_t(uint64_t(blk) >> 32), uint32_t(id),
                        uint32_t(id >> 32)};
                    philox4x32_10(c, uint32_t(seed), uint32_t(seed >> 32));
                    for (int q = 0; q < 4; ++q)
                        block[q] = c[q];
                    have = blk;
                }
                const int b = int(tm & 127);
                p += ((block[b >> 5] >> (b & 31)) & 1u) ? 1 : -1;
                ++tm;
                ++s;
                if (p == 0 || p == 100) {
                    term[i] = 1;
                    break;
                }
            }
            pos[i] = p;
            time[i] = tm;
        }
        finished += term[i] != 0 ? 1 : 0;
        longest = std::max(longest, s);
        total += s;
    }
    if (stats != nullptr) {
        stats[0] = finished;
        stats[1] = longest;
        stats[2] = total;
    }
    return 0;
}

// ------------------------------------------------------------ Lorenz, RKF7(8)
//
// Lorenz-63 (dx = sigma (y - x), dy = x (rho - z) - y, dz = x y - beta z) integrated
// by the adaptive Runge-Kutta-Fehlberg 7(8) attempt of eagle's perf card
// (benchmarks/perf_card/perf_card.py:131-138 controller constants, :255-278
// Fehlberg's tableau from NASA TR R-287, :289-309 stages with left-to-right term
// sums skipping zero coefficients and the mixed max-norm error ratio, :313-317
// sum_terms, :330-348 the attempt: clip the last step onto t_final, accept or reject,
// scale h by min(5, max(0.2, 0.9 ratio^expo)), count, stop at t_final).
//
// The controller's power ratio^expo is this build's deterministic pow (the library
// pow rounds differently on CPU and GPU): ln by exponent extraction and the series
// ln m = 2 atanh((m-1)/(m+1)) on m in [sqrt(1/2), sqrt(2)), exp by reduction to
// f = y - n ln2 and the Taylor series of e^f, then scaling by 2^n; every operation
// rounds once, in the same order on the device.

}  // extern "C"

namespace {

const double kLn2 = 0.6931471805599453;

double detLog(double r)
{
    uint64_t b;
    std::memcpy(&b, &r, sizeof b);
    int k = 0;
    if (((b >> 52) & 0x7ff) == 0) {  // subnormal: scale up exactly
        r = r * 18014398509481984.0;  // 2^54
        std::memcpy(&b, &r, sizeof b);
        k = -54;
    }
    k += int((b >> 52) & 0x7ff) - 1023;
    b = (b & 0x800FFFFFFFFFFFFFull) | (uint64_t(1023) << 52);  // m in [1, 2)
    double m;
    std::memcpy(&m, &b, sizeof m);
    if (m > 1.4142135623730951) {
        m = m * 0.5;
        k += 1;
    }
    const double u = (m - 1.0) / (m + 1.0);
    const double u2 = u * u;
    double p = 1.0 / 23.0;
    p = p * u2 + 1.0 / 21.0;
    p = p * u2 + 1.0 / 19.0;
    p = p * u2 + 1.0 / 17.0;
    p = p * u2 + 1.0 / 15.0;
    p = p * u2 + 1.0 / 13.0;
    p = p * u2 + 1.0 / 11.0;
    p = p * u2 + 1.0 / 9.0;
    p = p * u2 + 1.0 / 7.0;
    p = p * u2 + 1.0 / 5.0;
    p = p * u2 + 1.0 / 3.0;
    p = p * u2 + 1.0;
    const double lnm = (2.0 * u) * p;
    return lnm + double(k) * kLn2;
}

double detExp(double y)
{
    const double n = std::nearbyint(y / kLn2);
    const double f = y - n * kLn2;
    double p = 1.0 / 6402373705728000.0;  // 1/18!
    p = p * f + 1.0 / 355687428096000.0;
    p = p * f + 1.0 / 20922789888000.0;
    p = p * f + 1.0 / 1307674368000.0;
    p = p * f + 1.0 / 87178291200.0;
    p = p * f + 1.0 / 6227020800.0;
    p = p * f + 1.0 / 479001600.0;
    p = p * f + 1.0 / 39916800.0;
    p = p * f + 1.0 / 3628800.0;
    p = p * f + 1.0 / 362880.0;
    p = p * f + 1.0 / 40320.0;
    p = p * f + 1.0 / 5040.0;
    p = p * f + 1.0 / 720.0;
    p = p * f + 1.0 / 120.0;
    p = p * f + 1.0 / 24.0;
    p = p * f + 1.0 / 6.0;
    p = p * f + 1.0 / 2.0;
    p = p * f + 1.0;
    p = p * f + 1.0;
    const int e = int(n);
    if (e > 1000 || e < -1000)
        return e > 0 ? INFINITY : 0.0;
    const uint64_t sb = uint64_t(e + 1023) << 52;
    double scale;
    std::memcpy(&scale, &sb, sizeof scale);
    return p * scale;
}

double detPow(double r, double e)  // r >= 0 (or NaN), e < 0: the controller's power
{
    if (std::isnan(r))
        return r;
    if (r == 0.0)
        return INFINITY;
    if (std::isinf(r))
        return 0.0;
    return detExp(e * detLog(r));
}

// Fehlberg 7(8) (NASA TR R-287): the lower-triangular a, the 8th-order weights b, the
// error weights be (b_hat - b), as eagle's perf card lists them.
const double kA[12][12] = {
    {2. / 27},
    {1. / 36, 1. / 12},
    {1. / 24, 0, 1. / 8},
    {5. / 12, 0, -25. / 16, 25. / 16},
    {1. / 20, 0, 0, 1. / 4, 1. / 5},
    {-25. / 108, 0, 0, 125. / 108, -65. / 27, 125. / 54},
    {31. / 300, 0, 0, 0, 61. / 225, -2. / 9, 13. / 900},
    {2.0, 0, 0, -53. / 6, 704. / 45, -107. / 9, 67. / 90, 3.0},
    {-91. / 108, 0, 0, 23. / 108, -976. / 135, 311. / 54, -19. / 60, 17. / 6, -1. / 12},
    {2383. / 4100, 0, 0, -341. / 164, 4496. / 1025, -301. / 82, 2133. / 4100, 45. / 82, 45. / 164, 18. / 41},
    {3. / 205, 0, 0, 0, 0, -6. / 41, -3. / 205, -3. / 41, 3. / 41, 6. / 41, 0},
    {-1777. / 4100, 0, 0, -341. / 164, 4496. / 1025, -289. / 82, 2193. / 4100, 51. / 82, 33. / 164, 12. / 41, 0,
        1.0},
};
const double kB[13] = {0, 0, 0, 0, 0, 34. / 105, 9. / 35, 9. / 35, 9. / 280, 9. / 280, 0, 41. / 840, 41. / 840};
const double kBE[13] = {41. / 840, 0, 0, 0, 0, 0, 0, 0, 0, 0, 41. / 840, -41. / 840, -41. / 840};

inline void lorenzRhs(const double s[3], double sigma, double rho, double beta, double out[3])
{
    out[0] = sigma * (s[1] - s[0]);
    out[1] = s[0] * (rho - s[2]) - s[1];
    out[2] = s[0] * s[1] - beta * s[2];
}

// the weighted left-to-right sum of k[j][d] over the non-zero coefficients
inline double termSum(const double* coef, int count, double k[][3], int d)
{
    double total = 0.0;
    bool first = true;
    for (int j = 0; j < count; ++j) {
        if (coef[j] == 0.0)
            continue;
        const double term = coef[j] * k[j][d];
        total = first ? term : total + term;
        first = false;
    }
    return total;
}

// The scheme of one attempt of step h from s0: the 8th-order state, the error vector
// and the mixed max-norm ratio (the attempt below, before its controller).
void lorenzStages(const double s0[3], double step, double rho, double sigma, double beta, double rtol,
    double atol, double s8[3], double err[3], double* ratioOut)
{
    double k[13][3];
    lorenzRhs(s0, sigma, rho, beta, k[0]);
    for (int i = 0; i < 12; ++i) {
        double si[3];
        for (int d = 0; d < 3; ++d)
            si[d] = s0[d] + step * termSum(kA[i], i + 1, k, d);
        lorenzRhs(si, sigma, rho, beta, k[i + 1]);
    }
    for (int d = 0; d < 3; ++d) {
        s8[d] = s0[d] + step * termSum(kB, 13, k, d);
        err[d] = step * termSum(kBE, 13, k, d);
    }
    double ratio = 0.0;
    for (int d = 0; d < 3; ++d) {
        const double r = std::fabs(err[d]) / (atol + rtol * std::fmax(std::fabs(s8[d]), std::fabs(s0[d])));
        ratio = d == 0 ? r : std::fmax(ratio, r);
    }
    *ratioOut = ratio;
}

// One attempt; returns true when it was accepted.
bool lorenzAttempt(double s[3], double& t, double& h, double rho, double sigma, double beta, double tFinal,
    double rtol, double atol)
{
    const double s0[3] = {s[0], s[1], s[2]};
    const double t0 = t;
    const bool last = h >= tFinal - t0;
    const double step = last ? tFinal - t0 : h;
    double s8[3], err[3], ratio = 0.0;
    lorenzStages(s0, step, rho, sigma, beta, rtol, atol, s8, err, &ratio);
    const bool accept = ratio < 1.0;
    const double expo = accept ? -1.0 / 9.0 : -1.0 / 8.0;
    h = step * std::fmin(5.0, std::fmax(0.2, 0.9 * detPow(ratio, expo)));
    if (accept) {
        s[0] = s8[0];
        s[1] = s8[1];
        s[2] = s8[2];
        t = last ? tFinal : t0 + step;
    }
    return accept;
}

}  // namespace

extern "C" {

double oracle_det_pow(double r, double e) { return detPow(r, e); }

void oracle_lorenz_stages(const double s0[3], double step, double rho, double sigma, double beta, double rtol,
    double atol, double s8[3], double err[3], double* ratio)
{
    lorenzStages(s0, step, rho, sigma, beta, rtol, atol, s8, err, ratio);
}

int oracle_lorenz_run(int64_t n, const double* rho, double sigma, double beta, double t_final, double rtol,
    double atol, double* x, double* y, double* z, double* t, double* h, uint32_t* n_acc, uint32_t* n_rej,
    uint8_t* term, int64_t max_steps, int64_t* stats)
{
    if (n < 0 || max_steps < 0)
        return 2;
    int64_t finished = 0, longest = 0, total = 0;
#pragma omp parallel for schedule(dynamic, 64) reduction(+ : finished, total) reduction(max : longest)
    for (int64_t i = 0; i < n; ++i) {
        int64_t a = 0;
        if (term[i] == 0) {
            double s[3] = {x[i], y[i], z[i]};
            double tt = t[i], hh = h[i];
            uint32_t na = n_acc[i], nr = n_rej[i];
            while (a < max_steps) {
                const bool acc = lorenzAttempt(s, tt, hh, rho[i], sigma, beta, t_final, rtol, atol);
                na += acc ? 1u : 0u;
                nr += acc ? 0u : 1u;
                ++a;
                if (tt >= t_final) {
                    term[i] = 1;
                    break;
                }
            }
            x[i] = s[0];
            y[i] = s[1];
            z[i] = s[2];
            t[i] = tt;
            h[i] = hh;
            n_acc[i] = na;
            n_rej[i] = nr;
        }
        finished += term[i] != 0 ? 1 : 0;
        longest = std::max(longest, a);
        total += a;
    }
    if (stats != nullptr) {
        stats[0] = finished;
        stats[1] = longest;
        stats[2] = total;
    }
    return 0;
}

}  // extern "C"

extern "C" {

// ------------------------------------------------------- reference test corpora
//
// The inputs of eagle's canonical-reduction tests, regenerated with the same
// standard-library engines and distributions (libstdc++): the adversarial corpus
// of tests/CanonicalReduceCases.h:49-60 and the exact-sum fixture of :141-176
// (mirrored +-x pairs that cancel exactly, plus a residual on a 2^-10 grid whose
// exact sum is known).

void oracle_corpus_f64(int64_t n, uint64_t seed, double* out)
{
    std::mt19937_64 rng(seed);
    std::normal_distribution<double> nd(0.0, 1.0);
    std::uniform_int_distribution<int> ex(-8, 8);
    for (int64_t i = 0; i < n; ++i)
        out[i] = nd(rng) * std::pow(10.0, ex(rng));
}

void oracle_corpus_f32(int64_t n, uint64_t seed, float* out)
{
    std::mt19937_64 rng(seed);
    std::normal_distribution<double> nd(0.0, 1.0);
    std::uniform_int_distribution<int> ex(-8, 8);
    for (int64_t i = 0; i < n; ++i)
        out[i] = float(nd(rng) * std::pow(10.0, ex(rng)));
}

double oracle_fixture_f64(int64_t n, double kappa, double* x, double* reached)
{
    return fixtureOf<double>(n, kappa, x, reached);
}

double oracle_fixture_f32(int64_t n, double kappa, float* x, double* reached)
{
    return fixtureOf<float>(n, kappa, x, reached);
}

}  // extern "C"
