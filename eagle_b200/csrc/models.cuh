// The step bodies this backend carries in place of hawk-generated kernels.
//
// A model is a per-sample state held in registers plus a ``step`` that advances
// it one step and answers whether the sample terminated on that step (the
// ``terminated = ...`` assignment at the end of a hawk kernel body). The until-done
// semantics around it (docs/content/modules/filtering/run_until_done.rst:4-24) are
// the callers': a sample whose mask byte is set takes no step; a live sample steps
// until its step sets the mask or its budget runs out, and is counted once into
// ``finished_count`` when it is set.
#pragma once

#include "common.cuh"

namespace eb {

/** The Euler oscillator of eagle's README (README.md:89-97):
 *      x = x0 + dt * v0;  v = v0 - dt * omega * omega * x0;  t += dt;  terminated = t >= t_end
 *  in its written expression order. ``c = (dt * omega) * omega`` is the same
 *  product every step, so it is formed once per sample. With ``Fma`` the two
 *  multiply-adds are contracted (fma(dt, v0, x0), fma(-c, x0, v0)), as a device
 *  compiler contracts the hawk body by default; without it every operation
 *  rounds once as written (the reference's exact host profile). ``t`` never
 *  contracts, so the step counts are identical either way. */
template <bool Fma>
struct Oscillator {
    double x, v, t, c, te;
    static constexpr int kBlock = 8;

    static __device__ __forceinline__ double coeff(double dt, double omega)
    {
        return __dmul_rn(__dmul_rn(dt, omega), omega);
    }

    /** x and v one step on (t is advanced by the caller). */
    __device__ __forceinline__ void stepXV(double dt)
    {
        double x1, v1;
        if constexpr (Fma) {
            x1 = __fma_rn(dt, v, x);
            v1 = __fma_rn(-c, x, v);
        } else {
            x1 = __dadd_rn(x, __dmul_rn(dt, v));
            v1 = __dsub_rn(v, __dmul_rn(c, x));
        }
        x = x1;
        v = v1;
    }

    __device__ __forceinline__ void step(double dt)
    {
        stepXV(dt);
        t = __dadd_rn(t, dt);
    }

    /** x and v ``n`` (>= 0) steps on, t untouched: for a sample whose stop step is
     *  known in advance. */
    __device__ __forceinline__ void stepsXV(double dt, int n)
    {
        int k = 0;
        for (; k + kBlock <= n; k += kBlock) {
#pragma unroll
            for (int j = 0; j < kBlock; ++j)
                stepXV(dt);
        }
        for (; k < n; ++k)
            stepXV(dt);
    }

    /** Run at most ``budget`` (>= 0) steps; returns the steps run, ``fin`` true if
     *  the sample terminated on the last of them.
     *
     *  The stop test reads t only, and t advances by dt alone. With dt >= 0 the
     *  rounded sums t, t + dt, ... never decrease, so when t after a whole block of
     *  kBlock steps is still below t_end no step inside the block stopped: the
     *  block's t is formed first (the same additions, in the same order) and, if it
     *  stays below t_end, x and v take the block's steps with no per-step test.
     *  The block holding the stop, and any dt that is negative or NaN, take the
     *  steps one at a time with the test after each, as the model is written. */
    __device__ __forceinline__ int run(double dt, int budget, bool& fin)
    {
        int s = 0;
        fin = false;
        if (dt >= 0.0) {
            for (; s + kBlock <= budget; s += kBlock) {
                double tb = t;
#pragma unroll
                for (int k = 0; k < kBlock; ++k)
                    tb = __dadd_rn(tb, dt);
                if (tb >= te)
                    break;
#pragma unroll
                for (int k = 0; k < kBlock; ++k)
                    stepXV(dt);
                t = tb;
            }
        }
        for (; s < budget; ++s) {
            step(dt);
            if (t >= te) {
                fin = true;
                return s + 1;
            }
        }
        return s;
    }

    /** ``run`` for a 64-bit budget, in pieces of at most 2^30 steps. */
    __device__ __forceinline__ int64_t runLong(double dt, int64_t budget, bool& fin)
    {
        int64_t total = 0;
        fin = false;
        while (total < budget && !fin) {
            const int64_t left = budget - total;
            total += run(dt, left < (INT64_C(1) << 30) ? int(left) : (1 << 30), fin);
        }
        return total;
    }
};

}  // namespace eb

namespace eb {

/** Philox-4x32-10 (Salmon, Moraes, Dror and Shaw, SC'11): ten rounds of two
 *  32x32->64 multiplies and xors over a 4-word counter, the 2-word key bumped by
 *  the Weyl constants between rounds. */
__device__ __forceinline__ void philox4x32_10(uint32_t& c0, uint32_t& c1, uint32_t& c2, uint32_t& c3, uint32_t k0,
    uint32_t k1)
{
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        if (r > 0) {
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
        const uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
        const uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
        const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c0 = n0;
        c1 = lo1;
        c2 = n2;
        c3 = lo0;
    }
}

/** The gambler's-ruin walk: a position in (0, 100) moves +1 or -1 per step and the
 *  sample stops when it reaches 0 or 100; ``time`` counts its steps over its whole
 *  life. Step s (0-based) moves +1 when bit (s mod 128) of Philox-4x32-10 with
 *  counter (s / 128, id) and key ``seed`` is set (word s/32 mod 4, bit s mod 32). */
struct GamblerModel {
    int32_t* pos;
    int64_t* time;
    uint8_t* term;
    uint64_t seed;
    int64_t idBase;

    struct Sample {
        int32_t pos;
        int64_t time;
        uint64_t id;
    };

    __device__ __forceinline__ Sample load(int64_t i) const { return Sample{pos[i], time[i], uint64_t(idBase + i)}; }
    __device__ __forceinline__ void store(int64_t i, const Sample& s) const
    {
        pos[i] = s.pos;
        time[i] = s.time;
    }
    __device__ __forceinline__ void prepare(Sample&) const {}

    /** At most ``budget`` steps; returns the steps run, ``fin`` when it reached 0 or 100. */
    __device__ __forceinline__ int run(Sample& s, int budget, bool& fin) const
    {
        int done = 0;
        fin = false;
        int32_t p = s.pos;
        int64_t tm = s.time;
        while (done < budget) {
            const uint64_t blk = uint64_t(tm) >> 7;
            uint32_t c0 = uint32_t(blk), c1 = uint32_t(blk >> 32), c2 = uint32_t(s.id), c3 = uint32_t(s.id >> 32);
            philox4x32_10(c0, c1, c2, c3, uint32_t(seed), uint32_t(seed >> 32));
            // the block's remaining bits, one 32-bit word at a time
            int bit = int(tm & 127);
            while (bit < 128 && done < budget) {
                const int w = bit >> 5;
                uint32_t word = w == 0 ? c0 : (w == 1 ? c1 : (w == 2 ? c2 : c3));
                word >>= (bit & 31);
                int lim = 32 - (bit & 31);
                if (lim > budget - done)
                    lim = budget - done;
                for (int k = 0; k < lim; ++k) {
                    p += int32_t((word & 1u) << 1) - 1;
                    word >>= 1;
                    if (p == 0 || p == 100) {
                        fin = true;
                        done += k + 1;
                        tm += k + 1;
                        s.pos = p;
                        s.time = tm;
                        return done;
                    }
                }
                done += lim;
                tm += lim;
                bit += lim;
            }
        }
        s.pos = p;
        s.time = tm;
        return done;
    }
};

}  // namespace eb

namespace eb {

// ------------------------------------------------------------ Lorenz, RKF7(8)

/** The controller's deterministic power, the same operations in the same order as
 *  the host: ln by exponent extraction and ln m = 2 atanh((m-1)/(m+1)) on
 *  m in [sqrt(1/2), sqrt(2)) (a series in u^2 to degree 11), exp by reduction to
 *  f = y - n ln2 and the Taylor series of e^f to degree 18, scaled by 2^n. Every
 *  operation rounds once (no contraction). */
__device__ __forceinline__ double detLog(double r)
{
    constexpr double kLn2 = 0.6931471805599453;
    unsigned long long b = (unsigned long long)__double_as_longlong(r);
    int k = 0;
    if (((b >> 52) & 0x7ffull) == 0) {
        r = __dmul_rn(r, 18014398509481984.0);
        b = (unsigned long long)__double_as_longlong(r);
        k = -54;
    }
    k += int((b >> 52) & 0x7ffull) - 1023;
    b = (b & 0x800FFFFFFFFFFFFFull) | (1023ull << 52);
    double m = __longlong_as_double((long long)b);
    if (m > 1.4142135623730951) {
        m = __dmul_rn(m, 0.5);
        k += 1;
    }
    const double u = __ddiv_rn(__dadd_rn(m, -1.0), __dadd_rn(m, 1.0));
    const double u2 = __dmul_rn(u, u);
    double p = 1.0 / 23.0;
    p = __dadd_rn(__dmul_rn(p, u2), 1.0 / 21.0);
    p = __dadd_rn(__dmul_rn(p, u2), 1.0 / 19.0);
    p = __dadd_rn(__dmul_rn(p, u2), 1.0 / 17.0);
    p = __dadd_rn(__dmul_rn(p, u2), 1.0 / 15.0);
    p = __dadd_rn(__dmul_rn(p, u2), 1.0 / 13.0);
    p = __dadd_rn(__dmul_rn(p, u2), 1.0 / 11.0);
    p = __dadd_rn(__dmul_rn(p, u2), 1.0 / 9.0);
    p = __dadd_rn(__dmul_rn(p, u2), 1.0 / 7.0);
    p = __dadd_rn(__dmul_rn(p, u2), 1.0 / 5.0);
    p = __dadd_rn(__dmul_rn(p, u2), 1.0 / 3.0);
    p = __dadd_rn(__dmul_rn(p, u2), 1.0);
    const double lnm = __dmul_rn(__dmul_rn(2.0, u), p);
    return __dadd_rn(lnm, __dmul_rn(double(k), kLn2));
}

__device__ __forceinline__ double detExp(double y)
{
    constexpr double kLn2 = 0.6931471805599453;
    const double n = rint(__ddiv_rn(y, kLn2));
    const double f = __dadd_rn(y, -__dmul_rn(n, kLn2));
    double p = 1.0 / 6402373705728000.0;
    p = __dadd_rn(__dmul_rn(p, f), 1.0 / 355687428096000.0);
    p = __dadd_rn(__dmul_rn(p, f), 1.0 / 20922789888000.0);
    p = __dadd_rn(__dmul_rn(p, f), 1.0 / 1307674368000.0);
    p = __dadd_rn(__dmul_rn(p, f), 1.0 / 87178291200.0);
    p = __dadd_rn(__dmul_rn(p, f), 1.0 / 6227020800.0);
    p = __dadd_rn(__dmul_rn(p, f), 1.0 / 479001600.0);
    p = __dadd_rn(__dmul_rn(p, f), 1.0 / 39916800.0);
    p = __dadd_rn(__dmul_rn(p, f), 1.0 / 3628800.0);
    p = __dadd_rn(__dmul_rn(p, f), 1.0 / 362880.0);
    p = __dadd_rn(__dmul_rn(p, f), 1.0 / 40320.0);
    p = __dadd_rn(__dmul_rn(p, f), 1.0 / 5040.0);
    p = __dadd_rn(__dmul_rn(p, f), 1.0 / 720.0);
    p = __dadd_rn(__dmul_rn(p, f), 1.0 / 120.0);
    p = __dadd_rn(__dmul_rn(p, f), 1.0 / 24.0);
    p = __dadd_rn(__dmul_rn(p, f), 1.0 / 6.0);
    p = __dadd_rn(__dmul_rn(p, f), 1.0 / 2.0);
    p = __dadd_rn(__dmul_rn(p, f), 1.0);
    p = __dadd_rn(__dmul_rn(p, f), 1.0);
    const int e = int(n);
    if (e > 1000 || e < -1000)
        return e > 0 ? __longlong_as_double(0x7FF0000000000000ll) : 0.0;
    return __dmul_rn(p, __longlong_as_double((long long)((unsigned long long)(e + 1023) << 52)));
}

__device__ __forceinline__ double detPow(double r, double e)
{
    if (isnan(r))
        return r;
    if (r == 0.0)
        return __longlong_as_double(0x7FF0000000000000ll);
    if (isinf(r))
        return 0.0;
    return detExp(__dmul_rn(e, detLog(r)));
}

/** Fehlberg 7(8) (NASA TR R-287), as eagle's perf card lists it
 *  (benchmarks/perf_card/perf_card.py:262-278): a, b and be = b_hat - b. */
struct Rkf78 {
    static __host__ __device__ constexpr double a(int i, int j)
    {
        constexpr double t[12][12] = {
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
            {-1777. / 4100, 0, 0, -341. / 164, 4496. / 1025, -289. / 82, 2193. / 4100, 51. / 82, 33. / 164, 12. / 41,
                0, 1.0},
        };
        return t[i][j];
    }
    static __host__ __device__ constexpr double b(int j)
    {
        constexpr double t[13] = {0, 0, 0, 0, 0, 34. / 105, 9. / 35, 9. / 35, 9. / 280, 9. / 280, 0, 41. / 840,
            41. / 840};
        return t[j];
    }
    static __host__ __device__ constexpr double be(int j)
    {
        constexpr double t[13] = {41. / 840, 0, 0, 0, 0, 0, 0, 0, 0, 0, 41. / 840, -41. / 840, -41. / 840};
        return t[j];
    }
};

/** Lorenz-63 integrated by eagle's perf-card RKF7(8) attempt
 *  (benchmarks/perf_card/perf_card.py:330-348): clip the step onto t_final, 13
 *  stages (each component s0 + h * (left-to-right sum of the non-zero a_ij k_j)),
 *  the mixed max-norm error ratio, accept when ratio < 1, h scaled by
 *  min(5, max(0.2, 0.9 ratio^expo)) with expo -1/9 (accept) or -1/8 (reject).
 *  One attempt is one step of the until-done loop. */
struct LorenzModel {
    const double* rho;
    double sigma, beta, tFinal, rtol, atol;
    double* x;
    double* y;
    double* z;
    double* t;
    double* h;
    uint32_t* nacc;
    uint32_t* nrej;
    uint8_t* term;

    struct Sample {
        double s0, s1, s2, t, h, rho;
        uint32_t na, nr;
    };

    __device__ __forceinline__ Sample load(int64_t i) const
    {
        return Sample{x[i], y[i], z[i], t[i], h[i], rho[i], nacc[i], nrej[i]};
    }
    __device__ __forceinline__ void store(int64_t i, const Sample& s) const
    {
        x[i] = s.s0;
        y[i] = s.s1;
        z[i] = s.s2;
        t[i] = s.t;
        h[i] = s.h;
        nacc[i] = s.na;
        nrej[i] = s.nr;
    }
    __device__ __forceinline__ void prepare(Sample&) const {}

    __device__ __forceinline__ void rhs(double s0, double s1, double s2, double r, double* k) const
    {
        k[0] = __dmul_rn(sigma, __dadd_rn(s1, -s0));
        k[1] = __dadd_rn(__dmul_rn(s0, __dadd_rn(r, -s2)), -s1);
        k[2] = __dadd_rn(__dmul_rn(s0, s1), -__dmul_rn(beta, s2));
    }

    /** One attempt; true when accepted. */
    __device__ __forceinline__ bool attempt(Sample& s) const
    {
        const double x0[3] = {s.s0, s.s1, s.s2};
        const double t0 = s.t;
        const bool last = s.h >= __dadd_rn(tFinal, -t0);
        const double step = last ? __dadd_rn(tFinal, -t0) : s.h;
        double k[13][3];
        rhs(x0[0], x0[1], x0[2], s.rho, k[0]);
#pragma unroll
        for (int i = 0; i < 12; ++i) {
            double si[3];
#pragma unroll
            for (int d = 0; d < 3; ++d) {
                double total = 0.0;
                bool first = true;
#pragma unroll
                for (int j = 0; j <= i; ++j) {
                    if (Rkf78::a(i, j) == 0.0)
                        continue;
                    const double term = __dmul_rn(Rkf78::a(i, j), k[j][d]);
                    total = first ? term : __dadd_rn(total, term);
                    first = false;
                }
                si[d] = __dadd_rn(x0[d], __dmul_rn(step, total));
            }
            rhs(si[0], si[1], si[2], s.rho, k[i + 1]);
        }
        double s8[3], err[3];
#pragma unroll
        for (int d = 0; d < 3; ++d) {
            double tb = 0.0, te = 0.0;
            bool fb = true, fe = true;
#pragma unroll
            for (int j = 0; j < 13; ++j) {
                if (Rkf78::b(j) != 0.0) {
                    const double term = __dmul_rn(Rkf78::b(j), k[j][d]);
                    tb = fb ? term : __dadd_rn(tb, term);
                    fb = false;
                }
                if (Rkf78::be(j) != 0.0) {
                    const double term = __dmul_rn(Rkf78::be(j), k[j][d]);
                    te = fe ? term : __dadd_rn(te, term);
                    fe = false;
                }
            }
            s8[d] = __dadd_rn(x0[d], __dmul_rn(step, tb));
            err[d] = __dmul_rn(step, te);
        }
        double ratio = 0.0;
#pragma unroll
        for (int d = 0; d < 3; ++d) {
            const double den = __dadd_rn(atol, __dmul_rn(rtol, fmax(fabs(s8[d]), fabs(x0[d]))));
            const double r = __ddiv_rn(fabs(err[d]), den);
            ratio = d == 0 ? r : fmax(ratio, r);
        }
        const bool accept = ratio < 1.0;
        const double expo = accept ? -1.0 / 9.0 : -1.0 / 8.0;
        s.h = __dmul_rn(step, fmin(5.0, fmax(0.2, __dmul_rn(0.9, detPow(ratio, expo)))));
        if (accept) {
            s.s0 = s8[0];
            s.s1 = s8[1];
            s.s2 = s8[2];
            s.t = last ? tFinal : __dadd_rn(t0, step);
        }
        return accept;
    }

    /** At most ``budget`` attempts; returns the attempts run, ``fin`` once t >= t_final. */
    __device__ __forceinline__ int run(Sample& s, int budget, bool& fin) const
    {
        fin = false;
        for (int a = 0; a < budget; ++a) {
            const bool acc = attempt(s);
            s.na += acc ? 1u : 0u;
            s.nr += acc ? 0u : 1u;
            if (s.t >= tFinal) {
                fin = true;
                return a + 1;
            }
        }
        return budget;
    }
};

}  // namespace eb
