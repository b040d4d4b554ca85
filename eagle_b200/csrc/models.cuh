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

    static constexpr int kBlock = 8;

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
