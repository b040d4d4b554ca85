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
