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

    __device__ __forceinline__ bool step(double dt)
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
        t = __dadd_rn(t, dt);
        return t >= te;
    }

    /** Run at most ``budget`` steps; ``taken`` = steps run; true if the sample
     *  terminated on its last step. */
    __device__ __forceinline__ bool run(double dt, int64_t budget, int64_t& taken)
    {
        int64_t s = 0;
        bool fin = false;
#pragma unroll 4
        for (; s < budget;) {
            ++s;
            if (step(dt)) {
                fin = true;
                break;
            }
        }
        taken = s;
        return fin;
    }
};

}  // namespace eb
