// Lorenz-63 under adaptive RKF7(8): step entries in the hawk kernel ABI (see
// entries.cu for the packing). arg_spec:
//
//   ("per_sample", "rho"), ("uniform", "sigma"), ("uniform", "beta"),
//   ("uniform", "t_final"), ("uniform", "rtol"), ("uniform", "atol"),
//   ("terminated", "terminated"), ("mutable", "x"), ("mutable", "y"), ("mutable", "z"),
//   ("mutable", "t"), ("mutable", "h"), ("mutable", "n_acc") uint32,
//   ("mutable", "n_rej") uint32, ("lookup", "finished_count"), ("lookup", "fused_steps")
//
// then ``int64 base, count, nSamples`` and the _range / _persist tails. One step of
// the until-done loop is one attempt (accepted or rejected).
#include "schedule.cuh"

#include <map>
#include <string>

namespace eb {

#define EB_LORENZ_ROLES                                                                                        \
    ScalarHandle rho, double sigma, double beta, double tFinal, double rtol, double atol, ScalarHandle terminated, \
        ScalarHandle x, ScalarHandle y, ScalarHandle z, ScalarHandle t, ScalarHandle h, ScalarHandle nacc,         \
        ScalarHandle nrej, ScalarHandle finished, ScalarHandle fused, int64_t base, int64_t count, int64_t nSamples

#define EB_LORENZ_MODEL                                                                                        \
    LorenzModel{static_cast<const double*>(rho.data), sigma, beta, tFinal, rtol, atol,                        \
        static_cast<double*>(x.data), static_cast<double*>(y.data), static_cast<double*>(z.data),             \
        static_cast<double*>(t.data), static_cast<double*>(h.data), static_cast<uint32_t*>(nacc.data),       \
        static_cast<uint32_t*>(nrej.data), static_cast<uint8_t*>(terminated.data)}

__global__ __launch_bounds__(128) void lorenzPlain(EB_LORENZ_ROLES)
{
    (void)nSamples;
    rangeLoop(EB_LORENZ_MODEL, base, count, *static_cast<const int64_t*>(fused.data),
        static_cast<uint32_t*>(finished.data), nullptr, nullptr);
}

__global__ __launch_bounds__(128) void lorenzRange(EB_LORENZ_ROLES, uint32_t* hawkSteps,
    unsigned long long* hawkStepsum)
{
    (void)nSamples;
    rangeLoop(EB_LORENZ_MODEL, base, count, *static_cast<const int64_t*>(fused.data),
        static_cast<uint32_t*>(finished.data), hawkSteps, hawkStepsum);
}

__global__ __launch_bounds__(128) void lorenzPersist(EB_LORENZ_ROLES, uint32_t* hawkNext,
    unsigned long long* hawkUtil, uint32_t* hawkSteps, unsigned long long* hawkStepsum, uint32_t hawkChunk)
{
    (void)nSamples;
    const int chunk = hawkChunk == 0 ? 32 : int(hawkChunk < (1u << 20) ? hawkChunk : (1u << 20));
    persistLoop(EB_LORENZ_MODEL, base, count, *static_cast<const int64_t*>(fused.data), chunk, hawkNext, hawkUtil,
        static_cast<uint32_t*>(finished.data), hawkSteps, hawkStepsum);
}

void addLorenzEntries(std::map<std::string, const void*>& m)
{
    m["lorenz"] = reinterpret_cast<const void*>(&lorenzPlain);
    m["lorenz_range"] = reinterpret_cast<const void*>(&lorenzRange);
    m["lorenz_persist"] = reinterpret_cast<const void*>(&lorenzPersist);
}

}  // namespace eb
