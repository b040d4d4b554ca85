// The gambler's-ruin walk's step entries in the hawk kernel ABI (see entries.cu for
// the packing). arg_spec:
//
//   ("mutable", "pos") int32, ("mutable", "time") int64, ("terminated", "terminated"),
//   ("uniform", "seed") int64, ("uniform", "id_base") int64,
//   ("lookup", "finished_count"), ("lookup", "fused_steps")
//
// then ``int64 base, count, nSamples`` and the _range / _persist tails of
// python/eagle/_plan_binding.py:455-460, :582-591. ``id_base`` offsets the sample
// ids that key the random stream, so a shard of a larger batch draws the numbers
// its samples draw in the whole.
#include "schedule.cuh"

#include <map>
#include <string>

namespace eb {

#define EB_GAMBLER_ROLES                                                                                        \
    ScalarHandle pos, ScalarHandle time, ScalarHandle terminated, int64_t seed, int64_t idBase,                \
        ScalarHandle finished, ScalarHandle fused, int64_t base, int64_t count, int64_t nSamples

__device__ __forceinline__ GamblerModel gamblerOf(const ScalarHandle& pos, const ScalarHandle& time,
    const ScalarHandle& terminated, int64_t seed, int64_t idBase)
{
    return GamblerModel{static_cast<int32_t*>(pos.data), static_cast<int64_t*>(time.data),
        static_cast<uint8_t*>(terminated.data), uint64_t(seed), idBase};
}

__global__ __launch_bounds__(256) void gamblerPlain(EB_GAMBLER_ROLES)
{
    (void)nSamples;
    rangeLoop(gamblerOf(pos, time, terminated, seed, idBase), base, count, *static_cast<const int64_t*>(fused.data),
        static_cast<uint32_t*>(finished.data), nullptr, nullptr);
}

__global__ __launch_bounds__(256) void gamblerRange(EB_GAMBLER_ROLES, uint32_t* hawkSteps,
    unsigned long long* hawkStepsum)
{
    (void)nSamples;
    rangeLoop(gamblerOf(pos, time, terminated, seed, idBase), base, count, *static_cast<const int64_t*>(fused.data),
        static_cast<uint32_t*>(finished.data), hawkSteps, hawkStepsum);
}

__global__ __launch_bounds__(256) void gamblerPersist(EB_GAMBLER_ROLES, uint32_t* hawkNext,
    unsigned long long* hawkUtil, uint32_t* hawkSteps, unsigned long long* hawkStepsum, uint32_t hawkChunk)
{
    (void)nSamples;
    const int chunk = hawkChunk == 0 ? 32 : int(hawkChunk < (1u << 20) ? hawkChunk : (1u << 20));
    persistLoop(gamblerOf(pos, time, terminated, seed, idBase), base, count, *static_cast<const int64_t*>(fused.data),
        chunk, hawkNext, hawkUtil, static_cast<uint32_t*>(finished.data), hawkSteps, hawkStepsum);
}

void addGamblerEntries(std::map<std::string, const void*>& m)
{
    m["gambler"] = reinterpret_cast<const void*>(&gamblerPlain);
    m["gambler_range"] = reinterpret_cast<const void*>(&gamblerRange);
    m["gambler_persist"] = reinterpret_cast<const void*>(&gamblerPersist);
}

}  // namespace eb
