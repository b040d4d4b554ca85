// The FP64 issue probe: how many double-precision fused multiply-adds per second
// this GPU retires for a given instruction pattern and occupancy. The
// register-resident step kernels (the oscillator's two multiply-adds per
// sample-step, the RKF7(8) attempt) are bound by this rate, not by HBM, so it is
// the measured denominator of their roofline beside the derived lane peak (64 FP64
// lanes per SM per cycle).
//
// Patterns (``kind``):
//   0..3  1, 2, 4 or 8 independent chains per lane, c = fma(c, a, b) with a and b
//         kernel arguments (two of the three operands the same for every lane);
//   4..6  the oscillator's own step on 1, 2 or 3 samples per lane: x' = fma(dt, v, x),
//         v' = fma(-c, x, v), both results needed by the next step (two coupled
//         chains per sample, every operand but dt varying per lane).
#include "common.cuh"

#include <algorithm>

namespace eb {
namespace {

constexpr int kProbeThreads = 256;
constexpr int kProbeFmas = 1 << 16;  // multiply-adds per lane per launch, every pattern

template <int Chains>
__global__ __launch_bounds__(kProbeThreads) void fmaChainKernel(double* sink, double a, double b)
{
    double c[Chains];
#pragma unroll
    for (int k = 0; k < Chains; ++k)
        c[k] = double(threadIdx.x) * 1e-3 + double(k);
#pragma unroll 4
    for (int i = 0; i < kProbeFmas / Chains; ++i) {
#pragma unroll
        for (int k = 0; k < Chains; ++k)
            c[k] = fma(c[k], a, b);
    }
    double s = 0.0;
#pragma unroll
    for (int k = 0; k < Chains; ++k)
        s += c[k];
    if (s == -1.0)  // never true for the arguments given: keeps the chains from being dropped
        sink[blockIdx.x] = s;
}

template <int Samples>
__global__ __launch_bounds__(kProbeThreads) void fmaStepKernel(double* sink, double dt, double c0, int steps)
{
    double x[Samples], v[Samples], c[Samples];
#pragma unroll
    for (int p = 0; p < Samples; ++p) {
        x[p] = 1.0 + double(threadIdx.x) * 1e-6 + double(p);
        v[p] = 0.0;
        c[p] = c0 * (1.0 + double((threadIdx.x + p) & 7) * 1e-3);
    }
#pragma unroll 8
    for (int i = 0; i < steps; ++i) {
#pragma unroll
        for (int p = 0; p < Samples; ++p) {
            const double x1 = fma(dt, v[p], x[p]);
            const double v1 = fma(-c[p], x[p], v[p]);
            x[p] = x1;
            v[p] = v1;
        }
    }
    double s = 0.0;
#pragma unroll
    for (int p = 0; p < Samples; ++p)
        s += x[p] + v[p];
    if (s == -12345.0)
        sink[blockIdx.x] = s;
}

struct Pattern {
    const void* kernel;
    int fmasPerIter;  // per lane
    int iters;        // loop trips (the step kernels' ``steps``)
};

Pattern patternOf(uint32_t kind)
{
    switch (kind) {
    case 0: return {reinterpret_cast<const void*>(&fmaChainKernel<1>), 1, kProbeFmas};
    case 1: return {reinterpret_cast<const void*>(&fmaChainKernel<2>), 2, kProbeFmas / 2};
    case 2: return {reinterpret_cast<const void*>(&fmaChainKernel<4>), 4, kProbeFmas / 4};
    case 3: return {reinterpret_cast<const void*>(&fmaChainKernel<8>), 8, kProbeFmas / 8};
    case 4: return {reinterpret_cast<const void*>(&fmaStepKernel<1>), 2, kProbeFmas / 2};
    case 5: return {reinterpret_cast<const void*>(&fmaStepKernel<2>), 4, kProbeFmas / 4};
    default: return {reinterpret_cast<const void*>(&fmaStepKernel<3>), 6, kProbeFmas / 6};
    }
}

}  // namespace
}  // namespace eb

using namespace eb;

#define EB_API extern "C" __attribute__((visibility("default")))

EB_API eagle_backend_status eagle_backend_x_b200_probe_fp64(int32_t device, uint32_t kind, uint32_t ctas_per_sm,
    uint64_t stream, double* fma_per_s)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_b200_probe_fp64";
        if (fma_per_s == nullptr)
            invalid(std::string(who) + ": null output");
        if (kind > 6)
            invalid(std::string(who) + ": kind must lie in [0, 6]");
        int dev = device;
        if (dev < 0)
            cudaCheck(cudaGetDevice(&dev), "cudaGetDevice");
        DeviceScope scope(dev);
        const cudaStream_t s = seamStream(stream);
        const Pattern pat = patternOf(kind);
        int occ = 0;
        cudaCheck(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, pat.kernel, kProbeThreads, 0),
            "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
        occ = std::max(1, occ);
        const int perSm = ctas_per_sm == 0 ? occ : std::min(occ, int(ctas_per_sm));
        const unsigned grid = unsigned(perSm * smCount());
        double* sink = nullptr;  // never written (see the kernels); a valid address all the same
        cudaCheck(cudaMallocAsync(reinterpret_cast<void**>(&sink), sizeof(double) * grid, s), "cudaMallocAsync");
        cudaEvent_t e0 = nullptr, e1 = nullptr;
        cudaCheck(cudaEventCreate(&e0), "cudaEventCreate");
        cudaCheck(cudaEventCreate(&e1), "cudaEventCreate");
        double a = 0.999999999, b = 1e-9, dt = 1e-3, c0 = 4e-6;
        int steps = pat.iters;
        void* chainArgs[] = {&sink, &a, &b};
        void* stepArgs[] = {&sink, &dt, &c0, &steps};
        float best = 0.0f;
        for (int rep = 0; rep < 6; ++rep) {
            cudaCheck(cudaEventRecord(e0, s), "cudaEventRecord");
            cudaCheck(cudaLaunchKernel(pat.kernel, dim3(grid), dim3(kProbeThreads), kind < 4 ? chainArgs : stepArgs, 0,
                          s),
                "cudaLaunchKernel");
            cudaCheck(cudaEventRecord(e1, s), "cudaEventRecord");
            cudaCheck(cudaEventSynchronize(e1), "cudaEventSynchronize");
            float ms = 0.0f;
            cudaCheck(cudaEventElapsedTime(&ms, e0, e1), "cudaEventElapsedTime");
            if (rep > 0 && (best == 0.0f || ms < best))  // the first launch is a warm-up
                best = ms;
        }
        (void)cudaEventDestroy(e0);
        (void)cudaEventDestroy(e1);
        cudaCheck(cudaFreeAsync(sink, s), "cudaFreeAsync");
        const double fmas = double(grid) * kProbeThreads * double(pat.fmasPerIter) * double(pat.iters);
        *fma_per_s = fmas / (double(best) * 1e-3);
    });
}
