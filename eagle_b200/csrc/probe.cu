// The FP64 issue probe: how many double-precision fused multiply-adds per second
// this GPU retires when every lane runs independent chains. The register-resident
// step kernels (the oscillator's two multiply-adds per sample-step, the RKF7(8)
// attempt) are bound by this rate, not by HBM, so it is the measured denominator
// of their roofline beside the derived lane peak (64 FP64 lanes per SM per cycle).
#include "common.cuh"

#include <algorithm>

namespace eb {
namespace {

constexpr int kProbeThreads = 256;
constexpr int kProbeChains = 8;   // independent chains per thread: enough to cover the DFMA latency
constexpr int kProbeIters = 8192; // multiply-adds per chain per launch

__global__ __launch_bounds__(kProbeThreads) void fmaChainKernel(double* sink, double a, double b)
{
    double c[kProbeChains];
#pragma unroll
    for (int k = 0; k < kProbeChains; ++k)
        c[k] = double(threadIdx.x) * 1e-3 + double(k);
#pragma unroll 4
    for (int i = 0; i < kProbeIters; ++i) {
#pragma unroll
        for (int k = 0; k < kProbeChains; ++k)
            c[k] = fma(c[k], a, b);
    }
    double s = 0.0;
#pragma unroll
    for (int k = 0; k < kProbeChains; ++k)
        s += c[k];
    if (s == -1.0)  // never true for the arguments given: keeps the chains from being dropped
        sink[blockIdx.x] = s;
}

}  // namespace
}  // namespace eb

using namespace eb;

#define EB_API extern "C" __attribute__((visibility("default")))

EB_API eagle_backend_status eagle_backend_x_b200_probe_fp64(int32_t device, uint64_t stream, double* fma_per_s)
{
    return guarded([&] {
        constexpr const char* who = "eagle_backend_x_b200_probe_fp64";
        if (fma_per_s == nullptr)
            invalid(std::string(who) + ": null output");
        int dev = device;
        if (dev < 0)
            cudaCheck(cudaGetDevice(&dev), "cudaGetDevice");
        DeviceScope scope(dev);
        const cudaStream_t s = seamStream(stream);
        int occ = 0;
        cudaCheck(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fmaChainKernel, kProbeThreads, 0),
            "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
        const unsigned grid = unsigned(std::max(1, occ) * smCount());
        double* sink = nullptr;  // never written (see the kernel); a valid address all the same
        cudaCheck(cudaMallocAsync(reinterpret_cast<void**>(&sink), sizeof(double) * grid, s), "cudaMallocAsync");
        cudaEvent_t e0 = nullptr, e1 = nullptr;
        cudaCheck(cudaEventCreate(&e0), "cudaEventCreate");
        cudaCheck(cudaEventCreate(&e1), "cudaEventCreate");
        float best = 0.0f;
        for (int rep = 0; rep < 6; ++rep) {
            cudaCheck(cudaEventRecord(e0, s), "cudaEventRecord");
            fmaChainKernel<<<grid, kProbeThreads, 0, s>>>(sink, 0.999999999, 1e-9);
            launchCheck(who);
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
        const double fmas = double(grid) * kProbeThreads * kProbeChains * double(kProbeIters);
        *fma_per_s = fmas / (double(best) * 1e-3);
    });
}
