// Test infrastructure: cuRAND's Philox-4x32-10 block function on the device, so that
// the oracle's restatement of Philox (oracle.cpp, philox4x32_10: the generator the
// gambler's-ruin walk draws its steps from) can be checked against NVIDIA's own on the
// same counters and keys. Only tests call it; nothing in eagle_b200 links it.
//
// curand_Philox4x32_10(counter, key) is the ten-round block function of cuRAND's
// device API (curand_philox4x32_x.h), called here as a library function.
#include <cstdint>

#include <cuda_runtime.h>
#include <curand_kernel.h>

namespace {

__global__ void philoxKernel(const uint4* __restrict__ counters, const uint2* __restrict__ keys,
    uint4* __restrict__ out, int n)
{
    const int i = int(blockIdx.x) * int(blockDim.x) + int(threadIdx.x);
    if (i < n)
        out[i] = curand_Philox4x32_10(counters[i], keys[i]);
}

}  // namespace

/** out[4 i .. 4 i + 3] = Philox-4x32-10 of counter words counters[4 i .. 4 i + 3]
 *  under key words keys[2 i], keys[2 i + 1], for i < n (host arrays; the device
 *  copies are made and freed here). Returns the first CUDA error, 0 on success. */
extern "C" int curand_philox_ref(const uint32_t* counters, const uint32_t* keys, uint32_t* out, int n)
{
    if (n <= 0)
        return 0;
    uint4* dc = nullptr;
    uint2* dk = nullptr;
    uint4* dout = nullptr;
    cudaError_t e = cudaMalloc(&dc, sizeof(uint4) * size_t(n));
    if (e == cudaSuccess)
        e = cudaMalloc(&dk, sizeof(uint2) * size_t(n));
    if (e == cudaSuccess)
        e = cudaMalloc(&dout, sizeof(uint4) * size_t(n));
    if (e == cudaSuccess)
        e = cudaMemcpy(dc, counters, sizeof(uint4) * size_t(n), cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(dk, keys, sizeof(uint2) * size_t(n), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        philoxKernel<<<(n + 255) / 256, 256>>>(dc, dk, dout, n);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess)
        e = cudaMemcpy(out, dout, sizeof(uint4) * size_t(n), cudaMemcpyDeviceToHost);
    cudaFree(dc);
    cudaFree(dk);
    cudaFree(dout);
    return int(e);
}
