// Test infrastructure (oracle), not product code.
// Evaluates the reference's counter-based noise (cuda/ntc_noise.h, #included from the read-only
// reference tree by oracle/Makefile) on the GPU, compiled by the same nvcc and flags as the
// backend (no fast-math), so tests can check that the backend's device noise is bit-identical.
#include "ntc_noise.h"
#include <cuda_runtime.h>
#include <stdint.h>

__global__ void ref_noise_kernel(uint64_t seed, uint32_t stream, uint32_t step, uint32_t pair, uint64_t index0,
                                 size_t n, float* gauss, uint32_t* u32) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    gauss[i] = ntc_gauss(seed, stream, step, pair, index0 + i);
    u32[i] = ntc_noise_u32(seed, stream, step, pair, index0 + i);
}

// Host buffers in and out; returns the cudaError_t of the run (0 = success).
extern "C" int ref_device_noise(uint64_t seed, uint32_t stream, uint32_t step, uint32_t pair, uint64_t index0,
                                size_t n, float* gauss_host, uint32_t* u32_host) {
    float* g = nullptr; uint32_t* u = nullptr;
    cudaError_t e = cudaMalloc(&g, n * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&u, n * sizeof(uint32_t));
    if (e == cudaSuccess && n) {
        ref_noise_kernel<<<(unsigned)((n + 255) / 256), 256>>>(seed, stream, step, pair, index0, n, g, u);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(gauss_host, g, n * sizeof(float), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(u32_host, u, n * sizeof(uint32_t), cudaMemcpyDeviceToHost);
    cudaFree(g); cudaFree(u);
    return (int)e;
}
