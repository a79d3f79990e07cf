// kernels.h -- the part of ML_Engine's Includes/kernels.h that programs
// built on the engine use directly: the launch-shape constants and the
// fill / zero templates (Includes/kernels.h:7-30).  Every other kernel of the
// reference is replaced by the C ABI in mle_kernels.h, which the engine's
// op builders call.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>

using str = std::string;

static constexpr int BLOCK_SIZE = 32;
static constexpr int THREADSPERBLOCK = 512;
static constexpr float PIBY2 = 1.57079632679f;
static constexpr float PI = 3.14159265359f;

// data[i] = value for i < n, one element per thread.
template <typename T>
__global__ void fillKernel(T* data, T value, unsigned long long n) {
    const unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x;
    if (i < n) data[i] = value;
}

// Clears `total` elements of a device array on the legacy stream.
template <typename T>
void Zerograd(const str name, T* ptr, const unsigned long long total) {
    (void)name;
    if (!total) return;
    const int tpb = THREADSPERBLOCK;
    fillKernel<<<(unsigned int)((total + tpb - 1) / tpb), tpb>>>(ptr, (T)0.0f, total);
}
