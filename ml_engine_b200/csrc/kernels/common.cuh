// Shared helpers for the sm_100a kernels behind include/mle_kernels.h.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <unordered_set>
#include <utility>

#include "mle_kernels.h"

namespace mle {

inline cudaStream_t as_stream(mle_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Records the CUDA error of the most recent failing entry point (read back
// through mle_last_cuda_error).
void record_cuda_error(cudaError_t e);

// Returns MLE_OK if the last launch was accepted, else records and returns
// MLE_ERR_CUDA.
inline int launch_status() {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        record_cuda_error(e);
        return MLE_ERR_CUDA;
    }
    return MLE_OK;
}

constexpr int kSMs = 148;  // B200: 2 dies x 74 SMs

// Grid size for a grid-stride elementwise kernel of `n` work items with
// `per_block` items per block and pass, capped at a whole number of waves.
// Every kernel of the library is launched through launch_k:
//  * programmatic dependent launch -- the kernel may be scheduled while the
//    previous kernel on the stream finishes; every kernel therefore starts
//    with pdl_entry(), which waits for that kernel's writes before any
//    global memory is touched and lets the next kernel be scheduled;
//  * the maximum shared-memory carveout for every kernel, so the SMs keep
//    one L1/shared split across a step instead of switching between the
//    tensor-core GEMM (which needs it) and the streaming kernels.
__device__ __forceinline__ void pdl_entry() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

inline void prefer_max_shared(const void* fn) {
    static std::mutex mu;
    static std::unordered_set<const void*> done;
    std::lock_guard<std::mutex> lock(mu);
    if (done.insert(fn).second)
        cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args&&... args) {
    prefer_max_shared(reinterpret_cast<const void*>(kern));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// launch_k for kernels built of thread-block clusters of `cluster` CTAs
// along x (gridDim.x a multiple of it).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kc(void (*kern)(KArgs...), dim3 grid, dim3 block, int cluster, cudaStream_t st,
                             Args&&... args) {
    prefer_max_shared(reinterpret_cast<const void*>(kern));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

inline unsigned grid_for(int64_t n, int per_block, int max_waves = 16) {
    int64_t blocks = (n + per_block - 1) / per_block;
    int64_t cap = (int64_t)kSMs * max_waves;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (unsigned)blocks;
}

__host__ __device__ inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum for blockDim.x a multiple of 32 (<= 1024).  `scratch`
// holds 32 values.  Every thread receives the total.
template <typename T>
__device__ __forceinline__ T block_sum(T v, T* scratch) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) scratch[wid] = v;
    __syncthreads();
    T t = (lane < nw) ? scratch[lane] : T(0);
    t = warp_sum(t);
    return t;
}

}  // namespace mle
