// Data parallelism for sessions: gradient buckets summed with NCCL over
// NVLink.  NCCL is resolved at run time (dlopen of libnccl.so.2, reusing the
// copy already mapped into the process when there is one), so the runtime
// library loads on machines without NCCL.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>
#include <vector>

namespace mle {

class DataParallel {
   public:
    DataParallel() = default;
    ~DataParallel();
    // grads: (pointer, element count) of every parameter gradient, in the
    // order the backward pass finishes them last.
    int init(const uint8_t* id128, int rank, int world, const std::vector<std::pair<float*, int64_t>>& grads,
             int bucket_mb, cudaStream_t compute);
    // Sums every bucket over the ranks (on the comm stream, ordered after the
    // work already queued on `compute`) and makes `compute` wait for it.
    void reduce_remaining(cudaStream_t compute);
    int world() const { return world_; }

   private:
    struct Bucket {
        float* base;
        int64_t count;
    };
    std::vector<Bucket> buckets_;
    void* comm_ = nullptr;
    cudaStream_t comm_stream_ = nullptr;
    cudaEvent_t ready_ = nullptr, done_ = nullptr;
    int rank_ = 0, world_ = 1;
};

int nccl_unique_id(uint8_t* out128);

}  // namespace mle
