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

struct GradBucket {
    float* base;
    int64_t count;  // floats, from base
};

// One parameter gradient: its device address, float count and the
// allocation (arena chunk) that holds it.
struct GradSpan {
    float* base;
    int64_t count;
    const void* chunk;
};

// Buckets over the parameter gradients: spans are sorted by address and
// merged while they are contiguous (a gap of at most 64 floats -- one
// 256-byte arena pad, which belongs to no tensor -- is bridged), lie in the
// same allocation (one NCCL buffer may not span two cudaMalloc ranges that
// happen to be adjacent) and the bucket stays within bucket_mb MiB; a tensor
// larger than that forms a bucket of its own.  bucket_mb <= 0 picks the size
// from the gradient total (auto_bucket_mb).
std::vector<GradBucket> plan_buckets(std::vector<GradSpan> grads, int bucket_mb);

// Bucket size for `total_floats` of gradients: the smallest power of two of
// MiB that splits them into at most four buckets, between 1 and 32 MiB, so
// that a model whose gradients fit one 32 MiB bucket still reduces its first
// buckets while the backward runs.
int auto_bucket_mb(int64_t total_floats);

class DataParallel {
   public:
    DataParallel() = default;
    ~DataParallel();
    int init(const uint8_t* id128, int rank, int world, const std::vector<GradSpan>& grads, int bucket_mb,
             cudaStream_t compute);
    // Backward of one step starts: every bucket waits for all its tensors.
    void begin_backward();
    // `grads` are complete once the work queued on `compute` (and on the
    // parameter-gradient stream, when forked) so far has run: each bucket
    // whose last tensor this was is summed over the ranks on the comm
    // stream, overlapping the rest of the backward.
    void grads_done(const std::vector<float*>& grads, cudaStream_t compute);
    // Sums the buckets not started yet and makes `compute` wait for every
    // reduction (before clip and update).  Returns MLE_OK, or the status of
    // the first all-reduce NCCL refused during this step (later buckets of
    // that step are then not issued).
    int reduce_remaining(cudaStream_t compute);
    // A dense buffer summed over the ranks after the gradient buckets, in
    // every step (the data-parallel embedding-table update).
    int add_dense(float* p, int64_t n);
    int world() const { return world_; }
    int bucket_mb() const { return bucket_mb_; }
    int rank() const { return rank_; }
    int bucket_count() const { return (int)buckets_.size(); }

   private:
    void issue(int b, cudaStream_t compute);
    std::vector<GradBucket> buckets_;
    std::vector<int> members_, pending_;
    std::vector<char> issued_;
    std::vector<cudaEvent_t> ready_, ready_param_;
    std::vector<std::pair<float*, int>> bucket_of_;  // grad pointer -> bucket, sorted
    std::vector<GradBucket> dense_;
    std::vector<cudaEvent_t> dense_ready_;
    void* comm_ = nullptr;
    cudaStream_t comm_stream_ = nullptr;
    cudaEvent_t done_ = nullptr;
    int rank_ = 0, world_ = 1, bucket_mb_ = 0;
    int error_ = 0;
    bool nonblocking_ = false;  // communicator made with blocking = 0
};

int nccl_unique_id(uint8_t* out128);

}  // namespace mle
