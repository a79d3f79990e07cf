// NCCL gradient reduction for data-parallel sessions (see session_dp.h).
#include <dlfcn.h>
#include <nccl.h>
#include <stdio.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <thread>

#include "engine_internal.h"
#include "mle_engine.h"
#include "session_dp.h"

namespace mle {
namespace {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    // non-blocking initialisation (optional: older libraries lack them)
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    bool ok = false;
};

const NcclApi& nccl() {
    static NcclApi api;
    static bool tried = false;
    if (tried) return api;
    tried = true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        fprintf(stderr, "mle: libnccl.so.2 not found: data parallelism unavailable\n");
        return api;
    }
    api.GetUniqueId = (decltype(api.GetUniqueId))dlsym(h, "ncclGetUniqueId");
    api.CommInitRank = (decltype(api.CommInitRank))dlsym(h, "ncclCommInitRank");
    api.AllReduce = (decltype(api.AllReduce))dlsym(h, "ncclAllReduce");
    api.CommDestroy = (decltype(api.CommDestroy))dlsym(h, "ncclCommDestroy");
    api.GroupStart = (decltype(api.GroupStart))dlsym(h, "ncclGroupStart");
    api.GroupEnd = (decltype(api.GroupEnd))dlsym(h, "ncclGroupEnd");
    api.GetErrorString = (decltype(api.GetErrorString))dlsym(h, "ncclGetErrorString");
    api.CommInitRankConfig = (decltype(api.CommInitRankConfig))dlsym(h, "ncclCommInitRankConfig");
    api.CommGetAsyncError = (decltype(api.CommGetAsyncError))dlsym(h, "ncclCommGetAsyncError");
    api.CommAbort = (decltype(api.CommAbort))dlsym(h, "ncclCommAbort");
    api.ok = api.GetUniqueId && api.CommInitRank && api.AllReduce && api.CommDestroy && api.GroupStart &&
             api.GroupEnd;
    return api;
}

// Wall-clock limit of the communicator set-up and of each wait for a
// non-blocking NCCL call: MLE_DP_TIMEOUT_S seconds (default 300).
double dp_timeout_s() {
    const char* e = getenv("MLE_DP_TIMEOUT_S");
    const double v = e ? atof(e) : 0.0;
    return v > 0 ? v : 300.0;
}

// Polls a non-blocking communicator until its pending call finished, failed
// or the wall-clock limit passed; returns the final state (ncclInProgress
// on timeout).
ncclResult_t wait_comm(ncclComm_t c, double limit_s) {
    const NcclApi& n = nccl();
    const auto t0 = std::chrono::steady_clock::now();
    ncclResult_t st = ncclInProgress;
    while (true) {
        if (n.CommGetAsyncError(c, &st) != ncclSuccess) return ncclSystemError;
        if (st != ncclInProgress) return st;
        const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (el > limit_s) return ncclInProgress;
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

}  // namespace

int nccl_unique_id(uint8_t* out128) {
    const NcclApi& n = nccl();
    if (!n.ok) return MLE_ERR_UNSUPPORTED;
    ncclUniqueId id;
    if (n.GetUniqueId(&id) != ncclSuccess) return MLE_ERR_CUDA;
    static_assert(sizeof(id) == 128, "ncclUniqueId is 128 bytes");
    std::memcpy(out128, &id, 128);
    return MLE_OK;
}

int auto_bucket_mb(int64_t total_floats) {
    const double mib = (double)std::max<int64_t>(total_floats, 0) * 4.0 / (1 << 20);
    int mb = 1;
    while (mb < 32 && mb * 4.0 < mib) mb *= 2;
    return mb;
}

std::vector<GradBucket> plan_buckets(std::vector<GradSpan> g, int bucket_mb) {
    std::vector<GradBucket> out;
    if (bucket_mb <= 0) {
        int64_t total = 0;
        for (auto& e : g) total += std::max<int64_t>(e.count, 0);
        bucket_mb = auto_bucket_mb(total);
    }
    std::sort(g.begin(), g.end(), [](const GradSpan& a, const GradSpan& b) { return a.base < b.base; });
    const int64_t cap = (int64_t)bucket_mb * (1ll << 20) / 4;
    float* cur = nullptr;
    const void* cur_chunk = nullptr;
    int64_t len = 0;
    for (auto& e : g) {
        if (e.count <= 0) continue;
        if (cur && e.chunk == cur_chunk && e.base <= cur + len + 64 && (e.base + e.count) - cur <= cap) {
            len = std::max<int64_t>(len, (e.base + e.count) - cur);
        } else {
            if (cur) out.push_back({cur, len});
            cur = e.base;
            cur_chunk = e.chunk;
            len = e.count;
        }
    }
    if (cur) out.push_back({cur, len});
    return out;
}

DataParallel::~DataParallel() {
    if (comm_stream_) cudaStreamSynchronize(comm_stream_);
    if (comm_ && nccl().ok) {
        if (error_ != MLE_OK && nccl().CommAbort) nccl().CommAbort((ncclComm_t)comm_);
        else nccl().CommDestroy((ncclComm_t)comm_);
    }
    for (cudaEvent_t e : ready_) cudaEventDestroy(e);
    for (cudaEvent_t e : ready_param_) cudaEventDestroy(e);
    for (cudaEvent_t e : dense_ready_) cudaEventDestroy(e);
    if (done_) cudaEventDestroy(done_);
    if (comm_stream_) cudaStreamDestroy(comm_stream_);
}

int DataParallel::init(const uint8_t* id128, int rank, int world, const std::vector<GradSpan>& grads, int bucket_mb,
                       cudaStream_t compute) {
    (void)compute;
    const NcclApi& n = nccl();
    if (!n.ok) return MLE_ERR_UNSUPPORTED;
    rank_ = rank;
    world_ = world;
    ncclUniqueId id;
    std::memcpy(&id, id128, 128);
    ncclComm_t c = nullptr;
    nonblocking_ = n.CommInitRankConfig && n.CommGetAsyncError && n.CommAbort;
    if (nonblocking_) {
        // Non-blocking set-up: a rank that never joins makes the others give
        // up after the wall-clock limit (MLE_ERR_TIMEOUT) instead of waiting
        // inside NCCL for good.
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        cfg.blocking = 0;
        ncclResult_t r = n.CommInitRankConfig(&c, world, id, rank, &cfg);
        if (r == ncclInProgress || r == ncclSuccess) r = wait_comm(c, dp_timeout_s());
        if (r != ncclSuccess) {
            fprintf(stderr, "mle: ncclCommInitRankConfig %s: %s\n", r == ncclInProgress ? "timed out" : "failed",
                    r == ncclInProgress ? "a rank did not join" : (n.GetErrorString ? n.GetErrorString(r) : "?"));
            if (c) n.CommAbort(c);
            return r == ncclInProgress ? MLE_ERR_TIMEOUT : MLE_ERR_CUDA;
        }
    } else {
        const ncclResult_t r = n.CommInitRank(&c, world, id, rank);
        if (r != ncclSuccess) {
            fprintf(stderr, "mle: ncclCommInitRank failed: %s\n", n.GetErrorString ? n.GetErrorString(r) : "?");
            return MLE_ERR_CUDA;
        }
    }
    comm_ = c;
    if (cudaStreamCreateWithFlags(&comm_stream_, cudaStreamNonBlocking) != cudaSuccess) return MLE_ERR_CUDA;
    if (cudaEventCreateWithFlags(&done_, cudaEventDisableTiming) != cudaSuccess) return MLE_ERR_CUDA;
    if (bucket_mb <= 0) {
        int64_t total = 0;
        for (auto& gr : grads) total += std::max<int64_t>(gr.count, 0);
        bucket_mb = auto_bucket_mb(total);
    }
    bucket_mb_ = bucket_mb;
    buckets_ = plan_buckets(grads, bucket_mb);
    members_.assign(buckets_.size(), 0);
    ready_.assign(buckets_.size(), nullptr);
    ready_param_.assign(buckets_.size(), nullptr);
    for (auto& e : ready_)
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return MLE_ERR_CUDA;
    for (auto& e : ready_param_)
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return MLE_ERR_CUDA;
    for (auto& gr : grads) {
        if (gr.count <= 0) continue;
        for (int b = 0; b < (int)buckets_.size(); ++b) {
            if (gr.base >= buckets_[b].base && gr.base < buckets_[b].base + buckets_[b].count) {
                bucket_of_.push_back({gr.base, b});
                ++members_[b];
                break;
            }
        }
    }
    std::sort(bucket_of_.begin(), bucket_of_.end());
    begin_backward();
    return MLE_OK;
}

void DataParallel::begin_backward() {
    pending_ = members_;
    issued_.assign(buckets_.size(), 0);
    error_ = MLE_OK;
}

void DataParallel::issue(int b, cudaStream_t compute) {
    issued_[b] = 1;
    if (error_ != MLE_OK) return;  // the step already failed: issue nothing more
    check_cuda(cudaEventRecord(ready_[b], compute), "dp bucket ready");
    check_cuda(cudaStreamWaitEvent(comm_stream_, ready_[b], 0), "dp bucket wait");
    if (param_stream_pending()) {
        // parameter gradients produced on the parameter-gradient stream
        check_cuda(cudaEventRecord(ready_param_[b], param_stream()), "dp bucket ready");
        check_cuda(cudaStreamWaitEvent(comm_stream_, ready_param_[b], 0), "dp bucket wait");
    }
    ncclResult_t r = nccl().AllReduce(buckets_[b].base, buckets_[b].base, (size_t)buckets_[b].count, ncclFloat32,
                                      ncclSum, (ncclComm_t)comm_, comm_stream_);
    // a non-blocking communicator may still be enqueuing the call: wait for
    // that (host side only; the reduction itself runs on comm_stream_)
    if (nonblocking_ && r == ncclInProgress) r = wait_comm((ncclComm_t)comm_, dp_timeout_s());
    if (r != ncclSuccess) {
        fprintf(stderr, "mle: ncclAllReduce failed: %s\n", nccl().GetErrorString ? nccl().GetErrorString(r) : "?");
        error_ = MLE_ERR_CUDA;
    }
}

void DataParallel::grads_done(const std::vector<float*>& grads, cudaStream_t compute) {
    for (float* g : grads) {
        auto it = std::lower_bound(bucket_of_.begin(), bucket_of_.end(), std::make_pair(g, -1));
        if (it == bucket_of_.end() || it->first != g) continue;
        const int b = it->second;
        if (--pending_[b] == 0 && !issued_[b]) issue(b, compute);
    }
}

int DataParallel::add_dense(float* p, int64_t n) {
    cudaEvent_t e = nullptr;
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return MLE_ERR_CUDA;
    dense_.push_back({p, n});
    dense_ready_.push_back(e);
    return MLE_OK;
}

int DataParallel::reduce_remaining(cudaStream_t compute) {
    for (int b = 0; b < (int)buckets_.size(); ++b)
        if (!issued_[b]) issue(b, compute);
    for (size_t i = 0; i < dense_.size() && error_ == MLE_OK; ++i) {
        check_cuda(cudaEventRecord(dense_ready_[i], compute), "dp dense ready");
        check_cuda(cudaStreamWaitEvent(comm_stream_, dense_ready_[i], 0), "dp dense wait");
        ncclResult_t r = nccl().AllReduce(dense_[i].base, dense_[i].base, (size_t)dense_[i].count, ncclFloat32,
                                          ncclSum, (ncclComm_t)comm_, comm_stream_);
        if (nonblocking_ && r == ncclInProgress) r = wait_comm((ncclComm_t)comm_, dp_timeout_s());
        if (r != ncclSuccess) {
            fprintf(stderr, "mle: ncclAllReduce failed: %s\n", nccl().GetErrorString ? nccl().GetErrorString(r) : "?");
            error_ = MLE_ERR_CUDA;
        }
    }
    check_cuda(cudaEventRecord(done_, comm_stream_), "dp done");
    check_cuda(cudaStreamWaitEvent(compute, done_, 0), "dp join");
    return error_;
}

}  // namespace mle

extern "C" int mle_dp_plan_buckets(const uint64_t* addrs, const int64_t* counts, const uint64_t* chunks, int n,
                                   int bucket_mb, uint64_t* out_base, int64_t* out_count, int max_out, int* out_n) {
    if (n < 0 || (n > 0 && (!addrs || !counts)) || !out_n || max_out < 0 || (max_out > 0 && (!out_base || !out_count)))
        return MLE_ERR_ARG;
    std::vector<mle::GradSpan> g;
    for (int i = 0; i < n; ++i)
        g.push_back({reinterpret_cast<float*>(addrs[i]), counts[i],
                     chunks ? reinterpret_cast<const void*>(chunks[i]) : nullptr});
    const std::vector<mle::GradBucket> b = mle::plan_buckets(g, bucket_mb);
    *out_n = (int)b.size();
    if ((int)b.size() > max_out) return MLE_ERR_ARG;
    for (size_t i = 0; i < b.size(); ++i) {
        out_base[i] = reinterpret_cast<uint64_t>(b[i].base);
        out_count[i] = b[i].count;
    }
    return MLE_OK;
}

extern "C" int mle_dp_auto_bucket_mb(int64_t total_floats) { return mle::auto_bucket_mb(total_floats); }

extern "C" int mle_dp_unique_id(uint8_t* out128) {
    if (!out128) return MLE_ERR_ARG;
    return mle::nccl_unique_id(out128);
}
