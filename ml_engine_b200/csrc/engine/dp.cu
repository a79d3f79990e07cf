// NCCL gradient reduction for data-parallel sessions (see session_dp.h).
#include <dlfcn.h>
#include <nccl.h>
#include <stdio.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>

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
    api.ok = api.GetUniqueId && api.CommInitRank && api.AllReduce && api.CommDestroy && api.GroupStart &&
             api.GroupEnd;
    return api;
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

std::vector<GradBucket> plan_buckets(std::vector<std::pair<float*, int64_t>> g, int bucket_mb) {
    std::vector<GradBucket> out;
    std::sort(g.begin(), g.end());
    const int64_t cap = std::max<int64_t>(1, (int64_t)bucket_mb) * (1ll << 20) / 4;
    float* cur = nullptr;
    int64_t len = 0;
    for (auto& e : g) {
        if (e.second <= 0) continue;
        if (cur && e.first <= cur + len + 64 && (e.first + e.second) - cur <= cap) {
            len = std::max<int64_t>(len, (e.first + e.second) - cur);
        } else {
            if (cur) out.push_back({cur, len});
            cur = e.first;
            len = e.second;
        }
    }
    if (cur) out.push_back({cur, len});
    return out;
}

DataParallel::~DataParallel() {
    if (comm_stream_) cudaStreamSynchronize(comm_stream_);
    if (comm_ && nccl().ok) nccl().CommDestroy((ncclComm_t)comm_);
    for (cudaEvent_t e : ready_) cudaEventDestroy(e);
    for (cudaEvent_t e : ready_param_) cudaEventDestroy(e);
    if (done_) cudaEventDestroy(done_);
    if (comm_stream_) cudaStreamDestroy(comm_stream_);
}

int DataParallel::init(const uint8_t* id128, int rank, int world, const std::vector<std::pair<float*, int64_t>>& grads,
                       int bucket_mb, cudaStream_t compute) {
    (void)compute;
    const NcclApi& n = nccl();
    if (!n.ok) return MLE_ERR_UNSUPPORTED;
    rank_ = rank;
    world_ = world;
    ncclUniqueId id;
    std::memcpy(&id, id128, 128);
    ncclComm_t c;
    const ncclResult_t r = n.CommInitRank(&c, world, id, rank);
    if (r != ncclSuccess) {
        fprintf(stderr, "mle: ncclCommInitRank failed: %s\n", n.GetErrorString ? n.GetErrorString(r) : "?");
        return MLE_ERR_CUDA;
    }
    comm_ = c;
    if (cudaStreamCreateWithFlags(&comm_stream_, cudaStreamNonBlocking) != cudaSuccess) return MLE_ERR_CUDA;
    if (cudaEventCreateWithFlags(&done_, cudaEventDisableTiming) != cudaSuccess) return MLE_ERR_CUDA;
    buckets_ = plan_buckets(grads, bucket_mb);
    members_.assign(buckets_.size(), 0);
    ready_.assign(buckets_.size(), nullptr);
    ready_param_.assign(buckets_.size(), nullptr);
    for (auto& e : ready_)
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return MLE_ERR_CUDA;
    for (auto& e : ready_param_)
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return MLE_ERR_CUDA;
    for (auto& gr : grads) {
        if (gr.second <= 0) continue;
        for (int b = 0; b < (int)buckets_.size(); ++b) {
            if (gr.first >= buckets_[b].base && gr.first < buckets_[b].base + buckets_[b].count) {
                bucket_of_.push_back({gr.first, b});
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
}

void DataParallel::issue(int b, cudaStream_t compute) {
    check_cuda(cudaEventRecord(ready_[b], compute), "dp bucket ready");
    check_cuda(cudaStreamWaitEvent(comm_stream_, ready_[b], 0), "dp bucket wait");
    if (param_stream_pending()) {
        // parameter gradients produced on the parameter-gradient stream
        check_cuda(cudaEventRecord(ready_param_[b], param_stream()), "dp bucket ready");
        check_cuda(cudaStreamWaitEvent(comm_stream_, ready_param_[b], 0), "dp bucket wait");
    }
    const ncclResult_t r = nccl().AllReduce(buckets_[b].base, buckets_[b].base, (size_t)buckets_[b].count,
                                            ncclFloat32, ncclSum, (ncclComm_t)comm_, comm_stream_);
    if (r != ncclSuccess) {
        fprintf(stderr, "mle: ncclAllReduce failed: %s\n", nccl().GetErrorString ? nccl().GetErrorString(r) : "?");
        std::exit(1);
    }
    issued_[b] = 1;
}

void DataParallel::grads_done(const std::vector<float*>& grads, cudaStream_t compute) {
    for (float* g : grads) {
        auto it = std::lower_bound(bucket_of_.begin(), bucket_of_.end(), std::make_pair(g, -1));
        if (it == bucket_of_.end() || it->first != g) continue;
        const int b = it->second;
        if (--pending_[b] == 0 && !issued_[b]) issue(b, compute);
    }
}

void DataParallel::reduce_remaining(cudaStream_t compute) {
    for (int b = 0; b < (int)buckets_.size(); ++b)
        if (!issued_[b]) issue(b, compute);
    check_cuda(cudaEventRecord(done_, comm_stream_), "dp done");
    check_cuda(cudaStreamWaitEvent(compute, done_, 0), "dp join");
}

}  // namespace mle

extern "C" int mle_dp_plan_buckets(const uint64_t* addrs, const int64_t* counts, int n, int bucket_mb,
                                   uint64_t* out_base, int64_t* out_count, int max_out, int* out_n) {
    if (n < 0 || (n > 0 && (!addrs || !counts)) || !out_n || max_out < 0 || (max_out > 0 && (!out_base || !out_count)))
        return MLE_ERR_ARG;
    std::vector<std::pair<float*, int64_t>> g;
    for (int i = 0; i < n; ++i) g.push_back({reinterpret_cast<float*>(addrs[i]), counts[i]});
    const std::vector<mle::GradBucket> b = mle::plan_buckets(g, bucket_mb);
    *out_n = (int)b.size();
    if ((int)b.size() > max_out) return MLE_ERR_ARG;
    for (size_t i = 0; i < b.size(); ++i) {
        out_base[i] = reinterpret_cast<uint64_t>(b[i].base);
        out_count[i] = b[i].count;
    }
    return MLE_OK;
}

extern "C" int mle_dp_unique_id(uint8_t* out128) {
    if (!out128) return MLE_ERR_ARG;
    return mle::nccl_unique_id(out128);
}
