// NCCL gradient reduction for data-parallel sessions (see session_dp.h).
#include <dlfcn.h>
#include <nccl.h>
#include <stdio.h>

#include <algorithm>
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

DataParallel::~DataParallel() {
    if (comm_stream_) cudaStreamSynchronize(comm_stream_);
    if (comm_ && nccl().ok) nccl().CommDestroy((ncclComm_t)comm_);
    if (ready_) cudaEventDestroy(ready_);
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
    cudaEventCreateWithFlags(&ready_, cudaEventDisableTiming);
    cudaEventCreateWithFlags(&done_, cudaEventDisableTiming);
    // Buckets: contiguous runs of the parameter-gradient arena (gaps of at
    // most one 256-byte alignment pad are bridged; the pad bytes belong to no
    // tensor) of at most bucket_mb MiB.
    std::vector<std::pair<float*, int64_t>> g = grads;
    std::sort(g.begin(), g.end());
    const int64_t cap = std::max<int64_t>(1, (int64_t)bucket_mb) * (1ll << 20) / 4;
    float* cur = nullptr;
    int64_t len = 0;
    for (auto& e : g) {
        if (cur && e.first <= cur + len + 64 && (e.first + e.second) - cur <= cap) {
            len = std::max<int64_t>(len, (e.first + e.second) - cur);
        } else {
            if (cur) buckets_.push_back({cur, len});
            cur = e.first;
            len = e.second;
        }
    }
    if (cur) buckets_.push_back({cur, len});
    return MLE_OK;
}

void DataParallel::reduce_remaining(cudaStream_t compute) {
    const NcclApi& n = nccl();
    check_cuda(cudaEventRecord(ready_, compute), "dp ready");
    check_cuda(cudaStreamWaitEvent(comm_stream_, ready_, 0), "dp wait");
    n.GroupStart();
    for (auto& b : buckets_)
        n.AllReduce(b.base, b.base, (size_t)b.count, ncclFloat32, ncclSum, (ncclComm_t)comm_, comm_stream_);
    n.GroupEnd();
    check_cuda(cudaEventRecord(done_, comm_stream_), "dp done");
    check_cuda(cudaStreamWaitEvent(compute, done_, 0), "dp join");
}

}  // namespace mle

extern "C" int mle_dp_unique_id(uint8_t* out128) {
    if (!out128) return MLE_ERR_ARG;
    return mle::nccl_unique_id(out128);
}
