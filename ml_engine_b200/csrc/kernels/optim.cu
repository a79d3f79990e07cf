// Multi-tensor gradient-norm clip and Adam/AdamW.
//
// The reference launches SumSquared, SP and AdamWUpdate once per parameter
// tensor with one thread per element (Engine/engine.cu:283-302,
// Engine/kernels.cu:1486-1534).  Here a single launch covers up to
// kMaxTensors tensors: the tensor table travels in the kernel's parameter
// space (__grid_constant__), each block processes a fixed-size chunk of one
// tensor with 128-bit loads, and the block-to-tensor map is a prefix sum
// over chunk counts computed on the host.  Nothing is allocated.
//
// Per-element arithmetic keeps the reference's types and operation order:
//   m = b1*m + (1.0 - b1)*g            (product in float, sum in double)
//   v = b2*v + (1.0 - b2)*g*g
//   m_hat = m / (1.0 - pow(b1, t))     (pow(float,int), division in double)
//   AdamW: w -= lr*((m_hat/(sqrtf(v_hat)+eps)) + wd*w)
//   Adam : w -= lr*m_hat/(sqrtf(v_hat)+eps), bias terms with powf
// and the clip divides by (float)norm as SP does.
#include <math.h>

#include <mutex>

#include "common.cuh"

namespace mle {
namespace {

constexpr int kThreads = 256;
constexpr int kVecPerThread = 4;                              // float4 per thread per chunk
constexpr int kChunk = kThreads * 4 * kVecPerThread;          // 4096 elements per block
constexpr int kMaxTensors = 96;

struct TensorTable {
    int n;
    int64_t block_start[kMaxTensors + 1];
    mle_param_view p[kMaxTensors];
};

__device__ __forceinline__ int find_tensor(const TensorTable& tt, int64_t block) {
    int lo = 0, hi = tt.n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (tt.block_start[mid] <= block) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// ------------------------------- sum of squares -----------------------------
__global__ void __launch_bounds__(kThreads) sumsq_kernel(const __grid_constant__ TensorTable tt,
                                                         double* __restrict__ ws, double scale2) {
    pdl_entry();
    __shared__ double scratch[32];
    const int ti = find_tensor(tt, blockIdx.x);
    const mle_param_view& P = tt.p[ti];
    const int64_t begin = (int64_t)(blockIdx.x - tt.block_start[ti]) * kChunk;
    int64_t end = begin + kChunk;
    if (end > P.n) end = P.n;
    double acc = 0.0;
    const float* g = P.g;
    const bool vec = aligned16(g);
    if (vec) {
        const int64_t vb = begin, ve = begin + ((end - begin) & ~int64_t(3));
        for (int64_t i = vb + threadIdx.x * 4; i < ve; i += kThreads * 4) {
            const float4 v = *reinterpret_cast<const float4*>(g + i);
            acc += (double)v.x * (double)v.x;
            acc += (double)v.y * (double)v.y;
            acc += (double)v.z * (double)v.z;
            acc += (double)v.w * (double)v.w;
        }
        for (int64_t i = ve + threadIdx.x; i < end; i += kThreads) acc += (double)g[i] * (double)g[i];
    } else {
        for (int64_t i = begin + threadIdx.x; i < end; i += kThreads) acc += (double)g[i] * (double)g[i];
    }
    acc = block_sum(acc, scratch);
    if (threadIdx.x == 0) atomicAdd(ws, acc * scale2);
}

// Sqrt_Scale (Engine/kernels.cu:1763-1773) generalised to a max norm:
// ws = (sqrt(ws) > max_norm) ? sqrt(ws)/max_norm : 1; with max_norm == 1 this
// is the reference's (curr > 1.0) ? curr * 1.0 : 1.0.  A NaN stays NaN.
__global__ void clip_finalize_kernel(double* ws, double max_norm) {
    pdl_entry();
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const double x = ws[0];
    if (x != x) return;
    const double curr = sqrt(x);
    ws[0] = (curr > max_norm) ? curr / max_norm : 1.0;
}

// ---------------------------------- clip -----------------------------------
__global__ void __launch_bounds__(kThreads) clip_apply_kernel(const __grid_constant__ TensorTable tt,
                                                              const double* __restrict__ ws) {
    pdl_entry();
    const int ti = find_tensor(tt, blockIdx.x);
    const mle_param_view& P = tt.p[ti];
    const int64_t begin = (int64_t)(blockIdx.x - tt.block_start[ti]) * kChunk;
    int64_t end = begin + kChunk;
    if (end > P.n) end = P.n;
    const float f = (float)ws[0];
    for (int64_t i = begin + threadIdx.x; i < end; i += kThreads) P.g[i] /= f;
}

// ---------------------------------- Adam -----------------------------------
template <bool ADAMW>
__device__ __forceinline__ void adam_elem(float& w, float& m, float& v, float g, float b1, float b2, float eps,
                                          float wd, float lr, double bc1, double bc2) {
    m = b1 * m + (1.0 - b1) * g;
    v = b2 * v + (1.0 - b2) * g * g;
    const float m_hat = m / bc1;
    const float v_hat = v / bc2;
    const float v_hat_scale = sqrtf(v_hat);
    if (ADAMW) w -= lr * ((m_hat / (v_hat_scale + eps)) + wd * w);
    else w -= lr * m_hat / (v_hat_scale + eps);
}

template <bool ADAMW, bool CLIP, bool PRESCALE>
__global__ void __launch_bounds__(kThreads) adam_kernel(const __grid_constant__ TensorTable tt,
                                                        const double* __restrict__ clip_ws, float pre_scale,
                                                        float lr, int write_back) {
    pdl_entry();
    const int ti = find_tensor(tt, blockIdx.x);
    const mle_param_view& P = tt.p[ti];
    const int64_t chunk = blockIdx.x - tt.block_start[ti];
    const int64_t begin = chunk * kChunk;
    int64_t end = begin + kChunk;
    if (end > P.n) end = P.n;
    const float b1 = P.b1, b2 = P.b2, eps = P.eps, wd = P.weight_decay;
    // bias corrections: one thread per block evaluates the powers (the
    // same values every thread would compute)
    __shared__ double bc[2];
    if (threadIdx.x == 0) {
        const int t = *P.t;
        if (ADAMW) {
            bc[0] = 1.0 - pow(b1, t);   // pow(float, int) as in AdamWUpdate
            bc[1] = 1.0 - pow(b2, t);
        } else {
            bc[0] = 1.0 - powf(b1, (float)t);
            bc[1] = 1.0 - powf(b2, (float)t);
        }
    }
    __syncthreads();
    const double bc1 = bc[0], bc2 = bc[1];
    const float clip_f = CLIP ? (float)clip_ws[0] : 1.0f;
    float* __restrict__ W = P.w;
    float* __restrict__ G = P.g;
    float* __restrict__ M = P.m;
    float* __restrict__ V = P.v;
    const bool vec = aligned16(W) && aligned16(G) && aligned16(M) && aligned16(V);
    int64_t tail = begin;
    if (vec) {
        const int64_t ve = begin + ((end - begin) & ~int64_t(3));
        for (int64_t i = begin + threadIdx.x * 4; i < ve; i += kThreads * 4) {
            float4 g4 = *reinterpret_cast<const float4*>(G + i);
            float4 w4 = *reinterpret_cast<const float4*>(W + i);
            float4 m4 = *reinterpret_cast<const float4*>(M + i);
            float4 v4 = *reinterpret_cast<const float4*>(V + i);
            float gg[4] = {g4.x, g4.y, g4.z, g4.w};
            float ww[4] = {w4.x, w4.y, w4.z, w4.w};
            float mm[4] = {m4.x, m4.y, m4.z, m4.w};
            float vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (PRESCALE) gg[j] = gg[j] * pre_scale;
                if (CLIP) gg[j] /= clip_f;
                adam_elem<ADAMW>(ww[j], mm[j], vv[j], gg[j], b1, b2, eps, wd, lr, bc1, bc2);
            }
            *reinterpret_cast<float4*>(W + i) = make_float4(ww[0], ww[1], ww[2], ww[3]);
            *reinterpret_cast<float4*>(M + i) = make_float4(mm[0], mm[1], mm[2], mm[3]);
            *reinterpret_cast<float4*>(V + i) = make_float4(vv[0], vv[1], vv[2], vv[3]);
            if ((CLIP || PRESCALE) && write_back)
                *reinterpret_cast<float4*>(G + i) = make_float4(gg[0], gg[1], gg[2], gg[3]);
        }
        tail = ve;
    }
    for (int64_t i = tail + threadIdx.x; i < end; i += kThreads) {
        float g = G[i];
        if (PRESCALE) g = g * pre_scale;
        if (CLIP) g /= clip_f;
        float w = W[i], m = M[i], v = V[i];
        adam_elem<ADAMW>(w, m, v, g, b1, b2, eps, wd, lr, bc1, bc2);
        W[i] = w;
        M[i] = m;
        V[i] = v;
        if ((CLIP || PRESCALE) && write_back) G[i] = g;
    }
}

// t += 1 for every tensor of the table (run after the update; stream order
// makes every block of the update see the old value).
__global__ void step_increment_kernel(const __grid_constant__ TensorTable tt) {
    pdl_entry();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < tt.n) *tt.p[i].t += 1;
}

// Builds the table for tensors [first, first+count).  Returns the number of
// blocks, or -1 on a bad entry.
int64_t build_table(TensorTable& tt, const mle_param_view* params, int first, int count) {
    tt.n = count;
    int64_t blocks = 0;
    for (int i = 0; i < count; ++i) {
        const mle_param_view& p = params[first + i];
        if (p.n < 0 || (p.n > 0 && (!p.g))) return -1;
        tt.p[i] = p;
        tt.block_start[i] = blocks;
        blocks += (p.n + kChunk - 1) / kChunk;
        if (p.n == 0) blocks += 1;  // an empty tensor still owns one (idle) block
    }
    tt.block_start[count] = blocks;
    return blocks;
}

// ------------------------- clip without a caller workspace -------------------------
// Scratch of mle_clip_grad_norm_static: slots [0, blocks) hold the per-block
// sums of squares of one call, slot MLE_CLIP_STATIC_MAX_BLOCKS the clip
// coefficient.
static __device__ __align__(256) double g_clip_static[MLE_CLIP_STATIC_MAX_BLOCKS + 1];

__global__ void __launch_bounds__(kThreads) sumsq_partial_kernel(const __grid_constant__ TensorTable tt,
                                                                 double* __restrict__ partial) {
    pdl_entry();
    __shared__ double scratch[32];
    const int ti = find_tensor(tt, blockIdx.x);
    const mle_param_view& P = tt.p[ti];
    const int64_t begin = (int64_t)(blockIdx.x - tt.block_start[ti]) * kChunk;
    int64_t end = begin + kChunk;
    if (end > P.n) end = P.n;
    double acc = 0.0;
    for (int64_t i = begin + threadIdx.x; i < end; i += kThreads) acc += (double)P.g[i] * (double)P.g[i];
    acc = block_sum(acc, scratch);
    if (threadIdx.x == 0) partial[blockIdx.x] = acc;
}

// One block: thread i adds partials i, i + 256, ... in order, then a fixed
// shuffle tree; the coefficient follows clip_finalize_kernel.
__global__ void __launch_bounds__(kThreads) clip_finalize_static_kernel(double* __restrict__ scratch, int nblocks,
                                                                        double max_norm, double* coef_out) {
    pdl_entry();
    __shared__ double red[32];
    double acc = 0.0;
    for (int i = threadIdx.x; i < nblocks; i += kThreads) acc += scratch[i];
    acc = block_sum(acc, red);
    if (threadIdx.x == 0) {
        double c = acc;  // a NaN sum is left as it is
        if (acc == acc) {
            const double curr = sqrt(acc);
            c = (curr > max_norm) ? curr / max_norm : 1.0;
        }
        scratch[MLE_CLIP_STATIC_MAX_BLOCKS] = c;
        if (coef_out) *coef_out = c;
    }
}

}  // namespace
}  // namespace mle

using namespace mle;

namespace {
// Device address of g_clip_static, resolved once per device.
double* clip_static_scratch(int& status) {
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static double* addr[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        status = MLE_ERR_CUDA;
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_clip_static) != cudaSuccess || !p) {
            status = MLE_ERR_CUDA;
            return nullptr;
        }
        addr[dev] = static_cast<double*>(p);
    }
    status = MLE_OK;
    return addr[dev];
}
}  // namespace

extern "C" {

int mle_grad_sumsq(const mle_param_view* params, int n_tensors, double* norm_ws, double scale, mle_stream_t stream) {
    if (n_tensors < 0 || (n_tensors > 0 && !params) || !norm_ws) return MLE_ERR_ARG;
    cudaStream_t st = as_stream(stream);
    for (int first = 0; first < n_tensors; first += kMaxTensors) {
        const int count = (n_tensors - first < kMaxTensors) ? n_tensors - first : kMaxTensors;
        TensorTable tt;
        const int64_t blocks = build_table(tt, params, first, count);
        if (blocks < 0) return MLE_ERR_ARG;
        if (blocks == 0) continue;
        if (blocks > 0x7fffffffLL) return MLE_ERR_UNSUPPORTED;
        launch_k(sumsq_kernel, (unsigned)blocks, kThreads, 0, st, tt, norm_ws, scale * scale);
        const int s = launch_status();
        if (s) return s;
    }
    return MLE_OK;
}

int mle_clip_finalize(double* norm_ws, double max_norm, mle_stream_t stream) {
    if (!norm_ws || !(max_norm > 0.0)) return MLE_ERR_ARG;
    launch_k(clip_finalize_kernel, 1, 32, 0, as_stream(stream), norm_ws, max_norm);
    return launch_status();
}

int mle_clip_apply(const mle_param_view* params, int n_tensors, const double* norm_ws, mle_stream_t stream) {
    if (n_tensors < 0 || (n_tensors > 0 && !params) || !norm_ws) return MLE_ERR_ARG;
    cudaStream_t st = as_stream(stream);
    for (int first = 0; first < n_tensors; first += kMaxTensors) {
        const int count = (n_tensors - first < kMaxTensors) ? n_tensors - first : kMaxTensors;
        TensorTable tt;
        const int64_t blocks = build_table(tt, params, first, count);
        if (blocks < 0) return MLE_ERR_ARG;
        if (blocks == 0) continue;
        launch_k(clip_apply_kernel, (unsigned)blocks, kThreads, 0, st, tt, norm_ws);
        const int s = launch_status();
        if (s) return s;
    }
    return MLE_OK;
}

int mle_adam_update(const mle_param_view* params, int n_tensors, const double* clip_ws, float pre_scale, float lr,
                    int adamw, int write_back_grad, mle_stream_t stream) {
    if (n_tensors < 0 || (n_tensors > 0 && !params)) return MLE_ERR_ARG;
    for (int i = 0; i < n_tensors; ++i) {
        const mle_param_view& p = params[i];
        if (p.n > 0 && (!p.w || !p.g || !p.m || !p.v || !p.t)) return MLE_ERR_ARG;
        if (p.n == 0 && !p.t) return MLE_ERR_ARG;
    }
    cudaStream_t st = as_stream(stream);
    const bool clip = clip_ws != nullptr;
    const bool pres = pre_scale != 1.0f;
    for (int first = 0; first < n_tensors; first += kMaxTensors) {
        const int count = (n_tensors - first < kMaxTensors) ? n_tensors - first : kMaxTensors;
        TensorTable tt;
        const int64_t blocks = build_table(tt, params, first, count);
        if (blocks < 0) return MLE_ERR_ARG;
        if (blocks > 0) {
#define MLE_ADAM_LAUNCH(AW, CL, PS) \
    launch_k(adam_kernel<AW, CL, PS>, (unsigned)blocks, kThreads, 0, st, tt, clip_ws, pre_scale, lr, write_back_grad)
            if (adamw) {
                if (clip) { if (pres) MLE_ADAM_LAUNCH(true, true, true); else MLE_ADAM_LAUNCH(true, true, false); }
                else { if (pres) MLE_ADAM_LAUNCH(true, false, true); else MLE_ADAM_LAUNCH(true, false, false); }
            } else {
                if (clip) { if (pres) MLE_ADAM_LAUNCH(false, true, true); else MLE_ADAM_LAUNCH(false, true, false); }
                else { if (pres) MLE_ADAM_LAUNCH(false, false, true); else MLE_ADAM_LAUNCH(false, false, false); }
            }
#undef MLE_ADAM_LAUNCH
            int s = launch_status();
            if (s) return s;
        }
        launch_k(step_increment_kernel, (count + 127) / 128, 128, 0, st, tt);
        const int s = launch_status();
        if (s) return s;
    }
    return MLE_OK;
}

int mle_clip_grad_norm_static(const mle_param_view* params, int n_tensors, double max_norm, double* coef_out,
                              mle_stream_t stream) {
    if (n_tensors < 0 || (n_tensors > 0 && !params) || !(max_norm > 0.0)) return MLE_ERR_ARG;
    // size check first: the whole set must fit the static scratch
    int64_t total_blocks = 0;
    for (int i = 0; i < n_tensors; ++i) {
        if (params[i].n < 0 || (params[i].n > 0 && !params[i].g)) return MLE_ERR_ARG;
        total_blocks += params[i].n > 0 ? (params[i].n + kChunk - 1) / kChunk : 1;
    }
    if (total_blocks > MLE_CLIP_STATIC_MAX_BLOCKS) return MLE_ERR_ARG;
    int status = MLE_OK;
    double* scratch = clip_static_scratch(status);
    if (!scratch) return status;
    cudaStream_t st = as_stream(stream);
    int64_t offset = 0;
    for (int first = 0; first < n_tensors; first += kMaxTensors) {
        const int count = (n_tensors - first < kMaxTensors) ? n_tensors - first : kMaxTensors;
        TensorTable tt;
        const int64_t blocks = build_table(tt, params, first, count);
        if (blocks < 0) return MLE_ERR_ARG;
        if (blocks == 0) continue;
        launch_k(sumsq_partial_kernel, (unsigned)blocks, kThreads, 0, st, tt, scratch + offset);
        const int s = launch_status();
        if (s) return s;
        offset += blocks;
    }
    launch_k(clip_finalize_static_kernel, 1, kThreads, 0, st, scratch, (int)offset, max_norm, coef_out);
    int s = launch_status();
    if (s) return s;
    for (int first = 0; first < n_tensors; first += kMaxTensors) {
        const int count = (n_tensors - first < kMaxTensors) ? n_tensors - first : kMaxTensors;
        TensorTable tt;
        const int64_t blocks = build_table(tt, params, first, count);
        if (blocks <= 0) continue;
        launch_k(clip_apply_kernel, (unsigned)blocks, kThreads, 0, st, tt, scratch + MLE_CLIP_STATIC_MAX_BLOCKS);
        s = launch_status();
        if (s) return s;
    }
    return MLE_OK;
}

}  // extern "C"
