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

#include <algorithm>
#include <cstddef>
#include <cstring>
#include <mutex>
#include <vector>

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

// ---------------------- norm + clip + update in one launch ----------------------
// A cooperative grid (every block resident) splits the kFusedUnit-element
// units of all tensors into one contiguous range per block (blocks beyond
// the unit count return at once) and walks it twice: forwards for the
// per-block sum of squares, then, after one grid barrier, backwards for the
// update, so that the gradients the first walk read last are still in L2
// when the second walk starts.  After the barrier every block adds the
// partials in block order (the same coefficient in every block, and the same
// from run to run for a given grid).  The last block to finish the update (a
// counter, no waiting) increments the step counters and re-arms the counters
// for the next launch, so a run needs no memset.  The tensor table sits in
// the caller's device workspace: the count of tensors is not bounded by the
// kernel's parameter space.  A unit is two float4 of each array per thread,
// so that small models still spread over many SMs.
constexpr int kFusedUnit = kThreads * 8;  // 2048 elements
constexpr int kFusedMaxBlocks = 148 * 8;
constexpr int kFusedMinBlocksPerSM = 3;   // <= 80 registers a thread

struct FusedWs {
    int n;           // tensors      } one 16-byte load at kernel entry
    int status;      // 1: the barrier timed out; later launches return at once
    int64_t units;   // kFusedUnit-element units over all tensors
    unsigned bar;    // arrivals at the grid barrier of the current launch
    unsigned done;   // blocks that finished the current launch
    double partial[kFusedMaxBlocks];
};
static_assert(offsetof(FusedWs, n) == 0 && offsetof(FusedWs, status) == 4 && offsetof(FusedWs, units) == 8,
              "header read as one int4");

__host__ __device__ inline size_t fused_table_offset() { return (sizeof(FusedWs) + 255) & ~size_t(255); }
__host__ __device__ inline int64_t* fused_unit_start(void* ws) {
    return reinterpret_cast<int64_t*>(static_cast<char*>(ws) + fused_table_offset());
}
__host__ __device__ inline size_t fused_views_offset(int n) {
    return (fused_table_offset() + sizeof(int64_t) * (size_t)(n + 1) + 255) & ~size_t(255);
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Every active block arrives once (a reduction, no round trip) and polls
// the counter.  True when all `active` arrivals came within two seconds and
// no block gave up; otherwise the status word is set and the caller returns.
// The counter is re-armed by the launch's last block.
__device__ bool fused_grid_barrier(FusedWs* ws, unsigned active) {
    __shared__ int ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(&ws->bar, 1u);
        volatile unsigned* bar = &ws->bar;
        volatile int* status = &ws->status;
        const uint64_t t0 = global_ns();
        ok = 1;
        for (;;) {
            if (*bar >= active) break;
            if (*status) {
                ok = 0;
                break;
            }
            if (global_ns() - t0 > 2000000000ull) {
                atomicOr(&ws->status, 1);
                ok = 0;
                break;
            }
        }
        __threadfence();
    }
    __syncthreads();
    return ok != 0;
}

__device__ __forceinline__ int fused_find(const int64_t* us, int n, int64_t c) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (us[mid] <= c) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

template <bool ADAMW>
__device__ __forceinline__ void bias_corrections(const mle_param_view& P, double* bc) {
    const int t = *P.t;
    if (ADAMW) {
        bc[0] = 1.0 - pow(P.b1, t);  // pow(float, int) as in AdamWUpdate
        bc[1] = 1.0 - pow(P.b2, t);
    } else {
        bc[0] = 1.0 - powf(P.b1, (float)t);
        bc[1] = 1.0 - powf(P.b2, (float)t);
    }
}

__device__ __forceinline__ double sumsq4(double acc, const float4& x) {
    acc += (double)x.x * (double)x.x;
    acc += (double)x.y * (double)x.y;
    acc += (double)x.z * (double)x.z;
    acc += (double)x.w * (double)x.w;
    return acc;
}

// g' = g * pre_scale / clip, then the element update, for four elements
template <bool ADAMW, bool CLIP, bool PRESCALE>
__device__ __forceinline__ void adam1(float& g, float& w, float& m, float& v, const mle_param_view& P,
                                      float pre_scale, float clip_f, float lr, double bc1, double bc2) {
    if (PRESCALE) g = g * pre_scale;
    if (CLIP) g /= clip_f;
    adam_elem<ADAMW>(w, m, v, g, P.b1, P.b2, P.eps, P.weight_decay, lr, bc1, bc2);
}

template <bool ADAMW, bool CLIP, bool PRESCALE>
__device__ __forceinline__ void adam4(float4& g4, float4& w4, float4& m4, float4& v4, const mle_param_view& P,
                                      float pre_scale, float clip_f, float lr, double bc1, double bc2) {
    adam1<ADAMW, CLIP, PRESCALE>(g4.x, w4.x, m4.x, v4.x, P, pre_scale, clip_f, lr, bc1, bc2);
    adam1<ADAMW, CLIP, PRESCALE>(g4.y, w4.y, m4.y, v4.y, P, pre_scale, clip_f, lr, bc1, bc2);
    adam1<ADAMW, CLIP, PRESCALE>(g4.z, w4.z, m4.z, v4.z, P, pre_scale, clip_f, lr, bc1, bc2);
    adam1<ADAMW, CLIP, PRESCALE>(g4.w, w4.w, m4.w, v4.w, P, pre_scale, clip_f, lr, bc1, bc2);
}

template <bool ADAMW, bool CLIP, bool PRESCALE>
__global__ void __launch_bounds__(kThreads, kFusedMinBlocksPerSM)
    fused_clip_adam_kernel(void* wsv, float pre_scale, float lr, double max_norm, int write_back) {
    FusedWs* ws = static_cast<FusedWs*>(wsv);
    __shared__ double scratch[32];
    __shared__ double bc[2];
    __shared__ int last;
    const int4 hdr = __ldcg(static_cast<const int4*>(wsv));  // n, status, units
    if (hdr.y) return;  // a failed launch: nothing runs until the table is prepared again
    const int n = hdr.x;
    const int64_t units = (int64_t)(((uint64_t)(unsigned)hdr.w << 32) | (uint64_t)(unsigned)hdr.z);
    // blocks beyond the unit count have nothing to do and take no part
    const unsigned active = units < (int64_t)gridDim.x ? (unsigned)units : gridDim.x;
    if (blockIdx.x >= active) return;
    const int64_t* us = fused_unit_start(wsv);
    const mle_param_view* views =
        reinterpret_cast<const mle_param_view*>(static_cast<char*>(wsv) + fused_views_offset(n));
    const int64_t per = units / active, rem = units % active;
    const int64_t c0 = (int64_t)blockIdx.x * per + (blockIdx.x < rem ? blockIdx.x : rem);
    const int64_t c1 = c0 + per + (blockIdx.x < rem ? 1 : 0);  // c1 > c0
    const int tid4 = threadIdx.x * 4;
    // The first tensor the update visits: its bias corrections are taken by
    // a thread of the second warp while the first walk runs.  The table is
    // read only where a walk crosses into another tensor; the data loads
    // bypass L1 so that the table stays there.
    int ti = fused_find(us, n, c1 - 1);
    if (threadIdx.x == 32) bias_corrections<ADAMW>(views[ti], bc);
    float clip_f = 1.0f;
    if (CLIP) {
        double acc = 0.0;
        int tf = fused_find(us, n, c0);
        int64_t t_begin = us[tf], t_end = us[tf + 1];
        const float* g = views[tf].g;
        int64_t len = views[tf].n;
        for (int64_t c = c0; c < c1;) {
            if (c >= t_end) {
                do {
                    ++tf;
                    t_begin = t_end;
                    t_end = us[tf + 1];
                } while (c >= t_end);
                g = views[tf].g;
                len = views[tf].n;
            }
            const int64_t begin = (c - t_begin) * kFusedUnit;
            const int64_t left = len - begin;
            if (left >= 2 * kFusedUnit && c + 1 < c1 && aligned16(g)) {
                // two whole units of one tensor: four float4 in flight
                float4 x[4];
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    x[j] = __ldcg(reinterpret_cast<const float4*>(g + begin + j * kThreads * 4 + tid4));
#pragma unroll
                for (int j = 0; j < 4; ++j) acc = sumsq4(acc, x[j]);
                c += 2;
                continue;
            }
            const int64_t end = left < kFusedUnit ? len : begin + kFusedUnit;
            if (aligned16(g)) {
                const int64_t ve = begin + ((end - begin) & ~int64_t(3));
                for (int64_t i = begin + tid4; i < ve; i += kThreads * 4)
                    acc = sumsq4(acc, __ldcg(reinterpret_cast<const float4*>(g + i)));
                for (int64_t i = ve + threadIdx.x; i < end; i += kThreads) acc += (double)g[i] * (double)g[i];
            } else {
                for (int64_t i = begin + threadIdx.x; i < end; i += kThreads) acc += (double)g[i] * (double)g[i];
            }
            ++c;
        }
        acc = block_sum(acc, scratch);
        if (threadIdx.x == 0) ws->partial[blockIdx.x] = acc;
        if (!fused_grid_barrier(ws, active)) return;
        double tot = 0.0;
        for (int i = threadIdx.x; i < (int)active; i += kThreads) tot += __ldcg(&ws->partial[i]);
        tot = block_sum(tot, scratch) * ((double)pre_scale * (double)pre_scale);
        // Sqrt_Scale with a max norm; a NaN sum stays NaN
        double coef = tot;
        if (tot == tot) {
            const double curr = sqrt(tot);
            coef = (curr > max_norm) ? curr / max_norm : 1.0;
        }
        clip_f = (float)coef;
    } else {
        __syncthreads();  // bc of the first tensor
    }
    const bool wb = (CLIP || PRESCALE) && write_back;
    mle_param_view P = views[ti];
    int64_t t_begin = us[ti];
    double bc1 = bc[0], bc2 = bc[1];
    for (int64_t c = c1 - 1; c >= c0; --c) {
        if (c < t_begin) {  // block-uniform: the next tensor and its bias corrections
            do {
                --ti;
                t_begin = us[ti];
            } while (c < t_begin);
            P = views[ti];
            __syncthreads();
            if (threadIdx.x == 0) bias_corrections<ADAMW>(P, bc);
            __syncthreads();
            bc1 = bc[0];
            bc2 = bc[1];
        }
        const int64_t begin = (c - t_begin) * kFusedUnit;
        const int64_t end = begin + kFusedUnit < P.n ? begin + kFusedUnit : P.n;
        float* __restrict__ W = P.w;
        float* __restrict__ G = P.g;
        float* __restrict__ M = P.m;
        float* __restrict__ V = P.v;
        const bool vec = aligned16(W) && aligned16(G) && aligned16(M) && aligned16(V);
        if (vec && end - begin == kFusedUnit) {
            // a whole unit: every load of the thread in flight before the arithmetic
            float4 g4[2], w4[2], m4[2], v4[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int64_t i = begin + u * kThreads * 4 + tid4;
                g4[u] = __ldcg(reinterpret_cast<const float4*>(G + i));
                w4[u] = __ldcg(reinterpret_cast<const float4*>(W + i));
                m4[u] = __ldcg(reinterpret_cast<const float4*>(M + i));
                v4[u] = __ldcg(reinterpret_cast<const float4*>(V + i));
            }
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int64_t i = begin + u * kThreads * 4 + tid4;
                adam4<ADAMW, CLIP, PRESCALE>(g4[u], w4[u], m4[u], v4[u], P, pre_scale, clip_f, lr, bc1, bc2);
                *reinterpret_cast<float4*>(W + i) = w4[u];
                *reinterpret_cast<float4*>(M + i) = m4[u];
                *reinterpret_cast<float4*>(V + i) = v4[u];
                if (wb) *reinterpret_cast<float4*>(G + i) = g4[u];
            }
            continue;
        }
        int64_t tail = begin;
        if (vec) {
            const int64_t ve = begin + ((end - begin) & ~int64_t(3));
            for (int64_t i = begin + tid4; i < ve; i += kThreads * 4) {
                float4 g4 = __ldcg(reinterpret_cast<const float4*>(G + i));
                float4 w4 = __ldcg(reinterpret_cast<const float4*>(W + i));
                float4 m4 = __ldcg(reinterpret_cast<const float4*>(M + i));
                float4 v4 = __ldcg(reinterpret_cast<const float4*>(V + i));
                adam4<ADAMW, CLIP, PRESCALE>(g4, w4, m4, v4, P, pre_scale, clip_f, lr, bc1, bc2);
                *reinterpret_cast<float4*>(W + i) = w4;
                *reinterpret_cast<float4*>(M + i) = m4;
                *reinterpret_cast<float4*>(V + i) = v4;
                if (wb) *reinterpret_cast<float4*>(G + i) = g4;
            }
            tail = ve;
        }
        for (int64_t i = tail + threadIdx.x; i < end; i += kThreads) {
            float g = G[i];
            if (PRESCALE) g = g * pre_scale;
            if (CLIP) g /= clip_f;
            float w = W[i], m = M[i], v = V[i];
            adam_elem<ADAMW>(w, m, v, g, P.b1, P.b2, P.eps, P.weight_decay, lr, bc1, bc2);
            W[i] = w;
            M[i] = m;
            V[i] = v;
            if (wb) G[i] = g;
        }
    }
    // The last block to get here increments every step counter (every block
    // read the counters it needed before arriving) and re-arms the counters.
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(&ws->done, 1u) == active - 1;
        if (last) __threadfence();
    }
    __syncthreads();
    if (last) {
        for (int i = threadIdx.x; i < n; i += kThreads) *views[i].t += 1;
        if (threadIdx.x == 0) {
            ws->bar = 0;
            ws->done = 0;
        }
    }
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

int64_t mle_clip_adam_ws_bytes(int n_tensors) {
    if (n_tensors < 0) return -1;
    return (int64_t)(fused_views_offset(n_tensors) + sizeof(mle_param_view) * (size_t)n_tensors);
}

int mle_clip_adam_prepare(const mle_param_view* params, int n_tensors, void* ws, int64_t ws_bytes,
                          mle_stream_t stream) {
    if (n_tensors <= 0 || !params || !ws || ws_bytes < mle_clip_adam_ws_bytes(n_tensors)) return MLE_ERR_ARG;
    if (!aligned16(ws)) return MLE_ERR_ARG;
    cudaStream_t st = as_stream(stream);
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cap) != cudaSuccess) return launch_status();
    if (cap != cudaStreamCaptureStatusNone) return MLE_ERR_UNSUPPORTED;  // a copy of a host table
    std::vector<FusedWs> hbuf((size_t)(mle_clip_adam_ws_bytes(n_tensors) + sizeof(FusedWs) - 1) / sizeof(FusedWs));
    memset(static_cast<void*>(hbuf.data()), 0, hbuf.size() * sizeof(FusedWs));
    char* buf = reinterpret_cast<char*>(hbuf.data());
    FusedWs* hdr = hbuf.data();
    int64_t* us = fused_unit_start(buf);
    mle_param_view* views = reinterpret_cast<mle_param_view*>(buf + fused_views_offset(n_tensors));
    int64_t units = 0;
    for (int i = 0; i < n_tensors; ++i) {
        const mle_param_view& p = params[i];
        if (p.n < 0 || !p.t || (p.n > 0 && (!p.w || !p.g || !p.m || !p.v))) return MLE_ERR_ARG;
        views[i] = p;
        us[i] = units;
        units += p.n > 0 ? (p.n + kFusedUnit - 1) / kFusedUnit : 1;  // an empty tensor owns one idle unit
    }
    us[n_tensors] = units;
    hdr->n = n_tensors;
    hdr->units = units;  // status and the counters start at zero
    // pageable source: the runtime has taken its copy of `buf` when this returns
    if (cudaMemcpyAsync(ws, buf, (size_t)mle_clip_adam_ws_bytes(n_tensors), cudaMemcpyHostToDevice, st) != cudaSuccess)
        return launch_status();
    return launch_status();
}

int mle_clip_adam_run(void* ws, float max_norm, float pre_scale, float lr, int adamw, int write_back_grad,
                      mle_stream_t stream) {
    if (!ws || !aligned16(ws) || (adamw != 0 && adamw != 1))
        return MLE_ERR_ARG;
    cudaStream_t st = as_stream(stream);
    const bool clip = max_norm > 0.0f;
    const bool pres = pre_scale != 1.0f;
    auto go = [&](auto kern) -> int {
        static int grid = 0;  // one per instantiation: resident blocks on every SM
        if (grid == 0) {
            int per_sm = 0, dev = 0, sms = 0;
            if (cudaGetDevice(&dev) != cudaSuccess ||
                cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
                cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, 0) != cudaSuccess)
                return launch_status();
            grid = std::min(per_sm * sms, kFusedMaxBlocks);
            if (grid <= 0) return MLE_ERR_UNSUPPORTED;
        }
        // the counters were zeroed by prepare and are re-armed by each launch's last block
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)grid);
        cfg.blockDim = dim3(kThreads);
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaLaunchKernelEx(&cfg, kern, ws, pre_scale, lr, (double)max_norm, write_back_grad) != cudaSuccess)
            return launch_status();
        return launch_status();
    };
#define MLE_FCA(A, C, P) \
    if (adamw == A && clip == C && pres == P) return go(fused_clip_adam_kernel<A, C, P>);
    MLE_FCA(1, true, true)
    MLE_FCA(1, true, false)
    MLE_FCA(1, false, true)
    MLE_FCA(1, false, false)
    MLE_FCA(0, true, true)
    MLE_FCA(0, true, false)
    MLE_FCA(0, false, true)
    MLE_FCA(0, false, false)
#undef MLE_FCA
    return MLE_ERR_ARG;
}

int mle_clip_adam_status(void* ws, int* out_status, mle_stream_t stream) {
    if (!ws || !out_status) return MLE_ERR_ARG;
    FusedWs* w = static_cast<FusedWs*>(ws);
    int v = 0;
    cudaStream_t st = as_stream(stream);
    if (cudaMemcpyAsync(&v, &w->status, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return launch_status();
    *out_status = v;
    return v ? MLE_ERR_TIMEOUT : MLE_OK;
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
