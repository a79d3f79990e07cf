// LayerNorm / GroupNorm forward and backward.
//
// Both reference ops normalise contiguous segments of the [B,C,H,W] tensor:
// LayerNorm one segment of C*H*W per dim0 index (Engine/kernels.cu:541-572),
// GroupNorm one segment of (C/G)*H*W per (sample, group)
// (Engine/kernels.cu:607-639).  One kernel pair therefore serves both: a
// warp owns a segment when it fits in its registers (N <= 1024, N % 4 == 0),
// a cluster of up to 8 CTAs when it fits in theirs (N <= 65536), otherwise
// a 256-thread block streams it.  gamma = 1 and beta = 0 are the
// reference's fixed constants.
//
// The reference computes the forward scale as rsqrtf((1/N)*sqdev + eps)
// (LNorm/GNorm) and the backward scale as rsqrtf(sqdev/N + eps)
// (LayerBackward/GroupBackward); both expressions are kept.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace mle {
namespace {

constexpr int kBlock = 256;
// longest segment a warp holds (8 float4 per lane); longer ones go to a CTA
// or a cluster (a 2048-float row ran at 59 % of HBM on one warp)
constexpr int kWarpMaxN = 1024;

// ----------------------------- warp per segment ---------------------------
// RESID: the segment is x + r (the residual Add that feeds the norm), which
// is also written to xr; the sum is the Add's own x + 1.0f * r, so both
// outputs are bitwise those of the Add and the norm launched apart.
template <int V, bool RESID>  // V float4 per lane -> N <= 128 * V
__device__ __forceinline__ void norm_fwd_warp(const float* __restrict__ x, const float* __restrict__ r,
                                              float* __restrict__ xr, float* __restrict__ y,
                                              float* __restrict__ mean, float* __restrict__ sqdev, int64_t segs,
                                              int N, float eps) {
    const int lane = threadIdx.x & 31;
    const int64_t seg = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (seg >= segs) return;
    const float4* xs = reinterpret_cast<const float4*>(x + seg * N);
    float4 v[V];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int c = lane + 32 * i;
        if (c * 4 < N) {
            v[i] = xs[c];
            if constexpr (RESID) {
                const float4 w = reinterpret_cast<const float4*>(r + seg * N)[c];
                v[i].x = v[i].x + 1.0f * w.x;
                v[i].y = v[i].y + 1.0f * w.y;
                v[i].z = v[i].z + 1.0f * w.z;
                v[i].w = v[i].w + 1.0f * w.w;
                reinterpret_cast<float4*>(xr + seg * N)[c] = v[i];
            }
            s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
        } else {
            v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    s = warp_sum(s);
    const float mu = s / N;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int c = lane + 32 * i;
        if (c * 4 < N) {
            const float a = v[i].x - mu, b = v[i].y - mu, cc = v[i].z - mu, d = v[i].w - mu;
            q += (a * a + b * b) + (cc * cc + d * d);
        }
    }
    q = warp_sum(q);
    const float scale = rsqrtf((1.0f / N) * q + eps);
    float4* ys = reinterpret_cast<float4*>(y + seg * N);
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int c = lane + 32 * i;
        if (c * 4 < N) {
            float4 o;
            o.x = 1.0f * ((v[i].x - mu) * scale) + 0.0f;
            o.y = 1.0f * ((v[i].y - mu) * scale) + 0.0f;
            o.z = 1.0f * ((v[i].z - mu) * scale) + 0.0f;
            o.w = 1.0f * ((v[i].w - mu) * scale) + 0.0f;
            ys[c] = o;
        }
    }
    if (lane == 0) {
        if (mean) mean[seg] = mu;
        sqdev[seg] = q;
    }
}

template <int V>
__global__ void seg_norm_fwd_warp(const float* __restrict__ x, float* __restrict__ y, float* __restrict__ mean,
                                  float* __restrict__ sqdev, int64_t segs, int N, float eps) {
    pdl_entry();
    norm_fwd_warp<V, false>(x, nullptr, nullptr, y, mean, sqdev, segs, N, eps);
}

template <int V>
__global__ void add_norm_fwd_warp(const float* __restrict__ x, const float* __restrict__ r, float* __restrict__ xr,
                                  float* __restrict__ y, float* __restrict__ mean, float* __restrict__ sqdev,
                                  int64_t segs, int N, float eps) {
    pdl_entry();
    norm_fwd_warp<V, true>(x, r, xr, y, mean, sqdev, segs, N, eps);
}

template <int V>
__global__ void seg_norm_bwd_warp(const float* __restrict__ y, const float* __restrict__ gy,
                                  const float* __restrict__ sqdev, float* __restrict__ gx, int64_t segs, int N,
                                  float eps) {
    pdl_entry();
    const int lane = threadIdx.x & 31;
    const int64_t seg = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (seg >= segs) return;
    const float4* ys = reinterpret_cast<const float4*>(y + seg * N);
    const float4* gs = reinterpret_cast<const float4*>(gy + seg * N);
    float4 yv[V], gv[V];
    float sg = 0.f, sgy = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int c = lane + 32 * i;
        if (c * 4 < N) {
            yv[i] = ys[c];
            gv[i] = gs[c];
            sg += (gv[i].x + gv[i].y) + (gv[i].z + gv[i].w);
            sgy += (gv[i].x * yv[i].x + gv[i].y * yv[i].y) + (gv[i].z * yv[i].z + gv[i].w * yv[i].w);
        } else {
            yv[i] = gv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    sg = warp_sum(sg);
    sgy = warp_sum(sgy);
    const float rstd = rsqrtf(sqdev[seg] / N + eps);
    const float mg = sg / N, mgy = sgy / N;
    float4* xs = reinterpret_cast<float4*>(gx + seg * N);
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int c = lane + 32 * i;
        if (c * 4 < N) {
            float4 o = xs[c];
            o.x += rstd * (1.0f * gv[i].x - mg - yv[i].x * mgy);
            o.y += rstd * (1.0f * gv[i].y - mg - yv[i].y * mgy);
            o.z += rstd * (1.0f * gv[i].z - mg - yv[i].z * mgy);
            o.w += rstd * (1.0f * gv[i].w - mg - yv[i].w * mgy);
            xs[c] = o;
        }
    }
}

// ----------------------------- block per segment --------------------------
__global__ void seg_norm_fwd_block(const float* __restrict__ x, float* __restrict__ y, float* __restrict__ mean,
                                   float* __restrict__ sqdev, int N, float eps) {
    pdl_entry();
    __shared__ float scratch[32];
    const int64_t seg = blockIdx.x;
    const float* xs = x + seg * N;
    float s = 0.f;
    for (int i = threadIdx.x; i < N; i += blockDim.x) s += xs[i];
    s = block_sum(s, scratch);
    const float mu = s / N;
    float q = 0.f;
    for (int i = threadIdx.x; i < N; i += blockDim.x) {
        const float d = xs[i] - mu;
        q += d * d;
    }
    q = block_sum(q, scratch);
    const float scale = rsqrtf((1.0f / N) * q + eps);
    float* ys = y + seg * N;
    for (int i = threadIdx.x; i < N; i += blockDim.x) ys[i] = 1.0f * ((xs[i] - mu) * scale) + 0.0f;
    if (threadIdx.x == 0) {
        if (mean) mean[seg] = mu;
        sqdev[seg] = q;
    }
}

__global__ void seg_norm_bwd_block(const float* __restrict__ y, const float* __restrict__ gy,
                                   const float* __restrict__ sqdev, float* __restrict__ gx, int N, float eps) {
    pdl_entry();
    __shared__ float scratch[32];
    const int64_t seg = blockIdx.x;
    const float* ys = y + seg * N;
    const float* gs = gy + seg * N;
    float sg = 0.f, sgy = 0.f;
    for (int i = threadIdx.x; i < N; i += blockDim.x) {
        const float g = gs[i];
        sg += g;
        sgy += g * ys[i];
    }
    sg = block_sum(sg, scratch);
    sgy = block_sum(sgy, scratch);
    const float rstd = rsqrtf(sqdev[seg] / N + eps);
    const float mg = sg / N, mgy = sgy / N;
    float* xs = gx + seg * N;
    for (int i = threadIdx.x; i < N; i += blockDim.x) xs[i] += rstd * (1.0f * gs[i] - mg - ys[i] * mgy);
}

// --------------------------- cluster per segment ----------------------------
// A segment too long for one warp is split over the CL CTAs of a thread-block
// cluster (CTA `rank` owns floats [rank*slice, (rank+1)*slice)); each thread
// keeps its V float4 in registers, so the input is read once and the output
// written once.  The CTAs' partial sums meet in distributed shared memory and
// every CTA adds them in rank order, so all of them see the same totals.
// Statistics as the block path: mean first, then the squared deviations.
template <int V>
__global__ void __launch_bounds__(kBlock) seg_norm_fwd_cluster(const float* __restrict__ x, float* __restrict__ y,
                                                               float* __restrict__ mean, float* __restrict__ sqdev,
                                                               int N, int slice, float eps) {
    pdl_entry();
    cg::cluster_group cl = cg::this_cluster();
    __shared__ float scratch[32];
    __shared__ float part[2];
    const int CL = (int)cl.num_blocks(), rank = (int)cl.block_rank();
    const int64_t seg = blockIdx.x / CL;
    const int lo = rank * slice;
    const int n = min(slice, N - lo);
    const float4* xs = reinterpret_cast<const float4*>(x + seg * N + lo);
    float4 v[V];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int e = (i * kBlock + threadIdx.x) * 4;
        v[i] = e < n ? xs[e / 4] : make_float4(0.f, 0.f, 0.f, 0.f);
        s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    }
    s = block_sum(s, scratch);
    if (threadIdx.x == 0) part[0] = s;
    cl.sync();
    float tot = 0.f;
    for (int r = 0; r < CL; ++r) tot += *cl.map_shared_rank(&part[0], r);
    const float mu = tot / N;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int e = (i * kBlock + threadIdx.x) * 4;
        if (e < n) {
            const float a = v[i].x - mu, b = v[i].y - mu, c = v[i].z - mu, d = v[i].w - mu;
            q += (a * a + b * b) + (c * c + d * d);
        }
    }
    q = block_sum(q, scratch);
    if (threadIdx.x == 0) part[1] = q;
    cl.sync();
    float qt = 0.f;
    for (int r = 0; r < CL; ++r) qt += *cl.map_shared_rank(&part[1], r);
    const float scale = rsqrtf((1.0f / N) * qt + eps);
    float4* ys = reinterpret_cast<float4*>(y + seg * N + lo);
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int e = (i * kBlock + threadIdx.x) * 4;
        if (e < n)
            ys[e / 4] = make_float4((v[i].x - mu) * scale, (v[i].y - mu) * scale, (v[i].z - mu) * scale,
                                    (v[i].w - mu) * scale);
    }
    if (rank == 0 && threadIdx.x == 0) {
        if (mean) mean[seg] = mu;
        sqdev[seg] = qt;
    }
    cl.sync();  // peers may still be reading part[]
}

template <int V>
__global__ void __launch_bounds__(kBlock) seg_norm_bwd_cluster(const float* __restrict__ y,
                                                               const float* __restrict__ gy,
                                                               const float* __restrict__ sqdev,
                                                               float* __restrict__ gx, int N, int slice, float eps) {
    pdl_entry();
    cg::cluster_group cl = cg::this_cluster();
    __shared__ float scratch[32];
    __shared__ float part[2];
    const int CL = (int)cl.num_blocks(), rank = (int)cl.block_rank();
    const int64_t seg = blockIdx.x / CL;
    const int lo = rank * slice;
    const int n = min(slice, N - lo);
    const float4* ys = reinterpret_cast<const float4*>(y + seg * N + lo);
    const float4* gs = reinterpret_cast<const float4*>(gy + seg * N + lo);
    float4 yv[V], gv[V];
    float sg = 0.f, sgy = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int e = (i * kBlock + threadIdx.x) * 4;
        if (e < n) {
            yv[i] = ys[e / 4];
            gv[i] = gs[e / 4];
        } else {
            yv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            gv[i] = yv[i];
        }
        sg += (gv[i].x + gv[i].y) + (gv[i].z + gv[i].w);
        sgy += (gv[i].x * yv[i].x + gv[i].y * yv[i].y) + (gv[i].z * yv[i].z + gv[i].w * yv[i].w);
    }
    sg = block_sum(sg, scratch);
    sgy = block_sum(sgy, scratch);
    if (threadIdx.x == 0) {
        part[0] = sg;
        part[1] = sgy;
    }
    cl.sync();
    float tg = 0.f, tgy = 0.f;
    for (int r = 0; r < CL; ++r) {
        const float* pr = cl.map_shared_rank(part, r);
        tg += pr[0];
        tgy += pr[1];
    }
    const float rstd = rsqrtf(sqdev[seg] / N + eps);
    const float mg = tg / N, mgy = tgy / N;
    float4* xs = reinterpret_cast<float4*>(gx + seg * N + lo);
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int e = (i * kBlock + threadIdx.x) * 4;
        if (e < n) {
            float4 o = xs[e / 4];
            o.x += rstd * (1.0f * gv[i].x - mg - yv[i].x * mgy);
            o.y += rstd * (1.0f * gv[i].y - mg - yv[i].y * mgy);
            o.z += rstd * (1.0f * gv[i].z - mg - yv[i].z * mgy);
            o.w += rstd * (1.0f * gv[i].w - mg - yv[i].w * mgy);
            xs[e / 4] = o;
        }
    }
    cl.sync();  // peers may still be reading part[]
}

// Cluster shape for a segment of N floats: CL CTAs (<= 8, the portable
// cluster size) of V float4 per thread, V <= 8.  False if N is too long.
bool cluster_shape(int N, int& CL, int& V) {
    CL = 1;
    while (CL < 8 && (int64_t)CL * 4096 < N) CL *= 2;
    V = (N + CL * kBlock * 4 - 1) / (CL * kBlock * 4);
    return V <= 8;
}

// LayerBackward with channels > 1 keeps the reference's index map: only the
// first batch*row*col elements are updated and element idx uses the
// statistics of sample idx/(row*col) (Engine/kernels.cu:849-862), while the
// statistics themselves are sums over the whole sample (LayerMean over
// C*H*W).  Block b sums sample b and then updates elements
// [b*row*col, (b+1)*row*col); the sums read y and gy only, so no block reads
// what another writes.
__global__ void ln_bwd_channels_block(const float* __restrict__ y, const float* __restrict__ gy,
                                      const float* __restrict__ sqdev, float* __restrict__ gx, int64_t N, int64_t rc,
                                      float eps) {
    pdl_entry();
    __shared__ float scratch[32];
    const int64_t b = blockIdx.x;
    float sg = 0.f, sgy = 0.f;
    for (int64_t i = threadIdx.x; i < N; i += blockDim.x) {
        const float g = gy[b * N + i];
        sg += g;
        sgy += g * y[b * N + i];
    }
    sg = block_sum(sg, scratch);
    sgy = block_sum(sgy, scratch);
    const float Nf = (float)N;
    const float rstd = rsqrtf(sqdev[b] / Nf + eps);
    for (int64_t i = b * rc + threadIdx.x; i < (b + 1) * rc; i += blockDim.x)
        gx[i] += rstd * (1.0f * gy[i] - (sg / Nf) - y[i] * (sgy / Nf));
}

}  // namespace

static int seg_norm_fwd(const float* x, float* y, float* mean, float* sqdev, int64_t segs, int N, float eps,
                        cudaStream_t st) {
    if (segs == 0) return MLE_OK;
    if (N % 4 == 0 && N <= kWarpMaxN && aligned16(x) && aligned16(y)) {
        const int wpb = 8;  // warps per block
        const unsigned grid = (unsigned)((segs + wpb - 1) / wpb);
        if (N <= 128) launch_k(seg_norm_fwd_warp<1>, grid, 32 * wpb, 0, st, x, y, mean, sqdev, segs, N, eps);
        else if (N <= 256) launch_k(seg_norm_fwd_warp<2>, grid, 32 * wpb, 0, st, x, y, mean, sqdev, segs, N, eps);
        else if (N <= 512) launch_k(seg_norm_fwd_warp<4>, grid, 32 * wpb, 0, st, x, y, mean, sqdev, segs, N, eps);
        else launch_k(seg_norm_fwd_warp<8>, grid, 32 * wpb, 0, st, x, y, mean, sqdev, segs, N, eps);
    } else if (int CL, V; N % 4 == 0 && aligned16(x) && aligned16(y) && cluster_shape(N, CL, V)) {
        const int slice = V * kBlock * 4;
        const dim3 grid((unsigned)(segs * CL));
        if (V <= 1) launch_kc(seg_norm_fwd_cluster<1>, grid, kBlock, CL, st, x, y, mean, sqdev, N, slice, eps);
        else if (V <= 2) launch_kc(seg_norm_fwd_cluster<2>, grid, kBlock, CL, st, x, y, mean, sqdev, N, slice, eps);
        else if (V <= 4) launch_kc(seg_norm_fwd_cluster<4>, grid, kBlock, CL, st, x, y, mean, sqdev, N, slice, eps);
        else launch_kc(seg_norm_fwd_cluster<8>, grid, kBlock, CL, st, x, y, mean, sqdev, N, slice, eps);
    } else {
        launch_k(seg_norm_fwd_block, (unsigned)segs, kBlock, 0, st, x, y, mean, sqdev, N, eps);
    }
    return launch_status();
}

static int seg_norm_bwd(const float* y, const float* gy, const float* sqdev, float* gx, int64_t segs, int N, float eps,
                        cudaStream_t st) {
    if (segs == 0) return MLE_OK;
    if (N % 4 == 0 && N <= kWarpMaxN && aligned16(y) && aligned16(gy) && aligned16(gx)) {
        const int wpb = 8;
        const unsigned grid = (unsigned)((segs + wpb - 1) / wpb);
        if (N <= 128) launch_k(seg_norm_bwd_warp<1>, grid, 32 * wpb, 0, st, y, gy, sqdev, gx, segs, N, eps);
        else if (N <= 256) launch_k(seg_norm_bwd_warp<2>, grid, 32 * wpb, 0, st, y, gy, sqdev, gx, segs, N, eps);
        else if (N <= 512) launch_k(seg_norm_bwd_warp<4>, grid, 32 * wpb, 0, st, y, gy, sqdev, gx, segs, N, eps);
        else launch_k(seg_norm_bwd_warp<8>, grid, 32 * wpb, 0, st, y, gy, sqdev, gx, segs, N, eps);
    } else if (int CL, V; N % 4 == 0 && aligned16(y) && aligned16(gy) && aligned16(gx) && cluster_shape(N, CL, V)) {
        const int slice = V * kBlock * 4;
        const dim3 grid((unsigned)(segs * CL));
        if (V <= 1) launch_kc(seg_norm_bwd_cluster<1>, grid, kBlock, CL, st, y, gy, sqdev, gx, N, slice, eps);
        else if (V <= 2) launch_kc(seg_norm_bwd_cluster<2>, grid, kBlock, CL, st, y, gy, sqdev, gx, N, slice, eps);
        else if (V <= 4) launch_kc(seg_norm_bwd_cluster<4>, grid, kBlock, CL, st, y, gy, sqdev, gx, N, slice, eps);
        else launch_kc(seg_norm_bwd_cluster<8>, grid, kBlock, CL, st, y, gy, sqdev, gx, N, slice, eps);
    } else {
        launch_k(seg_norm_bwd_block, (unsigned)segs, kBlock, 0, st, y, gy, sqdev, gx, N, eps);
    }
    return launch_status();
}

}  // namespace mle

using namespace mle;

extern "C" {

int mle_layernorm_fwd(const float* x, float* y, float* mean, float* sqdev, int batch, int channels, int row, int col,
                      float eps, mle_stream_t stream) {
    if (batch < 0 || channels <= 0 || row <= 0 || col <= 0 || !x || !y || !sqdev) return MLE_ERR_ARG;
    const int64_t N = (int64_t)channels * row * col;
    if (N > (1ll << 30)) return MLE_ERR_UNSUPPORTED;
    return seg_norm_fwd(x, y, mean, sqdev, batch, (int)N, eps, as_stream(stream));
}

int mle_add_layernorm_fwd(const float* x, const float* r, float* xr, float* y, float* mean, float* sqdev, int batch,
                          int channels, int row, int col, float eps, mle_stream_t stream) {
    if (batch < 0 || channels <= 0 || row <= 0 || col <= 0 || !x || !r || !xr || !y || !sqdev) return MLE_ERR_ARG;
    const int64_t N = (int64_t)channels * row * col;
    if (N % 4 != 0 || N > kWarpMaxN || !aligned16(x) || !aligned16(r) || !aligned16(xr) || !aligned16(y))
        return MLE_ERR_UNSUPPORTED;
    if (batch == 0) return MLE_OK;
    const int wpb = 8;  // warps per block, one segment each
    const unsigned grid = (unsigned)((batch + wpb - 1) / wpb);
    const int n = (int)N;
    cudaStream_t st = as_stream(stream);
    const int64_t segs = batch;
    if (N <= 128) launch_k(add_norm_fwd_warp<1>, grid, 32 * wpb, 0, st, x, r, xr, y, mean, sqdev, segs, n, eps);
    else if (N <= 256) launch_k(add_norm_fwd_warp<2>, grid, 32 * wpb, 0, st, x, r, xr, y, mean, sqdev, segs, n, eps);
    else if (N <= 512) launch_k(add_norm_fwd_warp<4>, grid, 32 * wpb, 0, st, x, r, xr, y, mean, sqdev, segs, n, eps);
    else launch_k(add_norm_fwd_warp<8>, grid, 32 * wpb, 0, st, x, r, xr, y, mean, sqdev, segs, n, eps);
    return launch_status();
}

int mle_layernorm_bwd(const float* y, const float* gy, const float* sqdev, float* gx, int batch, int channels, int row,
                      int col, float eps, mle_stream_t stream) {
    if (batch < 0 || channels <= 0 || row <= 0 || col <= 0 || !y || !gy || !sqdev || !gx) return MLE_ERR_ARG;
    const int64_t N = (int64_t)channels * row * col;
    if (N > (1ll << 30)) return MLE_ERR_UNSUPPORTED;
    if (channels == 1) return seg_norm_bwd(y, gy, sqdev, gx, batch, (int)N, eps, as_stream(stream));
    if (batch == 0) return MLE_OK;
    launch_k(ln_bwd_channels_block, (unsigned)batch, kBlock, 0, as_stream(stream), y, gy, sqdev, gx, N,
                                                                             (int64_t)row * col, eps);
    return launch_status();
}

int mle_groupnorm_fwd(const float* x, float* y, float* mean, float* sqdev, int batch, int channels, int groups,
                      int row, int col, float eps, mle_stream_t stream) {
    if (batch < 0 || channels <= 0 || groups <= 0 || channels % groups != 0 || row <= 0 || col <= 0 || !x || !y ||
        !sqdev)
        return MLE_ERR_ARG;
    const int64_t N = (int64_t)(channels / groups) * row * col;
    if (N > (1ll << 30)) return MLE_ERR_UNSUPPORTED;
    return seg_norm_fwd(x, y, mean, sqdev, (int64_t)batch * groups, (int)N, eps, as_stream(stream));
}

int mle_groupnorm_bwd(const float* y, const float* gy, const float* sqdev, float* gx, int batch, int channels,
                      int groups, int row, int col, float eps, mle_stream_t stream) {
    if (batch < 0 || channels <= 0 || groups <= 0 || channels % groups != 0 || row <= 0 || col <= 0 || !y || !gy ||
        !sqdev || !gx)
        return MLE_ERR_ARG;
    const int64_t N = (int64_t)(channels / groups) * row * col;
    if (N > (1ll << 30)) return MLE_ERR_UNSUPPORTED;
    return seg_norm_bwd(y, gy, sqdev, gx, (int64_t)batch * groups, (int)N, eps, as_stream(stream));
}

}  // extern "C"
