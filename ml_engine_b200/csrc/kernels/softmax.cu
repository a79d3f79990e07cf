// Softmax (row- and column-wise), its backward, softmax cross-entropy and
// mean squared error.
//
// Column-wise softmax (the reference's "type 1", used by every attention
// block) assigns one thread per column and walks the rows in order, which is
// the reference's own summation order (FindMax / exponentiate[M] / SumRows /
// Scale_arr, Engine/kernels.cu:2003-2147), so its results are bitwise the
// reference's while the loads stay coalesced across the warp.  Row-wise
// softmax reduces a row with a block, which reorders the float sums.
#include <float.h>
#include <math.h>

#include "common.cuh"

namespace mle {
namespace {

constexpr int kColThreads = 128;
constexpr int kRowThreads = 256;

// ------------------------------ column-wise --------------------------------
__global__ void softmax_col_fwd(const float* __restrict__ x, float* __restrict__ y, int rows, int cols, int causal) {
    pdl_entry();
    const int64_t mat = blockIdx.y;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    const float* xm = x + mat * (int64_t)rows * cols;
    float* ym = y + mat * (int64_t)rows * cols;
    float m = -FLT_MAX;
    for (int r = 0; r < rows; ++r) m = fmaxf(m, xm[(int64_t)r * cols + c]);
    float s = 0.0f;
    for (int r = 0; r < rows; ++r) {
        const float e = (causal && c > r) ? 0.0f : expf(xm[(int64_t)r * cols + c] - m);
        ym[(int64_t)r * cols + c] = e;
        s += e;
    }
    if (s < 1e-45f) s = 1.0f;
    for (int r = 0; r < rows; ++r) ym[(int64_t)r * cols + c] /= s;
}

__global__ void softmax_col_bwd(const float* __restrict__ y, const float* __restrict__ gy, float* __restrict__ gx,
                                int rows, int cols) {
    pdl_entry();
    const int64_t mat = blockIdx.y;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    const int64_t base = mat * (int64_t)rows * cols + c;
    float dot = 0.0f;
    for (int r = 0; r < rows; ++r) dot += gy[base + (int64_t)r * cols] * y[base + (int64_t)r * cols];
    for (int r = 0; r < rows; ++r) {
        const int64_t i = base + (int64_t)r * cols;
        gx[i] += y[i] * (gy[i] - dot);
    }
}

// -------------------------------- row-wise ---------------------------------
// One block per row; each thread caches up to EPT values (float4-strided).
template <int EPT>
__device__ __forceinline__ void load_row(const float* __restrict__ row, int cols, float (&v)[EPT]) {
#pragma unroll
    for (int k = 0; k < EPT / 4; ++k) {
        const int c = (k * blockDim.x + threadIdx.x) * 4;
        if (c < cols) {
            const float4 t = *reinterpret_cast<const float4*>(row + c);
            v[4 * k] = t.x; v[4 * k + 1] = t.y; v[4 * k + 2] = t.z; v[4 * k + 3] = t.w;
        } else {
            v[4 * k] = v[4 * k + 1] = v[4 * k + 2] = v[4 * k + 3] = -FLT_MAX;
        }
    }
}

template <int EPT>
__device__ __forceinline__ float row_softmax_regs(float (&v)[EPT], int cols, int row_idx, int causal, float* scratch) {
    float m = -FLT_MAX;
#pragma unroll
    for (int k = 0; k < EPT; ++k) m = fmaxf(m, v[k]);
    // block max
    m = warp_max(m);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = m;
    __syncthreads();
    {
        const int nw = blockDim.x >> 5;
        float t = ((threadIdx.x & 31) < nw) ? scratch[threadIdx.x & 31] : -FLT_MAX;
        m = warp_max(t);
    }
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < EPT / 4; ++k) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int c = (k * blockDim.x + threadIdx.x) * 4 + j;
            float e = 0.f;
            if (c < cols && !(causal && c > row_idx)) e = expf(v[4 * k + j] - m);
            v[4 * k + j] = e;
            s += e;
        }
    }
    s = block_sum(s, scratch);
    if (s < 1e-45f) s = 1.0f;
    return s;
}

template <int EPT>
__global__ void softmax_row_fwd_cached(const float* __restrict__ x, float* __restrict__ y, int rows, int cols,
                                       int causal) {
    pdl_entry();
    __shared__ float scratch[32];
    const int64_t row = blockIdx.x;
    float v[EPT];
    load_row<EPT>(x + row * cols, cols, v);
    const float s = row_softmax_regs<EPT>(v, cols, (int)(row % rows), causal, scratch);
    float* yr = y + row * cols;
#pragma unroll
    for (int k = 0; k < EPT / 4; ++k) {
        const int c = (k * blockDim.x + threadIdx.x) * 4;
        if (c < cols)
            *reinterpret_cast<float4*>(yr + c) =
                make_float4(v[4 * k] / s, v[4 * k + 1] / s, v[4 * k + 2] / s, v[4 * k + 3] / s);
    }
}

__global__ void softmax_row_fwd_generic(const float* __restrict__ x, float* __restrict__ y, int rows, int cols,
                                        int causal) {
    pdl_entry();
    __shared__ float scratch[32];
    const int64_t row = blockIdx.x;
    const int r_in = (int)(row % rows);
    const float* xr = x + row * cols;
    float* yr = y + row * cols;
    float m = -FLT_MAX;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) m = fmaxf(m, xr[c]);
    m = warp_max(m);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = m;
    __syncthreads();
    {
        const int nw = blockDim.x >> 5;
        float t = ((threadIdx.x & 31) < nw) ? scratch[threadIdx.x & 31] : -FLT_MAX;
        m = warp_max(t);
    }
    float s = 0.f;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        const float e = (causal && c > r_in) ? 0.0f : expf(xr[c] - m);
        yr[c] = e;
        s += e;
    }
    s = block_sum(s, scratch);
    if (s < 1e-45f) s = 1.0f;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) yr[c] /= s;
}

__global__ void softmax_row_bwd(const float* __restrict__ y, const float* __restrict__ gy, float* __restrict__ gx,
                                int cols) {
    pdl_entry();
    __shared__ float scratch[32];
    const int64_t row = blockIdx.x;
    const float* yr = y + row * cols;
    const float* gr = gy + row * cols;
    float* xr = gx + row * cols;
    float dot = 0.f;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) dot += gr[c] * yr[c];
    dot = block_sum(dot, scratch);
    for (int c = threadIdx.x; c < cols; c += blockDim.x) xr[c] += yr[c] * (gr[c] - dot);
}

// ------------------------- softmax cross-entropy ---------------------------
// x / batch_div; binv = 1 / batch_div when that is exact (a power of two),
// then the product is the same number, else 0 and the quotient is taken.
__device__ __forceinline__ float div_batch(float x, float batch_div, float binv) {
    return binv != 0.0f ? x * binv : x / batch_div;
}

template <int EPT>
__global__ void smce_fwd_cached(const float* __restrict__ logits, const float* __restrict__ target,
                                float* __restrict__ probs, float* __restrict__ loss, float* __restrict__ grad,
                                float batch_div, float binv, int cols, double total) {
    pdl_entry();
    __shared__ float scratch[32];
    __shared__ double dscratch[32];
    const int64_t row = blockIdx.x;
    float v[EPT];
    load_row<EPT>(logits + row * cols, cols, v);
    const float inv_s = 1.0f / row_softmax_regs<EPT>(v, cols, 0, 0, scratch);
    double part = 0.0;
#pragma unroll
    for (int k = 0; k < EPT / 4; ++k) {
        const int c = (k * blockDim.x + threadIdx.x) * 4;
        if (c < cols) {
            const float4 t4 = *reinterpret_cast<const float4*>(target + row * cols + c);
            const float tt[4] = {t4.x, t4.y, t4.z, t4.w};
            float p[4], g[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                p[j] = v[4 * k + j] * inv_s;
                // -t*log(p+1e-27) is -0 where t == 0, so skipping those terms
                // leaves the double sum unchanged.
                if (tt[j] != 0.0f) part += -(double)tt[j] * log((double)p[j] + 1e-27);
                g[j] = div_batch(p[j] + (-1.0f) * tt[j], batch_div, binv);
            }
            if (probs) *reinterpret_cast<float4*>(probs + row * cols + c) = make_float4(p[0], p[1], p[2], p[3]);
            if (grad) *reinterpret_cast<float4*>(grad + row * cols + c) = make_float4(g[0], g[1], g[2], g[3]);
        }
    }
    part = block_sum(part, dscratch);
    if (threadIdx.x == 0) atomicAdd(loss, (float)(part / total));
}

// The same with the target given as one class index per row (the one-hot
// row of the reference's dense target: 1 at `label`, 0 elsewhere; a label
// outside [0, cols) is a row of zeros).  Each row's loss term and gradient
// are those of the dense kernel on the one-hot target, bit for bit.
template <int EPT>
__global__ void smce_index_fwd_cached(const float* __restrict__ logits, const int32_t* __restrict__ labels,
                                      float* __restrict__ probs, float* __restrict__ loss, float* __restrict__ grad,
                                      float batch_div, float binv, int cols, double total) {
    pdl_entry();
    __shared__ float scratch[32];
    const int64_t row = blockIdx.x;
    const int label = labels[row];
    float v[EPT];
    load_row<EPT>(logits + row * cols, cols, v);
    const float inv_s = 1.0f / row_softmax_regs<EPT>(v, cols, 0, 0, scratch);
#pragma unroll
    for (int k = 0; k < EPT / 4; ++k) {
        const int c = (k * blockDim.x + threadIdx.x) * 4;
        if (c < cols) {
            float p[4], g[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                p[j] = v[4 * k + j] * inv_s;
                const float tt = (c + j == label) ? 1.0f : 0.0f;
                // the row's one loss term (the dense kernel's block sum of
                // this term and zeros is this term), from the thread holding it
                if (tt != 0.0f) atomicAdd(loss, (float)(-(double)tt * log((double)p[j] + 1e-27) / total));
                g[j] = div_batch(p[j] + (-1.0f) * tt, batch_div, binv);
            }
            if (probs) *reinterpret_cast<float4*>(probs + row * cols + c) = make_float4(p[0], p[1], p[2], p[3]);
            if (grad) *reinterpret_cast<float4*>(grad + row * cols + c) = make_float4(g[0], g[1], g[2], g[3]);
        }
    }
}

__global__ void smce_index_bwd_kernel(const float* __restrict__ probs, const int32_t* __restrict__ labels,
                                      const float* __restrict__ upstream, float* __restrict__ grad, float batch_div,
                                      float binv, int cols, int64_t n) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const int64_t row = i / cols;
        const float tt = (int)(i - row * cols) == labels[row] ? 1.0f : 0.0f;
        float g = probs[i] + (-1.0f) * tt;
        if (upstream) g *= upstream[0];
        grad[i] = div_batch(g, batch_div, binv);
    }
}

__global__ void smce_fwd_generic(const float* __restrict__ logits, const float* __restrict__ target,
                                 float* __restrict__ probs, float* __restrict__ loss, float* __restrict__ grad,
                                 float batch_div, float binv, int cols, double total) {
    pdl_entry();
    __shared__ float scratch[32];
    __shared__ double dscratch[32];
    const int64_t row = blockIdx.x;
    const float* xr = logits + row * cols;
    const float* tr = target + row * cols;
    float m = -FLT_MAX;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) m = fmaxf(m, xr[c]);
    m = warp_max(m);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = m;
    __syncthreads();
    {
        const int nw = blockDim.x >> 5;
        float t = ((threadIdx.x & 31) < nw) ? scratch[threadIdx.x & 31] : -FLT_MAX;
        m = warp_max(t);
    }
    float s = 0.f;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) s += expf(xr[c] - m);
    s = block_sum(s, scratch);
    if (s < 1e-45f) s = 1.0f;
    double part = 0.0;
    const float inv_s = 1.0f / s;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        const float p = expf(xr[c] - m) * inv_s;
        const float t = tr[c];
        if (t != 0.0f) part += -(double)t * log((double)p + 1e-27);
        if (probs) probs[row * cols + c] = p;
        if (grad) grad[row * cols + c] = div_batch(p + (-1.0f) * t, batch_div, binv);
    }
    part = block_sum(part, dscratch);
    if (threadIdx.x == 0) atomicAdd(loss, (float)(part / total));
}

__global__ void smce_bwd_kernel(const float* __restrict__ probs, const float* __restrict__ target,
                                const float* __restrict__ upstream, float* __restrict__ grad, float batch_div,
                                float binv, int64_t n) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        float g = probs[i] + (-1.0f) * target[i];
        if (upstream) g *= upstream[0];
        grad[i] = div_batch(g, batch_div, binv);
    }
}

// ------------------------------------ MSE -----------------------------------
__global__ void mse_fwd_kernel(const float* __restrict__ x, const float* __restrict__ t, float* __restrict__ loss,
                               int64_t n) {
    pdl_entry();
    __shared__ double dscratch[32];
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    double part = 0.0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const double d = (double)t[i] - (double)x[i];
        part += d * d;
    }
    part = block_sum(part, dscratch);
    if (threadIdx.x == 0) atomicAdd(loss, (float)(part / (double)n));
}

__global__ void mse_bwd_kernel(const float* __restrict__ x, const float* __restrict__ t,
                               const float* __restrict__ upstream, float* __restrict__ gx, int64_t n) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const float nf = (float)n;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        if (!upstream) gx[i] += 2.0f * (x[i] - t[i]) / nf;
        else gx[i] += (2.0f * (x[i] - t[i]) * upstream[0]) / nf;
    }
}

}  // namespace
}  // namespace mle

using namespace mle;

extern "C" {

int mle_softmax_fwd(const float* x, float* y, int64_t bc, int rows, int cols, int axis, int causal,
                    mle_stream_t stream) {
    if (bc < 0 || rows <= 0 || cols <= 0 || (axis != 0 && axis != 1) || !x || !y) return MLE_ERR_ARG;
    if (bc == 0) return MLE_OK;
    cudaStream_t st = as_stream(stream);
    if (axis == 1) {
        if (bc > 65535) return MLE_ERR_UNSUPPORTED;
        dim3 grid((cols + kColThreads - 1) / kColThreads, (unsigned)bc);
        launch_k(softmax_col_fwd, grid, kColThreads, 0, st, x, y, rows, cols, causal);
        return launch_status();
    }
    const int64_t nrows = bc * rows;
    if (cols % 4 == 0 && cols <= 4 * kRowThreads * 4 && aligned16(x) && aligned16(y)) {
        if (cols <= 4 * kRowThreads)
            launch_k(softmax_row_fwd_cached<4>, (unsigned)nrows, kRowThreads, 0, st, x, y, rows, cols, causal);
        else if (cols <= 8 * kRowThreads)
            launch_k(softmax_row_fwd_cached<8>, (unsigned)nrows, kRowThreads, 0, st, x, y, rows, cols, causal);
        else
            launch_k(softmax_row_fwd_cached<16>, (unsigned)nrows, kRowThreads, 0, st, x, y, rows, cols, causal);
    } else {
        launch_k(softmax_row_fwd_generic, (unsigned)nrows, kRowThreads, 0, st, x, y, rows, cols, causal);
    }
    return launch_status();
}

int mle_softmax_bwd(const float* y, const float* gy, float* gx, int64_t bc, int rows, int cols, int axis,
                    mle_stream_t stream) {
    if (bc < 0 || rows <= 0 || cols <= 0 || (axis != 0 && axis != 1) || !y || !gy || !gx) return MLE_ERR_ARG;
    if (bc == 0) return MLE_OK;
    cudaStream_t st = as_stream(stream);
    if (axis == 1) {
        if (bc > 65535) return MLE_ERR_UNSUPPORTED;
        dim3 grid((cols + kColThreads - 1) / kColThreads, (unsigned)bc);
        launch_k(softmax_col_bwd, grid, kColThreads, 0, st, y, gy, gx, rows, cols);
    } else {
        launch_k(softmax_row_bwd, (unsigned)(bc * rows), kRowThreads, 0, st, y, gy, gx, cols);
    }
    return launch_status();
}

}  // extern "C"

// 1 / b when it is exact (b a power of two), else 0 (see div_batch)
static float exact_inverse(float b) {
    int e = 0;
    const float m = frexpf(b, &e);
    return (m == 0.5f || m == -0.5f) ? 1.0f / b : 0.0f;
}

extern "C" {

int mle_softmax_ce_fwd(const float* logits, const float* target, float* probs, float* loss, float* grad,
                       float batch_div, int64_t rows, int cols, mle_stream_t stream) {
    if (rows < 0 || cols <= 0 || !logits || !target || !loss || batch_div == 0.0f) return MLE_ERR_ARG;
    cudaStream_t st = as_stream(stream);
    if (cudaMemsetAsync(loss, 0, sizeof(float), st) != cudaSuccess) return launch_status();
    if (rows == 0) return MLE_OK;
    const double total = (double)rows * (double)cols;
    const float binv = exact_inverse(batch_div);
    const bool vec = cols % 4 == 0 && aligned16(logits) && aligned16(target) && (!probs || aligned16(probs)) &&
                     (!grad || aligned16(grad));
    if (vec && cols <= 4 * kRowThreads)
        launch_k(smce_fwd_cached<4>, (unsigned)rows, kRowThreads, 0, st, logits, target, probs, loss, grad, batch_div, binv, cols, total);
    else if (vec && cols <= 8 * kRowThreads)
        launch_k(smce_fwd_cached<8>, (unsigned)rows, kRowThreads, 0, st, logits, target, probs, loss, grad, batch_div, binv, cols, total);
    else if (vec && cols <= 16 * kRowThreads)
        launch_k(smce_fwd_cached<16>, (unsigned)rows, kRowThreads, 0, st, logits, target, probs, loss, grad, batch_div, binv,
                 cols, total);
    else if (vec && cols <= 32 * kRowThreads)  // two threads' share per thread of a 512-thread block
        launch_k(smce_fwd_cached<16>, (unsigned)rows, 2 * kRowThreads, 0, st, logits, target, probs, loss, grad,
                 batch_div, binv, cols, total);
    else
        launch_k(smce_fwd_generic, (unsigned)rows, kRowThreads, 0, st, logits, target, probs, loss, grad, batch_div, binv, cols,
                 total);
    return launch_status();
}

int mle_softmax_ce_index_fwd(const float* logits, const int32_t* labels, float* probs, float* loss, float* grad,
                             float batch_div, int64_t rows, int cols, mle_stream_t stream) {
    if (rows < 0 || cols <= 0 || !logits || !labels || !loss || batch_div == 0.0f) return MLE_ERR_ARG;
    const bool vec = cols % 4 == 0 && aligned16(logits) && (!probs || aligned16(probs)) && (!grad || aligned16(grad));
    if (!vec || cols > 32 * kRowThreads) return MLE_ERR_UNSUPPORTED;
    cudaStream_t st = as_stream(stream);
    if (cudaMemsetAsync(loss, 0, sizeof(float), st) != cudaSuccess) return launch_status();
    if (rows == 0) return MLE_OK;
    const double total = (double)rows * (double)cols;
    const float binv = exact_inverse(batch_div);
    if (cols <= 4 * kRowThreads)
        launch_k(smce_index_fwd_cached<4>, (unsigned)rows, kRowThreads, 0, st, logits, labels, probs, loss, grad,
                 batch_div, binv, cols, total);
    else if (cols <= 8 * kRowThreads)
        launch_k(smce_index_fwd_cached<8>, (unsigned)rows, kRowThreads, 0, st, logits, labels, probs, loss, grad,
                 batch_div, binv, cols, total);
    else if (cols <= 16 * kRowThreads)
        launch_k(smce_index_fwd_cached<16>, (unsigned)rows, kRowThreads, 0, st, logits, labels, probs, loss, grad,
                 batch_div, binv, cols, total);
    else
        launch_k(smce_index_fwd_cached<16>, (unsigned)rows, 2 * kRowThreads, 0, st, logits, labels, probs, loss, grad,
                 batch_div, binv, cols, total);
    return launch_status();
}

int mle_softmax_ce_index_bwd(const float* probs, const int32_t* labels, const float* upstream, float* grad,
                             float batch_div, int64_t rows, int cols, mle_stream_t stream) {
    if (rows < 0 || cols <= 0 || !probs || !labels || !grad || batch_div == 0.0f) return MLE_ERR_ARG;
    const int64_t n = rows * cols;
    if (n == 0) return MLE_OK;
    launch_k(smce_index_bwd_kernel, grid_for(n, 256), 256, 0, as_stream(stream), probs, labels, upstream, grad,
             batch_div, exact_inverse(batch_div), cols, n);
    return launch_status();
}

int mle_softmax_ce_bwd(const float* probs, const float* target, const float* upstream, float* grad, float batch_div,
                       int64_t n, mle_stream_t stream) {
    if (n < 0 || !probs || !target || !grad || batch_div == 0.0f) return MLE_ERR_ARG;
    if (n == 0) return MLE_OK;
    launch_k(smce_bwd_kernel, grid_for(n, 256), 256, 0, as_stream(stream), probs, target, upstream, grad, batch_div,
             exact_inverse(batch_div), n);
    return launch_status();
}

int mle_mse_fwd(const float* x, const float* target, float* loss, int64_t n, mle_stream_t stream) {
    if (n <= 0 || !x || !target || !loss) return MLE_ERR_ARG;
    cudaStream_t st = as_stream(stream);
    if (cudaMemsetAsync(loss, 0, sizeof(float), st) != cudaSuccess) return launch_status();
    launch_k(mse_fwd_kernel, grid_for(n, 256, 4), 256, 0, st, x, target, loss, n);
    return launch_status();
}

int mle_mse_bwd(const float* x, const float* target, const float* upstream, float* gx, int64_t n,
                mle_stream_t stream) {
    if (n <= 0 || !x || !target || !gx) return MLE_ERR_ARG;
    launch_k(mse_bwd_kernel, grid_for(n, 256), 256, 0, as_stream(stream), x, target, upstream, gx, n);
    return launch_status();
}

}  // extern "C"
