// Elementwise and gather/scatter kernels of the graph-op lambdas.
//
// All kernels are grid-stride loops sized to whole waves of the 148 SMs and
// use 128-bit accesses whenever every pointer is 16-byte aligned.  The
// arithmetic of each op follows the reference kernel named at its entry
// point in include/mle_kernels.h, operation for operation, so results are
// bitwise those of the reference for the elementwise ops.
#include <math.h>
#include <stdio.h>

#include "common.cuh"

namespace mle {

static cudaError_t g_last_cuda_error = cudaSuccess;

void record_cuda_error(cudaError_t e) { g_last_cuda_error = e; }

namespace {

constexpr int kThreads = 256;
constexpr float kPi = 3.14159265359f;  // the reference's float PI constant

// ---------------------------------------------------------------------------
// activation formulas (Engine/kernels.cu:1214-1328)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float act_forward(int kind, float x) {
    switch (kind) {
        case MLE_ACT_RELU: return (x < 0.f) ? 0.0f : x;
        case MLE_ACT_LEAKY_RELU: return (x < 0.f) ? 0.01f * x : x;
        case MLE_ACT_SILU: return x * (1.0f / (1.0f + expf(-x)));
        case MLE_ACT_TANH: return tanhf(x);
        case MLE_ACT_GELU: {
            const float val = sqrtf(2.0f / kPi) * (x + 0.044715f * x * x * x);
            const float th = tanhf(val);
            return 0.5f * x * (1.0f + th);
        }
        default: {  // sigmoid
            const float negexp = expf(-1.0f * x);
            return 1.0f / (1.0f + negexp);
        }
    }
}

// gx + gy * f'(x), with the reference's derivative expressions.
__device__ __forceinline__ float act_backward(int kind, float x, float gy, float gx) {
    switch (kind) {
        case MLE_ACT_RELU: {
            const float mask = (x > 0.0f) ? 1.0f : 0.0f;
            return gx + gy * mask;
        }
        case MLE_ACT_LEAKY_RELU: {
            const float mask = (x < 0.0f) ? 0.01f : 1.0f;
            return gx + gy * mask;
        }
        case MLE_ACT_SILU: {
            const float e = expf(x);
            const float ne = 1.0f / e;
            const float sigma = 1.0f / (1.0f + ne);
            const float d = sigma + (x / (e + ne + 2.0f));
            return gx + gy * d;
        }
        case MLE_ACT_TANH: {
            const float e2 = expf(2.0f * x);
            const float ne2 = 1.0f / e2;
            const float d = 4.0f / (e2 + ne2 + 2.0f);
            return gx + gy * d;
        }
        case MLE_ACT_GELU: {
            const float root = sqrtf(2.0f / kPi);
            const float u = root * (x + 0.044715f * x * x * x);
            const float du = root * (1.0f + 0.134145f * x * x);
            const float t = tanhf(u);
            return gx + (0.5f + 0.5f * t + 0.5f * x * (1.0f - t * t) * du) * gy;
        }
        default: {  // sigmoid
            const float e = expf(x);
            const float ne = 1.0f / e;
            const float d = 1.0f / (e + ne + 2.0f);
            return gx + gy * d;
        }
    }
}

// ---------------------------------------------------------------------------
// generic vectorised map kernels
// ---------------------------------------------------------------------------
__global__ void fill_kernel(float* __restrict__ x, float v, int64_t n) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t n4 = n >> 2;
    float4* x4 = reinterpret_cast<float4*>(x);
    for (int64_t j = i; j < n4; j += stride) x4[j] = make_float4(v, v, v, v);
    for (int64_t j = (n4 << 2) + i; j < n; j += stride) x[j] = v;
}

__global__ void fill_kernel_scalar(float* __restrict__ x, float v, int64_t n) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) x[i] = v;
}

// op codes for the binary map kernel
enum MapOp { OP_COPY = 0, OP_ACCUM = 1, OP_SCALE_WRITE = 2, OP_SCALE_ADD = 3, OP_MUL = 4, OP_MUL_ACC = 5 };

template <int OP>
__device__ __forceinline__ float map1(float x, float y_old, float other, float fscale, double dscale) {
    if (OP == OP_COPY) return x;
    if (OP == OP_ACCUM) return (float)((double)y_old + dscale * (double)x);  // Y += scale*X in double
    if (OP == OP_SCALE_WRITE) return fscale * x;
    if (OP == OP_MUL) return x * other;
    if (OP == OP_MUL_ACC) return y_old + x * other;
    return x + fscale * other;  // OP_SCALE_ADD: z = x + scale*y
}

template <int OP, bool VEC>
__global__ void map_kernel(const float* __restrict__ x, const float* __restrict__ other,
                           float* __restrict__ y, int64_t n, float fscale, double dscale) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t tail = 0;
    if (VEC) {
        const int64_t n4 = n >> 2;
        const float4* x4 = reinterpret_cast<const float4*>(x);
        const float4* o4 = reinterpret_cast<const float4*>(other);
        float4* y4 = reinterpret_cast<float4*>(y);
        for (int64_t j = i0; j < n4; j += stride) {
            const float4 a = x4[j];
            float4 yo = make_float4(0.f, 0.f, 0.f, 0.f), b = make_float4(0.f, 0.f, 0.f, 0.f);
            if (OP == OP_ACCUM || OP == OP_MUL_ACC) yo = y4[j];
            if (OP == OP_SCALE_ADD || OP == OP_MUL || OP == OP_MUL_ACC) b = o4[j];
            float4 r;
            r.x = map1<OP>(a.x, yo.x, b.x, fscale, dscale);
            r.y = map1<OP>(a.y, yo.y, b.y, fscale, dscale);
            r.z = map1<OP>(a.z, yo.z, b.z, fscale, dscale);
            r.w = map1<OP>(a.w, yo.w, b.w, fscale, dscale);
            y4[j] = r;
        }
        tail = n4 << 2;
    }
    for (int64_t j = tail + i0; j < n; j += stride) {
        const float yo = (OP == OP_ACCUM || OP == OP_MUL_ACC) ? y[j] : 0.f;
        const float b = (OP == OP_SCALE_ADD || OP == OP_MUL || OP == OP_MUL_ACC) ? other[j] : 0.f;
        y[j] = map1<OP>(x[j], yo, b, fscale, dscale);
    }
}

// AA / AB: ga / gb assigned (their previous contents count as zero: the
// result is bitwise 0 + g, as accumulating into a cleared buffer).
template <bool VEC, bool AA, bool AB>
__global__ void add_bwd_kernel_t(const float* __restrict__ g, float* __restrict__ ga,
                                 float* __restrict__ gb, int64_t n) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    int64_t tail = 0;
    if (VEC) {
        const int64_t n4 = n >> 2;
        const float4* g4 = reinterpret_cast<const float4*>(g);
        float4* a4 = reinterpret_cast<float4*>(ga);
        float4* b4 = reinterpret_cast<float4*>(gb);
        for (int64_t j = i0; j < n4; j += stride) {
            const float4 v = g4[j];
            float4 a = AA ? z : a4[j];
            a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
            a4[j] = a;
            float4 b = AB ? z : b4[j];
            b.x += v.x; b.y += v.y; b.z += v.z; b.w += v.w;
            b4[j] = b;
        }
        tail = n4 << 2;
    }
    for (int64_t j = tail + i0; j < n; j += stride) {
        const float v = g[j];
        ga[j] = (AA ? 0.f : ga[j]) + v;
        gb[j] = (AB ? 0.f : gb[j]) + v;
    }
}

template <bool VEC>
__global__ void add_bwd_kernel(const float* __restrict__ g, float* __restrict__ ga,
                               float* __restrict__ gb, int64_t n) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t tail = 0;
    if (VEC) {
        const int64_t n4 = n >> 2;
        const float4* g4 = reinterpret_cast<const float4*>(g);
        float4* a4 = reinterpret_cast<float4*>(ga);
        float4* b4 = reinterpret_cast<float4*>(gb);
        for (int64_t j = i0; j < n4; j += stride) {
            const float4 v = g4[j];
            float4 a = a4[j];
            a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
            a4[j] = a;
            float4 b = b4[j];
            b.x += v.x; b.y += v.y; b.z += v.z; b.w += v.w;
            b4[j] = b;
        }
        tail = n4 << 2;
    }
    for (int64_t j = tail + i0; j < n; j += stride) {
        const float v = g[j];
        ga[j] += v;
        gb[j] += v;
    }
}

template <bool VEC>
__global__ void act_fwd_kernel(int kind, const float* __restrict__ x, float* __restrict__ y, int64_t n) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t tail = 0;
    if (VEC) {
        const int64_t n4 = n >> 2;
        const float4* x4 = reinterpret_cast<const float4*>(x);
        float4* y4 = reinterpret_cast<float4*>(y);
        for (int64_t j = i0; j < n4; j += stride) {
            const float4 a = x4[j];
            y4[j] = make_float4(act_forward(kind, a.x), act_forward(kind, a.y), act_forward(kind, a.z),
                                act_forward(kind, a.w));
        }
        tail = n4 << 2;
    }
    for (int64_t j = tail + i0; j < n; j += stride) y[j] = act_forward(kind, x[j]);
}

// ASSIGN: gx's previous contents count as zero (not read): the result is
// bitwise that of accumulating into a cleared buffer.
template <bool VEC, bool ASSIGN = false>
__global__ void act_bwd_kernel(int kind, const float* __restrict__ x, const float* __restrict__ gy,
                               float* __restrict__ gx, int64_t n) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t tail = 0;
    if (VEC) {
        const int64_t n4 = n >> 2;
        const float4* x4 = reinterpret_cast<const float4*>(x);
        const float4* g4 = reinterpret_cast<const float4*>(gy);
        float4* o4 = reinterpret_cast<float4*>(gx);
        for (int64_t j = i0; j < n4; j += stride) {
            const float4 a = x4[j], g = g4[j];
            float4 o = ASSIGN ? make_float4(0.f, 0.f, 0.f, 0.f) : o4[j];
            o.x = act_backward(kind, a.x, g.x, o.x);
            o.y = act_backward(kind, a.y, g.y, o.y);
            o.z = act_backward(kind, a.z, g.z, o.z);
            o.w = act_backward(kind, a.w, g.w, o.w);
            o4[j] = o;
        }
        tail = n4 << 2;
    }
    for (int64_t j = tail + i0; j < n; j += stride) gx[j] = act_backward(kind, x[j], gy[j], ASSIGN ? 0.f : gx[j]);
}

// Column sums of a [rows, cols] matrix, optionally fused with the activation
// backward that produces it (gx = gx + gy*f'(x), summing the updated gx).
// A 256-thread block owns a strip of 128 columns (4 per lane, float4) or 32
// columns (1 per lane) and a chunk of rows; its 8 warps take rows
// round-robin, the partials meet in shared memory, and one atomicAdd per
// column per block publishes them -- the grid is sized so a column sees at
// most a few dozen atomics.
constexpr int kColWarps = 8;

template <bool ACT, bool VEC, bool ASSIGN = false>
__global__ void __launch_bounds__(256) colsum_kernel(int kind, const float* __restrict__ x,
                                                     const float* __restrict__ gy, float* __restrict__ g,
                                                     float* __restrict__ out, int64_t rows, int64_t cols,
                                                     int64_t rows_per_block, float scale) {
    pdl_entry();
    constexpr int W = VEC ? 4 : 1;  // columns per lane
    __shared__ float part[kColWarps][32 * W];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t c0 = (int64_t)blockIdx.x * (32 * W) + (int64_t)lane * W;
    const int64_t r_begin = (int64_t)blockIdx.y * rows_per_block;
    const int64_t r_end = (r_begin + rows_per_block < rows) ? r_begin + rows_per_block : rows;
    float s[W];
#pragma unroll
    for (int k = 0; k < W; ++k) s[k] = 0.f;
    if (c0 < cols) {
        if constexpr (VEC) {
            // U rows per pass, their loads issued together (bytes in flight:
            // the plain column sum reads one tensor, the fused one two)
            constexpr int U = ACT ? 4 : 8;
            for (int64_t r = r_begin + warp; r < r_end; r += U * kColWarps) {
                float4 o[U], a[U], d[U];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int64_t rr = r + (int64_t)u * kColWarps;
                    const int64_t idx = rr * cols + c0;
                    const bool in = rr < r_end;
                    o[u] = (!in || (ACT && ASSIGN)) ? make_float4(0.f, 0.f, 0.f, 0.f)
                                                    : *reinterpret_cast<const float4*>(g + idx);
                    if (ACT) {
                        a[u] = in ? *reinterpret_cast<const float4*>(x + idx) : make_float4(0.f, 0.f, 0.f, 0.f);
                        d[u] = in ? *reinterpret_cast<const float4*>(gy + idx) : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                }
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int64_t rr = r + (int64_t)u * kColWarps;
                    if (rr >= r_end) break;
                    if (ACT) {
                        o[u].x = act_backward(kind, a[u].x, d[u].x, o[u].x);
                        o[u].y = act_backward(kind, a[u].y, d[u].y, o[u].y);
                        o[u].z = act_backward(kind, a[u].z, d[u].z, o[u].z);
                        o[u].w = act_backward(kind, a[u].w, d[u].w, o[u].w);
                        *reinterpret_cast<float4*>(g + rr * cols + c0) = o[u];
                    }
                    s[0] += o[u].x;
                    s[1] += o[u].y;
                    s[2] += o[u].z;
                    s[3] += o[u].w;
                }
            }
        } else {
          for (int64_t r = r_begin + warp; r < r_end; r += kColWarps) {
            const int64_t idx = r * cols + c0;
            {
                float o = (ACT && ASSIGN) ? 0.f : g[idx];
                if (ACT) {
                    o = act_backward(kind, x[idx], gy[idx], o);
                    g[idx] = o;
                }
                s[0] += o;
            }
          }
        }
    }
#pragma unroll
    for (int k = 0; k < W; ++k) part[warp][lane * W + k] = s[k];
    __syncthreads();
    for (int t = threadIdx.x; t < 32 * W; t += blockDim.x) {
        const int64_t c = (int64_t)blockIdx.x * (32 * W) + t;
        if (c < cols) {
            float tot = 0.f;
#pragma unroll
            for (int w = 0; w < kColWarps; ++w) tot += part[w][t];
            atomicAdd(out + c, tot * scale);
        }
    }
}

// Launch shape for colsum_kernel: column strips x row chunks, each chunk at
// least 32 rows; about four waves of blocks for the plain column sum and
// eight for the one fused with an activation backward (all resident: the
// warps per SM keep enough loads in flight; measured on B200).
struct ColsumShape {
    dim3 grid;
    int64_t rpb;
};

inline ColsumShape colsum_shape(int64_t rows, int64_t cols, bool vec, bool act = false) {
    const int64_t strip = vec ? 128 : 32;
    const int64_t col_blocks = (cols + strip - 1) / strip;
    int64_t row_blocks = ((act ? 8 : 4) * kSMs + col_blocks - 1) / col_blocks;
    const int64_t max_rb = (rows + 31) / 32;
    if (row_blocks > max_rb) row_blocks = max_rb;
    if (row_blocks < 1) row_blocks = 1;
    const int64_t rpb = (rows + row_blocks - 1) / row_blocks;
    row_blocks = (rows + rpb - 1) / rpb;
    return {dim3((unsigned)col_blocks, (unsigned)row_blocks), rpb};
}

// y[r,c] = x[r,c] + b[c]
template <bool VEC>
__global__ void bias_add_kernel(const float* __restrict__ x, const float* __restrict__ b, float* __restrict__ y,
                                int64_t rows, int64_t cols) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (VEC) {
        const int64_t c4 = cols >> 2;
        const int64_t n4 = rows * c4;
        for (int64_t j = i0; j < n4; j += stride) {
            const int64_t c = (j % c4) << 2;
            float4 a = reinterpret_cast<const float4*>(x)[j];
            const float4 bb = *reinterpret_cast<const float4*>(b + c);
            a.x += bb.x; a.y += bb.y; a.z += bb.z; a.w += bb.w;
            reinterpret_cast<float4*>(y)[j] = a;
        }
    } else {
        const int64_t n = rows * cols;
        for (int64_t j = i0; j < n; j += stride) y[j] = x[j] + b[j % cols];
    }
}

// y[n,c,s] = x[n,c,s] + b[c]; Q consecutive s per thread (Q = 4: 16-byte
// accesses), 32-bit chunk index (the host checks the count)
template <int Q>
__global__ void channel_bias_fwd_kernel(const float* __restrict__ x, const float* __restrict__ b,
                                        float* __restrict__ y, unsigned channels, unsigned per_plane,
                                        unsigned chunks) {
    pdl_entry();
    for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < chunks; i += gridDim.x * blockDim.x) {
        const float bc = __ldg(b + (i / per_plane) % channels);
        if constexpr (Q == 4) {
            float4 v = reinterpret_cast<const float4*>(x)[i];
            v.x += bc;
            v.y += bc;
            v.z += bc;
            v.w += bc;
            reinterpret_cast<float4*>(y)[i] = v;
        } else {
            y[i] = x[i] + bc;
        }
    }
}

// One block per (channel, batch chunk): gb[c] += sum; optional gx += g.
// blockIdx.x runs over the reduced channels (the first gridDim.x of
// `channels`); float4 accesses when `vec` (spatial % 4 == 0, aligned).
__global__ void channel_bias_bwd_kernel(const float* __restrict__ g, float* __restrict__ gx,
                                        float* __restrict__ gb, int batch, int channels, int64_t spatial,
                                        int batch_per_block, int vec) {
    pdl_entry();
    __shared__ float scratch[32];
    const int c = blockIdx.x;
    const int n0 = blockIdx.y * batch_per_block;
    int n1 = n0 + batch_per_block;
    if (n1 > batch) n1 = batch;
    float s = 0.f;
    for (int n = n0; n < n1; ++n) {
        const int64_t base = ((int64_t)n * channels + c) * spatial;
        if (vec) {
            const float4* g4 = reinterpret_cast<const float4*>(g + base);
            float4* x4 = reinterpret_cast<float4*>(gx + base);
            for (int64_t k = threadIdx.x; k < spatial / 4; k += blockDim.x) {
                const float4 v = g4[k];
                s += (v.x + v.y) + (v.z + v.w);
                if (gx) {
                    float4 o = x4[k];
                    o.x += v.x;
                    o.y += v.y;
                    o.z += v.z;
                    o.w += v.w;
                    x4[k] = o;
                }
            }
        } else {
            for (int64_t k = threadIdx.x; k < spatial; k += blockDim.x) {
                const float v = g[base + k];
                s += v;
                if (gx) gx[base + k] += v;
            }
        }
    }
    s = block_sum(s, scratch);
    if (threadIdx.x == 0) atomicAdd(gb + c, s);
}

// MatPEncoding (Engine/kernels.cu:166-185): double-precision angle.
__global__ void matpe_kernel(const float* __restrict__ x, float* __restrict__ y, int rows, int cols,
                             int64_t total, int start_idx) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int pos = (int)((i % ((int64_t)rows * cols)) / cols) + start_idx;
        const int d = (int)(i % cols);
        const int half = d / 2;
        const double exponent = (2.0 * half) / cols;
        const double freq = 1.0 / pow(10000.0, exponent);
        const double angle = (double)pos * freq;
        y[i] = (d % 2 == 0) ? x[i] + (float)sin(angle) : x[i] + (float)cos(angle);
    }
}

// The positional term of MatPEncoding alone (x = 0): table[r, c].
__global__ void matpe_table_kernel(float* __restrict__ t, int rows, int cols, int start_idx) {
    pdl_entry();
    const int64_t total = (int64_t)rows * cols;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int pos = (int)(i / cols) + start_idx;
        const int d = (int)(i % cols);
        const double freq = 1.0 / pow(10000.0, (2.0 * (d / 2)) / cols);
        const double angle = (double)pos * freq;
        t[i] = (d % 2 == 0) ? (float)sin(angle) : (float)cos(angle);
    }
}

// y[b, i] = x[b, i] + table[i]
__global__ void rows_add_table_kernel(const float4* __restrict__ x, const float4* __restrict__ table,
                                      float4* __restrict__ y, int64_t total4, int64_t row4) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total4; i += stride) {
        float4 a = x[i];
        const float4 t = table[i % row4];
        a.x += t.x; a.y += t.y; a.z += t.z; a.w += t.w;
        y[i] = a;
    }
}

__global__ void rows_add_table_scalar(const float* __restrict__ x, const float* __restrict__ table,
                                      float* __restrict__ y, int64_t total, int64_t row) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride)
        y[i] = x[i] + table[i % row];
}

// PEncoding (Engine/kernels.cu:147-164)
__global__ void timestep_pe_kernel(float* __restrict__ y, int t, int dim) {
    pdl_entry();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= dim) return;
    const int half = dim / 2;
    const int f = (i < half) ? i : i - half;
    const double exponent = -(double)f * log(10000.0) / (half - 1);
    const double freq = exp(exponent);
    const double angle = (double)t * freq;
    y[i] = (i < half) ? (float)cos(angle) : (float)sin(angle);
}

// HeadifyColChannel (Engine/kernels.cu:1371-1406); the += forms touch each
// element once, so plain read-modify-write replaces the atomics.
__global__ void headify_kernel(const float* __restrict__ in, float* __restrict__ out, int heads, int seq,
                               int head_dim, int64_t total, int flag) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int embed = heads * head_dim;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
        const int d = (int)(idx % head_dim);
        const int s = (int)((idx / head_dim) % seq);
        const int h = (int)((idx / ((int64_t)head_dim * seq)) % heads);
        const int64_t b = idx / ((int64_t)head_dim * seq * heads);
        const int64_t hidx = idx;
        const int64_t fidx = b * ((int64_t)seq * embed) + (int64_t)s * embed + (int64_t)h * head_dim + d;
        if (flag == 0) out[hidx] = in[fidx];
        else if (flag == 1) out[fidx] += in[hidx];
        else if (flag == 2) out[fidx] = in[hidx];
        else out[hidx] += in[fidx];
    }
}

// float4 form of headify_kernel for head_dim % 4 == 0: thread i moves the
// 4-vector i of the head-major tensor; 32-bit index math (the entry point
// checks that the element count fits).
__global__ void headify4_kernel(const float4* __restrict__ in, float4* __restrict__ out, int heads, int seq, int hd4,
                                int total4, int flag) {
    pdl_entry();
    const int stride = gridDim.x * blockDim.x;
    const int row4 = heads * hd4;  // 4-vectors per token row
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total4; i += stride) {
        const int d4 = i % hd4;
        int t = i / hd4;
        const int s = t % seq;
        t /= seq;
        const int h = t % heads;
        const int b = t / heads;
        const int f = (b * seq + s) * row4 + h * hd4 + d4;
        if (flag == 0) {
            out[i] = in[f];
        } else if (flag == 2) {
            out[f] = in[i];
        } else if (flag == 1) {
            float4 o = out[f];
            const float4 v = in[i];
            o.x += v.x; o.y += v.y; o.z += v.z; o.w += v.w;
            out[f] = o;
        } else {
            float4 o = out[i];
            const float4 v = in[f];
            o.x += v.x; o.y += v.y; o.z += v.z; o.w += v.w;
            out[i] = o;
        }
    }
}

// Channel concatenation along dim1 and its adjoint: every (n, channel)
// plane is a contiguous run of `spatial` floats, so a thread moves Q
// consecutive floats of one plane (Q = 4: 16-byte accesses).  32-bit chunk
// index (the host checks the count).
template <int Q>
__global__ void channel_concat_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                      float* __restrict__ c, int c1, int c2, unsigned per_plane, unsigned chunks) {
    pdl_entry();
    const unsigned cc = (unsigned)(c1 + c2);
    for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < chunks; i += gridDim.x * blockDim.x) {
        const unsigned pl = i / per_plane, j = i - pl * per_plane;
        const unsigned n = pl / cc, ch = pl - n * cc;
        const float* src = ch < (unsigned)c1 ? a + ((int64_t)n * c1 + ch) * per_plane * Q
                                             : b + ((int64_t)n * c2 + (ch - c1)) * per_plane * Q;
        if constexpr (Q == 4)
            reinterpret_cast<float4*>(c)[i] = reinterpret_cast<const float4*>(src)[j];
        else
            c[i] = src[j];
    }
}

template <int Q>
__global__ void channel_split_kernel(float* __restrict__ ga, float* __restrict__ gb, const float* __restrict__ gc,
                                     int c1, int c2, unsigned per_plane, unsigned chunks) {
    pdl_entry();
    const unsigned cc = (unsigned)(c1 + c2);
    for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < chunks; i += gridDim.x * blockDim.x) {
        const unsigned pl = i / per_plane, j = i - pl * per_plane;
        const unsigned n = pl / cc, ch = pl - n * cc;
        float* dst = ch < (unsigned)c1 ? ga + ((int64_t)n * c1 + ch) * per_plane * Q
                                       : gb + ((int64_t)n * c2 + (ch - c1)) * per_plane * Q;
        if constexpr (Q == 4) {
            const float4 g = reinterpret_cast<const float4*>(gc)[i];
            float4 o = reinterpret_cast<float4*>(dst)[j];
            o.x += g.x;
            o.y += g.y;
            o.z += g.z;
            o.w += g.w;
            reinterpret_cast<float4*>(dst)[j] = o;
        } else {
            dst[j] += gc[i];
        }
    }
}

// CopynCrop: (a,b) -> (c,d) centre crop
__global__ void center_crop_kernel(const float* __restrict__ x, float* __restrict__ y, int depth, int a, int b,
                                   int c, int d, int64_t total) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int dr = (a - c) / 2, dc = (b - d) / 2;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int64_t nb = i / ((int64_t)depth * c * d);
        const int ch = (int)((i / ((int64_t)c * d)) % depth);
        const int t = (int)(i % ((int64_t)c * d));
        const int r = t / d, col = t % d;
        y[i] = x[nb * depth * (int64_t)a * b + (int64_t)ch * a * b + (int64_t)(r + dr) * b + col + dc];
    }
}

// PaddingCrop: (c,d) -> (a,b), accumulate
__global__ void pad_crop_kernel(const float* __restrict__ x, float* __restrict__ y, int depth, int a, int b,
                                int c, int d, int64_t total) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int dr = (a - c) / 2, dc = (b - d) / 2;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int64_t nb = i / ((int64_t)depth * a * b);
        const int ch = (int)((i / ((int64_t)a * b)) % depth);
        const int t = (int)(i % ((int64_t)a * b));
        const int xr = t / b - dr, xc = t % b - dc;
        if (xr >= 0 && xr < c && xc >= 0 && xc < d)
            y[i] += x[nb * depth * (int64_t)c * d + (int64_t)ch * c * d + (int64_t)xr * d + xc];
    }
}

__global__ void gather_kernel(const int32_t* __restrict__ keys, const float* __restrict__ table,
                              float* __restrict__ out, int64_t total, int dim) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int64_t row = i / dim;
        const int k = keys[row];
        out[i] = (k < 0) ? 0.0f : table[(int64_t)k * dim + (i % dim)];
    }
}

// out[r, :] = table[keys[r], :] (0 for a key < 0) + pe[r % seq, :]: the
// gather and the positional table's add in one pass, four floats a thread
__global__ void gather_add_kernel(const int32_t* __restrict__ keys, const float* __restrict__ table,
                                  const float* __restrict__ pe, float* __restrict__ out, int64_t total4, int dim4,
                                  int seq) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total4; i += stride) {
        const int64_t row = i / dim4;
        const int c = (int)(i - row * dim4);
        const int k = keys[row];
        const float4 e = (k < 0) ? make_float4(0.f, 0.f, 0.f, 0.f)
                                 : reinterpret_cast<const float4*>(table)[(int64_t)k * dim4 + c];
        const float4 q = reinterpret_cast<const float4*>(pe)[(row % seq) * dim4 + c];
        reinterpret_cast<float4*>(out)[i] = make_float4(e.x + q.x, e.y + q.y, e.z + q.z, e.w + q.w);
    }
}

// gsum[keys[r], :] += grad[r, :] for every gradient row r whose key is >= 0
// (token t of batch b reads its key at keys[b * key_stride + t]); rows that
// share a key meet in atomic adds.
__global__ void key_grad_scatter_kernel(const int32_t* __restrict__ keys, const float* __restrict__ grad,
                                        float* __restrict__ gsum, int64_t rows, int dim, int key_stride, int row_len,
                                        int vec) {
    pdl_entry();
    const int per_row = vec ? dim / 4 : dim;
    const int64_t total = rows * per_row;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int64_t r = i / per_row;
        const int c = (int)(i - r * per_row);
        const int64_t b = r / row_len, t = r - b * row_len;
        const int k = keys[b * key_stride + t];
        if (k < 0) continue;
        if (vec) atomicAdd(reinterpret_cast<float4*>(gsum + (int64_t)k * dim + 4 * c),
                           *reinterpret_cast<const float4*>(grad + r * dim + 4 * c));
        else atomicAdd(gsum + (int64_t)k * dim + c, grad[r * dim + c]);
    }
}

// table = fma(neg_lr, gsum, table): the reference's `EmbedSpace += -lr *
// grad` is one fused multiply-add per element, so a table row whose key
// occurred once gets exactly the reference's value.
__global__ void key_apply_kernel(float* __restrict__ table, const float* __restrict__ gsum, int64_t n, float neg_lr) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t n4 = n >> 2;
    float4* t4 = reinterpret_cast<float4*>(table);
    const float4* g4 = reinterpret_cast<const float4*>(gsum);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
        const float4 g = g4[i];
        float4 t = t4[i];
        t.x = __fmaf_rn(neg_lr, g.x, t.x);
        t.y = __fmaf_rn(neg_lr, g.y, t.y);
        t.z = __fmaf_rn(neg_lr, g.z, t.z);
        t.w = __fmaf_rn(neg_lr, g.w, t.w);
        t4[i] = t;
    }
    for (int64_t i = (n4 << 2) + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        table[i] = __fmaf_rn(neg_lr, gsum[i], table[i]);
}

// Number of NaN elements (a block-local count, one atomic per block).
__global__ void count_nan_kernel(const float* __restrict__ x, int64_t n, unsigned long long* __restrict__ count) {
    unsigned long long c = 0;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) c += (x[i] != x[i]);
    for (int o = 16; o > 0; o >>= 1) c += __shfl_down_sync(0xffffffffu, c, o);
    __shared__ unsigned long long part[32];
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = c;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long t = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[w];
        if (t) atomicAdd(count, t);
    }
}

// First index of the largest element (a strict > scan keeps the earliest of
// equal maxima, NaNs never win): one block, per-thread strided scan, then a
// shared-memory tree that prefers the lower index on ties.
__global__ void argmax_kernel(const float* __restrict__ x, int64_t n, int* __restrict__ out) {
    __shared__ float sv[1024];
    __shared__ int64_t si[1024];
    float best = -INFINITY;
    int64_t bi = -1;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = x[i];
        if (bi < 0 || v > best) {
            best = v;
            bi = i;
        }
    }
    sv[threadIdx.x] = best;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int off = blockDim.x / 2; off > 0; off >>= 1) {
        if ((int)threadIdx.x < off) {
            const float ov = sv[threadIdx.x + off];
            const int64_t oi = si[threadIdx.x + off];
            const float mv = sv[threadIdx.x];
            const int64_t mi = si[threadIdx.x];
            const bool take = oi >= 0 && (mi < 0 || ov > mv || (ov == mv && oi < mi) || (mv != mv && ov == ov));
            if (take) {
                sv[threadIdx.x] = ov;
                si[threadIdx.x] = oi;
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) *out = (int)(si[0] < 0 ? 0 : si[0]);
}

// Counter-based noise (not the reference's cuRAND stream: the values differ,
// the distributions do not): splitmix64 of (seed, index) -> two uniforms;
// kind 0 Gaussian (Box-Muller) mean + std * z, kind 1 uniform mean + std * u
// with u in [0, 1) (GaussianNoise / UnifNoise, Engine/engine.cu:3936-3944).
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void noise_kernel(float* __restrict__ x, int64_t n, float mean, float stdv, int kind, uint64_t seed) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint64_t r = mix64(seed ^ mix64((uint64_t)i));
        const float u1 = ((uint32_t)(r >> 40) + 0.5f) * (1.0f / 16777216.0f);          // (0, 1)
        const float u2 = ((uint32_t)(r & 0xFFFFFFu)) * (1.0f / 16777216.0f);            // [0, 1)
        if (kind == 0) x[i] = mean + stdv * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
        else x[i] = mean + stdv * u2;
    }
}

__global__ void one_hot_kernel(const int32_t* __restrict__ keys, float* __restrict__ out, int64_t n, int vocab) {
    pdl_entry();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const int k = keys[i];
        if (k >= 0 && k < vocab) out[i * vocab + k] = 1.0f;
    }
}

inline bool vec_ok(int64_t n, const void* a, const void* b = nullptr, const void* c = nullptr) {
    (void)n;
    return aligned16(a) && (b == nullptr || aligned16(b)) && (c == nullptr || aligned16(c));
}

}  // namespace
}  // namespace mle

using namespace mle;

extern "C" {

const char* mle_status_string(int status) {
    switch (status) {
        case MLE_OK: return "ok";
        case MLE_ERR_ARG: return "invalid argument";
        case MLE_ERR_CUDA: return "CUDA error";
        case MLE_ERR_UNSUPPORTED: return "unsupported shape or flag";
        case MLE_ERR_TIMEOUT: return "a bounded wait timed out";
        default: return "unknown status";
    }
}

int mle_last_cuda_error(void) { return (int)g_last_cuda_error; }

int mle_abi_version(void) { return 1; }

int mle_fill(float* x, float value, int64_t n, mle_stream_t stream) {
    if (n < 0 || (n > 0 && !x)) return MLE_ERR_ARG;
    if (n == 0) return MLE_OK;
    if (aligned16(x)) launch_k(fill_kernel, grid_for(n / 4 + 1, kThreads), kThreads, 0, as_stream(stream), x, value, n);
    else launch_k(fill_kernel_scalar, grid_for(n, kThreads), kThreads, 0, as_stream(stream), x, value, n);
    return launch_status();
}

#define MLE_MAP_LAUNCH(OP, X, O, Y, N, FS, DS)                                                        \
    do {                                                                                          \
        if (vec_ok(N, X, O, Y))                                                                   \
            launch_k(map_kernel<OP, true>, grid_for((N) / 4 + 1, kThreads), kThreads, 0, as_stream(stream),  \
                X, O, Y, N, FS, DS);                                                              \
        else                                                                                      \
            launch_k(map_kernel<OP, false>, grid_for(N, kThreads), kThreads, 0, as_stream(stream), X, O, Y, N, \
                                                                                        FS, DS);  \
    } while (0)

int mle_copy(const float* x, float* y, int64_t n, mle_stream_t stream) {
    if (n < 0 || (n > 0 && (!x || !y))) return MLE_ERR_ARG;
    if (n == 0) return MLE_OK;
    MLE_MAP_LAUNCH(OP_COPY, x, (const float*)nullptr, y, n, 1.f, 1.0);
    return launch_status();
}

int mle_accumulate(const float* x, float* y, int64_t n, double scale, mle_stream_t stream) {
    if (n < 0 || (n > 0 && (!x || !y))) return MLE_ERR_ARG;
    if (n == 0) return MLE_OK;
    MLE_MAP_LAUNCH(OP_ACCUM, x, (const float*)nullptr, y, n, 1.f, scale);
    return launch_status();
}

int mle_scale_write(const float* x, float* y, int64_t n, float scale, mle_stream_t stream) {
    if (n < 0 || (n > 0 && (!x || !y))) return MLE_ERR_ARG;
    if (n == 0) return MLE_OK;
    MLE_MAP_LAUNCH(OP_SCALE_WRITE, x, (const float*)nullptr, y, n, scale, 1.0);
    return launch_status();
}

int mle_scale_add(const float* x, const float* y, float* z, float scale, int64_t n, mle_stream_t stream) {
    if (n < 0 || (n > 0 && (!x || !y || !z))) return MLE_ERR_ARG;
    if (n == 0) return MLE_OK;
    MLE_MAP_LAUNCH(OP_SCALE_ADD, x, y, z, n, scale, 1.0);
    return launch_status();
}

int mle_add_bwd(const float* g, float* ga, float* gb, int64_t n, mle_stream_t stream) {
    if (n < 0 || (n > 0 && (!g || !ga || !gb))) return MLE_ERR_ARG;
    if (n == 0) return MLE_OK;
    if (vec_ok(n, g, ga, gb))
        launch_k(add_bwd_kernel<true>, grid_for(n / 4 + 1, kThreads), kThreads, 0, as_stream(stream), g, ga, gb, n);
    else
        launch_k(add_bwd_kernel<false>, grid_for(n, kThreads), kThreads, 0, as_stream(stream), g, ga, gb, n);
    return launch_status();
}

int mle_add_bwd_assign(const float* g, float* ga, float* gb, int64_t n, int assign_mask, mle_stream_t stream) {
    if (n < 0 || (n > 0 && (!g || !ga || !gb)) || assign_mask < 0 || assign_mask > 3) return MLE_ERR_ARG;
    if (n == 0) return MLE_OK;
    if (assign_mask == 0) return mle_add_bwd(g, ga, gb, n, stream);
    if (ga == gb) return MLE_ERR_ARG;  // x + x accumulates twice into one buffer
    const bool vec = vec_ok(n, g, ga, gb);
    const unsigned grid = vec ? grid_for(n / 4 + 1, kThreads) : grid_for(n, kThreads);
    cudaStream_t st = as_stream(stream);
#define MLE_ADDB(V, A, B) launch_k(add_bwd_kernel_t<V, A, B>, grid, kThreads, 0, st, g, ga, gb, n)
    if (vec) {
        if (assign_mask == 1) MLE_ADDB(true, true, false);
        else if (assign_mask == 2) MLE_ADDB(true, false, true);
        else MLE_ADDB(true, true, true);
    } else {
        if (assign_mask == 1) MLE_ADDB(false, true, false);
        else if (assign_mask == 2) MLE_ADDB(false, false, true);
        else MLE_ADDB(false, true, true);
    }
#undef MLE_ADDB
    return launch_status();
}

int mle_act_fwd(int kind, const float* x, float* y, int64_t n, mle_stream_t stream) {
    if (kind < 0 || kind > MLE_ACT_SIGMOID || n < 0 || (n > 0 && (!x || !y))) return MLE_ERR_ARG;
    if (n == 0) return MLE_OK;
    if (vec_ok(n, x, y))
        launch_k(act_fwd_kernel<true>, grid_for(n / 4 + 1, kThreads), kThreads, 0, as_stream(stream), kind, x, y, n);
    else
        launch_k(act_fwd_kernel<false>, grid_for(n, kThreads), kThreads, 0, as_stream(stream), kind, x, y, n);
    return launch_status();
}

extern "C++" {
namespace {
template <bool ASSIGN>
int act_bwd(int kind, const float* x, const float* gy, float* gx, int64_t n, float* bias_grad, int64_t rows,
            int64_t cols, mle_stream_t stream) {
    if (kind < 0 || kind > MLE_ACT_SIGMOID || n < 0 || (n > 0 && (!x || !gy || !gx))) return MLE_ERR_ARG;
    if (n == 0) return MLE_OK;
    if (!bias_grad) {
        if (vec_ok(n, x, gy, gx))
            launch_k(act_bwd_kernel<true, ASSIGN>, grid_for(n / 4 + 1, kThreads), kThreads, 0, as_stream(stream), kind,
                     x, gy, gx, n);
        else
            launch_k(act_bwd_kernel<false, ASSIGN>, grid_for(n, kThreads), kThreads, 0, as_stream(stream), kind, x, gy,
                     gx, n);
        return launch_status();
    }
    if (rows <= 0 || cols <= 0 || rows * cols != n) return MLE_ERR_ARG;
    const bool vec = (cols % 4 == 0) && vec_ok(n, x, gy, gx);
    const ColsumShape sh = colsum_shape(rows, cols, vec, true);
    if (vec)
        launch_k(colsum_kernel<true, true, ASSIGN>, sh.grid, 256, 0, as_stream(stream), kind, x, gy, gx, bias_grad,
                 rows, cols, sh.rpb, 1.0f);
    else
        launch_k(colsum_kernel<true, false, ASSIGN>, sh.grid, 256, 0, as_stream(stream), kind, x, gy, gx, bias_grad,
                 rows, cols, sh.rpb, 1.0f);
    return launch_status();
}
}  // namespace
}  // extern "C++"

int mle_act_bwd(int kind, const float* x, const float* gy, float* gx, int64_t n, float* bias_grad, int64_t rows,
                int64_t cols, mle_stream_t stream) {
    return act_bwd<false>(kind, x, gy, gx, n, bias_grad, rows, cols, stream);
}

int mle_act_bwd_assign(int kind, const float* x, const float* gy, float* gx, int64_t n, float* bias_grad,
                       int64_t rows, int64_t cols, mle_stream_t stream) {
    return act_bwd<true>(kind, x, gy, gx, n, bias_grad, rows, cols, stream);
}

int mle_bias_add_fwd(const float* x, const float* bias, float* y, int64_t rows, int64_t cols, mle_stream_t stream) {
    if (rows < 0 || cols <= 0 || !x || !bias || !y) return MLE_ERR_ARG;
    if (rows == 0) return MLE_OK;
    const int64_t n = rows * cols;
    if (cols % 4 == 0 && vec_ok(n, x, bias, y))
        launch_k(bias_add_kernel<true>, grid_for(n / 4, kThreads), kThreads, 0, as_stream(stream), x, bias, y, rows, cols);
    else
        launch_k(bias_add_kernel<false>, grid_for(n, kThreads), kThreads, 0, as_stream(stream), x, bias, y, rows, cols);
    return launch_status();
}

int mle_bias_grad(const float* g, float* bias_grad, int64_t rows, int64_t cols, float scale, mle_stream_t stream) {
    if (rows < 0 || cols <= 0 || !g || !bias_grad) return MLE_ERR_ARG;
    if (rows == 0) return MLE_OK;
    const bool vec = cols % 4 == 0 && aligned16(g);
    const ColsumShape sh = colsum_shape(rows, cols, vec);
    float* gm = const_cast<float*>(g);  // read-only when ACT == false
    if (vec)
        launch_k(colsum_kernel<false, true>, sh.grid, 256, 0, as_stream(stream), 0, nullptr, nullptr, gm, bias_grad, rows,
                                                                           cols, sh.rpb, scale);
    else
        launch_k(colsum_kernel<false, false>, sh.grid, 256, 0, as_stream(stream), 0, nullptr, nullptr, gm, bias_grad, rows,
                                                                            cols, sh.rpb, scale);
    return launch_status();
}

int mle_channel_bias_fwd(const float* x, const float* b, float* y, int batch, int channels, int64_t spatial,
                         mle_stream_t stream) {
    if (batch < 0 || channels <= 0 || spatial <= 0 || !x || !b || !y) return MLE_ERR_ARG;
    const int Q = (spatial % 4 == 0 && aligned16(x) && aligned16(y)) ? 4 : 1;
    const int64_t chunks = (int64_t)batch * channels * spatial / Q;
    if (chunks == 0) return MLE_OK;
    if (chunks > INT32_MAX) return MLE_ERR_UNSUPPORTED;
    const unsigned per = (unsigned)(spatial / Q), grid = grid_for(chunks, kThreads);
    if (Q == 4)
        launch_k(channel_bias_fwd_kernel<4>, grid, kThreads, 0, as_stream(stream), x, b, y, (unsigned)channels, per,
                 (unsigned)chunks);
    else
        launch_k(channel_bias_fwd_kernel<1>, grid, kThreads, 0, as_stream(stream), x, b, y, (unsigned)channels, per,
                 (unsigned)chunks);
    return launch_status();
}

static int channel_sums(const float* g, float* gx, float* gb, int batch, int channels, int first, int64_t spatial,
                        cudaStream_t st) {
    if (batch == 0 || first == 0) return MLE_OK;
    int chunks = (2 * kSMs + first - 1) / first;
    if (chunks > batch) chunks = batch;
    const int bpb = (batch + chunks - 1) / chunks;
    chunks = (batch + bpb - 1) / bpb;
    const int vec = (spatial % 4 == 0) && aligned16(g) && (gx == nullptr || aligned16(gx));
    dim3 grid((unsigned)first, (unsigned)chunks);
    launch_k(channel_bias_bwd_kernel, grid, kThreads, 0, st, g, gx, gb, batch, channels, spatial, bpb, vec);
    return launch_status();
}

int mle_channel_bias_bwd(const float* g, float* gx, float* gb, int batch, int channels, int64_t spatial,
                         mle_stream_t stream) {
    if (batch < 0 || channels <= 0 || spatial <= 0 || !g || !gb) return MLE_ERR_ARG;
    return channel_sums(g, gx, gb, batch, channels, channels, spatial, as_stream(stream));
}

int mle_channel_bias_bwd_first(const float* g, float* gb, int batch, int channels, int first, int64_t spatial,
                               mle_stream_t stream) {
    if (batch < 0 || channels <= 0 || first < 0 || first > channels || spatial <= 0 || !g || !gb)
        return MLE_ERR_ARG;
    return channel_sums(g, nullptr, gb, batch, channels, first, spatial, as_stream(stream));
}

int mle_matpe_fwd(const float* x, float* y, int batch, int rows, int cols, int start_idx, mle_stream_t stream) {
    if (batch < 0 || rows <= 0 || cols <= 0 || !x || !y) return MLE_ERR_ARG;
    const int64_t total = (int64_t)batch * rows * cols;
    if (total == 0) return MLE_OK;
    launch_k(matpe_kernel, grid_for(total, kThreads), kThreads, 0, as_stream(stream), x, y, rows, cols, total, start_idx);
    return launch_status();
}

int mle_matpe_table(float* table, int rows, int cols, int start_idx, mle_stream_t stream) {
    if (rows <= 0 || cols <= 0 || !table) return MLE_ERR_ARG;
    launch_k(matpe_table_kernel, grid_for((int64_t)rows * cols, kThreads), kThreads, 0, as_stream(stream), table, rows, cols,
                                                                                                     start_idx);
    return launch_status();
}

int mle_rows_add_table(const float* x, const float* table, float* y, int64_t batch, int64_t row_elems,
                       mle_stream_t stream) {
    if (batch < 0 || row_elems <= 0 || !x || !table || !y) return MLE_ERR_ARG;
    const int64_t total = batch * row_elems;
    if (total == 0) return MLE_OK;
    if (row_elems % 4 == 0 && aligned16(x) && aligned16(table) && aligned16(y))
        launch_k(rows_add_table_kernel, grid_for(total / 4, kThreads), kThreads, 0, as_stream(stream), 
            reinterpret_cast<const float4*>(x), reinterpret_cast<const float4*>(table), reinterpret_cast<float4*>(y),
            total / 4, row_elems / 4);
    else
        launch_k(rows_add_table_scalar, grid_for(total, kThreads), kThreads, 0, as_stream(stream), x, table, y, total,
                                                                                             row_elems);
    return launch_status();
}

int mle_timestep_pe(float* y, int t, int dim, mle_stream_t stream) {
    if (dim <= 2 || !y) return MLE_ERR_ARG;
    launch_k(timestep_pe_kernel, (dim + kThreads - 1) / kThreads, kThreads, 0, as_stream(stream), y, t, dim);
    return launch_status();
}

int mle_headify(const float* in, float* out, int batch, int heads, int seq, int head_dim, int flag,
                mle_stream_t stream) {
    if (batch < 0 || heads <= 0 || seq <= 0 || head_dim <= 0 || flag < 0 || flag > 3 || !in || !out)
        return MLE_ERR_ARG;
    const int64_t total = (int64_t)batch * heads * seq * head_dim;
    if (total == 0) return MLE_OK;
    if (head_dim % 4 == 0 && aligned16(in) && aligned16(out) && total / 4 < (1ll << 31)) {
        const int total4 = (int)(total / 4);
        launch_k(headify4_kernel, grid_for(total4, kThreads), kThreads, 0, as_stream(stream), 
            reinterpret_cast<const float4*>(in), reinterpret_cast<float4*>(out), heads, seq, head_dim / 4, total4,
            flag);
    } else {
        launch_k(headify_kernel, grid_for(total, kThreads), kThreads, 0, as_stream(stream), in, out, heads, seq, head_dim,
                                                                                      total, flag);
    }
    return launch_status();
}

int mle_channel_concat(const float* a, const float* b, float* c, int batch, int c1, int c2, int64_t spatial,
                       mle_stream_t stream) {
    if (batch < 0 || c1 < 0 || c2 < 0 || spatial <= 0 || !a || !b || !c) return MLE_ERR_ARG;
    const int Q = (spatial % 4 == 0 && aligned16(a) && aligned16(b) && aligned16(c)) ? 4 : 1;
    const int64_t chunks = (int64_t)batch * (c1 + c2) * spatial / Q;
    if (chunks == 0) return MLE_OK;
    if (chunks > INT32_MAX) return MLE_ERR_UNSUPPORTED;
    const unsigned per = (unsigned)(spatial / Q), grid = grid_for(chunks, kThreads);
    if (Q == 4)
        launch_k(channel_concat_kernel<4>, grid, kThreads, 0, as_stream(stream), a, b, c, c1, c2, per,
                 (unsigned)chunks);
    else
        launch_k(channel_concat_kernel<1>, grid, kThreads, 0, as_stream(stream), a, b, c, c1, c2, per,
                 (unsigned)chunks);
    return launch_status();
}

int mle_channel_split(float* ga, float* gb, const float* gc, int batch, int c1, int c2, int64_t spatial,
                      mle_stream_t stream) {
    if (batch < 0 || c1 < 0 || c2 < 0 || spatial <= 0 || !ga || !gb || !gc) return MLE_ERR_ARG;
    const int Q = (spatial % 4 == 0 && aligned16(ga) && aligned16(gb) && aligned16(gc)) ? 4 : 1;
    const int64_t chunks = (int64_t)batch * (c1 + c2) * spatial / Q;
    if (chunks == 0) return MLE_OK;
    if (chunks > INT32_MAX) return MLE_ERR_UNSUPPORTED;
    const unsigned per = (unsigned)(spatial / Q), grid = grid_for(chunks, kThreads);
    if (Q == 4)
        launch_k(channel_split_kernel<4>, grid, kThreads, 0, as_stream(stream), ga, gb, gc, c1, c2, per,
                 (unsigned)chunks);
    else
        launch_k(channel_split_kernel<1>, grid, kThreads, 0, as_stream(stream), ga, gb, gc, c1, c2, per,
                 (unsigned)chunks);
    return launch_status();
}

int mle_center_crop(const float* x, float* y, int batch, int depth, int a, int b, int c, int d,
                    mle_stream_t stream) {
    if (batch < 0 || depth <= 0 || c <= 0 || d <= 0 || c > a || d > b || !x || !y) return MLE_ERR_ARG;
    const int64_t total = (int64_t)batch * depth * c * d;
    if (total == 0) return MLE_OK;
    launch_k(center_crop_kernel, grid_for(total, kThreads), kThreads, 0, as_stream(stream), x, y, depth, a, b, c, d, total);
    return launch_status();
}

int mle_pad_crop(const float* x, float* y, int batch, int depth, int a, int b, int c, int d, mle_stream_t stream) {
    if (batch < 0 || depth <= 0 || a <= 0 || b <= 0 || !x || !y) return MLE_ERR_ARG;
    const int64_t total = (int64_t)batch * depth * a * b;
    if (total == 0) return MLE_OK;
    launch_k(pad_crop_kernel, grid_for(total, kThreads), kThreads, 0, as_stream(stream), x, y, depth, a, b, c, d, total);
    return launch_status();
}

int mle_embedding_gather(const int32_t* keys, const float* table, float* out, int64_t n_keys, int dim,
                         mle_stream_t stream) {
    if (n_keys < 0 || dim <= 0 || !keys || !table || !out) return MLE_ERR_ARG;
    const int64_t total = n_keys * dim;
    if (total == 0) return MLE_OK;
    launch_k(gather_kernel, grid_for(total, kThreads), kThreads, 0, as_stream(stream), keys, table, out, total, dim);
    return launch_status();
}

int mle_embedding_gather_add(const int32_t* keys, const float* table, const float* pe, float* out, int64_t n_keys,
                             int dim, int seq, mle_stream_t stream) {
    if (n_keys < 0 || dim <= 0 || seq <= 0 || !keys || !table || !pe || !out) return MLE_ERR_ARG;
    if (dim % 4 != 0 || !aligned16(table) || !aligned16(pe) || !aligned16(out)) return MLE_ERR_UNSUPPORTED;
    if (n_keys == 0) return MLE_OK;
    const int64_t total4 = n_keys * (dim / 4);
    launch_k(gather_add_kernel, grid_for(total4, kThreads), kThreads, 0, as_stream(stream), keys, table, pe, out,
             total4, dim / 4, seq);
    return launch_status();
}

int mle_embedding_grad_scatter(const int32_t* keys, const float* grad, float* gsum, int64_t rows, int dim,
                               int row_len, int key_stride, mle_stream_t stream) {
    if (rows < 0 || dim <= 0 || row_len <= 0 || key_stride < row_len || !keys || !grad || !gsum) return MLE_ERR_ARG;
    if (rows == 0) return MLE_OK;
    const int vec = (dim % 4 == 0 && aligned16(grad) && aligned16(gsum)) ? 1 : 0;
    const int64_t total = rows * (vec ? dim / 4 : dim);
    launch_k(key_grad_scatter_kernel, grid_for(total, kThreads), kThreads, 0, as_stream(stream), keys, grad, gsum,
             rows, dim, key_stride, row_len, vec);
    return launch_status();
}

int mle_embedding_apply(float* table, const float* gsum, int64_t n, float neg_lr, mle_stream_t stream) {
    if (n < 0 || (n > 0 && (!table || !gsum)) || !aligned16(table) || !aligned16(gsum)) return MLE_ERR_ARG;
    if (n == 0) return MLE_OK;
    launch_k(key_apply_kernel, grid_for(n / 4 + 1, kThreads), kThreads, 0, as_stream(stream), table, gsum, n, neg_lr);
    return launch_status();
}

int mle_embedding_update(const int32_t* keys, const float* grad, float* table, float* gsum, int vocab, int64_t rows,
                         int dim, int row_len, int key_stride, float lr, mle_stream_t stream) {
    if (vocab <= 0 || dim <= 0 || !gsum) return MLE_ERR_ARG;
    const int64_t n = (int64_t)vocab * dim;
    if (cudaMemsetAsync(gsum, 0, (size_t)n * sizeof(float), as_stream(stream)) != cudaSuccess) return MLE_ERR_CUDA;
    int st = mle_embedding_grad_scatter(keys, grad, gsum, rows, dim, row_len, key_stride, stream);
    if (st != MLE_OK) return st;
    return mle_embedding_apply(table, gsum, n, -lr, stream);
}

int mle_mul(const float* x, const float* y, float* z, int64_t n, int accumulate, mle_stream_t stream) {
    if (n < 0 || (n > 0 && (!x || !y || !z))) return MLE_ERR_ARG;
    if (n == 0) return MLE_OK;
    if (accumulate) MLE_MAP_LAUNCH(OP_MUL_ACC, x, y, z, n, 1.f, 1.0);
    else MLE_MAP_LAUNCH(OP_MUL, x, y, z, n, 1.f, 1.0);
    return launch_status();
}

int mle_count_nan(const float* x, int64_t n, unsigned long long* count, mle_stream_t stream) {
    if (n < 0 || !count || (n > 0 && !x)) return MLE_ERR_ARG;
    if (cudaMemsetAsync(count, 0, sizeof(unsigned long long), as_stream(stream)) != cudaSuccess) return MLE_ERR_CUDA;
    if (n == 0) return MLE_OK;
    count_nan_kernel<<<grid_for(n, kThreads), kThreads, 0, as_stream(stream)>>>(x, n, count);
    return launch_status();
}

int mle_argmax(const float* x, int64_t n, int* out, mle_stream_t stream) {
    if (n <= 0 || !x || !out) return MLE_ERR_ARG;
    argmax_kernel<<<1, 1024, 0, as_stream(stream)>>>(x, n, out);
    return launch_status();
}

int mle_fill_noise(float* x, int64_t n, float mean, float stdv, int kind, uint64_t seed, mle_stream_t stream) {
    if (n < 0 || (n > 0 && !x) || (kind != 0 && kind != 1)) return MLE_ERR_ARG;
    if (n == 0) return MLE_OK;
    noise_kernel<<<grid_for(n, kThreads), kThreads, 0, as_stream(stream)>>>(x, n, mean, stdv, kind, seed);
    return launch_status();
}

int mle_one_hot(const int32_t* keys, float* out, int64_t n_keys, int vocab, mle_stream_t stream) {
    if (n_keys < 0 || vocab <= 0 || !keys || !out) return MLE_ERR_ARG;
    if (n_keys == 0) return MLE_OK;
    launch_k(one_hot_kernel, grid_for(n_keys, kThreads), kThreads, 0, as_stream(stream), keys, out, n_keys, vocab);
    return launch_status();
}

}  // extern "C"
