// 2-D convolution and transposed convolution (Convolute2D / Convolute2DT,
// Engine/engine.cu:3723-3912) on the tensor-core GEMM.
//
// The reference computes every output with one thread looping over
// (channel, kh, kw) or over the whole batch (CV2D, GV2D, CV2D_GradInput,
// CVT2D, GVT2D, CVT2D_GradInput, Engine/kernels.cu:985-1212).  Here each of
// them is a GEMM over an im2col matrix:
//   cols[n][(c, kh, kw)][(oy, ox)] = x[n][c][oy*s - p + kh][ox*s - p + kw]
// (zero outside the image), so for a convolution with weights
// W[Cout][Cin][KH][KW]
//   forward  y[n]  = W · cols(x)[n]                  (M=Cout, N=OH*OW, K=Cin*KH*KW)
//   dW            = sum_n dy[n] · cols(x)[n]^T         (assigned, as GV2D)
//   dx      += col2im(W^T · dy[n])                     (gather, as CV2D_GradInput)
// and the transposed convolution (weights W[Cout][Cin][KH][KW] with Cin the
// input channels) is the adjoint geometry: its forward is col2im of
// W'^T · x with W' = W with its first two dimensions swapped, its input
// gradient a convolution of dy, its weight gradient a reduction over the
// batch.  The column index k = c*KH*KW + kh*KW + kw ascends in the
// reference's loop order, so the fp32 GEMM mode sums the forward in the
// reference's order.
#include <string.h>

#include <stdint.h>

#include <algorithm>

#include "common.cuh"
#include "gemm.cuh"

namespace mle {
namespace {

constexpr int kT = 256;

constexpr int kRowThreads = 256;

// cols[n][(c, kh, kw)][(oy, ox)]: one thread per Q consecutive ox of one
// column row (Q = 4 when OW % 4 == 0: one 16-byte store).  The thread index
// runs over (row, chunk) pairs; 32-bit index arithmetic (the host checks
// that the chunk count fits).
template <int Q>
__global__ void im2col_kernel(const float* __restrict__ x, float* __restrict__ cols, int C, int H, int W, int KH,
                              int KW, int OH, int OW, int pad, int stride, unsigned chunks) {
    pdl_entry();
    const unsigned per_row = (unsigned)(OH * OW) / Q;
    for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < chunks; i += gridDim.x * blockDim.x) {
        const unsigned row = i / per_row;
        const int p0 = (int)(i - row * per_row) * Q;
        const int oy = p0 / OW, ox0 = p0 - oy * OW;
        const int kw = (int)(row % (unsigned)KW);
        const unsigned r = row / (unsigned)KW;
        const int kh = (int)(r % (unsigned)KH);
        const float* xp = x + (int64_t)(r / (unsigned)KH) * H * W;  // plane n * C + c
        const int iy = oy * stride - pad + kh;
        const bool row_in = iy >= 0 && iy < H;
        float v[Q];
#pragma unroll
        for (int u = 0; u < Q; ++u) {
            const int ix = (ox0 + u) * stride - pad + kw;
            v[u] = (row_in && ix >= 0 && ix < W) ? __ldg(xp + (int64_t)iy * W + ix) : 0.f;
        }
        float* dst = cols + (int64_t)i * Q;
        if constexpr (Q == 4) {
            *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
#pragma unroll
            for (int u = 0; u < Q; ++u) dst[u] = v[u];
        }
    }
}

// x[n][c][h][w] (=|+=) sum over the taps (kh, kw) that reach (h, w) of
// cols[n][(c,kh,kw)][(oy,ox)], h = oy*s - p + kh, w = ox*s - p + kw.  One
// thread per Q consecutive w of one image row (n, c, h).
template <int Q>
__global__ void col2im_kernel(const float* __restrict__ cols, float* __restrict__ x, int C, int H, int W, int KH,
                              int KW, int OH, int OW, int pad, int stride, int accumulate, unsigned chunks) {
    pdl_entry();
    const int P = OH * OW;
    const unsigned per_row = (unsigned)W / Q;
    for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < chunks; i += gridDim.x * blockDim.x) {
        const unsigned row = i / per_row;
        const int w0 = (int)(i - row * per_row) * Q;
        const int h = (int)(row % (unsigned)H);
        const unsigned nc = row / (unsigned)H;
        const float* base = cols + (int64_t)nc * KH * KW * P;
        // only taps congruent to h + pad (w + pad) modulo the stride reach
        // (h, w): walk them in ascending order (the gather order of the
        // reference) with the output coordinate stepping down by one
        float s[Q];
        int kw0[Q], ox0[Q];
#pragma unroll
        for (int u = 0; u < Q; ++u) {
            s[u] = 0.f;
            kw0[u] = (w0 + u + pad) % stride;
            ox0[u] = (w0 + u + pad - kw0[u]) / stride;
        }
        const int kh0 = (h + pad) % stride;
        int oy = (h + pad - kh0) / stride;
        for (int kh = kh0; kh < KH && oy >= 0; kh += stride, --oy) {
            if (oy >= OH) continue;
            const float* rowp = base + (int64_t)kh * KW * P + (int64_t)oy * OW;
#pragma unroll
            for (int u = 0; u < Q; ++u) {
                int ox = ox0[u];
                for (int kw = kw0[u]; kw < KW && ox >= 0; kw += stride, --ox)
                    if (ox < OW) s[u] += __ldg(rowp + (int64_t)kw * P + ox);
            }
        }
        float* dst = x + (int64_t)i * Q;
        if constexpr (Q == 4) {
            float4 o = make_float4(s[0], s[1], s[2], s[3]);
            if (accumulate) {
                const float4 a = *reinterpret_cast<const float4*>(dst);
                o.x += a.x;
                o.y += a.y;
                o.z += a.z;
                o.w += a.w;
            }
            *reinterpret_cast<float4*>(dst) = o;
        } else {
#pragma unroll
            for (int u = 0; u < Q; ++u) dst[u] = accumulate ? dst[u] + s[u] : s[u];
        }
    }
}

// dst[b][n][c][y][x] = src[n][c][y][x + b + shift] (0 outside the source
// row), b < KW, x < WD: the horizontally shifted copies an implicit-GEMM
// convolution reads its taps from.  One thread per 4 consecutive x of one
// row; WD % 4 == 0.
__global__ void shift_copies_kernel(const float* __restrict__ src, float* __restrict__ dst, int rows, int WS, int WD,
                                    int KW, int shift, int64_t copy_stride) {
    pdl_entry();
    const int q4 = WD >> 2;
    const int64_t total = (int64_t)rows * q4;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += step) {
        const int row = (int)(i / q4);
        const int x0 = (int)(i - (int64_t)row * q4) * 4;
        const float* s = src + (int64_t)row * WS;
        float v[4 + 15];
        const int lo = x0 + shift;
#pragma unroll 4
        for (int u = 0; u < KW + 3; ++u) {
            const int xs = lo + u;
            v[u] = (xs >= 0 && xs < WS) ? __ldg(s + xs) : 0.f;
        }
        float* d = dst + (int64_t)row * WD + x0;
        for (int b = 0; b < KW; ++b)
            *reinterpret_cast<float4*>(d + (int64_t)b * copy_stride) = make_float4(v[b], v[b + 1], v[b + 2], v[b + 3]);
    }
}

// Weight layouts for the implicit GEMM (taps t = kh*KW + kw, T taps):
//   mode 0: out[t][co][ld] = w[co][ci][t]          (0 for ci >= Cin)
//   mode 1: out[t][ci][ld] = w[co][ci][T - 1 - t]  (0 for co >= Cout)
//   mode 2: out[co][ci][t] = in[t][co][ci] (row pitch ld)  -- dW back to [Cout][Cin][KH][KW]
__global__ void conv_weight_pack_kernel(const float* __restrict__ in, float* __restrict__ out, int Cout, int Cin,
                                        int T, int ld, int mode, int64_t total) {
    pdl_entry();
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += step) {
        if (mode == 0) {
            const int c = (int)(i % ld);
            const int64_t r = i / ld;
            const int co = (int)(r % Cout), t = (int)(r / Cout);
            out[i] = c < Cin ? in[((int64_t)co * Cin + c) * T + t] : 0.f;
        } else if (mode == 1) {
            const int co = (int)(i % ld);
            const int64_t r = i / ld;
            const int ci = (int)(r % Cin), t = (int)(r / Cin);
            out[i] = co < Cout ? in[((int64_t)co * Cin + ci) * T + (T - 1 - t)] : 0.f;
        } else {
            const int t = (int)(i % T);
            const int64_t r = i / T;
            const int ci = (int)(r % Cin), co = (int)(r / Cin);
            out[i] = in[((int64_t)t * Cout + co) * ld + ci];
        }
    }
}

// ------------------------------------------------------------ stride 2
// A stride-2 convolution is a stride-1 convolution over the polyphase
// sub-images of its input: phase (py, px) holds x[2Y + py][2X + px], and a
// tap (kh, kw) with kh - pad = 2a + py, kw - pad = 2b + px reads phase
// (py, px) at (oy + a, ox + b).  The phases in use (those some tap reads)
// become the channels of one image, c' = phase * Cin + ci, and the taps
// collapse onto a KH2 x KW2 kernel whose top/left padding is -min a.
struct PhaseGeom {
    int h2, w2;        // phase image size
    int py0, npy;      // rows phases in use: py0 .. py0 + npy - 1
    int px0, npx;
    int k2, pad2;      // virtual square kernel and its top/left padding
    int oh, ow;        // the stride-2 output size
    int nph() const { return npy * npx; }
};

__host__ __device__ inline int floor_half(int a) { return a >= 0 ? a / 2 : -((1 - a) / 2); }

// false where the virtual kernel is not square with one padding
bool phase_geom(int h, int w, int kh, int kw, int pad, PhaseGeom& g) {
    auto axis = [&](int k, int& p0, int& np, int& k2, int& pad2) {
        const int amin = floor_half(-pad), amax = floor_half(k - 1 - pad);
        k2 = amax - amin + 1;
        pad2 = -amin;
        const int r0 = ((-pad) % 2 + 2) % 2;  // phase of tap 0
        np = k > 1 ? 2 : 1;
        p0 = np == 2 ? 0 : r0;
    };
    int k2h, p2h, k2w, p2w;
    axis(kh, g.py0, g.npy, k2h, p2h);
    axis(kw, g.px0, g.npx, k2w, p2w);
    if (k2h != k2w || p2h != p2w) return false;
    g.k2 = k2h;
    g.pad2 = p2h;
    g.h2 = (h + 1) / 2;
    g.w2 = (w + 1) / 2;
    g.oh = (h + 2 * pad - kh) / 2 + 1;
    g.ow = (w + 2 * pad - kw) / 2 + 1;
    return g.oh > 0 && g.ow > 0;
}

// P[n][(iy * npx + ix) * C + c][Y][X] = x[n][c][2Y + py0 + iy][2X + px0 + ix] (0 outside)
__global__ void phase_split_kernel(const float* __restrict__ x, float* __restrict__ P, int C, int H, int W, int H2,
                                   int W2, int py0, int npy, int px0, int npx, int64_t total) {
    pdl_entry();
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += step) {
        const int X = (int)(i % W2);
        int64_t r = i / W2;
        const int Y = (int)(r % H2);
        r /= H2;
        const int cp = (int)(r % ((int64_t)npy * npx * C));
        const int64_t n = r / ((int64_t)npy * npx * C);
        const int ph = cp / C, c = cp - ph * C;
        const int y = 2 * Y + py0 + ph / npx, xx = 2 * X + px0 + ph % npx;
        P[i] = (y < H && xx < W) ? x[((n * C + c) * H + y) * W + xx] : 0.f;
    }
}

// dx[n][c][y][x] (= or +=) dP[n][phase(y, x) * C + c][y / 2][x / 2]; a
// pixel of an unused phase receives nothing (0 when assigned)
__global__ void phase_merge_kernel(const float* __restrict__ dP, float* __restrict__ dx, int C, int H, int W, int H2,
                                   int W2, int py0, int npy, int px0, int npx, int accumulate, int64_t total) {
    pdl_entry();
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += step) {
        const int xx = (int)(i % W);
        int64_t r = i / W;
        const int y = (int)(r % H);
        r /= H;
        const int c = (int)(r % C);
        const int64_t n = r / C;
        const int iy = (y & 1) - py0, ix = (xx & 1) - px0;
        float v = 0.f;
        if (iy >= 0 && iy < npy && ix >= 0 && ix < npx)
            v = dP[((n * npy * npx + iy * npx + ix) * C + c) * (int64_t)H2 * W2 + (int64_t)(y >> 1) * W2 + (xx >> 1)];
        dx[i] = accumulate ? dx[i] + v : v;
    }
}

// mode 0 (expand): W2[co][(iy*npx+ix)*Cin + ci][th][tw] = W[co][ci][kh][kw],
//   kh = 2 (th - pad2) + py0 + iy + pad (0 where kh or kw falls outside);
// mode 1 (contract): W[co][ci][kh][kw] = W2[co][c'][th][tw] for the one
//   virtual tap each real tap maps to (assigned)
__global__ void phase_weights_kernel(const float* __restrict__ in, float* __restrict__ out, int Cout, int Cin, int KH,
                                     int KW, int pad, int k2, int pad2, int py0, int npy, int px0, int npx, int mode,
                                     int64_t total) {
    pdl_entry();
    const int nph = npy * npx;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += step) {
        if (mode == 0) {
            const int tw = (int)(i % k2);
            int64_t r = i / k2;
            const int th = (int)(r % k2);
            r /= k2;
            const int cp = (int)(r % ((int64_t)nph * Cin));
            const int co = (int)(r / ((int64_t)nph * Cin));
            const int ph = cp / Cin, ci = cp - ph * Cin;
            const int kh = 2 * (th - pad2) + py0 + ph / npx + pad, kw = 2 * (tw - pad2) + px0 + ph % npx + pad;
            out[i] = (kh >= 0 && kh < KH && kw >= 0 && kw < KW) ? in[(((int64_t)co * Cin + ci) * KH + kh) * KW + kw]
                                                                 : 0.f;
        } else {
            const int kw = (int)(i % KW);
            int64_t r = i / KW;
            const int kh = (int)(r % KH);
            r /= KH;
            const int ci = (int)(r % Cin);
            const int co = (int)(r / Cin);
            const int ah = floor_half(kh - pad), aw = floor_half(kw - pad);
            const int py = kh - pad - 2 * ah, px = kw - pad - 2 * aw;
            const int ph = (py - py0) * npx + (px - px0);
            const int th = ah + pad2, tw = aw + pad2;
            out[i] = in[((((int64_t)co * nph + ph) * Cin + ci) * k2 + th) * k2 + tw];
        }
    }
}

// out = in with two of its three dimensions exchanged:
//   mode 0: [A][B][C] -> [B][A][C];  mode 1: [A][B][C] -> [A][C][B]
__global__ void swap_dims_kernel(const float* __restrict__ in, float* __restrict__ out, int A, int B, int C, int mode,
                                 int64_t total) {
    pdl_entry();
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += step) {
        const int c = (int)(i % C);
        const int b = (int)((i / C) % B);
        const int a = (int)(i / ((int64_t)B * C));
        const int64_t o = mode == 0 ? ((int64_t)b * A + a) * C + c : ((int64_t)a * C + c) * B + b;
        out[o] = in[i];
    }
}

int im2col(const float* x, float* cols, int n, int c, int h, int w, int kh, int kw, int oh, int ow, int pad,
           int stride, cudaStream_t st) {
    const bool v4 = ow % 4 == 0 && aligned16(cols);
    const int64_t chunks = (int64_t)n * c * kh * kw * oh * ow / (v4 ? 4 : 1);
    if (chunks == 0) return MLE_OK;
    if (chunks > INT32_MAX || (int64_t)h * w > INT32_MAX) return MLE_ERR_UNSUPPORTED;
    const unsigned grid = grid_for(chunks, kRowThreads);
    if (v4)
        launch_k(im2col_kernel<4>, grid, kRowThreads, 0, st, x, cols, c, h, w, kh, kw, oh, ow, pad, stride,
                 (unsigned)chunks);
    else
        launch_k(im2col_kernel<1>, grid, kRowThreads, 0, st, x, cols, c, h, w, kh, kw, oh, ow, pad, stride,
                 (unsigned)chunks);
    return launch_status();
}

int col2im(const float* cols, float* x, int n, int c, int h, int w, int kh, int kw, int oh, int ow, int pad,
           int stride, int accumulate, cudaStream_t st) {
    const bool v4 = w % 4 == 0 && aligned16(x);
    const int64_t chunks = (int64_t)n * c * h * w / (v4 ? 4 : 1);
    if (chunks == 0) return MLE_OK;
    if (chunks > INT32_MAX || (int64_t)oh * ow > INT32_MAX) return MLE_ERR_UNSUPPORTED;
    const unsigned grid = grid_for(chunks, kRowThreads);
    if (v4)
        launch_k(col2im_kernel<4>, grid, kRowThreads, 0, st, cols, x, c, h, w, kh, kw, oh, ow, pad, stride, accumulate,
                 (unsigned)chunks);
    else
        launch_k(col2im_kernel<1>, grid, kRowThreads, 0, st, cols, x, c, h, w, kh, kw, oh, ow, pad, stride, accumulate,
                 (unsigned)chunks);
    return launch_status();
}

int shift_copies(const float* src, float* dst, int rows, int ws, int wd, int kw, int shift, cudaStream_t st) {
    const int64_t total = (int64_t)rows * (wd / 4);
    if (total == 0) return MLE_OK;
    launch_k(shift_copies_kernel, grid_for(total, kT), kT, 0, st, src, dst, rows, ws, wd, kw, shift,
             (int64_t)rows * wd);
    return launch_status();
}

int weight_pack(const float* in, float* out, int cout, int cin, int taps, int ld, int mode, cudaStream_t st) {
    const int64_t total = mode == 0   ? (int64_t)taps * cout * ld
                          : mode == 1 ? (int64_t)taps * cin * ld
                                      : (int64_t)cout * cin * taps;
    if (total == 0) return MLE_OK;
    launch_k(conv_weight_pack_kernel, grid_for(total, kT), kT, 0, st, in, out, cout, cin, taps, ld, mode, total);
    return launch_status();
}

int swap_dims(const float* in, float* out, int a, int b, int c, int mode, cudaStream_t st) {
    const int64_t total = (int64_t)a * b * c;
    if (total == 0) return MLE_OK;
    launch_k(swap_dims_kernel, grid_for(total, kT), kT, 0, st, in, out, a, b, c, mode, total);
    return launch_status();
}

bool conv_shape_ok(int batch, int cin, int h, int w, int cout, int kh, int kw, int pad, int stride) {
    return batch > 0 && cin > 0 && h > 0 && w > 0 && cout > 0 && kh > 0 && kw > 0 && pad >= 0 && stride > 0;
}

int64_t r4(int64_t n) { return (n + 3) & ~int64_t(3); }

// Implicit-GEMM plan of a stride-1 Convolute2D (ConvGemm, gemm.cuh):
//   forward y = kind 1 over S = KW shifted copies of x (width OW), weights
//               packed [tap][Cout][Cin4];
//   dW        = kind 2 over the same S and dy, into [tap][Cout][Cin4], then
//               unpacked to [Cout][Cin][KH][KW];
//   dx       += kind 1 over KW shifted copies of dy (width W) with the taps
//               flipped, weights packed [tap][Cin][Cout4], row offset KH-1-pad.
// A 1x1 unpadded convolution reads x and dy in place.  The workspace holds
// S (kept from the forward for the backward), the packed weights (also the
// dW staging) and the copies of dy.
struct ConvPlan {
    int h, oh, ow, taps, cin4, cout4;
    bool in_place;            // KW == 1 and pad == 0: no shifted copies
    int64_t xs, wp, wd, dys;  // workspace offsets (floats)
    int64_t floats;
};

// oh, ow >= 0: an output smaller than the padded one (the stride-2 phase
// form, whose padding is top/left only)
ConvPlan conv_plan(int batch, int cin, int h, int w, int cout, int kh, int kw, int pad, int oh = -1, int ow = -1) {
    ConvPlan p;
    p.h = h;
    p.oh = oh >= 0 ? oh : h + 2 * pad - kh + 1;
    p.ow = ow >= 0 ? ow : w + 2 * pad - kw + 1;
    p.taps = kh * kw;
    p.cin4 = (int)r4(cin);
    p.cout4 = (int)r4(cout);
    p.in_place = kw == 1 && pad == 0;
    const int64_t n_xs = p.in_place ? 0 : (int64_t)kw * batch * cin * h * p.ow;
    const int64_t n_dys = p.in_place ? 0 : (int64_t)kw * batch * cout * p.oh * w;
    p.xs = 0;
    p.wp = r4(n_xs);
    p.wd = p.wp + r4((int64_t)p.taps * cout * p.cin4);
    p.dys = p.wd + r4((int64_t)p.taps * cin * p.cout4);
    p.floats = p.dys + r4(n_dys);
    return p;
}

ConvGemm conv_fwd_gemm(const ConvPlan& p, const float* x, const float* ws, float* y, int batch, int cin, int h,
                       int cout, int kh, int kw, int pad) {
    ConvGemm g;
    memset(&g, 0, sizeof(g));
    g.kind = 1;
    g.A = ws + p.wp;
    g.S = p.in_place ? x : ws + p.xs;
    g.out = y;
    g.M = cout;
    g.C = cin;
    g.HS = h;
    g.WS = p.ow;
    g.KH = kh;
    g.KW = kw;
    g.pad = pad;
    g.nb = batch;
    g.P = p.oh * p.ow;
    g.lda = p.cin4;
    return g;
}

ConvGemm conv_dw_gemm(const ConvPlan& p, const float* x, const float* dy, float* ws, int batch, int cin, int h,
                      int cout, int kh, int kw, int pad) {
    ConvGemm g = conv_fwd_gemm(p, x, ws, ws + p.wp, batch, cin, h, cout, kh, kw, pad);
    g.kind = 2;
    g.A = dy;
    g.ldc = p.cin4;
    return g;
}

ConvGemm conv_dx_gemm(const ConvPlan& p, const float* dy, float* ws, float* dx, int batch, int cin, int w,
                      int cout, int kh, int kw, int pad) {
    ConvGemm g;
    memset(&g, 0, sizeof(g));
    g.kind = 1;
    g.A = ws + p.wd;
    g.S = p.in_place ? dy : ws + p.dys;
    g.out = dx;
    g.M = cin;
    g.C = cout;
    g.HS = p.oh;
    g.WS = w;
    g.KH = kh;
    g.KW = kw;
    g.pad = kh - 1 - pad;
    g.nb = batch;
    g.P = p.h * w;
    g.lda = p.cout4;
    g.accumulate = 1;
    return g;
}

// The implicit path runs for stride 1 when all three products are supported
// (tensor-core mode, widths whose 32-pixel blocks TMA can address).  The
// choice depends only on the shape, the GEMM mode and x / ws, which the
// forward and the backward share, so both take the same path; a gradient
// pointer that TMA cannot address then fails the call.
bool conv_implicit_ok(const float* x, float* ws, int batch, int cin, int h, int w, int cout, int kh, int kw, int pad,
                      int stride) {
    if (stride != 1 || kw - 1 - pad < 0 || kh - 1 - pad < 0) return false;
    const ConvPlan p = conv_plan(batch, cin, h, w, cout, kh, kw, pad);
    if (p.oh <= 0 || p.ow <= 0) return false;
    const ConvGemm f = conv_fwd_gemm(p, x, ws, ws, batch, cin, h, cout, kh, kw, pad);
    const ConvGemm d = conv_dx_gemm(p, p.in_place ? x : ws, ws, ws, batch, cin, w, cout, kh, kw, pad);
    const ConvGemm g = conv_dw_gemm(p, x, ws, ws, batch, cin, h, cout, kh, kw, pad);
    return conv_gemm_supported(f) && conv_gemm_supported(d) && conv_gemm_supported(g);
}

// Plan of the stride-2 phase form: the stride-1 plan over the phase image
// (nph * Cin channels of h2 x w2, a k2 x k2 kernel, top/left padding pad2,
// the stride-2 output size), plus the phase image (dP in the backward), the
// expanded weights and the expanded dW.
struct PhasePlan {
    PhaseGeom g;
    ConvPlan p;
    int cin2;
    int64_t pP, pdP, pWe, pWd, floats;
};

bool phase_plan(int batch, int cin, int h, int w, int cout, int kh, int kw, int pad, PhasePlan& q) {
    if (!phase_geom(h, w, kh, kw, pad, q.g)) return false;
    const PhaseGeom& g = q.g;
    if (g.k2 - 1 - g.pad2 < 0) return false;
    q.cin2 = g.nph() * cin;
    q.p = conv_plan(batch, q.cin2, g.h2, g.w2, cout, g.k2, g.k2, g.pad2, g.oh, g.ow);
    const int64_t nw = (int64_t)cout * q.cin2 * g.k2 * g.k2;
    q.pP = q.p.floats;
    // dP apart from the phase image: dW may read the image (in place) while dx runs
    q.pdP = q.pP + r4((int64_t)batch * q.cin2 * g.h2 * g.w2);
    q.pWe = q.pdP + r4((int64_t)batch * q.cin2 * g.h2 * g.w2);
    q.pWd = q.pWe + r4(nw);
    q.floats = q.pWd + r4(nw);
    return true;
}

// The phase form runs for stride 2 when its three products are supported,
// on the same conditions as the stride-1 implicit path (the forward and the
// backward make the same choice).
// stride 2 through the phase form: 0 never (im2col, the default: it
// measured faster on the U-Net step), 1 where the phase kernel has no empty
// taps (phases x taps of the phase kernel = the real taps: 1x1 and 2x2
// kernels; a 3x3 kernel at pad 1 runs 16 products per output for 9), 2
// always
static thread_local int g_conv_phase = 0;

bool phase_implicit_ok(float* ws, int batch, int cin, int h, int w, int cout, int kh, int kw, int pad, int stride) {
    PhasePlan q;
    if (!g_conv_phase || stride != 2 || !phase_plan(batch, cin, h, w, cout, kh, kw, pad, q)) return false;
    if (g_conv_phase == 1 && q.g.nph() * q.g.k2 * q.g.k2 != kh * kw) return false;
    const ConvPlan& p = q.p;
    const PhaseGeom& g = q.g;
    const float* P = ws + q.pP;
    const ConvGemm f = conv_fwd_gemm(p, P, ws, ws, batch, q.cin2, g.h2, cout, g.k2, g.k2, g.pad2);
    const ConvGemm d = conv_dx_gemm(p, p.in_place ? P : ws, ws, ws + q.pdP, batch, q.cin2, g.w2, cout, g.k2, g.k2,
                                    g.pad2);
    const ConvGemm gw = conv_dw_gemm(p, P, ws, ws, batch, q.cin2, g.h2, cout, g.k2, g.k2, g.pad2);
    return conv_gemm_supported(f) && conv_gemm_supported(d) && conv_gemm_supported(gw);
}

int phase_split(const float* x, float* P, int n, int c, int h, int w, const PhaseGeom& g, cudaStream_t st) {
    const int64_t total = (int64_t)n * g.nph() * c * g.h2 * g.w2;
    launch_k(phase_split_kernel, grid_for(total, kT), kT, 0, st, x, P, c, h, w, g.h2, g.w2, g.py0, g.npy, g.px0,
             g.npx, total);
    return launch_status();
}

int phase_merge(const float* dP, float* dx, int n, int c, int h, int w, const PhaseGeom& g, int accumulate,
                cudaStream_t st) {
    const int64_t total = (int64_t)n * c * h * w;
    launch_k(phase_merge_kernel, grid_for(total, kT), kT, 0, st, dP, dx, c, h, w, g.h2, g.w2, g.py0, g.npy, g.px0,
             g.npx, accumulate, total);
    return launch_status();
}

int phase_weights(const float* in, float* out, int cout, int cin, int kh, int kw, int pad, const PhaseGeom& g,
                  int mode, cudaStream_t st) {
    const int64_t total = mode == 0 ? (int64_t)cout * g.nph() * cin * g.k2 * g.k2 : (int64_t)cout * cin * kh * kw;
    launch_k(phase_weights_kernel, grid_for(total, kT), kT, 0, st, in, out, cout, cin, kh, kw, pad, g.k2, g.pad2,
             g.py0, g.npy, g.px0, g.npx, mode, total);
    return launch_status();
}

}  // namespace
}  // namespace mle

using namespace mle;

extern "C" {

int mle_set_conv_phase(int enable) {
    if (enable < 0 || enable > 2) return MLE_ERR_ARG;
    g_conv_phase = enable;
    return MLE_OK;
}

int mle_get_conv_phase(void) { return g_conv_phase; }

int mle_conv_out_size(int in, int k, int pad, int stride) {
    if (stride <= 0 || in + 2 * pad < k) return -1;
    return (in + 2 * pad - k) / stride + 1;
}

int mle_convT_out_size(int in, int k, int pad, int stride) { return (in - 1) * stride - 2 * pad + k; }

int mle_im2col(const float* x, float* cols, int batch, int channels, int h, int w, int kh, int kw, int pad, int stride,
               mle_stream_t stream) {
    if (!x || !cols || batch < 0 || channels <= 0 || kh <= 0 || kw <= 0 || stride <= 0 || pad < 0) return MLE_ERR_ARG;
    const int oh = mle_conv_out_size(h, kh, pad, stride), ow = mle_conv_out_size(w, kw, pad, stride);
    if (oh <= 0 || ow <= 0) return MLE_ERR_ARG;
    return im2col(x, cols, batch, channels, h, w, kh, kw, oh, ow, pad, stride, as_stream(stream));
}

int mle_col2im(const float* cols, float* x, int batch, int channels, int h, int w, int kh, int kw, int pad, int stride,
               int accumulate, mle_stream_t stream) {
    if (!x || !cols || batch < 0 || channels <= 0 || kh <= 0 || kw <= 0 || stride <= 0 || pad < 0) return MLE_ERR_ARG;
    const int oh = mle_conv_out_size(h, kh, pad, stride), ow = mle_conv_out_size(w, kw, pad, stride);
    if (oh <= 0 || ow <= 0) return MLE_ERR_ARG;
    return col2im(cols, x, batch, channels, h, w, kh, kw, oh, ow, pad, stride, accumulate, as_stream(stream));
}

int mle_swap_dims(const float* in, float* out, int a, int b, int c, int mode, mle_stream_t stream) {
    if (!in || !out || a < 0 || b < 0 || c < 0 || (mode != 0 && mode != 1) || in == out) return MLE_ERR_ARG;
    return swap_dims(in, out, a, b, c, mode, as_stream(stream));
}

int64_t mle_conv2d_workspace_floats(int batch, int cin, int h, int w, int cout, int kh, int kw, int pad, int stride) {
    const int oh = mle_conv_out_size(h, kh, pad, stride), ow = mle_conv_out_size(w, kw, pad, stride);
    if (batch <= 0 || cin <= 0 || cout <= 0 || kh <= 0 || kw <= 0 || oh <= 0 || ow <= 0) return -1;
    // room for either path: the choice also depends on the GEMM mode and
    // pointer alignment at call time.  The column path keeps the forward's
    // columns (read by dW) and the input gradient's columns apart, so the
    // dx and dw/db parts of the backward may run concurrently.
    int64_t n = 2 * (int64_t)batch * cin * kh * kw * oh * ow;
    if (stride == 1) n = std::max(n, conv_plan(batch, cin, h, w, cout, kh, kw, pad).floats);
    PhasePlan q;
    if (stride == 2 && phase_plan(batch, cin, h, w, cout, kh, kw, pad, q)) n = std::max(n, q.floats);
    return n;
}

int mle_conv2d_fwd(const float* x, const float* wgt, const float* bias, float* y, float* ws, int batch, int cin,
                   int h, int w, int cout, int kh, int kw, int pad, int stride, mle_stream_t stream) {
    if (!x || !wgt || !y || !ws || !conv_shape_ok(batch, cin, h, w, cout, kh, kw, pad, stride)) return MLE_ERR_ARG;
    const int oh = mle_conv_out_size(h, kh, pad, stride), ow = mle_conv_out_size(w, kw, pad, stride);
    if (oh <= 0 || ow <= 0) return MLE_ERR_ARG;
    cudaStream_t st = as_stream(stream);
    const int64_t P = (int64_t)oh * ow, K = (int64_t)cin * kh * kw;
    int s;
    if (phase_implicit_ok(ws, batch, cin, h, w, cout, kh, kw, pad, stride)) {
        // stride 2: the stride-1 implicit GEMM over the phase image
        PhasePlan q;
        phase_plan(batch, cin, h, w, cout, kh, kw, pad, q);
        const ConvPlan& p = q.p;
        const PhaseGeom& g = q.g;
        float* Pimg = ws + q.pP;
        s = phase_split(x, Pimg, batch, cin, h, w, g, st);
        if (s) return s;
        if (!p.in_place) {
            s = shift_copies(Pimg, ws + p.xs, batch * q.cin2 * g.h2, g.w2, p.ow, g.k2, -g.pad2, st);
            if (s) return s;
        }
        s = phase_weights(wgt, ws + q.pWe, cout, cin, kh, kw, pad, g, 0, st);
        if (s) return s;
        s = weight_pack(ws + q.pWe, ws + p.wp, cout, q.cin2, p.taps, p.cin4, 0, st);
        if (s) return s;
        ConvGemm gm = conv_fwd_gemm(p, Pimg, ws, y, batch, q.cin2, g.h2, cout, g.k2, g.k2, g.pad2);
        gm.bias = bias;
        return run_conv_gemm(gm, st);
    }
    if (conv_implicit_ok(x, ws, batch, cin, h, w, cout, kh, kw, pad, stride)) {
        const ConvPlan p = conv_plan(batch, cin, h, w, cout, kh, kw, pad);
        if (!p.in_place) {
            s = shift_copies(x, ws + p.xs, batch * cin * h, w, p.ow, kw, -pad, st);
            if (s) return s;
        }
        s = weight_pack(wgt, ws + p.wp, cout, cin, p.taps, p.cin4, 0, st);
        if (s) return s;
        ConvGemm g = conv_fwd_gemm(p, x, ws, y, batch, cin, h, cout, kh, kw, pad);
        g.bias = bias;  // added by the GEMM
        return run_conv_gemm(g, st);
    } else {
        s = im2col(x, ws, batch, cin, h, w, kh, kw, oh, ow, pad, stride, st);
        if (s) return s;
        // y[n][Cout][P] = W[Cout][K] * cols[n][K][P]
        s = mle_gemm(wgt, ws, y, nullptr, batch, cout, P, K, K, P, P, 0, K * P, cout * P, 0, 0, 1.0f, 0.0f, stream);
    }
    if (s || !bias) return s;
    return mle_channel_bias_fwd(y, bias, y, batch, cout, P, stream);
}

int mle_conv2d_bwd(const float* x, const float* wgt, const float* dy, float* dx, float* dw, float* db, float* ws,
                   int batch, int cin, int h, int w, int cout, int kh, int kw, int pad, int stride,
                   mle_stream_t stream) {
    return mle_conv2d_bwd_assign(x, wgt, dy, dx, dw, db, ws, batch, cin, h, w, cout, kh, kw, pad, stride, 0, stream);
}

int mle_conv2d_bwd_assign(const float* x, const float* wgt, const float* dy, float* dx, float* dw, float* db,
                          float* ws, int batch, int cin, int h, int w, int cout, int kh, int kw, int pad, int stride,
                          int assign_dx, mle_stream_t stream) {
    if (assign_dx != 0 && assign_dx != 1) return MLE_ERR_ARG;
    if (!x || !wgt || !dy || !ws || !conv_shape_ok(batch, cin, h, w, cout, kh, kw, pad, stride)) return MLE_ERR_ARG;
    const int oh = mle_conv_out_size(h, kh, pad, stride), ow = mle_conv_out_size(w, kw, pad, stride);
    if (oh <= 0 || ow <= 0) return MLE_ERR_ARG;
    cudaStream_t st = as_stream(stream);
    const int64_t P = (int64_t)oh * ow, K = (int64_t)cin * kh * kw;
    int s;
    if (db) {
        s = mle_channel_bias_bwd(dy, nullptr, db, batch, cout, P, stream);
        if (s) return s;
    }
    if (phase_implicit_ok(ws, batch, cin, h, w, cout, kh, kw, pad, stride)) {
        PhasePlan q;
        phase_plan(batch, cin, h, w, cout, kh, kw, pad, q);
        const ConvPlan& p = q.p;
        const PhaseGeom& g = q.g;
        float* Pimg = ws + q.pP;  // the forward's phase image
        float* dP = ws + q.pdP;
        const int taps2 = p.taps;
        if (dw) {
            // dW' over the forward's shifted phase copies (or the phase image
            // itself), staged [tap][Cout][Cin2_4], unpacked to the expanded
            // layout, then folded back onto the real taps (assigned)
            if (cudaMemsetAsync(ws + p.wp, 0, sizeof(float) * (size_t)taps2 * cout * p.cin4, st) != cudaSuccess)
                return launch_status();
            s = run_conv_gemm(conv_dw_gemm(p, Pimg, dy, ws, batch, q.cin2, g.h2, cout, g.k2, g.k2, g.pad2), st);
            if (s) return s;
            s = weight_pack(ws + p.wp, ws + q.pWd, cout, q.cin2, taps2, p.cin4, 2, st);
            if (s) return s;
            s = phase_weights(ws + q.pWd, dw, cout, cin, kh, kw, pad, g, 1, st);
            if (s) return s;
        }
        if (dx) {
            if (!p.in_place) {
                s = shift_copies(dy, ws + p.dys, batch * cout * p.oh, p.ow, g.w2, g.k2, -(g.k2 - 1 - g.pad2), st);
                if (s) return s;
            }
            s = phase_weights(wgt, ws + q.pWe, cout, cin, kh, kw, pad, g, 0, st);
            if (s) return s;
            s = weight_pack(ws + q.pWe, ws + p.wd, cout, q.cin2, taps2, p.cout4, 1, st);
            if (s) return s;
            ConvGemm gm = conv_dx_gemm(p, dy, ws, dP, batch, q.cin2, g.w2, cout, g.k2, g.k2, g.pad2);
            gm.accumulate = 0;
            s = run_conv_gemm(gm, st);
            if (s) return s;
            return phase_merge(dP, dx, batch, cin, h, w, g, assign_dx ? 0 : 1, st);
        }
        return MLE_OK;
    }
    if (conv_implicit_ok(x, ws, batch, cin, h, w, cout, kh, kw, pad, stride)) {
        const ConvPlan p = conv_plan(batch, cin, h, w, cout, kh, kw, pad);
        if (dw) {
            // dW staged as [tap][Cout][Cin4] (reduce-added over images and
            // pixels), then assigned in the reference layout (as GV2D)
            if (cudaMemsetAsync(ws + p.wp, 0, sizeof(float) * (size_t)p.taps * cout * p.cin4, st) != cudaSuccess)
                return launch_status();
            s = run_conv_gemm(conv_dw_gemm(p, x, dy, ws, batch, cin, h, cout, kh, kw, pad), st);
            if (s) return s;
            s = weight_pack(ws + p.wp, dw, cout, cin, p.taps, p.cin4, 2, st);
            if (s) return s;
        }
        if (dx) {
            if (!p.in_place) {
                s = shift_copies(dy, ws + p.dys, batch * cout * oh, ow, w, kw, -(kw - 1 - pad), st);
                if (s) return s;
            }
            s = weight_pack(wgt, ws + p.wd, cout, cin, p.taps, p.cout4, 1, st);
            if (s) return s;
            ConvGemm g = conv_dx_gemm(p, dy, ws, dx, batch, cin, w, cout, kh, kw, pad);
            g.accumulate = assign_dx ? 0 : 1;
            return run_conv_gemm(g, st);
        }
        return MLE_OK;
    }
    if (dw) {
        // the forward left cols(x) in ws
        // dW[Cout][K] = sum_n dy[n][Cout][P] * cols[n][K][P]^T  (assigned, as GV2D)
        if (cudaMemsetAsync(dw, 0, sizeof(float) * (size_t)(cout * K), st) != cudaSuccess) return launch_status();
        s = mle_gemm(dy, ws, dw, nullptr, batch, cout, K, P, P, P, K, cout * P, K * P, 0, 0, 1, 1.0f, 1.0f, stream);
        if (s) return s;
    }
    if (dx) {
        // input-gradient columns after the forward's: dcols[n][K][P] = W^T * dy[n], then dx += col2im
        float* dcols = ws + (int64_t)batch * K * P;
        s = mle_gemm(wgt, dy, dcols, nullptr, batch, K, P, cout, K, P, P, 0, cout * P, K * P, 1, 0, 1.0f, 0.0f,
                     stream);
        if (s) return s;
        return col2im(dcols, dx, batch, cin, h, w, kh, kw, oh, ow, pad, stride, assign_dx ? 0 : 1, st);
    }
    return MLE_OK;
}

int64_t mle_convT2d_workspace_floats(int batch, int cin, int h, int w, int cout, int kh, int kw, int pad, int stride) {
    const int oh = mle_convT_out_size(h, kh, pad, stride), ow = mle_convT_out_size(w, kw, pad, stride);
    if (batch <= 0 || cin <= 0 || cout <= 0 || oh <= 0 || ow <= 0 || stride <= 0) return -1;
    const int64_t KK = (int64_t)cout * kh * kw;
    return 2 * KK * cin + (int64_t)batch * KK * h * w;
}

int mle_convT2d_fwd(const float* x, const float* wgt, const float* bias, float* y, float* ws, int batch, int cin,
                    int h, int w, int cout, int kh, int kw, int pad, int stride, mle_stream_t stream) {
    if (!x || !wgt || !y || !ws || !conv_shape_ok(batch, cin, h, w, cout, kh, kw, pad, stride)) return MLE_ERR_ARG;
    const int oh = mle_convT_out_size(h, kh, pad, stride), ow = mle_convT_out_size(w, kw, pad, stride);
    if (oh <= 0 || ow <= 0 || mle_conv_out_size(oh, kh, pad, stride) != h || mle_conv_out_size(ow, kw, pad, stride) != w)
        return MLE_ERR_ARG;
    cudaStream_t st = as_stream(stream);
    const int64_t P = (int64_t)h * w, KK = (int64_t)cout * kh * kw;
    float* wswap = ws;                 // [Cin][Cout][KH][KW]
    float* cols = ws + 2 * KK * cin;   // [n][Cout*KH*KW][h*w]
    int s = swap_dims(wgt, wswap, cout, cin, kh * kw, 0, st);
    if (s) return s;
    // cols[n][(oc,kh,kw)][p] = sum_ic W[oc][ic][kh][kw] x[n][ic][p]
    s = mle_gemm(wswap, x, cols, nullptr, batch, KK, P, cin, KK, P, P, 0, (int64_t)cin * P, KK * P, 1, 0, 1.0f, 0.0f,
                 stream);
    if (s) return s;
    // the output image is the "input" of the adjoint convolution geometry
    s = col2im(cols, y, batch, cout, oh, ow, kh, kw, h, w, pad, stride, 0, st);
    if (s || !bias) return s;
    return mle_channel_bias_fwd(y, bias, y, batch, cout, (int64_t)oh * ow, stream);
}

int mle_convT2d_bwd(const float* x, const float* wgt, const float* dy, float* dx, float* dw, float* db, float* ws,
                    int batch, int cin, int h, int w, int cout, int kh, int kw, int pad, int stride,
                    mle_stream_t stream) {
    if (!x || !wgt || !dy || !ws || !conv_shape_ok(batch, cin, h, w, cout, kh, kw, pad, stride)) return MLE_ERR_ARG;
    const int oh = mle_convT_out_size(h, kh, pad, stride), ow = mle_convT_out_size(w, kw, pad, stride);
    if (oh <= 0 || ow <= 0 || mle_conv_out_size(oh, kh, pad, stride) != h || mle_conv_out_size(ow, kw, pad, stride) != w)
        return MLE_ERR_ARG;
    cudaStream_t st = as_stream(stream);
    const int64_t P = (int64_t)h * w, KK = (int64_t)cout * kh * kw;
    float* wswap = ws;
    float* tmp = ws + KK * cin;        // [(oc,kh,kw)][ic]
    float* cols = ws + 2 * KK * cin;   // im2col of dy over the input positions
    int s = im2col(dy, cols, batch, cout, oh, ow, kh, kw, h, w, pad, stride, st);
    if (s) return s;
    if (dw) {
        // tmp[(oc,kh,kw)][ic] = sum_n cols[n][(oc,kh,kw)][p] x[n][ic][p]; dW = tmp
        // with its last two dimensions exchanged (assigned, as GVT2D)
        if (cudaMemsetAsync(tmp, 0, sizeof(float) * (size_t)(KK * cin), st) != cudaSuccess) return launch_status();
        s = mle_gemm(cols, x, tmp, nullptr, batch, KK, cin, P, P, P, cin, KK * P, (int64_t)cin * P, 0, 0, 1, 1.0f, 1.0f,
                     stream);
        if (s) return s;
        s = swap_dims(tmp, dw, cout, kh * kw, cin, 1, st);
        if (s) return s;
    }
    if (db) {
        s = mle_channel_bias_bwd(dy, nullptr, db, batch, cout, (int64_t)oh * ow, stream);
        if (s) return s;
    }
    if (dx) {
        // dx[n][ic][p] = sum_(oc,kh,kw) W[oc][ic][kh][kw] cols[n][(oc,kh,kw)][p]  (assigned, as CVT2D_GradInput)
        s = swap_dims(wgt, wswap, cout, cin, kh * kw, 0, st);
        if (s) return s;
        return mle_gemm(wswap, cols, dx, nullptr, batch, cin, P, KK, KK, P, P, 0, KK * P, (int64_t)cin * P, 0, 0, 1.0f,
                        0.0f, stream);
    }
    return MLE_OK;
}

}  // extern "C"
