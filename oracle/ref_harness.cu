/*
 * Reference-kernel harness -- TEST INFRASTRUCTURE ONLY.
 *
 * Compiled together with the reference's own Engine/kernels.cu (from the
 * ML_Engine source tree, by oracle/build_ref.py) into oracle/_ref/libmle_ref.so.
 * Each extern "C" function launches the reference kernels exactly as the
 * reference's graph lambdas do (same kernels, same grid/block shapes, same
 * order), on device buffers the caller owns and sizes correctly.  The tests
 * use it to pin oracle/mle_oracle.c and to generate tests/golden/ fixtures.
 *
 * Why not the reference's GraphOperations directly: SoftMaxCrossEntropy
 * allocates its softmax buffer with the loss node's total (1 float,
 * Engine/engine.cu:2074-2079) and then writes the full prediction tensor into
 * it (:2094), an out-of-bounds device write; that node is never run here.
 * ref_smce_* below issue the same kernels with a correctly sized buffer.
 *
 * All functions launch on the legacy default stream and return
 * cudaGetLastError().
 */
#include <cuda_runtime.h>

#include "kernels.h"

static inline int blocks(long long n, int tpb) { return (int)((n + tpb - 1) / tpb); }

extern "C" {

int ref_bcmm(int variant, const float* A, const float* B, float* C, int batch, int channels, int m, int n, int p,
             int backward, int A_case, int B_case, int C_case, float scale) {
    dim3 block(BLOCK_SIZE, BLOCK_SIZE);
    dim3 grid((p + BLOCK_SIZE - 1) / BLOCK_SIZE, (m + BLOCK_SIZE - 1) / BLOCK_SIZE, batch * channels);
    switch (variant) {
        case 0: bcmm<<<grid, block>>>(A, B, C, batch, channels, m, n, p, backward, A_case, B_case, C_case, scale); break;
        case 1: bcmmABT<<<grid, block>>>(A, B, C, batch, channels, m, n, p, backward, A_case, B_case, C_case, scale); break;
        case 2: bcmmATB<<<grid, block>>>(A, B, C, batch, channels, m, n, p, backward, A_case, B_case, C_case, scale); break;
        default: bcmmT<<<grid, block>>>(A, B, C, batch, channels, m, n, p, backward, A_case, B_case, C_case, scale); break;
    }
    return (int)cudaGetLastError();
}

/* Linear forward/backward lambdas (Engine/engine.cu:3534-3563) on
 * X [batch, channels, m, n], W [n, p]. */
int ref_linear_fwd(const float* X, const float* W, const float* B1, float* Y, int batch, int channels, int m, int n,
                   int p, int bias) {
    dim3 block(BLOCK_SIZE, BLOCK_SIZE);
    dim3 grid((p + BLOCK_SIZE - 1) / BLOCK_SIZE, (m + BLOCK_SIZE - 1) / BLOCK_SIZE, batch * channels);
    bcmm<<<grid, block>>>(X, W, Y, batch, channels, m, n, p, 0, 3, 0, 3);
    if (bias) BCumAdd<<<(THREADSPERBLOCK + batch * channels * m - 1) / THREADSPERBLOCK, THREADSPERBLOCK>>>(Y, B1, batch, channels, m, p);
    return (int)cudaGetLastError();
}

int ref_linear_bwd(const float* X, const float* W, const float* dY, float* dX, float* dW, float* dB, int batch,
                   int channels, int m, int n, int p, int bias) {
    dim3 block(BLOCK_SIZE, BLOCK_SIZE);
    dim3 grid_dA((n + BLOCK_SIZE - 1) / BLOCK_SIZE, (m + BLOCK_SIZE - 1) / BLOCK_SIZE, batch * channels);
    dim3 grid_dB((p + BLOCK_SIZE - 1) / BLOCK_SIZE, (n + BLOCK_SIZE - 1) / BLOCK_SIZE, batch * channels);
    bcmmABT<<<grid_dA, block>>>(dY, W, dX, batch, channels, m, p, n, 1, 3, 0, 3);
    bcmmATB<<<grid_dB, block>>>(X, dY, dW, batch, channels, n, m, p, 1, 3, 3, 0);
    if (bias) BCompress<<<p, THREADSPERBLOCK>>>(dY, dB, batch, channels, m, p);
    return (int)cudaGetLastError();
}

int ref_act_fwd(int kind, const float* x, float* y, int n) {
    const int g = blocks(n, THREADSPERBLOCK);
    switch (kind) {
        case 0: ReLU<<<g, THREADSPERBLOCK>>>(x, y, n); break;
        case 1: LeakyReLU<<<g, THREADSPERBLOCK>>>(x, y, n); break;
        case 2: SiLU<<<g, THREADSPERBLOCK>>>(x, y, n); break;
        case 3: TaNH<<<g, THREADSPERBLOCK>>>(x, y, n); break;
        case 4: GeLU<<<g, THREADSPERBLOCK>>>(x, y, n); break;
        default: Sigmoid<<<g, THREADSPERBLOCK>>>(x, y, n); break;
    }
    return (int)cudaGetLastError();
}

int ref_act_bwd(int kind, const float* x, const float* gy, float* gx, int n) {
    const int g = blocks(n, THREADSPERBLOCK);
    switch (kind) {
        case 0: deriv_ReLU<<<g, THREADSPERBLOCK>>>(x, gy, gx, n); break;
        case 1: deriv_LeakyReLU<<<g, THREADSPERBLOCK>>>(x, gy, gx, n); break;
        case 2: deriv_SiLU<<<g, THREADSPERBLOCK>>>(x, gy, gx, n); break;
        case 3: deriv_TaNH<<<g, THREADSPERBLOCK>>>(x, gy, gx, n); break;
        case 4: deriv_GeLU<<<g, THREADSPERBLOCK>>>(x, gy, gx, n); break;
        default: deriv_Sigmoid<<<g, THREADSPERBLOCK>>>(x, gy, gx, n); break;
    }
    return (int)cudaGetLastError();
}

int ref_accumulate(const float* x, float* y, long long n, double scale) {
    Accumulate<<<blocks(n, THREADSPERBLOCK), THREADSPERBLOCK>>>(x, y, (unsigned long long)n, scale);
    return (int)cudaGetLastError();
}

/* Scale forward (Engine/engine.cu:2533-2538) */
int ref_scale_write(const float* x, float* y, long long n, float scale) {
    Scale_Write<<<blocks(n, THREADSPERBLOCK), THREADSPERBLOCK>>>(x, y, (unsigned long long)n, scale);
    return (int)cudaGetLastError();
}

int ref_bcompress(const float* g, float* db, int batch, int channels, int rows, int cols) {
    BCompress<<<cols, THREADSPERBLOCK>>>(g, db, batch, channels, rows, cols);
    return (int)cudaGetLastError();
}

int ref_headify(const float* in, float* out, int b, int heads, int seq, int head_dim, int flag) {
    const long long total = (long long)b * heads * seq * head_dim;
    HeadifyColChannel<<<blocks(total, THREADSPERBLOCK), THREADSPERBLOCK>>>(in, out, b, heads, seq, head_dim, flag);
    return (int)cudaGetLastError();
}

int ref_matpe(const float* x, float* y, int batch, int rows, int cols, int start_idx) {
    const int total = batch * rows * cols;
    MatPEncoding<<<blocks(total, THREADSPERBLOCK), THREADSPERBLOCK>>>(x, y, batch, rows, cols, total, start_idx);
    return (int)cudaGetLastError();
}

/* LayerNorm forward lambda (Engine/engine.cu:3099-3113) */
int ref_layernorm_fwd(const float* x, float* y, float* mean, float* stdv, int a, int b, int c, int d) {
    const long long total = (long long)a * b * c * d;
    const int bpg = blocks(total, THREADSPERBLOCK);
    Write<<<bpg, THREADSPERBLOCK>>>(x, y, total);
    LayerMean<<<a, THREADSPERBLOCK>>>(x, mean, a, b, c, d);
    LayerStd<<<a, THREADSPERBLOCK>>>(x, mean, stdv, a, b, c, d);
    LNorm<<<bpg, THREADSPERBLOCK>>>(y, mean, stdv, a, b, c, d, 1.0f, 0.0f, 1e-5f);
    return (int)cudaGetLastError();
}

/* LayerNorm backward lambda (Engine/engine.cu:3116-3130); ggamma and
 * ggammanode hold a*b*c*d floats, the two means a floats each. */
int ref_layernorm_bwd(float* xgrad, const float* y, const float* gy, const float* stdv, float* ggamma,
                      float* ggammanode, float* ggamma_mean, float* ggammanode_mean, int a, int b, int c, int d) {
    const long long total = (long long)a * b * c * d;
    const int bpg = blocks(total, THREADSPERBLOCK);
    Scale_Write<<<bpg, THREADSPERBLOCK>>>(gy, ggamma, total, 1.0f);
    mulKernel<<<bpg, THREADSPERBLOCK>>>(ggamma, y, ggammanode, total);
    LayerMean<<<a, THREADSPERBLOCK>>>(ggamma, ggamma_mean, a, b, c, d, false);
    LayerMean<<<a, THREADSPERBLOCK>>>(ggammanode, ggammanode_mean, a, b, c, d, false);
    LayerBackward<<<bpg, THREADSPERBLOCK>>>(xgrad, y, gy, ggamma_mean, ggammanode_mean, stdv, 1.0f, 1e-5f, a, b, c, d);
    return (int)cudaGetLastError();
}

/* GroupNorm forward/backward lambdas (Engine/engine.cu:3232-3270) */
int ref_groupnorm_fwd(const float* x, float* y, float* mean, float* stdv, int a, int b, int c, int d, int group) {
    const long long total = (long long)a * b * c * d;
    const int bpg = blocks(total, THREADSPERBLOCK);
    Write<<<bpg, THREADSPERBLOCK>>>(x, y, total);
    GroupMean<<<a * group, THREADSPERBLOCK>>>(x, mean, a, b, group, c, d);
    GroupStd<<<a * group, THREADSPERBLOCK>>>(x, mean, stdv, a, b, group, c, d);
    GNorm<<<bpg, THREADSPERBLOCK>>>(y, mean, stdv, a, b, group, c, d, 1.0f, 0.0f, 1e-5f);
    return (int)cudaGetLastError();
}

int ref_groupnorm_bwd(float* xgrad, const float* y, const float* gy, const float* stdv, float* ggamma,
                      float* ggammanode, float* ggamma_mean, float* ggammanode_mean, int a, int b, int c, int d,
                      int group) {
    const long long total = (long long)a * b * c * d;
    const int bpg = blocks(total, THREADSPERBLOCK);
    Scale_Write<<<bpg, THREADSPERBLOCK>>>(gy, ggamma, total, 1.0f);
    mulKernel<<<bpg, THREADSPERBLOCK>>>(ggamma, y, ggammanode, total);
    GroupMean<<<a * group, THREADSPERBLOCK>>>(ggamma, ggamma_mean, a, b, group, c, d, false);
    GroupMean<<<a * group, THREADSPERBLOCK>>>(ggammanode, ggammanode_mean, a, b, group, c, d, false);
    GroupBackward<<<bpg, THREADSPERBLOCK>>>(xgrad, y, gy, ggamma_mean, ggammanode_mean, stdv, 1.0f, 1e-5f, a, b, group,
                                            c, d);
    return (int)cudaGetLastError();
}

/* SOFTMAX / SOFTMASK forward and backward lambdas (Engine/engine.cu:2430-2493);
 * arr and maxArr hold a*b*c (type 0) or a*b*d (type 1) floats. */
int ref_softmax_fwd(const float* x, float* arr, float* y, float* maxArr, int a, int b, int c, int d, int type,
                    int mask) {
    if (mask) SoftMask(x, arr, y, maxArr, a, b, c, d, type);
    else SoftMax(x, arr, y, maxArr, a, b, c, d, type);
    return (int)cudaGetLastError();
}

int ref_softmax_bwd(const float* y, const float* gy, float* gx, int a, int b, int c, int d, int type) {
    deriv_SoftMax(y, gy, gx, a, b, c, d, type);
    return (int)cudaGetLastError();
}

/* SoftMaxCrossEntropy forward/backward (Engine/engine.cu:2090-2111) with a
 * softmax buffer of the prediction's size. */
int ref_smce_fwd(const float* pred, const float* target, float* softmax, float* arr, float* maxArr, float* loss,
                 int batch, int channels, int c, int d) {
    const long long total = (long long)batch * channels * c * d;
    SoftMax(pred, arr, softmax, maxArr, batch, channels, c, d, 0);
    cudaMemset(loss, 0, sizeof(float));
    scalar_ce_kernel<<<blocks(total, THREADSPERBLOCK), THREADSPERBLOCK>>>(softmax, target, loss, total);
    return (int)cudaGetLastError();
}

int ref_smce_bwd(const float* softmax, const float* target, float* pred_grad, long long total, int batch) {
    ScaleAdd<<<blocks(total, THREADSPERBLOCK), THREADSPERBLOCK>>>(softmax, target, pred_grad, -1.0f, total);
    ScaleValue(pred_grad, (float)batch, total, 1);
    return (int)cudaGetLastError();
}

/* MeanSquaredError (Engine/engine.cu:1927-1944) with last = true */
int ref_mse_fwd(const float* pred, const float* target, float* loss, long long total) {
    cudaMemset(loss, 0, sizeof(float));
    scalar_mse_kernel<<<blocks(total, THREADSPERBLOCK), THREADSPERBLOCK>>>(pred, target, loss, total);
    return (int)cudaGetLastError();
}

int ref_mse_bwd(const float* pred, const float* target, const float* node_grad, float* pred_grad, long long total) {
    deriv_mse_kernel<<<blocks(total, THREADSPERBLOCK), THREADSPERBLOCK>>>(pred, target, node_grad, pred_grad, total,
                                                                          true, false);
    return (int)cudaGetLastError();
}

int ref_channel_squeeze(const float* g, float* db, int batch, int depth, int a, int b) {
    Channel_Squeeze1D<<<depth, THREADSPERBLOCK>>>(g, db, batch, depth, a, b);
    return (int)cudaGetLastError();
}

/* clip: AdamParameter::accumulate_grad (Engine/engine.cu:294-300),
 * Sqrt_Scale<<<1,1>>> (:3367), AdamParameter::gradnorm (:302) */
int ref_sumsq(double* ws, const float* g, long long n) {
    SumSquared<<<blocks(n, THREADSPERBLOCK), THREADSPERBLOCK>>>(ws, g, (unsigned long long)n);
    return (int)cudaGetLastError();
}

int ref_clip_finalize(double* ws) {
    Sqrt_Scale<<<1, 1>>>(ws, 1.0f, 0);
    return (int)cudaGetLastError();
}

int ref_clip_apply(float* g, const double* ws, long long n) {
    ScalePtr(g, ws, (unsigned long long)n, 1);
    return (int)cudaGetLastError();
}

/* AdamParameter::update (Engine/engine.cu:283-292) for one tensor */
int ref_adam(float* w, const float* g, int n, int t, float* m, float* v, float b1, float b2, float eps, float wd,
             float lr, int adamw) {
    const int bpg = blocks(n, THREADSPERBLOCK);
    if (adamw) AdamWUpdate<<<bpg, THREADSPERBLOCK>>>(w, g, n, t, m, v, b1, b2, eps, wd, lr);
    else AdamUpdate<<<bpg, THREADSPERBLOCK>>>(w, g, n, t, m, v, b1, b2, eps, lr);
    return (int)cudaGetLastError();
}

/* TextualEmbedding::EmbeddingUpdate (Engine/transformer.cu:233-245) on a
 * [batch, 1, clen, dim] embedding node's gradient. */
int ref_key_update(float* table, const float* grad, const int* keys, int clen, int max_clen, int dim, float lr,
                   long long total) {
    KeyUpdate<<<blocks(total, THREADSPERBLOCK), THREADSPERBLOCK>>>(table, grad, keys, clen, max_clen, dim, lr,
                                                                   (unsigned long long)total);
    return (int)cudaGetLastError();
}

int ref_sync(void) { return (int)cudaDeviceSynchronize(); }


/* Convolute2D / Convolute2DT kernels with the launch shapes of their
 * lambdas (Engine/engine.cu:3751-3773, 3850-3874). */
int ref_conv2d_fwd(const float* x, const float* k, const float* bias, float* y, int n, int cout, int cin, int h, int w,
                   int kh, int kw, int pad, int stride) {
    const int oh = (2 * pad + h - kh) / stride + 1, ow = (2 * pad + w - kw) / stride + 1;
    dim3 block(8, 8, 16);
    dim3 grid((ow + block.x - 1) / block.x, (oh + block.y - 1) / block.y, (n * cout + block.z - 1) / block.z);
    CV2D<<<grid, block>>>(x, k, bias, y, n, cout, cin, h, w, kh, kw, pad, stride);
    return (int)cudaGetLastError();
}

int ref_conv2d_bwd_k(const float* x, const float* dz, float* dk, int n, int cout, int cin, int h, int w, int kh,
                     int kw, int pad, int stride) {
    dim3 block(16, 16, 4);
    dim3 grid((cout + block.x - 1) / block.x, (cin + block.y - 1) / block.y, (kh * kw + block.z - 1) / block.z);
    GV2D<<<grid, block>>>(x, dz, dk, n, cout, cin, h, w, kh, kw, pad, stride);
    return (int)cudaGetLastError();
}

int ref_conv2d_bwd_x(const float* dy, const float* k, float* dx, int n, int cout, int cin, int h, int w, int kh,
                     int kw, int pad, int stride) {
    const int oh = (2 * pad + h - kh) / stride + 1, ow = (2 * pad + w - kw) / stride + 1;
    dim3 block(8, 8, 16);
    dim3 grid((w + block.x - 1) / block.x, (h + block.y - 1) / block.y, (n * cin + block.z - 1) / block.z);
    CV2D_GradInput<<<grid, block>>>(dy, k, dx, n, cout, cin, h, w, kh, kw, oh, ow, pad, stride);
    return (int)cudaGetLastError();
}

int ref_convT2d_fwd(const float* x, const float* wt, const float* bias, float* y, int n, int cout, int cin, int h,
                    int w, int kh, int kw, int pad, int stride) {
    const int oh = (h - 1) * stride - 2 * pad + kh, ow = (w - 1) * stride - 2 * pad + kw;
    dim3 block(8, 8, 16);
    dim3 grid((ow + block.x - 1) / block.x, (oh + block.y - 1) / block.y, (n * cout + block.z - 1) / block.z);
    CVT2D<<<grid, block>>>(x, wt, bias, y, n, cout, cin, h, w, kh, kw, pad, stride);
    return (int)cudaGetLastError();
}

int ref_convT2d_bwd_w(const float* x, const float* gout, float* gw, int n, int cout, int cin, int h, int w, int kh,
                      int kw, int pad, int stride) {
    GVT2D<<<cout, THREADSPERBLOCK>>>(x, gout, gw, n, cout, cin, h, w, kh, kw, pad, stride);
    return (int)cudaGetLastError();
}

int ref_convT2d_bwd_x(const float* gout, const float* wt, float* gx, int n, int cout, int cin, int h, int w, int kh,
                      int kw, int pad, int stride) {
    dim3 block(8, 8, 16);
    dim3 grid((w + block.x - 1) / block.x, (h + block.y - 1) / block.y, (n * cin + block.z - 1) / block.z);
    CVT2D_GradInput<<<grid, block>>>(gout, wt, gx, n, cout, cin, h, w, kh, kw, pad, stride);
    return (int)cudaGetLastError();
}

}  // extern "C"
