/*
 * CPU oracle for the ML_Engine training hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's CUDA kernels on the path
 * (Engine/kernels.cu, Engine/engine.cu of VicVibin/ML_Engine), one function
 * per kernel family, each citing the lines it restates.  It is the checker
 * for the sm_100a kernels (tests/, __graft_entry__.smoke) and the timed CPU
 * baseline of bench.py; no product code path may call it.
 *
 * Parity pin: the reference ships no tests or golden vectors.  This file is
 * pinned against the reference's own kernels, compiled from source into
 * oracle/_ref and run on a B200 by tests/test_oracle_pin.py, and against the
 * fixtures those runs produced (tests/golden/).
 *
 * Arithmetic: elementwise formulas keep the reference's float expressions;
 * matrix products and reductions accumulate in double (more accurate than
 * the reference's float sums, never less).  OpenMP parallelises the outer
 * loops.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* Threads of the parallel loops below: n > 0 sets it for the calling
 * thread's later regions (a launcher may have pinned OMP_NUM_THREADS to 1);
 * returns the count in force. */
int oracle_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}

#define ORACLE_PI 3.14159265359f

/* ------------------------------------------------------------------------ */
/* activations: Engine/kernels.cu:1214-1328                                  */
/* ------------------------------------------------------------------------ */
static float act_f(int kind, float x) {
    switch (kind) {
        case 0: return x < 0.f ? 0.0f : x;                               /* ReLU   :1214 */
        case 1: return x < 0.f ? 0.01f * x : x;                          /* Leaky  :1231 */
        case 2: return x * (1.0f / (1.0f + expf(-x)));                   /* SiLU   :1248 */
        case 3: return tanhf(x);                                         /* TaNH   :1268 */
        case 4: {                                                        /* GeLU   :1286 */
            const float v = sqrtf(2.0f / ORACLE_PI) * (x + 0.044715f * x * x * x);
            return 0.5f * x * (1.0f + tanhf(v));
        }
        default: return 1.0f / (1.0f + expf(-1.0f * x));                /* Sigmoid:1309 */
    }
}

static float act_d(int kind, float x) {
    switch (kind) {
        case 0: return x > 0.0f ? 1.0f : 0.0f;                           /* deriv_ReLU  :1223 */
        case 1: return x < 0.0f ? 0.01f : 1.0f;                          /* deriv_Leaky :1240 */
        case 2: {                                                        /* deriv_SiLU  :1257 */
            const float e = expf(x), ne = 1.0f / e;
            return 1.0f / (1.0f + ne) + x / (e + ne + 2.0f);
        }
        case 3: {                                                        /* deriv_TaNH  :1277 */
            const float e2 = expf(2.0f * x), ne2 = 1.0f / e2;
            return 4.0f / (e2 + ne2 + 2.0f);
        }
        case 4: {                                                        /* deriv_GeLU  :1296 */
            const float root = sqrtf(2.0f / ORACLE_PI);
            const float u = root * (x + 0.044715f * x * x * x);
            const float du = root * (1.0f + 0.134145f * x * x);
            const float t = tanhf(u);
            return 0.5f + 0.5f * t + 0.5f * x * (1.0f - t * t) * du;
        }
        default: {                                                       /* deriv_Sigmoid:1318 */
            const float e = expf(x), ne = 1.0f / e;
            return 1.0f / (e + ne + 2.0f);
        }
    }
}

void oracle_act_fwd(int kind, const float* x, float* y, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) y[i] = act_f(kind, x[i]);
}

/* gx += gy * f'(x)  (lambdas Engine/engine.cu:2666-2842) */
void oracle_act_bwd(int kind, const float* x, const float* gy, float* gx, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) gx[i] += gy[i] * act_d(kind, x[i]);
}

/* ------------------------------------------------------------------------ */
/* elementwise glue                                                          */
/* ------------------------------------------------------------------------ */
/* Accumulate (Engine/kernels.cu:1702): Y += scale*X in double */
void oracle_accumulate(const float* x, float* y, int64_t n, double scale) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) y[i] = (float)((double)y[i] + scale * (double)x[i]);
}

/* ScaleAdd (Engine/kernels.cu:1718): Z = X + scale*Y */
void oracle_scale_add(const float* x, const float* y, float* z, float scale, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) z[i] = x[i] + scale * y[i];
}

/* Scale_Write (Engine/kernels.cu:1677) */
void oracle_scale_write(const float* x, float* y, int64_t n, float scale) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) y[i] = scale * x[i];
}

/* BCumAdd (Engine/kernels.cu:1586): X[r, c] += Y[c] */
void oracle_bias_add(float* x, const float* b, int64_t rows, int64_t cols) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < cols; ++c) x[r * cols + c] += b[c];
}

/* BCompress (Engine/kernels.cu:1562): Y[c] += scale * sum_r X[r, c] */
void oracle_bias_grad(const float* g, float* db, int64_t rows, int64_t cols, float scale) {
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < cols; ++c) {
        double s = 0.0;
        for (int64_t r = 0; r < rows; ++r) s += g[r * cols + c];
        db[c] += (float)s * scale;
    }
}

/* broadcast_add (Engine/kernels.cu:1661) */
void oracle_channel_bias_fwd(const float* x, const float* b, float* y, int batch, int channels, int64_t spatial) {
    const int64_t total = (int64_t)batch * channels * spatial;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < total; ++i) y[i] = x[i] + b[(i / spatial) % channels];
}

/* Channel_Squeeze1D (Engine/kernels.cu:1734) and, if gx, Accumulate */
void oracle_channel_bias_bwd(const float* g, float* gx, float* gb, int batch, int channels, int64_t spatial) {
#pragma omp parallel for schedule(static)
    for (int c = 0; c < channels; ++c) {
        double s = 0.0;
        for (int n = 0; n < batch; ++n) {
            const int64_t base = ((int64_t)n * channels + c) * spatial;
            for (int64_t k = 0; k < spatial; ++k) {
                s += g[base + k];
                if (gx) gx[base + k] += g[base + k];
            }
        }
        gb[c] += (float)s;
    }
}

/* MatPEncoding (Engine/kernels.cu:166-185) */
void oracle_matpe(const float* x, float* y, int batch, int rows, int cols, int start_idx) {
    const int64_t total = (int64_t)batch * rows * cols;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < total; ++i) {
        const int pos = (int)((i % ((int64_t)rows * cols)) / cols) + start_idx;
        const int d = (int)(i % cols);
        const double freq = 1.0 / pow(10000.0, (2.0 * (d / 2)) / cols);
        const double angle = (double)pos * freq;
        y[i] = (d % 2 == 0) ? x[i] + (float)sin(angle) : x[i] + (float)cos(angle);
    }
}

/* PEncoding (Engine/kernels.cu:147-164) */
void oracle_timestep_pe(float* y, int t, int dim) {
    const int half = dim / 2;
    for (int i = 0; i < dim; ++i) {
        const int f = i < half ? i : i - half;
        const double freq = exp(-(double)f * log(10000.0) / (half - 1));
        const double angle = (double)t * freq;
        y[i] = i < half ? (float)cos(angle) : (float)sin(angle);
    }
}

/* HeadifyColChannel (Engine/kernels.cu:1371-1406) */
void oracle_headify(const float* in, float* out, int batch, int heads, int seq, int head_dim, int flag) {
    const int64_t total = (int64_t)batch * heads * seq * head_dim;
    const int embed = heads * head_dim;
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < total; ++idx) {
        const int d = (int)(idx % head_dim);
        const int s = (int)((idx / head_dim) % seq);
        const int h = (int)((idx / ((int64_t)head_dim * seq)) % heads);
        const int64_t b = idx / ((int64_t)head_dim * seq * heads);
        const int64_t f = b * ((int64_t)seq * embed) + (int64_t)s * embed + (int64_t)h * head_dim + d;
        if (flag == 0) out[idx] = in[f];
        else if (flag == 1) out[f] += in[idx];
        else if (flag == 2) out[f] = in[idx];
        else out[idx] += in[f];
    }
}

/* Channel_Concat / Channel_Split (Engine/kernels.cu:1408-1432) */
void oracle_channel_concat(const float* a, const float* b, float* c, int batch, int c1, int c2, int64_t spatial) {
    const int cc = c1 + c2;
    for (int n = 0; n < batch; ++n)
        for (int ch = 0; ch < cc; ++ch)
            for (int64_t s = 0; s < spatial; ++s)
                c[((int64_t)n * cc + ch) * spatial + s] =
                    ch < c1 ? a[((int64_t)n * c1 + ch) * spatial + s] : b[((int64_t)n * c2 + ch - c1) * spatial + s];
}

void oracle_channel_split(float* ga, float* gb, const float* gc, int batch, int c1, int c2, int64_t spatial) {
    const int cc = c1 + c2;
    for (int n = 0; n < batch; ++n)
        for (int ch = 0; ch < cc; ++ch)
            for (int64_t s = 0; s < spatial; ++s) {
                const float v = gc[((int64_t)n * cc + ch) * spatial + s];
                if (ch < c1) ga[((int64_t)n * c1 + ch) * spatial + s] += v;
                else gb[((int64_t)n * c2 + ch - c1) * spatial + s] += v;
            }
}

/* GatherEmbeddings (Engine/kernels.cu:2279) / OneHotEmbeddings (:1551) */
void oracle_embedding_gather(const int32_t* keys, const float* table, float* out, int64_t n_keys, int dim) {
    for (int64_t i = 0; i < n_keys; ++i)
        for (int d = 0; d < dim; ++d) out[i * dim + d] = keys[i] < 0 ? 0.0f : table[(int64_t)keys[i] * dim + d];
}

/* KeyUpdate (Engine/kernels.cu:1536-1549): EmbedSpace[key * D + d] +=
 * -lr * grad[i] for every gradient element whose token key is >= 0; token t
 * of batch b reads its key at keys[b * max_clen + t].  Sequential, so rows
 * sharing a key all contribute (in row order), which is what the kernel
 * computes when its threads do not race. */
void oracle_key_update(float* table, const float* grad, const int32_t* keys, int clen, int max_clen, int dim,
                       float lr, int64_t total) {
    for (int64_t i = 0; i < total; ++i) {
        const int64_t b = i / ((int64_t)clen * dim);
        const int64_t kr = i % ((int64_t)clen * dim);
        const int64_t t = kr / dim, d = kr % dim;
        const int key = keys[b * max_clen + t];
        if (key < 0) continue;
        /* the kernel's `+= -lr * grad` compiles to one fused multiply-add */
        table[(int64_t)key * dim + d] = fmaf(-lr, grad[i], table[(int64_t)key * dim + d]);
    }
}

void oracle_one_hot(const int32_t* keys, float* out, int64_t n_keys, int vocab) {
    for (int64_t i = 0; i < n_keys; ++i)
        if (keys[i] >= 0 && keys[i] < vocab) out[i * vocab + keys[i]] = 1.0f;
}

/* ------------------------------------------------------------------------ */
/* batched GEMM with broadcast flags: bcmm/bcmmABT/bcmmATB/bcmmT             */
/* (Engine/kernels.cu:371-539)                                               */
/* ------------------------------------------------------------------------ */
static int64_t bc_off(int flag, int b, int c, int channels, int64_t inner) {
    const int hb = flag & 1, hc = (flag >> 1) & 1;
    const int64_t cs = hc ? channels : 1;
    return (hb ? (int64_t)b * cs : 0) * inner + (hc ? (int64_t)c : 0) * inner;
}

/* variant 0 AB, 1 ABT, 2 ATB, 3 ATBT.  C[m,p] (=|+=) scale * sum_k a(r,k) b(k,col) */
void oracle_bcmm(int variant, const float* A, const float* B, float* C, int batch, int channels, int m, int n, int p,
                 int backward, int A_case, int B_case, int C_case, float scale) {
    const int at = (variant == 2 || variant == 3), bt = (variant == 1 || variant == 3);
    for (int z = 0; z < batch * channels; ++z) {
        const int b = z / channels, c = z % channels;
        const float* a = A + bc_off(A_case, b, c, channels, (int64_t)m * n);
        const float* bb = B + bc_off(B_case, b, c, channels, (int64_t)n * p);
        float* cc = C + bc_off(C_case, b, c, channels, (int64_t)m * p);
#pragma omp parallel for schedule(static)
        for (int r = 0; r < m; ++r) {
            for (int col = 0; col < p; ++col) {
                double s = 0.0;
                for (int k = 0; k < n; ++k) {
                    const float av = at ? a[(int64_t)k * m + r] : a[(int64_t)r * n + k];
                    const float bv = bt ? bb[(int64_t)col * n + k] : bb[(int64_t)k * p + col];
                    s += (double)av * (double)bv;
                }
                const float v = scale * (float)s;
                if (backward) cc[(int64_t)r * p + col] += v;
                else cc[(int64_t)r * p + col] = v;
            }
        }
    }
}

/* Plain row-major GEMM used by the Linear layer oracles: C (=|+=) op(A) op(B) */
void oracle_gemm(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K, int trans_a, int trans_b,
                 int accumulate) {
#pragma omp parallel
    {
    /* one row of double accumulators per thread, on the heap: a row of a
     * wide product does not fit a thread's stack */
    double* acc = (double*)malloc(sizeof(double) * (size_t)(N > 0 ? N : 1));
#pragma omp for schedule(static)
    for (int64_t r = 0; r < M; ++r) {
        for (int64_t col = 0; col < N; ++col) acc[col] = 0.0;
        for (int64_t k = 0; k < K; ++k) {
            const double av = trans_a ? A[k * M + r] : A[r * K + k];
            if (av == 0.0) continue;
            if (!trans_b) {
                const float* brow = B + k * N;
                for (int64_t col = 0; col < N; ++col) acc[col] += av * brow[col];
            } else {
                for (int64_t col = 0; col < N; ++col) acc[col] += av * B[col * K + k];
            }
        }
        for (int64_t col = 0; col < N; ++col) {
            if (accumulate) C[r * N + col] += (float)acc[col];
            else C[r * N + col] = (float)acc[col];
        }
    }
    free(acc);
    }
}

/* ------------------------------------------------------------------------ */
/* normalisation                                                             */
/* ------------------------------------------------------------------------ */
/* segment normalisation shared by LayerNorm (segment = dim0 index,
 * Engine/kernels.cu:541-572,670-699,794-804) and GroupNorm (segment =
 * (sample, group), :607-639,732-763,818-834). */
static void seg_norm_fwd(const float* x, float* y, float* mean, float* sqdev, int64_t segs, int64_t N, float eps) {
#pragma omp parallel for schedule(static)
    for (int64_t s = 0; s < segs; ++s) {
        const float* xs = x + s * N;
        double sum = 0.0;
        for (int64_t i = 0; i < N; ++i) sum += xs[i];
        const float mu = (float)sum / (float)N;
        double q = 0.0;
        for (int64_t i = 0; i < N; ++i) {
            const float d = xs[i] - mu;
            q += (double)d * d;
        }
        const float qf = (float)q;
        const float scale = 1.0f / sqrtf((1.0f / (float)N) * qf + eps);
        for (int64_t i = 0; i < N; ++i) y[s * N + i] = (xs[i] - mu) * scale;
        if (mean) mean[s] = mu;
        sqdev[s] = qf;
    }
}

void oracle_layernorm_fwd(const float* x, float* y, float* mean, float* sqdev, int batch, int channels, int row,
                          int col, float eps) {
    seg_norm_fwd(x, y, mean, sqdev, batch, (int64_t)channels * row * col, eps);
}

void oracle_groupnorm_fwd(const float* x, float* y, float* mean, float* sqdev, int batch, int channels, int groups,
                          int row, int col, float eps) {
    seg_norm_fwd(x, y, mean, sqdev, (int64_t)batch * groups, (int64_t)(channels / groups) * row * col, eps);
}

/* LayerNorm backward lambda (Engine/engine.cu:3116-3130) with LayerBackward's
 * index map (Engine/kernels.cu:849-862): elements idx < batch*row*col, sample
 * idx/(row*col), sums over the whole sample. */
void oracle_layernorm_bwd(const float* y, const float* gy, const float* sqdev, float* gx, int batch, int channels,
                          int row, int col, float eps) {
    const int64_t N = (int64_t)channels * row * col, rc = (int64_t)row * col;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < batch; ++b) {
        double sg = 0.0, sgy = 0.0;
        for (int64_t i = 0; i < N; ++i) {
            sg += gy[b * N + i];
            sgy += (double)gy[b * N + i] * y[b * N + i];
        }
        const float Nf = (float)N;
        const float rstd = 1.0f / sqrtf(sqdev[b] / Nf + eps);
        const float mg = (float)sg / Nf, mgy = (float)sgy / Nf;
        for (int64_t i = b * rc; i < (b + 1) * rc; ++i) gx[i] += rstd * (gy[i] - mg - y[i] * mgy);
    }
}

/* GroupNorm backward lambda (Engine/engine.cu:3255-3270), GroupBackward
 * (Engine/kernels.cu:877-896) */
void oracle_groupnorm_bwd(const float* y, const float* gy, const float* sqdev, float* gx, int batch, int channels,
                          int groups, int row, int col, float eps) {
    const int64_t N = (int64_t)(channels / groups) * row * col, segs = (int64_t)batch * groups;
#pragma omp parallel for schedule(static)
    for (int64_t s = 0; s < segs; ++s) {
        double sg = 0.0, sgy = 0.0;
        for (int64_t i = 0; i < N; ++i) {
            sg += gy[s * N + i];
            sgy += (double)gy[s * N + i] * y[s * N + i];
        }
        const float Nf = (float)N;
        const float rstd = 1.0f / sqrtf(sqdev[s] / Nf + eps);
        const float mg = (float)sg / Nf, mgy = (float)sgy / Nf;
        for (int64_t i = s * N; i < (s + 1) * N; ++i) gx[i] += rstd * (gy[i] - mg - y[i] * mgy);
    }
}

/* ------------------------------------------------------------------------ */
/* softmax: SoftMax/SoftMask (Engine/kernels.cu:2183-2235), deriv (:2149)    */
/* ------------------------------------------------------------------------ */
void oracle_softmax_fwd(const float* x, float* y, int64_t bc, int rows, int cols, int axis, int causal) {
#pragma omp parallel for schedule(static)
    for (int64_t mtx = 0; mtx < bc; ++mtx) {
        const float* xm = x + mtx * (int64_t)rows * cols;
        float* ym = y + mtx * (int64_t)rows * cols;
        const int lines = axis == 0 ? rows : cols, len = axis == 0 ? cols : rows;
        for (int l = 0; l < lines; ++l) {
            float mx = -3.402823466e+38f;
            for (int k = 0; k < len; ++k) {
                const int r = axis == 0 ? l : k, c = axis == 0 ? k : l;
                if (xm[(int64_t)r * cols + c] > mx) mx = xm[(int64_t)r * cols + c];
            }
            float s = 0.f;
            for (int k = 0; k < len; ++k) {
                const int r = axis == 0 ? l : k, c = axis == 0 ? k : l;
                const float e = (causal && c > r) ? 0.0f : expf(xm[(int64_t)r * cols + c] - mx);
                ym[(int64_t)r * cols + c] = e;
                s += e;
            }
            if (s < 1e-45f) s = 1.0f;
            for (int k = 0; k < len; ++k) {
                const int r = axis == 0 ? l : k, c = axis == 0 ? k : l;
                ym[(int64_t)r * cols + c] /= s;
            }
        }
    }
}

void oracle_softmax_bwd(const float* y, const float* gy, float* gx, int64_t bc, int rows, int cols, int axis) {
#pragma omp parallel for schedule(static)
    for (int64_t mtx = 0; mtx < bc; ++mtx) {
        const int64_t base = mtx * (int64_t)rows * cols;
        const int lines = axis == 0 ? rows : cols, len = axis == 0 ? cols : rows;
        for (int l = 0; l < lines; ++l) {
            double dot = 0.0;
            for (int k = 0; k < len; ++k) {
                const int64_t i = base + (axis == 0 ? (int64_t)l * cols + k : (int64_t)k * cols + l);
                dot += (double)gy[i] * y[i];
            }
            const float d = (float)dot;
            for (int k = 0; k < len; ++k) {
                const int64_t i = base + (axis == 0 ? (int64_t)l * cols + k : (int64_t)k * cols + l);
                gx[i] += y[i] * (gy[i] - d);
            }
        }
    }
}

/* SoftMaxCrossEntropy forward (Engine/engine.cu:2090-2102): row softmax then
 * scalar_ce_kernel (Engine/kernels.cu:1818-1826). */
float oracle_smce_fwd(const float* logits, const float* target, float* probs, int64_t rows, int cols) {
    oracle_softmax_fwd(logits, probs, 1, (int)rows, cols, 0, 0);
    double s = 0.0;
#pragma omp parallel for reduction(+ : s) schedule(static)
    for (int64_t i = 0; i < rows * cols; ++i)
        if (target[i] != 0.0f) s += -(double)target[i] * log((double)probs[i] + 1e-27);
    return (float)(s / ((double)rows * cols));
}

/* SoftMaxCrossEntropy backward (Engine/engine.cu:2104-2111): grad = (p - t)
 * [* upstream] / batch (assign). */
void oracle_smce_bwd(const float* probs, const float* target, const float* upstream, float* grad, float batch_div,
                     int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        float g = probs[i] + (-1.0f) * target[i];
        if (upstream) g *= upstream[0];
        grad[i] = g / batch_div;
    }
}

/* scalar_mse_kernel / deriv_mse_kernel (Engine/kernels.cu:1808-1848) */
float oracle_mse_fwd(const float* x, const float* t, int64_t n) {
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        const double d = (double)t[i] - (double)x[i];
        s += d * d;
    }
    return (float)(s / (double)n);
}

void oracle_mse_bwd(const float* x, const float* t, const float* upstream, float* gx, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        if (!upstream) gx[i] += 2.0f * (x[i] - t[i]) / (float)n;
        else gx[i] += (2.0f * (x[i] - t[i]) * upstream[0]) / (float)n;
    }
}

/* ------------------------------------------------------------------------ */
/* grad-norm clip and Adam/AdamW                                             */
/* ------------------------------------------------------------------------ */
/* SumSquared (Engine/kernels.cu:1486-1506): *acc += sum g^2 in double */
void oracle_sumsq(double* acc, const float* g, int64_t n) {
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i) s += (double)g[i] * (double)g[i];
    *acc += s;
}

/* Sqrt_Scale(X, 1.0, 0) (Engine/kernels.cu:1763-1773) */
void oracle_clip_finalize(double* acc) {
    const double x = acc[0];
    if (x != x) return;
    const double curr = sqrt(x);
    acc[0] = curr > 1.0 ? curr * 1.0 : 1.0;
}

/* SP via ScalePtr(grad, g, n, 1) (Includes/kernels.h:293-300) */
void oracle_clip_apply(float* g, int64_t n, const double* acc) {
    const float f = (float)acc[0];
    for (int64_t i = 0; i < n; ++i) g[i] /= f;
}

/* AdamWUpdate / AdamUpdate (Engine/kernels.cu:1508-1534) */
void oracle_adam(float* w, const float* g, float* m, float* v, int64_t n, int t, float b1, float b2, float eps,
                 float wd, float lr, int adamw) {
    const double bc1 = adamw ? 1.0 - (double)(float)pow((double)b1, t) : 1.0 - (double)powf(b1, (float)t);
    const double bc2 = adamw ? 1.0 - (double)(float)pow((double)b2, t) : 1.0 - (double)powf(b2, (float)t);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        const float gi = g[i];
        m[i] = (float)((double)(b1 * m[i]) + (1.0 - b1) * gi);
        v[i] = (float)((double)(b2 * v[i]) + (1.0 - b2) * gi * gi);
        const float m_hat = (float)(m[i] / bc1);
        const float v_hat = (float)(v[i] / bc2);
        const float vs = sqrtf(v_hat);
        if (adamw) w[i] -= lr * ((m_hat / (vs + eps)) + wd * w[i]);
        else w[i] -= lr * m_hat / (vs + eps);
    }
}

/* ------------------------------------------------------------------------ */
/* 2-D convolution and transposed convolution (NCHW); weights [O][I][KH][KW] */
/* ------------------------------------------------------------------------ */
/* CV2D (Engine/kernels.cu:985-1019): y = sum_{ci,kh,kw} x*k (+ bias), assigned */
void oracle_conv2d_fwd(const float* x, const float* k, const float* bias, float* y, int N, int Cout, int Cin, int H,
                       int W, int KH, int KW, int pad, int stride) {
    const int OH = (2 * pad + H - KH) / stride + 1, OW = (2 * pad + W - KW) / stride + 1;
#pragma omp parallel for collapse(2) schedule(static)
    for (int n = 0; n < N; ++n)
        for (int co = 0; co < Cout; ++co)
            for (int oy = 0; oy < OH; ++oy)
                for (int ox = 0; ox < OW; ++ox) {
                    double s = 0.0;
                    for (int ci = 0; ci < Cin; ++ci)
                        for (int kh = 0; kh < KH; ++kh)
                            for (int kw = 0; kw < KW; ++kw) {
                                const int iy = oy * stride - pad + kh, ix = ox * stride - pad + kw;
                                if (iy < 0 || iy >= H || ix < 0 || ix >= W) continue;
                                s += (double)x[(((int64_t)n * Cin + ci) * H + iy) * W + ix] *
                                     (double)k[(((int64_t)co * Cin + ci) * KH + kh) * KW + kw];
                            }
                    const float v = (float)s;
                    y[(((int64_t)n * Cout + co) * OH + oy) * OW + ox] = bias ? v + bias[co] : v;
                }
}

/* GV2D (Engine/kernels.cu:1021-1051): dK = sum_{n,oy,ox} x*dZ, assigned */
void oracle_conv2d_bwd_k(const float* x, const float* dz, float* dk, int N, int Cout, int Cin, int H, int W, int KH,
                         int KW, int pad, int stride) {
    const int OH = (2 * pad + H - KH) / stride + 1, OW = (2 * pad + W - KW) / stride + 1;
#pragma omp parallel for collapse(2) schedule(static)
    for (int co = 0; co < Cout; ++co)
        for (int ci = 0; ci < Cin; ++ci)
            for (int kh = 0; kh < KH; ++kh)
                for (int kw = 0; kw < KW; ++kw) {
                    double s = 0.0;
                    for (int n = 0; n < N; ++n)
                        for (int oy = 0; oy < OH; ++oy)
                            for (int ox = 0; ox < OW; ++ox) {
                                const int iy = oy * stride - pad + kh, ix = ox * stride - pad + kw;
                                if (iy < 0 || iy >= H || ix < 0 || ix >= W) continue;
                                s += (double)x[(((int64_t)n * Cin + ci) * H + iy) * W + ix] *
                                     (double)dz[(((int64_t)n * Cout + co) * OH + oy) * OW + ox];
                            }
                    dk[(((int64_t)co * Cin + ci) * KH + kh) * KW + kw] = (float)s;
                }
}

/* CV2D_GradInput (Engine/kernels.cu:1053-1089): dX += sum_{oc,kh,kw} dY*K */
void oracle_conv2d_bwd_x(const float* dy, const float* k, float* dx, int N, int Cout, int Cin, int H, int W, int KH,
                         int KW, int pad, int stride) {
    const int OH = (2 * pad + H - KH) / stride + 1, OW = (2 * pad + W - KW) / stride + 1;
#pragma omp parallel for collapse(2) schedule(static)
    for (int n = 0; n < N; ++n)
        for (int ci = 0; ci < Cin; ++ci)
            for (int ih = 0; ih < H; ++ih)
                for (int iw = 0; iw < W; ++iw) {
                    double s = 0.0;
                    for (int oc = 0; oc < Cout; ++oc)
                        for (int kh = 0; kh < KH; ++kh) {
                            const int ry = ih + pad - kh;
                            if (ry < 0 || ry % stride != 0 || ry / stride >= OH) continue;
                            for (int kw = 0; kw < KW; ++kw) {
                                const int rx = iw + pad - kw;
                                if (rx < 0 || rx % stride != 0 || rx / stride >= OW) continue;
                                s += (double)dy[(((int64_t)n * Cout + oc) * OH + ry / stride) * OW + rx / stride] *
                                     (double)k[(((int64_t)oc * Cin + ci) * KH + kh) * KW + kw];
                            }
                        }
                    float* o = &dx[(((int64_t)n * Cin + ci) * H + ih) * W + iw];
                    *o += (float)s;
                }
}

/* CVT2D (Engine/kernels.cu:1091-1135): transposed conv forward, assigned */
void oracle_convT2d_fwd(const float* x, const float* w, const float* bias, float* y, int N, int Cout, int Cin, int H,
                        int W, int KH, int KW, int pad, int stride) {
    const int OH = (H - 1) * stride - 2 * pad + KH, OW = (W - 1) * stride - 2 * pad + KW;
#pragma omp parallel for collapse(2) schedule(static)
    for (int n = 0; n < N; ++n)
        for (int oc = 0; oc < Cout; ++oc)
            for (int row = 0; row < OH; ++row)
                for (int col = 0; col < OW; ++col) {
                    double s = 0.0;
                    for (int ic = 0; ic < Cin; ++ic)
                        for (int kh = 0; kh < KH; ++kh)
                            for (int kw = 0; kw < KW; ++kw) {
                                int r = row + pad - kh, c = col + pad - kw;
                                if (r % stride != 0 || c % stride != 0) continue;
                                r /= stride;
                                c /= stride;
                                if (r < 0 || r >= H || c < 0 || c >= W) continue;
                                s += (double)x[(((int64_t)n * Cin + ic) * H + r) * W + c] *
                                     (double)w[(((int64_t)oc * Cin + ic) * KH + kh) * KW + kw];
                            }
                    const float v = (float)s;
                    y[(((int64_t)n * Cout + oc) * OH + row) * OW + col] = bias ? v + bias[oc] : v;
                }
}

/* GVT2D (Engine/kernels.cu:1137-1176): transposed conv weight grad, assigned */
void oracle_convT2d_bwd_w(const float* x, const float* gout, float* gw, int N, int Cout, int Cin, int H, int W, int KH,
                          int KW, int pad, int stride) {
    const int OH = (H - 1) * stride - 2 * pad + KH, OW = (W - 1) * stride - 2 * pad + KW;
#pragma omp parallel for collapse(2) schedule(static)
    for (int oc = 0; oc < Cout; ++oc)
        for (int ic = 0; ic < Cin; ++ic)
            for (int kh = 0; kh < KH; ++kh)
                for (int kw = 0; kw < KW; ++kw) {
                    double s = 0.0;
                    for (int n = 0; n < N; ++n)
                        for (int r = 0; r < H; ++r)
                            for (int c = 0; c < W; ++c) {
                                const int orow = r * stride - pad + kh, ocol = c * stride - pad + kw;
                                if (orow < 0 || orow >= OH || ocol < 0 || ocol >= OW) continue;
                                s += (double)x[(((int64_t)n * Cin + ic) * H + r) * W + c] *
                                     (double)gout[(((int64_t)n * Cout + oc) * OH + orow) * OW + ocol];
                            }
                    gw[(((int64_t)oc * Cin + ic) * KH + kh) * KW + kw] = (float)s;
                }
}

/* CVT2D_GradInput (Engine/kernels.cu:1178-1212): assigned */
void oracle_convT2d_bwd_x(const float* gout, const float* w, float* gx, int N, int Cout, int Cin, int H, int W,
                          int KH, int KW, int pad, int stride) {
    const int OH = (H - 1) * stride - 2 * pad + KH, OW = (W - 1) * stride - 2 * pad + KW;
#pragma omp parallel for collapse(2) schedule(static)
    for (int n = 0; n < N; ++n)
        for (int ic = 0; ic < Cin; ++ic)
            for (int r = 0; r < H; ++r)
                for (int c = 0; c < W; ++c) {
                    double s = 0.0;
                    for (int oc = 0; oc < Cout; ++oc)
                        for (int kh = 0; kh < KH; ++kh)
                            for (int kw = 0; kw < KW; ++kw) {
                                const int orow = r * stride - pad + kh, ocol = c * stride - pad + kw;
                                if (orow < 0 || orow >= OH || ocol < 0 || ocol >= OW) continue;
                                s += (double)gout[(((int64_t)n * Cout + oc) * OH + orow) * OW + ocol] *
                                     (double)w[(((int64_t)oc * Cin + ic) * KH + kh) * KW + kw];
                            }
                    gx[(((int64_t)n * Cin + ic) * H + r) * W + c] = (float)s;
                }
}
