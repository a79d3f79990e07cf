// Attention sub-graph of MultiHeadAttention (Engine/transformer.cu:647-675):
//   scores = Q K^T, scaled = scale*scores, P = softmax_axis(scaled), O = P V.
//
// Fused path (column-wise softmax, the reference's "type 1", head_dim 16/32/64,
// Sq, Sk <= 256).  A column of that softmax runs over every query row, a
// row of O, dQ or of the reference's key gradient over every key, so each
// direction is two kernels, one per axis:
//   forward : probs  — CTA per (batch*head, 32 keys): scaled scores of all
//                      query rows, the column softmax, P stored;
//             pv     — CTA per (batch*head, 32 queries): O = P V;
//   backward: cols   — CTA per (batch*head, 32 keys): dP = dO V^T, the column
//                      dot, dScores = scale * P (dP - dot) into a workspace,
//                      dV (and the true dK), complete for these keys;
//             rows   — CTA per (batch*head, 32 queries): dQ = dScores K and
//                      the reference's key gradient dScores Q.
// Every sum is one FMA chain in the order the reference kernels use (bcmm*:
// k ascending; SumRows / deriv_softmax: rows ascending), so P, O and the
// gradients are bitwise those of the reference's kernel chain.  Q, K, V, O
// and the gradients are read and written token-major ([B, S, H*hd], the
// Linear layout) or head-major through strides, so no head copies are made.
//
// Tensor-core path (TF32 GEMM mode; chosen for long sequences, where the
// CUDA-core kernels' serial sums dominate the step, or on request through
// mle_set_attention_path): the two forward and four backward products run
// on the tcgen05 GEMM, which reads Q, K, V, dO and writes O, dQ, dK, dV in
// either layout through strides, P and the score gradients [B,H,Sq,Sk] in
// between; the column softmax and its backward read each 32-column slab of
// a matrix once into registers (columns up to 512 rows; longer ones take
// multi-pass column-block kernels), 16-byte accesses.  The reference's key gradient (memory of
// dScores read as [Sk,Sq], result laid out [hd,Sk] in the head's block) is
// one GEMM whose output columns are split over rows of the head block.
//
// Other shapes run the composed path on the tensor-core GEMM (head-major).
#include <float.h>

#include <algorithm>
#include <initializer_list>
#include <type_traits>

#include "common.cuh"
#include "gemm.cuh"

namespace mle {
namespace {

constexpr int kNT = 256;     // threads per CTA
constexpr int kTC = 32;      // key columns per column-block CTA
constexpr int kTR = 64;      // query rows per row-block CTA
constexpr int kWarps = kNT / 32;
constexpr int kMaxSeq = 256;

struct AttnArgs {
    const float *Q, *K, *V, *P, *dO;
    float *Pout, *O, *dQ, *dK, *dV, *dPout, *dSout;
    float* dScores;  // [B*H, Sq, Sk] workspace of the backward
    int B, H, Sq, Sk;
    float scale;
    int causal, key_mode;
    // element strides (b, h, s); the head_dim stride is 1
    int64_t qb, qh, qs;  // Q, dQ, O, dO
    int64_t kb, kh, ks;  // K, V, dK, dV
};

inline void strides_for(int layout, int H, int S, int hd, int64_t& sb, int64_t& sh, int64_t& ss) {
    if (layout == MLE_ATTN_TOKEN_MAJOR) {
        sb = (int64_t)S * H * hd;
        sh = hd;
        ss = (int64_t)H * hd;
    } else {
        sb = (int64_t)H * S * hd;
        sh = (int64_t)S * hd;
        ss = hd;
    }
}

// Shared-memory tiles are row-major with rows padded to a multiple of four
// floats plus four (so every row starts 16-byte aligned and consecutive rows
// start four banks apart): operand products read 128-bit vectors along the
// contiguous axis.
template <int HD>
__host__ __device__ constexpr int hd_pitch() { return HD + 4; }
constexpr int kColPitch = kTC + 4;
__host__ __device__ inline int seq_pitch(int S) { return ((S + 3) & ~3) + 4; }

__device__ __forceinline__ float4 lds4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float f4(const float4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

// rows [0, rows) of a [*, HD] operand (row stride rs) into shared rows of
// hd_pitch<HD>() floats; rows >= valid are zero-filled
template <int HD>
__device__ __forceinline__ void load_rows(float* dst, const float* __restrict__ src, int rows, int valid, int64_t rs) {
    constexpr int P = hd_pitch<HD>();
    for (int i = threadIdx.x; i < rows * (HD / 4); i += kNT) {
        const int r = i / (HD / 4), d4 = (i % (HD / 4)) * 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < valid) v = *reinterpret_cast<const float4*>(src + (int64_t)r * rs + d4);
        *reinterpret_cast<float4*>(dst + r * P + d4) = v;
    }
}

// [rows, kTC] tile of a head's [Sq, Sk] matrix (column offset c0) into
// shared rows of kColPitch floats, zero beyond Sk
__device__ __forceinline__ void load_col_tile(float* dst, const float* __restrict__ src, int rows, int Sk, int c0) {
    for (int i = threadIdx.x; i < rows * kTC; i += kNT) {
        const int r = i / kTC, c = i % kTC;
        dst[r * kColPitch + c] = (c0 + c < Sk) ? src[(int64_t)r * Sk + c0 + c] : 0.f;
    }
}

// [kTR, Sk] rows r0.. of a head's [Sq, Sk] matrix into shared rows of
// seq_pitch(Sk) floats, zero beyond Sk and below the tr valid rows
__device__ __forceinline__ void load_row_tile(float* dst, const float* __restrict__ src, int tr, int Sk) {
    const int ld = seq_pitch(Sk), w = ld - 4;
    for (int i = threadIdx.x; i < kTR * w; i += kNT) {
        const int r = i / w, c = i % w;
        dst[r * ld + c] = (r < tr && c < Sk) ? src[(int64_t)r * Sk + c] : 0.f;
    }
}

// Register-tiled products.  Every output is one FMA chain over its
// reduction index in ascending order (the reference kernels' order); a
// thread keeps several such chains, and zero-padded tails only add exact
// zero products.

// out[r][c] = sum_k A[r][k] * B[c][k] (k < HD) for every query row r < Sq
// and the kTC columns c of a block (A: [Sq] rows, B: [kTC] rows, both of
// hd_pitch).  Thread: columns c = t%8 + 8j, rows r = t/8 + 32i (4 x 4
// chains per pass of 128 rows); k advances four at a time with 128-bit
// loads.
template <int HD, typename Epi>
__device__ __forceinline__ void rows_times_cols(const float* As, const float* Bs, int Sq, Epi&& epi) {
    constexpr int P = hd_pitch<HD>();
    const int tx = threadIdx.x & 7, ty = threadIdx.x >> 3;
    for (int rb = 0; rb < Sq; rb += 128) {
        float acc[4][4];
        int ra[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            ra[i] = min(rb + ty + 32 * i, Sq - 1) * P;
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
        }
#pragma unroll 2
        for (int k = 0; k < HD; k += 4) {
            float4 a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = lds4(As + ra[i] + k);
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = lds4(Bs + (tx + 8 * j) * P + k);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(f4(a[i], kk), f4(b[j], kk), acc[i][j]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = rb + ty + 32 * i;
            if (r < Sq) {
#pragma unroll
                for (int j = 0; j < 4; ++j) epi(r, tx + 8 * j, acc[i][j]);
            }
        }
    }
}

// out[x][d] = sum_y M[y][x] * R[y][d] (y < ny) for the kTC columns x of a
// block (M: [ny] rows of kColPitch, R: [ny] rows of hd_pitch).  Thread:
// XV consecutive x (one vector load of M) by DV d's, XV * DV = HD / 8.
template <int HD, typename Epi>
__device__ __forceinline__ void cols_t_times_rows(const float* Ms, const float* Rs, int ny, int nx, Epi&& epi) {
    constexpr int P = hd_pitch<HD>();
    constexpr int XV = HD >= 32 ? 4 : 2, DV = HD / 8 / XV;
    constexpr int XG = kTC / XV;                       // x groups
    const int xg = threadIdx.x % XG, dg = threadIdx.x / XG;
    const int x0 = xg * XV;
    float acc[XV][DV];
#pragma unroll
    for (int u = 0; u < XV; ++u)
#pragma unroll
        for (int v = 0; v < DV; ++v) acc[u][v] = 0.f;
#pragma unroll 4
    for (int y = 0; y < ny; ++y) {
        float m[XV];
        if (XV == 4) {
            const float4 q = lds4(Ms + y * kColPitch + x0);
            m[0] = q.x;
            m[1] = q.y;
            m[XV > 2 ? 2 : 0] = q.z;
            m[XV > 3 ? 3 : 1] = q.w;
        } else {
            const float2 q = *reinterpret_cast<const float2*>(Ms + y * kColPitch + x0);
            m[0] = q.x;
            m[1] = q.y;
        }
        float r[DV];
#pragma unroll
        for (int v = 0; v < DV; ++v) r[v] = Rs[y * P + dg + (kNT / XG) * v];
#pragma unroll
        for (int u = 0; u < XV; ++u)
#pragma unroll
            for (int v = 0; v < DV; ++v) acc[u][v] = fmaf(m[u], r[v], acc[u][v]);
    }
#pragma unroll
    for (int u = 0; u < XV; ++u) {
        const int x = x0 + u;
        if (x < nx) {
#pragma unroll
            for (int v = 0; v < DV; ++v) epi(x, dg + (kNT / XG) * v, acc[u][v]);
        }
    }
}

// out_p[r][d] = sum_c M[r][c] * R_p[c][d] (c < nc) for the kTR rows r of a
// block and one or two right operands R_p ([nc] rows of hd_pitch); M:
// [kTR] rows of ldm (a multiple of 4).  Thread: four consecutive d (one
// vector load of each R_p row) by RI rows; c advances four at a time (one
// vector load of each M row).  Results land in shared tiles O_p [kTR] rows
// of hd_pitch, which may overlay M (the block synchronises first).
template <int HD, int NP>
__device__ __forceinline__ void rows_times_rows(const float* Ms, int ldm, const float* R0, const float* R1, int nc,
                                                float* O0, float* O1) {
    constexpr int P = hd_pitch<HD>();
    constexpr int DG = HD / 4, RG = kNT / DG, RI = kTR / RG;
    const int dg = threadIdx.x % DG, rg = threadIdx.x / DG;
    const int d0 = dg * 4;
    float acc[NP][RI][4];
#pragma unroll
    for (int p = 0; p < NP; ++p)
#pragma unroll
        for (int i = 0; i < RI; ++i)
#pragma unroll
            for (int v = 0; v < 4; ++v) acc[p][i][v] = 0.f;
    const int nc4 = (nc + 3) & ~3;
#pragma unroll 1
    for (int c = 0; c < nc4; c += 4) {
        float4 m[RI];
#pragma unroll
        for (int i = 0; i < RI; ++i) m[i] = lds4(Ms + (rg + RG * i) * ldm + c);
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
            const float4 r0 = lds4(R0 + (c + cc) * P + d0);
            float4 r1 = r0;
            if (NP > 1) r1 = lds4(R1 + (c + cc) * P + d0);
#pragma unroll
            for (int i = 0; i < RI; ++i) {
                const float mv = f4(m[i], cc);
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    acc[0][i][v] = fmaf(mv, f4(r0, v), acc[0][i][v]);
                    if (NP > 1) acc[NP - 1][i][v] = fmaf(mv, f4(r1, v), acc[NP - 1][i][v]);
                }
            }
        }
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < RI; ++i) {
        const int o = (rg + RG * i) * P + d0;
        *reinterpret_cast<float4*>(O0 + o) = make_float4(acc[0][i][0], acc[0][i][1], acc[0][i][2], acc[0][i][3]);
        if (NP > 1)
            *reinterpret_cast<float4*>(O1 + o) =
                make_float4(acc[NP - 1][i][0], acc[NP - 1][i][1], acc[NP - 1][i][2], acc[NP - 1][i][3]);
    }
}

// ------------------------------------------------------------------ forward
// grid (B*H, ceil(Sk / kTC)): P[:, c0:c0+kTC] of one head
template <int HD>
__global__ void __launch_bounds__(kNT) attn_probs_kernel(const AttnArgs a) {
    pdl_entry();
    extern __shared__ __align__(16) float sm[];
    constexpr int P = hd_pitch<HD>();
    const int Sq = a.Sq, Sk = a.Sk, c0 = blockIdx.y * kTC, tc = min(kTC, Sk - c0);
    float* Qs = sm;                      // [Sq][P]
    float* Ks = Qs + Sq * P;             // [kTC][P]
    float* Ss = Ks + kTC * P;            // [Sq][kColPitch]
    float* cred = Ss + Sq * kColPitch;   // [kWarps][kTC]
    const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H, t = threadIdx.x;
    load_rows<HD>(Qs, a.Q + b * a.qb + h * a.qh, Sq, Sq, a.qs);
    load_rows<HD>(Ks, a.K + b * a.kb + h * a.kh + (int64_t)c0 * a.ks, kTC, tc, a.ks);
    __syncthreads();
    // scaled scores (bcmmABT chain, then Scale_Write's product)
    const float scale = a.scale;
    rows_times_cols<HD>(Qs, Ks, Sq, [&](int r, int c, float s) { Ss[r * kColPitch + c] = scale * s; });
    __syncthreads();
    // column max over every row, masked ones included (FindMax); max is
    // exact in any order
    const int lane = t & 31, w = t >> 5;
    {
        float m = -FLT_MAX;
        for (int r = w; r < Sq; r += kWarps) m = fmaxf(m, Ss[r * kColPitch + lane]);
        cred[w * kTC + lane] = m;
    }
    __syncthreads();
    {
        float m = cred[lane];
#pragma unroll
        for (int i = 1; i < kWarps; ++i) m = fmaxf(m, cred[i * kTC + lane]);
        for (int r = w; r < Sq; r += kWarps) {
            float* e = &Ss[r * kColPitch + lane];
            *e = (a.causal && c0 + lane > r) ? 0.0f : expf(*e - m);
        }
    }
    __syncthreads();
    // rows summed in order (SumRows); an all-zero column is divided by 1
    if (t < kTC) {
        float s = 0.f;
#pragma unroll 8
        for (int r = 0; r < Sq; ++r) s += Ss[r * kColPitch + t];
        if (s < 1e-45f) s = 1.0f;
        cred[t] = s;
    }
    __syncthreads();
    float* Pg = a.Pout + (int64_t)bh * Sq * Sk + c0;
    for (int i = t; i < Sq * kTC; i += kNT) {
        const int r = i / kTC, c = i % kTC;
        if (c < tc) Pg[(int64_t)r * Sk + c] = Ss[r * kColPitch + c] / cred[c];
    }
}

// grid (B*H, ceil(Sq / kTR)): O[r0:r0+kTR] = P V
template <int HD>
__global__ void __launch_bounds__(kNT) attn_pv_kernel(const AttnArgs a) {
    pdl_entry();
    extern __shared__ __align__(16) float sm[];
    constexpr int P = hd_pitch<HD>();
    const int Sq = a.Sq, Sk = a.Sk, r0 = blockIdx.y * kTR, tr = min(kTR, Sq - r0);
    const int ldp = seq_pitch(Sk), nk4 = (Sk + 3) & ~3;
    float* Ps = sm;                                   // [kTR][ldp]
    float* Os = sm;                                   // [kTR][P], overlays Ps
    float* Vs = Ps + kTR * max(ldp, P);               // [nk4][P], rows >= Sk zero
    const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H;
    load_row_tile(Ps, a.Pout + ((int64_t)bh * Sq + r0) * Sk, tr, Sk);
    load_rows<HD>(Vs, a.V + b * a.kb + h * a.kh, nk4, Sk, a.ks);
    __syncthreads();
    rows_times_rows<HD, 1>(Ps, ldp, Vs, nullptr, Sk, Os, nullptr);
    __syncthreads();
    float* Og = a.O + b * a.qb + h * a.qh + (int64_t)r0 * a.qs;
    for (int i = threadIdx.x; i < tr * (HD / 4); i += kNT) {
        const int r = i / (HD / 4), d = (i % (HD / 4)) * 4;
        *reinterpret_cast<float4*>(Og + (int64_t)r * a.qs + d) = lds4(Os + r * P + d);
    }
}

// ----------------------------------------------------------------- backward
// grid (B*H, ceil(Sk / kTC)): everything that sums over query rows for the
// keys c0 .. c0+kTC
template <int HD>
__global__ void __launch_bounds__(kNT) attn_bwd_cols_kernel(const AttnArgs a) {
    pdl_entry();
    extern __shared__ __align__(16) float sm[];
    constexpr int P = hd_pitch<HD>();
    const int Sq = a.Sq, Sk = a.Sk, c0 = blockIdx.y * kTC, tc = min(kTC, Sk - c0);
    const bool true_dk = a.key_mode == MLE_KEYGRAD_TRUE;
    float* dOs = sm;                        // [Sq][P]
    float* Vs = dOs + Sq * P;               // [kTC][P]
    float* Ps = Vs + kTC * P;               // [Sq][kColPitch]
    float* Ds = Ps + Sq * kColPitch;        // [Sq][kColPitch]  dP, then dScores
    float* Qs = Ds + Sq * kColPitch;        // [Sq][P]  (true key gradient only)
    float* dot = Qs + (true_dk ? Sq * P : 0);   // [kTC]
    const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H, t = threadIdx.x;
    const int64_t qoff = b * a.qb + h * a.qh, koff = b * a.kb + h * a.kh + (int64_t)c0 * a.ks;
    const int64_t soff = (int64_t)bh * Sq * Sk + c0;
    load_rows<HD>(dOs, a.dO + qoff, Sq, Sq, a.qs);
    load_rows<HD>(Vs, a.V + koff, kTC, tc, a.ks);
    if (true_dk) load_rows<HD>(Qs, a.Q + qoff, Sq, Sq, a.qs);
    load_col_tile(Ps, a.P + (int64_t)bh * Sq * Sk, Sq, Sk, c0);
    __syncthreads();
    // dP = dO V^T (bcmmABT: k = head_dim ascending)
    rows_times_cols<HD>(dOs, Vs, Sq, [&](int r, int c, float s) { Ds[r * kColPitch + c] = s; });
    __syncthreads();
    // deriv_softmax type 1: per column dot over rows in order
    if (t < kTC) {
        float s = 0.f;
#pragma unroll 8
        for (int r = 0; r < Sq; ++r) s = fmaf(Ds[r * kColPitch + t], Ps[r * kColPitch + t], s);
        dot[t] = s;
    }
    __syncthreads();
    // dScaled = P (dP - dot); dScores = (float)(scale * dScaled) as Accumulate
    const double dscale = (double)a.scale;
    for (int i = t; i < Sq * kTC; i += kNT) {
        const int r = i / kTC, c = i % kTC;
        float v = 0.f;
        if (c < tc) {
            const float dp = Ds[r * kColPitch + c];
            if (a.dPout) a.dPout[soff + (int64_t)r * Sk + c] += dp;
            const float ds = Ps[r * kColPitch + c] * (dp - dot[c]);
            if (a.dSout) a.dSout[soff + (int64_t)r * Sk + c] += ds;
            v = (float)(0.0 + dscale * (double)ds);
            a.dScores[soff + (int64_t)r * Sk + c] = v;
        }
        Ds[r * kColPitch + c] = v;
    }
    __syncthreads();
    // dV = P^T dO and the true dK = dScores^T Q for these keys
    // (bcmmATB: k = query row ascending)
    float* dVg = a.dV + koff;
    const int64_t ks = a.ks;
    cols_t_times_rows<HD>(Ps, dOs, Sq, tc, [&](int x, int d, float v) { dVg[(int64_t)x * ks + d] += v; });
    if (true_dk) {
        float* dKg = a.dK + koff;
        cols_t_times_rows<HD>(Ds, Qs, Sq, tc, [&](int x, int d, float v) { dKg[(int64_t)x * ks + d] += v; });
    }
}

// grid (B*H, ceil(Sq / kTR)): sums over keys for the query rows r0 ..
// r0+kTR: dQ = dScores K (bcmm) and the reference key gradient
// dScores Q (bcmmT)
template <int HD>
__global__ void __launch_bounds__(kNT) attn_bwd_rows_kernel(const AttnArgs a) {
    pdl_entry();
    extern __shared__ __align__(16) float sm[];
    constexpr int P = hd_pitch<HD>();
    const int Sq = a.Sq, Sk = a.Sk, r0 = blockIdx.y * kTR, tr = min(kTR, Sq - r0);
    const bool ref_dk = a.key_mode == MLE_KEYGRAD_REFERENCE;
    const int ldm = seq_pitch(Sk), nk4 = (Sk + 3) & ~3;
    float* Ms = sm;                                    // [kTR][ldm] dScores rows
    float* Oq = sm;                                    // [kTR][P] dQ rows, overlays Ms
    float* Ok = Oq + kTR * P;                          // [kTR][P] reference key gradient
    float* Ks = Ms + kTR * max(ldm, 2 * P);            // [nk4][P]
    float* Qs = Ks + nk4 * P;                          // [nk4][P]  (reference key gradient; Sq == Sk)
    const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H;
    load_row_tile(Ms, a.dScores + ((int64_t)bh * Sq + r0) * Sk, tr, Sk);
    const int64_t qoff = b * a.qb + h * a.qh, koff = b * a.kb + h * a.kh;
    load_rows<HD>(Ks, a.K + koff, nk4, Sk, a.ks);
    if (ref_dk) load_rows<HD>(Qs, a.Q + qoff, nk4, Sk, a.qs);
    __syncthreads();
    if (ref_dk) rows_times_rows<HD, 2>(Ms, ldm, Ks, Qs, Sk, Oq, Ok);
    else rows_times_rows<HD, 1>(Ms, ldm, Ks, nullptr, Sk, Oq, nullptr);
    __syncthreads();
    float* dQg = a.dQ + qoff + (int64_t)r0 * a.qs;
    for (int i = threadIdx.x; i < tr * (HD / 4); i += kNT) {
        const int r = i / (HD / 4), d = (i % (HD / 4)) * 4;
        float4* g = reinterpret_cast<float4*>(dQg + (int64_t)r * a.qs + d);
        float4 o = *g;
        const float4 v = lds4(Oq + r * P + d);
        o.x += v.x;
        o.y += v.y;
        o.z += v.z;
        o.w += v.w;
        *g = o;
    }
    if (ref_dk) {
        // bcmmT(Q, dScores, Kh.grad, hd, Sq, Sk) writes element (row d, col
        // r) of its [hd, Sk] result at d*Sk + r of the head's [Sk, hd]
        // gradient block: consecutive r are consecutive there
        float* dKg = a.dK + koff;
        for (int i = threadIdx.x; i < tr * HD; i += kNT) {
            const int d = i / tr, r = i % tr;
            const int pos = d * Sk + r0 + r;
            dKg[(int64_t)(pos / HD) * a.ks + pos % HD] += Ok[r * P + d];
        }
    }
}

template <int HD>
size_t probs_smem(int Sq) {
    return sizeof(float) * ((size_t)Sq * hd_pitch<HD>() + kTC * hd_pitch<HD>() + (size_t)Sq * kColPitch + kWarps * kTC);
}
template <int HD>
size_t pv_smem(int Sk) {
    const size_t nk4 = (size_t)((Sk + 3) & ~3);
    return sizeof(float) * ((size_t)kTR * std::max(seq_pitch(Sk), hd_pitch<HD>()) + nk4 * hd_pitch<HD>());
}
template <int HD>
size_t bwd_cols_smem(int Sq, bool true_dk) {
    return sizeof(float) * ((size_t)Sq * hd_pitch<HD>() * (true_dk ? 2 : 1) + kTC * hd_pitch<HD>() +
                            2 * (size_t)Sq * kColPitch + kTC);
}
template <int HD>
size_t bwd_rows_smem(int Sk, bool ref_dk) {
    const size_t nk4 = (size_t)((Sk + 3) & ~3);
    return sizeof(float) * ((size_t)kTR * std::max(seq_pitch(Sk), 2 * hd_pitch<HD>()) +
                            nk4 * hd_pitch<HD>() * (ref_dk ? 2 : 1));
}

constexpr size_t kMaxSmem = 227 * 1024;

template <typename K>
int set_smem(K kern, bool& done) {
    if (!done) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem) != cudaSuccess)
            return launch_status();
        done = true;
    }
    return MLE_OK;
}

template <int HD>
int launch_fwd(const AttnArgs& a, cudaStream_t st) {
    const size_t s1 = probs_smem<HD>(a.Sq), s2 = pv_smem<HD>(a.Sk);
    if (s1 > kMaxSmem || s2 > kMaxSmem) return MLE_ERR_UNSUPPORTED;
    static bool c1 = false, c2 = false;
    int s = set_smem(attn_probs_kernel<HD>, c1);
    if (s == MLE_OK) s = set_smem(attn_pv_kernel<HD>, c2);
    if (s) return s;
    launch_k(attn_probs_kernel<HD>, dim3(a.B * a.H, (a.Sk + kTC - 1) / kTC), kNT, s1, st, a);
    s = launch_status();
    if (s) return s;
    launch_k(attn_pv_kernel<HD>, dim3(a.B * a.H, (a.Sq + kTR - 1) / kTR), kNT, s2, st, a);
    return launch_status();
}

template <int HD>
int launch_bwd(const AttnArgs& a, cudaStream_t st) {
    const bool true_dk = a.key_mode == MLE_KEYGRAD_TRUE;
    const size_t s1 = bwd_cols_smem<HD>(a.Sq, true_dk), s2 = bwd_rows_smem<HD>(a.Sk, !true_dk);
    if (s1 > kMaxSmem || s2 > kMaxSmem) return MLE_ERR_UNSUPPORTED;
    static bool c1 = false, c2 = false;
    int s = set_smem(attn_bwd_cols_kernel<HD>, c1);
    if (s == MLE_OK) s = set_smem(attn_bwd_rows_kernel<HD>, c2);
    if (s) return s;
    launch_k(attn_bwd_cols_kernel<HD>, dim3(a.B * a.H, (a.Sk + kTC - 1) / kTC), kNT, s1, st, a);
    s = launch_status();
    if (s) return s;
    launch_k(attn_bwd_rows_kernel<HD>, dim3(a.B * a.H, (a.Sq + kTR - 1) / kTR), kNT, s2, st, a);
    return launch_status();
}

bool fused_ok(int axis, int Sq, int Sk, int hd, int B, int H) {
    return axis == 1 && Sq >= 1 && Sq <= kMaxSeq && Sk >= 1 && Sk <= kMaxSeq && (hd == 16 || hd == 32 || hd == 64) &&
           (int64_t)B * H < (1ll << 31);
}

bool ptrs_aligned(std::initializer_list<const float*> ps) {
    for (const float* q : ps)
        if (!aligned16(q)) return false;
    return true;
}

template <typename F>
int dispatch_hd(int hd, F&& f) {
    switch (hd) {
        case 16: return f(std::integral_constant<int, 16>());
        case 32: return f(std::integral_constant<int, 32>());
        default: return f(std::integral_constant<int, 64>());
    }
}

// ------------------------------ tensor-core path -----------------------------
thread_local int g_attn_path = MLE_ATTN_PATH_AUTO;
// 1: the tensor-core path computes P (forward) and the score gradient
// (backward) with the keys-on-lanes kernels of gemm_tcgen05.cu; 0: product
// to HBM, then the column softmax (or its backward) in place
thread_local int g_attn_keys = 1;
// 1: graph attention nodes use the flash entry points where supported
thread_local int g_attn_flash = 1;

// Column softmax of each [rows, cols] matrix in place (the reference's type
// 1, causal entries key > query zeroed after the max over the whole column,
// as SoftMask does), the form for columns of more than 512 rows (the
// single-pass register kernels below take the rest).  A 256-thread block owns (matrix, 128 columns): lane l
// holds columns 4l..4l+3 (16-byte accesses), warp w the rows w, w + 8, ...
// Three passes over the block's rows, the later two served by L2: the
// column max, the sum of the exponentials, the probabilities; the 8 warps'
// partials merge in shared memory.  Every pass is a short dependency chain
// per element, so the loads of several rows stay in flight.  cols % 4 == 0.
constexpr int kSmThreads = 256;

__global__ void __launch_bounds__(kSmThreads) col_softmax_vec(float* __restrict__ P, int rows, int cols, int causal,
                                                              int mats) {
    pdl_entry();
    __shared__ float red[8][128 + 4];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c0 = blockIdx.x * 128 + lane * 4;
    const bool live = c0 < cols;
    for (int mat = blockIdx.y; mat < mats; mat += gridDim.y) {
        float* Pm = P + (int64_t)mat * rows * cols + c0;
        float m[4] = {-FLT_MAX, -FLT_MAX, -FLT_MAX, -FLT_MAX};
        if (live) {
#pragma unroll 8
            for (int r = warp; r < rows; r += 8) {
                const float4 v = *reinterpret_cast<const float4*>(Pm + (int64_t)r * cols);
                m[0] = fmaxf(m[0], v.x);
                m[1] = fmaxf(m[1], v.y);
                m[2] = fmaxf(m[2], v.z);
                m[3] = fmaxf(m[3], v.w);
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) red[warp][lane * 4 + j] = m[j];
        __syncthreads();
#pragma unroll
        for (int j = 0; j < 4; ++j)
            for (int w = 0; w < 8; ++w) m[j] = fmaxf(m[j], red[w][lane * 4 + j]);
        __syncthreads();
        float sum[4] = {0.f, 0.f, 0.f, 0.f};
        if (live) {
#pragma unroll 8
            for (int r = warp; r < rows; r += 8) {
                const float4 v4 = *reinterpret_cast<const float4*>(Pm + (int64_t)r * cols);
                const float v[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) sum[j] += (causal && c0 + j > r) ? 0.f : expf(v[j] - m[j]);
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) red[warp][lane * 4 + j] = sum[j];
        __syncthreads();
        float inv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float t = 0.f;
            for (int w = 0; w < 8; ++w) t += red[w][lane * 4 + j];
            if (t < 1e-45f) t = 1.0f;
            inv[j] = 1.0f / t;
        }
        __syncthreads();
        if (live) {
#pragma unroll 8
            for (int r = warp; r < rows; r += 8) {
                float4* p4 = reinterpret_cast<float4*>(Pm + (int64_t)r * cols);
                const float4 v4 = *p4;
                const float v[4] = {v4.x, v4.y, v4.z, v4.w};
                float o[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) o[j] = (causal && c0 + j > r) ? 0.f : expf(v[j] - m[j]) * inv[j];
                *p4 = make_float4(o[0], o[1], o[2], o[3]);
            }
        }
    }
}

// G (dP on entry) becomes dS = P (dP - sum over the column of P dP); same
// block shape, pass 1 the column dots, pass 2 the update.
__global__ void __launch_bounds__(kSmThreads) col_softmax_bwd_vec(const float* __restrict__ P, float* __restrict__ G,
                                                                  int rows, int cols, int mats) {
    pdl_entry();
    __shared__ float red[8][128 + 4];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c0 = blockIdx.x * 128 + lane * 4;
    const bool live = c0 < cols;
    for (int mat = blockIdx.y; mat < mats; mat += gridDim.y) {
        const float* Pm = P + (int64_t)mat * rows * cols + c0;
        float* Gm = G + (int64_t)mat * rows * cols + c0;
        float dot[4] = {0.f, 0.f, 0.f, 0.f};
        if (live) {
#pragma unroll 8
            for (int r = warp; r < rows; r += 8) {
                const float4 p = *reinterpret_cast<const float4*>(Pm + (int64_t)r * cols);
                const float4 g = *reinterpret_cast<const float4*>(Gm + (int64_t)r * cols);
                dot[0] += p.x * g.x;
                dot[1] += p.y * g.y;
                dot[2] += p.z * g.z;
                dot[3] += p.w * g.w;
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) red[warp][lane * 4 + j] = dot[j];
        __syncthreads();
        float D[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            D[j] = 0.f;
            for (int w = 0; w < 8; ++w) D[j] += red[w][lane * 4 + j];
        }
        __syncthreads();
        if (live) {
#pragma unroll 8
            for (int r = warp; r < rows; r += 8) {
                const float4 p = *reinterpret_cast<const float4*>(Pm + (int64_t)r * cols);
                float4* g4 = reinterpret_cast<float4*>(Gm + (int64_t)r * cols);
                const float4 g = *g4;
                *g4 = make_float4(p.x * (g.x - D[0]), p.y * (g.y - D[1]), p.z * (g.z - D[2]), p.w * (g.w - D[3]));
            }
        }
    }
}

// Single-pass forms for columns of at most 512 rows: a block of 8 * RG
// threads owns (matrix, 32 columns); lane l = tid % 8 holds columns
// 4l..4l+3, row group g = tid / 8 the rows g, g + RG, ... (RPT of them), all
// in registers, so every element is read once and written once.  Each warp
// load covers four full 128-byte rows.  The column partials merge across
// the warp's four row groups with shuffles, then across warps in shared
// memory.
__device__ __forceinline__ float4 max4(float4 a, float4 b) {
    return make_float4(fmaxf(a.x, b.x), fmaxf(a.y, b.y), fmaxf(a.z, b.z), fmaxf(a.w, b.w));
}
__device__ __forceinline__ float4 add4(float4 a, float4 b) {
    return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}
__device__ __forceinline__ float4 shfl_xor4(float4 v, int m) {
    return make_float4(__shfl_xor_sync(0xffffffffu, v.x, m), __shfl_xor_sync(0xffffffffu, v.y, m),
                       __shfl_xor_sync(0xffffffffu, v.z, m), __shfl_xor_sync(0xffffffffu, v.w, m));
}

template <int RG, int RPT>
__global__ void __launch_bounds__(8 * RG) col_softmax_reg(float* __restrict__ P, int rows, int cols, int causal,
                                                          int mats) {
    pdl_entry();
    constexpr int kWarps = RG / 4;
    __shared__ float4 red[kWarps][8];
    const int l = threadIdx.x & 7, g = threadIdx.x >> 3, warp = threadIdx.x >> 5;
    const int c0 = blockIdx.x * 32 + l * 4;
    const bool live = c0 < cols;
    for (int mat = blockIdx.y; mat < mats; mat += gridDim.y) {
        float* Pm = P + (int64_t)mat * rows * cols + c0;
        float4 v[RPT];
        float4 m = make_float4(-FLT_MAX, -FLT_MAX, -FLT_MAX, -FLT_MAX);
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
            const int r = g + i * RG;
            if (live && r < rows) {
                v[i] = *reinterpret_cast<const float4*>(Pm + (int64_t)r * cols);
                m = max4(m, v[i]);
            }
        }
        m = max4(m, shfl_xor4(m, 8));
        m = max4(m, shfl_xor4(m, 16));
        if ((threadIdx.x & 31) < 8) red[warp][l] = m;
        __syncthreads();
        m = red[0][l];
#pragma unroll
        for (int w = 1; w < kWarps; ++w) m = max4(m, red[w][l]);
        __syncthreads();
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
            const int r = g + i * RG;
            if (live && r < rows) {
                float4 e;
                e.x = (causal && c0 + 0 > r) ? 0.f : expf(v[i].x - m.x);
                e.y = (causal && c0 + 1 > r) ? 0.f : expf(v[i].y - m.y);
                e.z = (causal && c0 + 2 > r) ? 0.f : expf(v[i].z - m.z);
                e.w = (causal && c0 + 3 > r) ? 0.f : expf(v[i].w - m.w);
                v[i] = e;
                s = add4(s, e);
            }
        }
        s = add4(s, shfl_xor4(s, 8));
        s = add4(s, shfl_xor4(s, 16));
        if ((threadIdx.x & 31) < 8) red[warp][l] = s;
        __syncthreads();
        s = red[0][l];
#pragma unroll
        for (int w = 1; w < kWarps; ++w) s = add4(s, red[w][l]);
        __syncthreads();
        const float4 inv = make_float4(1.0f / (s.x < 1e-45f ? 1.0f : s.x), 1.0f / (s.y < 1e-45f ? 1.0f : s.y),
                                       1.0f / (s.z < 1e-45f ? 1.0f : s.z), 1.0f / (s.w < 1e-45f ? 1.0f : s.w));
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
            const int r = g + i * RG;
            if (live && r < rows)
                *reinterpret_cast<float4*>(Pm + (int64_t)r * cols) =
                    make_float4(v[i].x * inv.x, v[i].y * inv.y, v[i].z * inv.z, v[i].w * inv.w);
        }
    }
}

template <int RG, int RPT>
__global__ void __launch_bounds__(8 * RG) col_softmax_bwd_reg(const float* __restrict__ P, float* __restrict__ G,
                                                              int rows, int cols, int mats) {
    pdl_entry();
    constexpr int kWarps = RG / 4;
    __shared__ float4 red[kWarps][8];
    const int l = threadIdx.x & 7, g = threadIdx.x >> 3, warp = threadIdx.x >> 5;
    const int c0 = blockIdx.x * 32 + l * 4;
    const bool live = c0 < cols;
    for (int mat = blockIdx.y; mat < mats; mat += gridDim.y) {
        const float* Pm = P + (int64_t)mat * rows * cols + c0;
        float* Gm = G + (int64_t)mat * rows * cols + c0;
        float4 p[RPT], q[RPT];
        float4 d = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
            const int r = g + i * RG;
            if (live && r < rows) {
                p[i] = *reinterpret_cast<const float4*>(Pm + (int64_t)r * cols);
                q[i] = *reinterpret_cast<const float4*>(Gm + (int64_t)r * cols);
            }
        }
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
            const int r = g + i * RG;
            if (live && r < rows)
                d = make_float4(d.x + p[i].x * q[i].x, d.y + p[i].y * q[i].y, d.z + p[i].z * q[i].z,
                                d.w + p[i].w * q[i].w);
        }
        d = add4(d, shfl_xor4(d, 8));
        d = add4(d, shfl_xor4(d, 16));
        if ((threadIdx.x & 31) < 8) red[warp][l] = d;
        __syncthreads();
        d = red[0][l];
#pragma unroll
        for (int w = 1; w < kWarps; ++w) d = add4(d, red[w][l]);
        __syncthreads();
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
            const int r = g + i * RG;
            if (live && r < rows)
                *reinterpret_cast<float4*>(Gm + (int64_t)r * cols) =
                    make_float4(p[i].x * (q[i].x - d.x), p[i].y * (q[i].y - d.y), p[i].z * (q[i].z - d.z),
                                p[i].w * (q[i].w - d.w));
        }
    }
}

// Calls f(std::integral_constant<int, RG>, std::integral_constant<int, RPT>)
// for the single-pass shape covering `rows`; false above 512 rows.
template <typename F>
bool col_shape(int rows, F&& f) {
    using std::integral_constant;
    if (rows <= 32) return f(integral_constant<int, 32>(), integral_constant<int, 1>()), true;
    if (rows <= 64) return f(integral_constant<int, 32>(), integral_constant<int, 2>()), true;
    if (rows <= 128) return f(integral_constant<int, 32>(), integral_constant<int, 4>()), true;
    if (rows <= 256) return f(integral_constant<int, 32>(), integral_constant<int, 8>()), true;
    if (rows <= 512) return f(integral_constant<int, 64>(), integral_constant<int, 8>()), true;
    return false;
}

int tc_col_softmax(float* P, int64_t mats, int rows, int cols, int causal, cudaStream_t st) {
    const unsigned gy = (unsigned)std::min<int64_t>(mats, 65535);
    const bool single = col_shape(rows, [&](auto rg, auto rpt) {
        launch_k(col_softmax_reg<decltype(rg)::value, decltype(rpt)::value>, dim3((unsigned)((cols + 31) / 32), gy),
                 8 * decltype(rg)::value, 0, st, P, rows, cols, causal, (int)mats);
    });
    if (!single)
        launch_k(col_softmax_vec, dim3((unsigned)((cols + 127) / 128), gy), kSmThreads, 0, st, P, rows, cols, causal,
                 (int)mats);
    return launch_status();
}

int tc_col_softmax_bwd(const float* P, float* G, int64_t mats, int rows, int cols, cudaStream_t st) {
    const unsigned gy = (unsigned)std::min<int64_t>(mats, 65535);
    const bool single = col_shape(rows, [&](auto rg, auto rpt) {
        launch_k(col_softmax_bwd_reg<decltype(rg)::value, decltype(rpt)::value>,
                 dim3((unsigned)((cols + 31) / 32), gy), 8 * decltype(rg)::value, 0, st, P, G, rows, cols, (int)mats);
    });
    if (!single)
        launch_k(col_softmax_bwd_vec, dim3((unsigned)((cols + 127) / 128), gy), kSmThreads, 0, st, P, G, rows, cols,
                 (int)mats);
    return launch_status();
}

GemmProblem attn_gemm(const float* A, const float* B, float* C, int M, int N, int K, int64_t lda, int64_t ldb,
                      int64_t ldc, int ta, int tb, int nb, int nh, int64_t a_sb, int64_t a_sh, int64_t b_sb,
                      int64_t b_sh, int64_t c_sb, int64_t c_sh, float alpha, int mode) {
    GemmProblem p;
    memset(&p, 0, sizeof(p));
    p.A = A;
    p.B = B;
    p.C = C;
    p.M = M;
    p.N = N;
    p.K = K;
    p.lda = lda;
    p.ldb = ldb;
    p.ldc = ldc;
    p.trans_a = ta;
    p.trans_b = tb;
    p.nbatch = nb;
    p.channels = nh;
    p.a_sb = a_sb;
    p.a_sc = a_sh;
    p.b_sb = b_sb;
    p.b_sc = b_sh;
    p.c_sb = c_sb;
    p.c_sc = c_sh;
    p.alpha = alpha;
    p.mode = mode;
    return p;
}

// Whether the tensor-core path can run these sizes (GEMM operand strides and
// softmax rows in whole 16-byte units, the reference key gradient's
// head-block split in whole 32-column blocks) and is the one to take.
bool tc_attention_ok(int axis, int Sq, int Sk, int hd, int64_t BH, bool bwd, int key_mode) {
    if (g_attn_path == MLE_ATTN_PATH_FUSED || mle_get_gemm_mode() != MLE_GEMM_MODE_TF32) return false;
    if (axis != 1 || hd % 4 || Sq % 4 || Sk % 4 || BH > INT32_MAX) return false;
    if (bwd && key_mode == MLE_KEYGRAD_REFERENCE && !(Sq == Sk && hd % 32 == 0 && Sk % hd == 0)) return false;
    if (g_attn_path == MLE_ATTN_PATH_TENSOR) return true;
    // the CUDA-core kernels win below about 256K multiply-adds per head
    // product (measured: configs[1], 128 x 128 x 32, ran 10 % faster per
    // step on the tensor-core path)
    return (int64_t)Sq * Sk * hd >= (1ll << 18) || !fused_ok(axis, Sq, Sk, hd, 1, 1);
}

int tc_attention_fwd(const float* Q, const float* K, const float* V, float* P, float* O, int B, int H, int Sq, int Sk,
                     int hd, float scale, int causal, int layout, cudaStream_t st) {
    int64_t qb, qh, qs, kb, kh, ks;
    strides_for(layout, H, Sq, hd, qb, qh, qs);
    strides_for(layout, H, Sk, hd, kb, kh, ks);
    const int64_t pb = (int64_t)H * Sq * Sk, ph = (int64_t)Sq * Sk;
    int s = MLE_ERR_UNSUPPORTED;
    // P = softmax over each column of scale Q K^T: in one kernel with the
    // keys on the TMEM lanes (the scores stay on chip), or as a product
    // written to P and softmaxed in place
    if (g_attn_keys && attn_keys_supported(Sq, Sk, hd, (int64_t)B * H))
        s = run_attn_keys(0, K, Q, nullptr, P, B, H, Sq, Sk, hd, kb, kh, ks, qb, qh, qs, scale, causal, st);
    if (s == MLE_ERR_UNSUPPORTED) {
        s = run_gemm(attn_gemm(Q, K, P, Sq, Sk, hd, qs, ks, Sk, 0, 1, B, H, qb, qh, kb, kh, pb, ph, scale, 0), st);
        if (s) return s;
        s = tc_col_softmax(P, (int64_t)B * H, Sq, Sk, causal, st);
    }
    if (s) return s;
    // O = P V
    return run_gemm(attn_gemm(P, V, O, Sq, hd, Sk, Sk, ks, qs, 0, 0, B, H, pb, ph, kb, kh, qb, qh, 1.0f, 0), st);
}

// assign: bit 0 dQ, bit 1 dK, bit 2 dV written (not accumulated)
int tc_attention_bwd(const float* Q, const float* K, const float* V, const float* P, const float* dO, float* dQ,
                     float* dK, float* dV, float* dP_out, float* dS_out, float* W, int B, int H, int Sq, int Sk,
                     int hd, float scale, int key_mode, int layout, cudaStream_t st, int assign = 0) {
    const int mq = (assign & 1) ? 0 : 1, mk = (assign & 2) ? 0 : 1, mv = (assign & 4) ? 0 : 1;
    int64_t qb, qh, qs, kb, kh, ks;
    strides_for(layout, H, Sq, hd, qb, qh, qs);
    strides_for(layout, H, Sk, hd, kb, kh, ks);
    const int64_t pb = (int64_t)H * Sq * Sk, ph = (int64_t)Sq * Sk, ns = (int64_t)B * pb;
    int s = MLE_ERR_UNSUPPORTED;
    // W = P (dP - column sums of P dP), the score gradient, dP = dO V^T the
    // softmax node's gradient: in one kernel with the keys on the TMEM lanes
    // (dP stays on chip), or dP written to W and transformed in place
    if (g_attn_keys && !dP_out && attn_keys_supported(Sq, Sk, hd, (int64_t)B * H))
        s = run_attn_keys(1, V, dO, P, W, B, H, Sq, Sk, hd, kb, kh, ks, qb, qh, qs, 1.0f, 0, st);
    if (s == MLE_ERR_UNSUPPORTED) {
        s = run_gemm(attn_gemm(dO, V, W, Sq, Sk, hd, qs, ks, Sk, 0, 1, B, H, qb, qh, kb, kh, pb, ph, 1.0f, 0), st);
        if (s) return s;
        if (dP_out && (s = mle_accumulate(W, dP_out, ns, 1.0, st)) != 0) return s;
        s = tc_col_softmax_bwd(P, W, (int64_t)B * H, Sq, Sk, st);
    }
    if (s) return s;
    if (dS_out && (s = mle_accumulate(W, dS_out, ns, 1.0, st)) != 0) return s;
    // dV += P^T dO
    s = run_gemm(attn_gemm(P, dO, dV, Sk, hd, Sq, Sk, qs, ks, 1, 0, B, H, pb, ph, qb, qh, kb, kh, 1.0f, mv), st);
    if (s) return s;
    // dQ += scale W K
    s = run_gemm(attn_gemm(W, K, dQ, Sq, hd, Sk, Sk, ks, qs, 0, 0, B, H, pb, ph, kb, kh, qb, qh, scale, mq), st);
    if (s) return s;
    if (key_mode == MLE_KEYGRAD_TRUE)  // dK += scale W^T Q
        return run_gemm(attn_gemm(W, Q, dK, Sk, hd, Sq, Sk, qs, ks, 1, 0, B, H, pb, ph, qb, qh, kb, kh, scale, mk),
                        st);
    // reference: the head block of dK receives scale * Q^T M^T as [hd, Sk],
    // M = W's memory read as [Sk, Sq]; block element (d, i) lives at row
    // d*(Sk/hd) + i/hd, column i % hd of the head in `layout`
    GemmProblem g = attn_gemm(Q, W, dK, hd, Sk, Sq, qs, Sq, (int64_t)(Sk / hd) * ks, 1, 1, B, H, qb, qh, pb, ph, kb,
                              kh, scale, mk);
    g.c_split = hd;
    g.c_split_ld = ks;
    return run_gemm(g, st);
}

}  // namespace
}  // namespace mle

using namespace mle;

extern "C" {

int mle_set_attention_path(int path) {
    if (path != MLE_ATTN_PATH_AUTO && path != MLE_ATTN_PATH_FUSED && path != MLE_ATTN_PATH_TENSOR)
        return MLE_ERR_ARG;
    g_attn_path = path;
    return MLE_OK;
}

int mle_get_attention_path(void) { return g_attn_path; }

int mle_set_attention_keys_kernel(int enable) {
    if (enable != 0 && enable != 1) return MLE_ERR_ARG;
    g_attn_keys = enable;
    return MLE_OK;
}

int mle_get_attention_keys_kernel(void) { return g_attn_keys; }

int mle_set_attention_flash(int enable) {
    if (enable != 0 && enable != 1) return MLE_ERR_ARG;
    g_attn_flash = enable;
    return MLE_OK;
}

int mle_get_attention_flash(void) { return g_attn_flash; }

int mle_attention_flash_supported(int seq_q, int seq_k, int head_dim, int softmax_axis, int key_grad_mode) {
    if (!g_attn_flash || softmax_axis != 1 || mle_get_gemm_mode() != MLE_GEMM_MODE_TF32) return 0;
    if (key_grad_mode != MLE_KEYGRAD_REFERENCE && key_grad_mode != MLE_KEYGRAD_TRUE) return 0;
    return attn_flash_supported(seq_q, seq_k, head_dim, 1, key_grad_mode) ? 1 : 0;
}

int mle_attention_flash_fwd(const float* Q, const float* K, const float* V, float* O, float* stats, int batch,
                            int heads, int seq_q, int seq_k, int head_dim, float scale, int causal, int layout,
                            mle_stream_t stream) {
    if (!Q || !K || !V || !O || !stats || batch <= 0 || heads <= 0) return MLE_ERR_ARG;
    if (layout != MLE_ATTN_HEAD_MAJOR && layout != MLE_ATTN_TOKEN_MAJOR) return MLE_ERR_ARG;
    if (!mle_attention_flash_supported(seq_q, seq_k, head_dim, 1, MLE_KEYGRAD_TRUE) ||
        !ptrs_aligned({Q, K, V, O, stats}))
        return MLE_ERR_UNSUPPORTED;
    int64_t qb, qh, qs, kb, kh, ks;
    strides_for(layout, heads, seq_q, head_dim, qb, qh, qs);
    strides_for(layout, heads, seq_k, head_dim, kb, kh, ks);
    return run_attn_flash_fwd(Q, K, V, O, stats, batch, heads, seq_q, seq_k, head_dim, qb, qh, qs, kb, kh, ks, scale,
                              causal ? 1 : 0, as_stream(stream));
}

int mle_attention_flash_bwd(const float* Q, const float* K, const float* V, const float* dO, const float* stats,
                            float* dvec, float* dQ, float* dK, float* dV, int batch, int heads, int seq_q,
                            int seq_k, int head_dim, float scale, int causal, int key_grad_mode, int layout,
                            int assign_mask, mle_stream_t stream) {
    if (!Q || !K || !V || !dO || !stats || !dvec || !dQ || !dK || !dV || batch <= 0 || heads <= 0)
        return MLE_ERR_ARG;
    if (layout != MLE_ATTN_HEAD_MAJOR && layout != MLE_ATTN_TOKEN_MAJOR) return MLE_ERR_ARG;
    if (assign_mask < 0 || assign_mask > 7) return MLE_ERR_ARG;
    if ((dQ == dK && (assign_mask & 3)) || (dQ == dV && (assign_mask & 5)) || (dK == dV && (assign_mask & 6)))
        return MLE_ERR_ARG;
    if (!mle_attention_flash_supported(seq_q, seq_k, head_dim, 1, key_grad_mode) ||
        !ptrs_aligned({Q, K, V, dO, stats, dvec, dQ, dK, dV}))
        return MLE_ERR_UNSUPPORTED;
    int64_t qb, qh, qs, kb, kh, ks;
    strides_for(layout, heads, seq_q, head_dim, qb, qh, qs);
    strides_for(layout, heads, seq_k, head_dim, kb, kh, ks);
    return run_attn_flash_bwd(Q, K, V, dO, stats, dvec, dQ, dK, dV, batch, heads, seq_q, seq_k, head_dim, qb, qh, qs,
                              kb, kh, ks, scale, causal ? 1 : 0, key_grad_mode, assign_mask, as_stream(stream));
}

int mle_attention_fused_supported(int seq_q, int seq_k, int head_dim, int softmax_axis, int key_grad_mode) {
    if (!fused_ok(softmax_axis, seq_q, seq_k, head_dim, 1, 1)) return 0;
    if (key_grad_mode == MLE_KEYGRAD_REFERENCE && seq_q != seq_k) return 0;
    const bool t = key_grad_mode == MLE_KEYGRAD_TRUE;
    const int ok = dispatch_hd(head_dim, [&](auto hd) {
        constexpr int HD = decltype(hd)::value;
        return (int)(probs_smem<HD>(seq_q) <= kMaxSmem && pv_smem<HD>(seq_k) <= kMaxSmem &&
                     bwd_cols_smem<HD>(seq_q, t) <= kMaxSmem && bwd_rows_smem<HD>(seq_k, !t) <= kMaxSmem);
    });
    return ok;
}

int mle_attention_fwd(const float* Q, const float* K, const float* V, float* P, float* O, int batch, int heads,
                      int seq_q, int seq_k, int head_dim, float scale, int causal, int softmax_axis, int layout,
                      mle_stream_t stream) {
    if (!Q || !K || !V || !P || !O) return MLE_ERR_ARG;
    if (batch <= 0 || heads <= 0 || seq_q <= 0 || seq_k <= 0 || head_dim <= 0) return MLE_ERR_ARG;
    if ((softmax_axis != 0 && softmax_axis != 1) || (layout != MLE_ATTN_HEAD_MAJOR && layout != MLE_ATTN_TOKEN_MAJOR))
        return MLE_ERR_ARG;
    cudaStream_t st = as_stream(stream);
    if (tc_attention_ok(softmax_axis, seq_q, seq_k, head_dim, (int64_t)batch * heads, false, MLE_KEYGRAD_TRUE) &&
        ptrs_aligned({Q, K, V, P, O})) {
        const int s = tc_attention_fwd(Q, K, V, P, O, batch, heads, seq_q, seq_k, head_dim, scale, causal, layout, st);
        if (s != MLE_ERR_UNSUPPORTED) return s;
    }
    if (fused_ok(softmax_axis, seq_q, seq_k, head_dim, batch, heads) && ptrs_aligned({Q, K, V, O})) {
        AttnArgs a{};
        a.Q = Q;
        a.K = K;
        a.V = V;
        a.Pout = P;
        a.O = O;
        a.B = batch;
        a.H = heads;
        a.Sq = seq_q;
        a.Sk = seq_k;
        a.scale = scale;
        a.causal = causal;
        strides_for(layout, heads, seq_q, head_dim, a.qb, a.qh, a.qs);
        strides_for(layout, heads, seq_k, head_dim, a.kb, a.kh, a.ks);
        const int s = dispatch_hd(head_dim, [&](auto hd) { return launch_fwd<decltype(hd)::value>(a, st); });
        if (s != MLE_ERR_UNSUPPORTED) return s;
    }
    if (layout != MLE_ATTN_HEAD_MAJOR) return MLE_ERR_UNSUPPORTED;
    // composed: P = scale * Q K^T (tensor cores), softmax in place, O = P V
    int s = mle_bcmm(MLE_GEMM_ABT, Q, K, P, batch, heads, seq_q, head_dim, seq_k, 0, 3, 3, 3, scale, stream);
    if (s) return s;
    s = mle_softmax_fwd(P, P, (int64_t)batch * heads, seq_q, seq_k, softmax_axis, causal, stream);
    if (s) return s;
    return mle_bcmm(MLE_GEMM_AB, P, V, O, batch, heads, seq_q, seq_k, head_dim, 0, 3, 3, 3, 1.0f, stream);
}

int mle_attention_bwd(const float* Q, const float* K, const float* V, const float* P, const float* dO, float* dQ,
                      float* dK, float* dV, float* dP_out, float* dS_out, float* workspace, int batch, int heads,
                      int seq_q, int seq_k, int head_dim, float scale, int causal, int softmax_axis,
                      int key_grad_mode, int layout, mle_stream_t stream) {
    return mle_attention_bwd_assign(Q, K, V, P, dO, dQ, dK, dV, dP_out, dS_out, workspace, batch, heads, seq_q, seq_k,
                                    head_dim, scale, causal, softmax_axis, key_grad_mode, layout, 0, stream);
}

int mle_attention_bwd_assign(const float* Q, const float* K, const float* V, const float* P, const float* dO,
                             float* dQ, float* dK, float* dV, float* dP_out, float* dS_out, float* workspace,
                             int batch, int heads, int seq_q, int seq_k, int head_dim, float scale, int causal,
                             int softmax_axis, int key_grad_mode, int layout, int assign_mask, mle_stream_t stream) {
    (void)causal;  // P is exactly zero where the mask applied, so dS is too
    if (assign_mask < 0 || assign_mask > 7) return MLE_ERR_ARG;
    if ((dQ == dK && (assign_mask & 3)) || (dQ == dV && (assign_mask & 5)) || (dK == dV && (assign_mask & 6)))
        return MLE_ERR_ARG;  // an assigned gradient may not also receive another one
    if (!Q || !K || !V || !P || !dO || !dQ || !dK || !dV) return MLE_ERR_ARG;
    if (batch <= 0 || heads <= 0 || seq_q <= 0 || seq_k <= 0 || head_dim <= 0) return MLE_ERR_ARG;
    if ((softmax_axis != 0 && softmax_axis != 1) || (layout != MLE_ATTN_HEAD_MAJOR && layout != MLE_ATTN_TOKEN_MAJOR))
        return MLE_ERR_ARG;
    if (key_grad_mode != MLE_KEYGRAD_REFERENCE && key_grad_mode != MLE_KEYGRAD_TRUE) return MLE_ERR_ARG;
    cudaStream_t st = as_stream(stream);
    // every check of the tensor-core path precedes its first write, so a
    // refusal (MLE_ERR_UNSUPPORTED) leaves the gradients untouched
    if (workspace &&
        tc_attention_ok(softmax_axis, seq_q, seq_k, head_dim, (int64_t)batch * heads, true, key_grad_mode) &&
        ptrs_aligned({Q, K, V, P, dO, dQ, dK, dV, workspace})) {
        const int s = tc_attention_bwd(Q, K, V, P, dO, dQ, dK, dV, dP_out, dS_out, workspace, batch, heads, seq_q,
                                       seq_k, head_dim, scale, key_grad_mode, layout, st, assign_mask);
        if (s != MLE_ERR_UNSUPPORTED) return s;
    }
    // the other paths accumulate: assigned gradients start cleared
    const size_t nq = sizeof(float) * (size_t)batch * heads * seq_q * head_dim;
    const size_t nk = sizeof(float) * (size_t)batch * heads * seq_k * head_dim;
    if (((assign_mask & 1) && cudaMemsetAsync(dQ, 0, nq, st) != cudaSuccess) ||
        ((assign_mask & 2) && cudaMemsetAsync(dK, 0, nk, st) != cudaSuccess) ||
        ((assign_mask & 4) && cudaMemsetAsync(dV, 0, nk, st) != cudaSuccess))
        return launch_status();
    const bool ref_shape_ok = key_grad_mode == MLE_KEYGRAD_TRUE || seq_q == seq_k;
    if (fused_ok(softmax_axis, seq_q, seq_k, head_dim, batch, heads) && ref_shape_ok &&
        ptrs_aligned({Q, K, V, dO, dQ, dK, dV})) {
        if (!workspace) return MLE_ERR_ARG;
        AttnArgs a{};
        a.Q = Q;
        a.K = K;
        a.V = V;
        a.P = P;
        a.dO = dO;
        a.dQ = dQ;
        a.dK = dK;
        a.dV = dV;
        a.dPout = dP_out;
        a.dSout = dS_out;
        a.dScores = workspace;
        a.B = batch;
        a.H = heads;
        a.Sq = seq_q;
        a.Sk = seq_k;
        a.scale = scale;
        a.key_mode = key_grad_mode;
        strides_for(layout, heads, seq_q, head_dim, a.qb, a.qh, a.qs);
        strides_for(layout, heads, seq_k, head_dim, a.kb, a.kh, a.ks);
        const int s = dispatch_hd(head_dim, [&](auto hd) { return launch_bwd<decltype(hd)::value>(a, st); });
        if (s != MLE_ERR_UNSUPPORTED) return s;
    }
    // composed path: head-major operands and explicit score gradients
    if (layout != MLE_ATTN_HEAD_MAJOR || !dP_out || !dS_out) return MLE_ERR_UNSUPPORTED;
    int s;
    // dP[Sq,Sk] += dO[Sq,hd] * V[Sk,hd]^T
    s = mle_bcmm(MLE_GEMM_ABT, dO, V, dP_out, batch, heads, seq_q, head_dim, seq_k, 1, 3, 3, 3, 1.0f, stream);
    if (s) return s;
    // dV[Sk,hd] += P[Sq,Sk]^T * dO[Sq,hd]
    s = mle_bcmm(MLE_GEMM_ATB, P, dO, dV, batch, heads, seq_k, seq_q, head_dim, 1, 3, 3, 3, 1.0f, stream);
    if (s) return s;
    s = mle_softmax_bwd(P, dP_out, dS_out, (int64_t)batch * heads, seq_q, seq_k, softmax_axis, stream);
    if (s) return s;
    // dQ[Sq,hd] += scale * dS[Sq,Sk] * K[Sk,hd]
    s = mle_bcmm(MLE_GEMM_AB, dS_out, K, dQ, batch, heads, seq_q, seq_k, head_dim, 1, 3, 3, 3, scale, stream);
    if (s) return s;
    if (key_grad_mode == MLE_KEYGRAD_TRUE)  // dK[Sk,hd] += scale * dS[Sq,Sk]^T * Q[Sq,hd]
        return mle_bcmm(MLE_GEMM_ATB, dS_out, Q, dK, batch, heads, seq_k, seq_q, head_dim, 1, 3, 3, 3, scale, stream);
    // the reference's call: bcmmT(A=Q, B=dScores, C=K.grad, m=hd, n=Sq, p=Sk)
    return mle_bcmm(MLE_GEMM_ATBT, Q, dS_out, dK, batch, heads, head_dim, seq_q, seq_k, 1, 3, 3, 3, scale, stream);
}

}  // extern "C"
