// Attention sub-graph of MultiHeadAttention (Engine/transformer.cu:647-675):
//   scores = Q K^T, scaled = scale*scores, P = softmax_axis(scaled), O = P V.
//
// Fused path (column-wise softmax, the reference's "type 1", head_dim 16/32/64,
// Sq <= 256): one 256-thread CTA per (batch, head) keeps Q (and dO) in shared
// memory and walks the key axis in blocks of 32 columns.  A column of the
// softmax needs every query row, which the CTA holds, so each key block is
// finished inside the block loop; products that sum over keys (O, dQ and the
// reference's key gradient) accumulate in registers across blocks in key
// order.  Every sum is one FMA chain in the order the reference kernels use
// (bcmm*: k ascending; SumRows / deriv_softmax: rows ascending), so P, O and
// the gradients are bitwise those of the reference's kernel chain.  Q, K, V,
// O and the gradients are read and written token-major ([B, S, H*hd], the
// Linear layout) or head-major through strides, so no head copies are made.
//
// Other shapes run the composed path on the tensor-core GEMM (head-major).
#include <float.h>

#include <type_traits>

#include "common.cuh"

namespace mle {
namespace {

constexpr int kNT = 256;  // threads per CTA
constexpr int kTC = 32;   // key columns per block

struct AttnArgs {
    const float *Q, *K, *V, *P, *dO;
    float *Pout, *O, *dQ, *dK, *dV, *dPout, *dSout;
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

template <int HD>
__device__ __forceinline__ void load_rows(float* dst, const float* __restrict__ src, int rows, int64_t rs) {
    for (int i = threadIdx.x; i < rows * HD; i += kNT) {
        const int r = i / HD, d = i % HD;
        dst[r * (HD + 1) + d] = src[(int64_t)r * rs + d];
    }
}

// ------------------------------------------------------------------ forward
template <int HD>
__global__ void __launch_bounds__(kNT) attn_fwd_col_kernel(const AttnArgs a) {
    extern __shared__ float sm[];
    const int Sq = a.Sq, Sk = a.Sk;
    float* Qs = sm;                        // [Sq][HD+1]
    float* Ks = Qs + Sq * (HD + 1);        // [TC][HD+1]
    float* Vs = Ks + kTC * (HD + 1);       // [TC][HD+1]
    float* Ss = Vs + kTC * (HD + 1);       // [Sq][TC+1]
    float* csum = Ss + Sq * (kTC + 1);     // [TC]
    const int b = blockIdx.x / a.H, h = blockIdx.x % a.H, t = threadIdx.x;
    const float* Qg = a.Q + b * a.qb + h * a.qh;
    const float* Kg = a.K + b * a.kb + h * a.kh;
    const float* Vg = a.V + b * a.kb + h * a.kh;
    float* Pg = a.Pout + ((int64_t)b * a.H + h) * Sq * Sk;
    float* Og = a.O + b * a.qb + h * a.qh;
    load_rows<HD>(Qs, Qg, Sq, a.qs);

    // O accumulators: thread owns column d and rows r0, r0 + kNT/HD, ...
    constexpr int RSTEP = kNT / HD;
    constexpr int MAXJ = 256 / RSTEP;
    const int d = t % HD, r0 = t / HD;
    float acc[MAXJ];
#pragma unroll
    for (int j = 0; j < MAXJ; ++j) acc[j] = 0.f;

    for (int c0 = 0; c0 < Sk; c0 += kTC) {
        const int tc = min(kTC, Sk - c0);
        __syncthreads();
        for (int i = t; i < kTC * HD; i += kNT) {
            const int c = i / HD, dd = i % HD;
            const bool in = c < tc;
            Ks[c * (HD + 1) + dd] = in ? Kg[(int64_t)(c0 + c) * a.ks + dd] : 0.f;
            Vs[c * (HD + 1) + dd] = in ? Vg[(int64_t)(c0 + c) * a.ks + dd] : 0.f;
        }
        __syncthreads();
        // scaled scores: one k-ordered FMA chain per entry, then Scale_Write
        for (int i = t; i < Sq * kTC; i += kNT) {
            const int r = i / kTC, c = i % kTC;
            float s = 0.f;
#pragma unroll
            for (int k = 0; k < HD; ++k) s = fmaf(Qs[r * (HD + 1) + k], Ks[c * (HD + 1) + k], s);
            Ss[r * (kTC + 1) + c] = a.scale * s;
        }
        __syncthreads();
        // column softmax: max over every row (masked ones too, as FindMax),
        // exp, rows summed in order (SumRows), all-zero column divided by 1
        if (t < tc) {
            float m = -FLT_MAX;
            for (int r = 0; r < Sq; ++r) m = fmaxf(m, Ss[r * (kTC + 1) + t]);
            float s = 0.f;
            for (int r = 0; r < Sq; ++r) {
                const float e = (a.causal && c0 + t > r) ? 0.0f : expf(Ss[r * (kTC + 1) + t] - m);
                Ss[r * (kTC + 1) + t] = e;
                s += e;
            }
            if (s < 1e-45f) s = 1.0f;
            csum[t] = s;
        }
        __syncthreads();
        for (int i = t; i < Sq * kTC; i += kNT) {
            const int r = i / kTC, c = i % kTC;
            if (c < tc) {
                const float p = Ss[r * (kTC + 1) + c] / csum[c];
                Ss[r * (kTC + 1) + c] = p;
                Pg[(int64_t)r * Sk + c0 + c] = p;
            } else {
                Ss[r * (kTC + 1) + c] = 0.f;
            }
        }
        __syncthreads();
        // O += P_blk V_blk, keys in order
#pragma unroll
        for (int j = 0; j < MAXJ; ++j) {
            const int r = r0 + j * RSTEP;
            if (r < Sq) {
                float o = acc[j];
                for (int c = 0; c < tc; ++c) o = fmaf(Ss[r * (kTC + 1) + c], Vs[c * (HD + 1) + d], o);
                acc[j] = o;
            }
        }
    }
#pragma unroll
    for (int j = 0; j < MAXJ; ++j) {
        const int r = r0 + j * RSTEP;
        if (r < Sq) Og[(int64_t)r * a.qs + d] = acc[j];
    }
}

// ----------------------------------------------------------------- backward
template <int HD>
__global__ void __launch_bounds__(kNT) attn_bwd_col_kernel(const AttnArgs a) {
    extern __shared__ float sm[];
    const int Sq = a.Sq, Sk = a.Sk;
    float* Qs = sm;                        // [Sq][HD+1]
    float* dOs = Qs + Sq * (HD + 1);       // [Sq][HD+1]
    float* Ks = dOs + Sq * (HD + 1);       // [TC][HD+1]
    float* Vs = Ks + kTC * (HD + 1);       // [TC][HD+1]
    float* Ps = Vs + kTC * (HD + 1);       // [Sq][TC+1]
    float* Ds = Ps + Sq * (kTC + 1);       // [Sq][TC+1]  dP, then dScores
    float* dot = Ds + Sq * (kTC + 1);      // [TC]
    const int b = blockIdx.x / a.H, h = blockIdx.x % a.H, t = threadIdx.x;
    const int64_t qoff = b * a.qb + h * a.qh, koff = b * a.kb + h * a.kh;
    const float* Pg = a.P + ((int64_t)b * a.H + h) * Sq * Sk;
    const int64_t soff = ((int64_t)b * a.H + h) * Sq * Sk;
    load_rows<HD>(Qs, a.Q + qoff, Sq, a.qs);
    load_rows<HD>(dOs, a.dO + qoff, Sq, a.qs);

    constexpr int RSTEP = kNT / HD;
    constexpr int MAXJ = 256 / RSTEP;
    const int d = t % HD, r0 = t / HD;
    float accq[MAXJ], acck[MAXJ];
#pragma unroll
    for (int j = 0; j < MAXJ; ++j) accq[j] = acck[j] = 0.f;
    const double dscale = (double)a.scale;

    for (int c0 = 0; c0 < Sk; c0 += kTC) {
        const int tc = min(kTC, Sk - c0);
        __syncthreads();
        for (int i = t; i < kTC * HD; i += kNT) {
            const int c = i / HD, dd = i % HD;
            const bool in = c < tc;
            Ks[c * (HD + 1) + dd] = in ? a.K[koff + (int64_t)(c0 + c) * a.ks + dd] : 0.f;
            Vs[c * (HD + 1) + dd] = in ? a.V[koff + (int64_t)(c0 + c) * a.ks + dd] : 0.f;
        }
        for (int i = t; i < Sq * kTC; i += kNT) {
            const int r = i / kTC, c = i % kTC;
            Ps[r * (kTC + 1) + c] = (c < tc) ? Pg[(int64_t)r * Sk + c0 + c] : 0.f;
        }
        __syncthreads();
        // dP = dO V^T (bcmmABT: k = head_dim ascending)
        for (int i = t; i < Sq * kTC; i += kNT) {
            const int r = i / kTC, c = i % kTC;
            float s = 0.f;
#pragma unroll
            for (int k = 0; k < HD; ++k) s = fmaf(dOs[r * (HD + 1) + k], Vs[c * (HD + 1) + k], s);
            Ds[r * (kTC + 1) + c] = s;
            if (a.dPout && c < tc) a.dPout[soff + (int64_t)r * Sk + c0 + c] += s;
        }
        __syncthreads();
        // deriv_softmax type 1: per column dot over rows in order
        if (t < tc) {
            float s = 0.f;
            for (int r = 0; r < Sq; ++r) s = fmaf(Ds[r * (kTC + 1) + t], Ps[r * (kTC + 1) + t], s);
            dot[t] = s;
        }
        __syncthreads();
        // dScaled = P (dP - dot); dScores = (float)(scale * dScaled) as Accumulate
        for (int i = t; i < Sq * kTC; i += kNT) {
            const int r = i / kTC, c = i % kTC;
            if (c < tc) {
                const float ds = Ps[r * (kTC + 1) + c] * (Ds[r * (kTC + 1) + c] - dot[c]);
                if (a.dSout) a.dSout[soff + (int64_t)r * Sk + c0 + c] += ds;
                Ds[r * (kTC + 1) + c] = (float)(0.0 + dscale * (double)ds);
            } else {
                Ds[r * (kTC + 1) + c] = 0.f;
            }
        }
        __syncthreads();
        // per-key products of this block: dV = P^T dO, true dK = dS^T Q
        // (bcmmATB: k = query row ascending)
        for (int i = t; i < tc * HD; i += kNT) {
            const int c = i / HD, dd = i % HD;
            float sv = 0.f;
            for (int r = 0; r < Sq; ++r) sv = fmaf(Ps[r * (kTC + 1) + c], dOs[r * (HD + 1) + dd], sv);
            a.dV[koff + (int64_t)(c0 + c) * a.ks + dd] += sv;
            if (a.key_mode == MLE_KEYGRAD_TRUE) {
                float sk = 0.f;
                for (int r = 0; r < Sq; ++r) sk = fmaf(Ds[r * (kTC + 1) + c], Qs[r * (HD + 1) + dd], sk);
                a.dK[koff + (int64_t)(c0 + c) * a.ks + dd] += sk;
            }
        }
        // sums over keys, continued across blocks in key order:
        //   dQ = dScores K (bcmm), reference key gradient (dScores Q) of bcmmT
#pragma unroll
        for (int j = 0; j < MAXJ; ++j) {
            const int r = r0 + j * RSTEP;
            if (r < Sq) {
                float q = accq[j], kr = acck[j];
                for (int c = 0; c < tc; ++c) {
                    const float ds = Ds[r * (kTC + 1) + c];
                    q = fmaf(ds, Ks[c * (HD + 1) + d], q);
                    if (a.key_mode == MLE_KEYGRAD_REFERENCE) kr = fmaf(ds, Qs[(c0 + c) * (HD + 1) + d], kr);
                }
                accq[j] = q;
                acck[j] = kr;
            }
        }
    }
#pragma unroll
    for (int j = 0; j < MAXJ; ++j) {
        const int r = r0 + j * RSTEP;
        if (r < Sq) {
            a.dQ[qoff + (int64_t)r * a.qs + d] += accq[j];
            if (a.key_mode == MLE_KEYGRAD_REFERENCE) {
                // bcmmT(Q, dScores, Kh.grad, hd, Sq, Sk) writes element
                // (row d, col r) of its [hd, Sk] result at d*Sk + r of the
                // head's [Sk, hd] gradient block (Sq == Sk here)
                const int pos = d * Sk + r;
                a.dK[koff + (int64_t)(pos / HD) * a.ks + pos % HD] += acck[j];
            }
        }
    }
}

template <int HD>
size_t fwd_smem(int Sq) {
    return sizeof(float) * ((size_t)Sq * (HD + 1) + 2 * kTC * (HD + 1) + (size_t)Sq * (kTC + 1) + kTC);
}
template <int HD>
size_t bwd_smem(int Sq) {
    return sizeof(float) * (2 * (size_t)Sq * (HD + 1) + 2 * kTC * (HD + 1) + 2 * (size_t)Sq * (kTC + 1) + kTC);
}

constexpr size_t kMaxSmem = 227 * 1024;

template <int HD>
int launch_fwd(const AttnArgs& a, cudaStream_t st) {
    const size_t smem = fwd_smem<HD>(a.Sq);
    if (smem > kMaxSmem) return MLE_ERR_UNSUPPORTED;
    static bool cfg = false;
    if (!cfg) {
        if (cudaFuncSetAttribute(attn_fwd_col_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem) !=
            cudaSuccess)
            return launch_status();
        cfg = true;
    }
    attn_fwd_col_kernel<HD><<<a.B * a.H, kNT, smem, st>>>(a);
    return launch_status();
}

template <int HD>
int launch_bwd(const AttnArgs& a, cudaStream_t st) {
    const size_t smem = bwd_smem<HD>(a.Sq);
    if (smem > kMaxSmem) return MLE_ERR_UNSUPPORTED;
    static bool cfg = false;
    if (!cfg) {
        if (cudaFuncSetAttribute(attn_bwd_col_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem) !=
            cudaSuccess)
            return launch_status();
        cfg = true;
    }
    attn_bwd_col_kernel<HD><<<a.B * a.H, kNT, smem, st>>>(a);
    return launch_status();
}

bool fused_ok(int axis, int Sq, int hd, int B, int H) {
    return axis == 1 && Sq >= 1 && Sq <= 256 && (hd == 16 || hd == 32 || hd == 64) && (int64_t)B * H < (1ll << 31);
}

template <typename F>
int dispatch_hd(int hd, F&& f) {
    switch (hd) {
        case 16: return f(std::integral_constant<int, 16>());
        case 32: return f(std::integral_constant<int, 32>());
        default: return f(std::integral_constant<int, 64>());
    }
}

}  // namespace
}  // namespace mle

using namespace mle;

extern "C" {

int mle_attention_fused_supported(int seq_q, int seq_k, int head_dim, int softmax_axis, int key_grad_mode) {
    if (seq_k <= 0 || !fused_ok(softmax_axis, seq_q, head_dim, 1, 1)) return 0;
    if (key_grad_mode == MLE_KEYGRAD_REFERENCE && seq_q != seq_k) return 0;
    const size_t smem = head_dim == 16 ? bwd_smem<16>(seq_q) : head_dim == 32 ? bwd_smem<32>(seq_q) : bwd_smem<64>(seq_q);
    return smem <= kMaxSmem ? 1 : 0;
}

int mle_attention_fwd(const float* Q, const float* K, const float* V, float* P, float* O, int batch, int heads,
                      int seq_q, int seq_k, int head_dim, float scale, int causal, int softmax_axis, int layout,
                      mle_stream_t stream) {
    if (!Q || !K || !V || !P || !O) return MLE_ERR_ARG;
    if (batch <= 0 || heads <= 0 || seq_q <= 0 || seq_k <= 0 || head_dim <= 0) return MLE_ERR_ARG;
    if ((softmax_axis != 0 && softmax_axis != 1) || (layout != MLE_ATTN_HEAD_MAJOR && layout != MLE_ATTN_TOKEN_MAJOR))
        return MLE_ERR_ARG;
    cudaStream_t st = as_stream(stream);
    if (fused_ok(softmax_axis, seq_q, head_dim, batch, heads)) {
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
                      float* dK, float* dV, float* dP_out, float* dS_out, int batch, int heads, int seq_q, int seq_k,
                      int head_dim, float scale, int causal, int softmax_axis, int key_grad_mode, int layout,
                      mle_stream_t stream) {
    (void)causal;  // P is exactly zero where the mask applied, so dS is too
    if (!Q || !K || !V || !P || !dO || !dQ || !dK || !dV) return MLE_ERR_ARG;
    if (batch <= 0 || heads <= 0 || seq_q <= 0 || seq_k <= 0 || head_dim <= 0) return MLE_ERR_ARG;
    if ((softmax_axis != 0 && softmax_axis != 1) || (layout != MLE_ATTN_HEAD_MAJOR && layout != MLE_ATTN_TOKEN_MAJOR))
        return MLE_ERR_ARG;
    if (key_grad_mode != MLE_KEYGRAD_REFERENCE && key_grad_mode != MLE_KEYGRAD_TRUE) return MLE_ERR_ARG;
    cudaStream_t st = as_stream(stream);
    const bool ref_shape_ok = key_grad_mode == MLE_KEYGRAD_TRUE || seq_q == seq_k;
    if (fused_ok(softmax_axis, seq_q, head_dim, batch, heads) && ref_shape_ok) {
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
