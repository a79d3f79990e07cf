// Problem description shared by the tensor-core GEMM and its CUDA-core
// fallback.
#pragma once

#include "common.cuh"

namespace mle {

struct GemmProblem {
    const float* A;
    const float* B;
    float* C;
    const float* bias;
    int M, N, K;
    int64_t lda, ldb, ldc;
    int trans_a, trans_b;  // A stored [K][M]; B stored [N][K]
    // batch decomposition z = b * channels + c
    int nbatch, channels;
    int64_t a_sb, a_sc, b_sb, b_sc, c_sb, c_sc;  // element strides, 0 = broadcast
    float alpha;
    int mode;  // 0 assign, 1 +=, 2 atomic add
    // > 0: C's column n lives at (n % c_split) + (n / c_split) * c_split_ld
    // (tensor-core path only; c_split a multiple of 32 dividing N)
    int c_split = 0;
    int64_t c_split_ld = 0;
    // non-null: also colsum[n] += sum_k B[k][n] (B stored [K][N] with
    // ldb == N, one product).  The tensor-core path sums B's tiles in shared
    // memory while they pass through (a Linear's bias gradient beside its
    // weight gradient); where it cannot, a column-sum launch follows.
    float* colsum = nullptr;
};

// Implicit-GEMM convolution at stride 1 over KW horizontally shifted
// copies of an image, S[kw][n][c][y][x] = src[n][c][y][x + kw + shift]
// (0 outside), so that every tap's operand tile is a TMA box of S, whose
// image planes are addressed flattened: the tap moves the pixel index by
// (kh - pad) whole rows, a multiple of 4 elements when WS % 4 == 0, and rows
// above or below the image read as 0:
//   kind 1: C[n][m][p] (= or +=) sum over taps t = (kh, kw) and channels c
//           of A[t][m][c] * S[kw][n][c][oy + kh - pad][ox],  p = oy*WS + ox
//   kind 2: C[t][m][c] += sum over images n and pixels p of
//           A[n][m][p] * S[kw][n][c][oy + kh - pad][ox]
struct ConvGemm {
    int kind;
    const float* A;  // kind 1: [KH*KW][M][lda]; kind 2: [nb][M][P]
    const float* S;  // [KW][nb][C][HS][WS]
    float* out;      // kind 1: [nb][M][P]; kind 2: [KH*KW][M][ldc]
    int M, C, HS, WS, KH, KW, pad, nb;
    int P;           // pixels per image of the output (kind 1) / of A (kind 2)
    int64_t lda, ldc;
    int accumulate;  // kind 1 only (kind 2 always adds)
    const float* bias;  // kind 1 only: added per output channel m (assigned output)
};

// Attention scores with the column softmax on the tensor cores (keys on
// the TMEM lanes, one CTA per batch, head and 128 keys; gemm_tcgen05.cu).
// Operands are (hd, S, H, B) views with element strides (s, h, b) per
// row, head and batch.  mode 0: out = column softmax of scale * Q K^T
// (keys_src = K, rows_src = Q); mode 1: out = P (dP - column sums of P dP)
// with dP = dO V^T (keys_src = V, rows_src = dO).  P and out are
// [B, H, Sq, Sk]; mode 0 may leave out null and write only `stats` (column
// max [B*H*Sk], then inverse column sum [B*H*Sk]).  MLE_ERR_UNSUPPORTED
// (nothing launched) outside Sq <= 256, hd in {32, 64, 128}.
bool attn_keys_supported(int Sq, int Sk, int hd, int64_t BH);
int run_attn_keys(int mode, const float* keys_src, const float* rows_src, const float* P, float* out, int B, int H,
                  int Sq, int Sk, int hd, int64_t key_b, int64_t key_h, int64_t key_s, int64_t row_b, int64_t row_h,
                  int64_t row_s, float scale, int causal, cudaStream_t st, float* stats = nullptr);

// Attention with the column softmax without the score matrices in HBM
// (gemm_tcgen05.cu): the forward writes O and per-key statistics (column
// max, inverse column sum: stats[2 * B*H*Sk]); the backward recomputes the
// probabilities from them and writes dQ, dK, dV (dvec: B*H*Sk floats of
// workspace holding sum_q P dP per key).  Operand and output strides as for
// run_attn_keys; `assign` bit 0 dQ, bit 1 dK, bit 2 dV written rather than
// accumulated.  MLE_ERR_UNSUPPORTED outside Sq <= 256, Sk <= 512,
// hd in {32, 64} (and Sq == Sk, Sk % hd == 0 for the reference key gradient).
bool attn_flash_supported(int Sq, int Sk, int hd, int64_t BH, int key_mode);
int run_attn_flash_fwd(const float* Q, const float* K, const float* V, float* O, float* stats, int B, int H, int Sq,
                       int Sk, int hd, int64_t qb, int64_t qh, int64_t qs, int64_t kb, int64_t kh, int64_t ks,
                       float scale, int causal, cudaStream_t st);
int run_attn_flash_bwd(const float* Q, const float* K, const float* V, const float* dO, const float* stats,
                       float* dvec, float* dQ, float* dK, float* dV, int B, int H, int Sq, int Sk, int hd, int64_t qb,
                       int64_t qh, int64_t qs, int64_t kb, int64_t kh, int64_t ks, float scale, int causal,
                       int key_mode, int assign, cudaStream_t st);

int simt_gemm(const GemmProblem& p, cudaStream_t st);
// false when the shapes or pointers rule out the tensor-core implicit path
bool conv_gemm_supported(const ConvGemm& c);
int run_conv_gemm(const ConvGemm& c, cudaStream_t st);
int run_gemm(const GemmProblem& p, cudaStream_t st);
int run_gemm_group(const GemmProblem* ps, int n, bool shared_c, cudaStream_t st);
// C (= or +=) sum_g A_g B_g as one product over the concatenated reduction
// (problems sharing C, M, N, layouts, mode and alpha; unbatched, K_g % 64
// == 0); otherwise the group launch above with C shared.
int run_gemm_kcat(const GemmProblem* ps, int n, cudaStream_t st);

}  // namespace mle
