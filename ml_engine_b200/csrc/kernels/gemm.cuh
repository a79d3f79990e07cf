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
};

int simt_gemm(const GemmProblem& p, cudaStream_t st);
int run_gemm(const GemmProblem& p, cudaStream_t st);
int run_gemm_group(const GemmProblem* ps, int n, bool shared_c, cudaStream_t st);

}  // namespace mle
