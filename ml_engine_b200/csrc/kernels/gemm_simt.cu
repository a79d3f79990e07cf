// CUDA-core GEMM for the shapes the TMA path cannot describe: row strides
// that are not a multiple of 16 bytes, unaligned bases, or tiny N/M such as
// the 10-way classifier of the MNIST MLP.  64x64 output tile per 256-thread
// block, 4x4 outputs per thread, k-slices of 16 staged in shared memory;
// products of at most 8 rows take one warp per output instead.
// Operand access follows the same GemmProblem description as the tensor-core
// path (transposes, batch/channel strides, assign / += / atomic epilogue).
#include <stdint.h>

#include "gemm.cuh"

namespace mle {

namespace {

constexpr int TM = 64, TN = 64, TK = 16;

__global__ void __launch_bounds__(256) simt_gemm_kernel(const GemmProblem p) {
    pdl_entry();
    __shared__ float As[TK][TM + 4];
    __shared__ float Bs[TK][TN + 4];
    const int z = blockIdx.z;
    const int cidx = z % p.channels, bidx = z / p.channels;
    const float* A = p.A + (int64_t)bidx * p.a_sb + (int64_t)cidx * p.a_sc;
    const float* B = p.B + (int64_t)bidx * p.b_sb + (int64_t)cidx * p.b_sc;
    float* C = p.C + (int64_t)bidx * p.c_sb + (int64_t)cidx * p.c_sc;
    const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

    for (int k0 = 0; k0 < p.K; k0 += TK) {
        // 64x16 A slice and 16x64 B slice, 4 elements per thread each
        for (int e = threadIdx.x; e < TM * TK; e += 256) {
            int mm, kk;
            if (p.trans_a) { kk = e / TM; mm = e % TM; } else { mm = e / TK; kk = e % TK; }
            const int gm = m0 + mm, gk = k0 + kk;
            float v = 0.f;
            if (gm < p.M && gk < p.K) v = p.trans_a ? A[(int64_t)gk * p.lda + gm] : A[(int64_t)gm * p.lda + gk];
            As[kk][mm] = v;
        }
        for (int e = threadIdx.x; e < TN * TK; e += 256) {
            int nn, kk;
            if (p.trans_b) { nn = e / TK; kk = e % TK; } else { kk = e / TN; nn = e % TN; }
            const int gn = n0 + nn, gk = k0 + kk;
            float v = 0.f;
            if (gn < p.N && gk < p.K) v = p.trans_b ? B[(int64_t)gn * p.ldb + gk] : B[(int64_t)gk * p.ldb + gn];
            Bs[kk][nn] = v;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < TK; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] += a[i] * b[j];
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int gm = m0 + ty * 4 + i;
        if (gm >= p.M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int gn = n0 + tx * 4 + j;
            if (gn >= p.N) continue;
            float v = p.alpha * acc[i][j];
            if (p.bias) v += p.bias[gn];
            float* dst = C + (int64_t)gm * p.ldc + gn;
            if (p.mode == 0) *dst = v;
            else if (p.mode == 1) *dst += v;
            else atomicAdd(dst, v);
        }
    }
}

// Products with at most kSkinnyM rows (a [1, in] time embedding through a
// Linear layer): one warp per output element, the lanes striding over k
// and meeting in a butterfly sum.  blockIdx.z indexes (batch, channel).
constexpr int kSkinnyM = 8;

__global__ void __launch_bounds__(256) skinny_gemm_kernel(const GemmProblem p) {
    pdl_entry();
    const int z = blockIdx.z;
    const int cidx = z % p.channels, bidx = z / p.channels;
    const float* A = p.A + (int64_t)bidx * p.a_sb + (int64_t)cidx * p.a_sc;
    const float* B = p.B + (int64_t)bidx * p.b_sb + (int64_t)cidx * p.b_sc;
    float* C = p.C + (int64_t)bidx * p.c_sb + (int64_t)cidx * p.c_sc;
    const int lane = threadIdx.x & 31;
    const int64_t out = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (out >= (int64_t)p.M * p.N) return;
    const int m = (int)(out / p.N), n = (int)(out - (int64_t)m * p.N);
    float acc = 0.f;
    for (int k = lane; k < p.K; k += 32) {
        const float a = p.trans_a ? A[(int64_t)k * p.lda + m] : A[(int64_t)m * p.lda + k];
        const float b = p.trans_b ? B[(int64_t)n * p.ldb + k] : B[(int64_t)k * p.ldb + n];
        acc += a * b;
    }
    acc = warp_sum(acc);
    if (lane == 0) {
        float v = p.alpha * acc;
        if (p.bias) v += p.bias[n];
        float* dst = C + (int64_t)m * p.ldc + n;
        if (p.mode == 0) *dst = v;
        else if (p.mode == 1) *dst += v;
        else atomicAdd(dst, v);
    }
}

}  // namespace

int simt_gemm(const GemmProblem& p, cudaStream_t st) {
    const int64_t z = (int64_t)p.nbatch * p.channels;
    if (z > 65535) return MLE_ERR_UNSUPPORTED;
    if (p.M <= kSkinnyM) {
        const int64_t blocks = ((int64_t)p.M * p.N + 7) / 8;
        if (blocks > INT32_MAX) return MLE_ERR_UNSUPPORTED;
        launch_k(skinny_gemm_kernel, dim3((unsigned)blocks, 1, (unsigned)z), 256, 0, st, p);
        return launch_status();
    }
    dim3 grid((p.N + TN - 1) / TN, (p.M + TM - 1) / TM, (unsigned)z);
    if (grid.y > 65535) return MLE_ERR_UNSUPPORTED;
    launch_k(simt_gemm_kernel, grid, 256, 0, st, p);
    return launch_status();
}

}  // namespace mle
