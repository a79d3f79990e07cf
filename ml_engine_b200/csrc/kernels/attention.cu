// Backward of the attention sub-graph that MultiHeadAttention::forward and
// cross_forward build from graph ops (Engine/transformer.cu:647-675):
//   scores = Q K^T, scaled = scale*scores, P = softmax_axis(scaled), O = P V.
// The reference runs it as six launches per head batch (BMM backward: two
// bcmm*; deriv_softmax; Accumulate for Scale; BMMABT backward: two bcmm*).
//
// This entry point runs the chain on the tensor-core GEMM with the scale
// folded into the last two GEMMs' alpha:
//   dP  += dO V^T                     (dP_out, the softmax node's grad)
//   dV  += P^T dO
//   dS  += P o (dP - sum_axis(dP o P)) (dS_out, the Scale node's grad)
//   dQ  += scale * dS K
//   dK  += scale * dS^T Q                  (MLE_KEYGRAD_TRUE)
//   dK  <- bcmmT(Q, scale*dS) semantics     (MLE_KEYGRAD_REFERENCE, the
//          reference's BMMABT backward, Engine/engine.cu:2307)
#include "common.cuh"

extern "C" {

int mle_attention_bwd(const float* Q, const float* K, const float* V, const float* P, const float* dO, float* dQ,
                      float* dK, float* dV, float* dP_out, float* dS_out, int batch, int heads, int seq_q, int seq_k,
                      int head_dim, float scale, int causal, int softmax_axis, int key_grad_mode,
                      mle_stream_t stream) {
    (void)causal;  // P is exactly zero where the mask applied, so dS is too
    if (!Q || !K || !V || !P || !dO || !dQ || !dK || !dV || !dP_out || !dS_out) return MLE_ERR_ARG;
    if (batch <= 0 || heads <= 0 || seq_q <= 0 || seq_k <= 0 || head_dim <= 0) return MLE_ERR_ARG;
    if (softmax_axis != 0 && softmax_axis != 1) return MLE_ERR_ARG;
    if (key_grad_mode != MLE_KEYGRAD_REFERENCE && key_grad_mode != MLE_KEYGRAD_TRUE) return MLE_ERR_ARG;
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
