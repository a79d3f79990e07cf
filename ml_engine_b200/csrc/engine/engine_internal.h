// Internal plumbing shared by the runtime translation units.
#pragma once

#include <vector>

#include "engine.h"

namespace mle {

void* st();                                    // compute stream as mle_stream_t
void check_cuda(cudaError_t e, const str& what);

// Parameters touched by per-node lambdas while one fused launch is built.
struct ParamUpdate {
    AdamParameter* p;
    float lr;
    bool adamw;
};
struct ParamCollector {
    std::vector<ParamUpdate> update;
    std::vector<AdamParameter*> sumsq;
    std::vector<AdamParameter*> clip;
};
extern ParamCollector* g_collector;

// SoftMaxCrossEntropy keeps its probabilities for a later forward without
// calc_loss (the reference's softmax buffer); a session that always
// computes the loss switches this off to save one tensor write per step.
extern bool g_keep_softmax;
// Loss nodes copy their value into GraphOperations::loss (a device sync)
// when last, as the reference does; sessions read the loss themselves.
extern bool g_loss_readback;
void set_keep_softmax(bool keep);

// Op tags used by the fusion pass.
enum OpKind {
    OP_GENERIC = 0,
    OP_LINEAR = 1,
    OP_ACTIVATION = 2,
    OP_SMCE = 3,
    OP_ATTENTION = 4,  // ScaledDotAttention on the token-major kernels
    OP_ADD = 5,
    OP_CONV = 6,       // Convolute2D
    OP_LAYERNORM = 7,
};

// Per-node fusion state decided by prepare_fusions() before a backward pass.
struct NodeExt {
    int kind = OP_GENERIC;
    float* linear_bias_grad = nullptr;   // Linear with bias: B1.grad
    bool bias_grad_fused = false;        // Linear: the consumer adds the bias grad
    float* fused_bias_target = nullptr;  // activation: bias grad to accumulate
    long long fused_rows = 0, fused_cols = 0;
    std::vector<float*> param_grads;     // parameter gradients complete once this node's backward ran
    int assign_inputs = 0;               // bit i: backward writes (not adds to) inputs[i]'s gradient
    // forward: an Add whose sum feeds a LayerNorm computes both in one pass
    const NodeBackProp* fused_norm = nullptr;  // Add: the LayerNorm it also produces
    bool add_is_loss = false;                  // Add: the loss sum (read back; not fused)
    bool norm_done = false;                    // LayerNorm: its Add wrote its output this forward
    float* ln_mean = nullptr;                  // LayerNorm: its statistics buffers and shape
    float* ln_sq = nullptr;
    int ln_dims[4] = {0, 0, 0, 0};
    float ln_eps = 0.0f;
    // MatrixPositionalEncoding: its table; output written by the gather
    // that feeds it (pe_fed), its forward then idle
    const float* pe_table = nullptr;
    bool pe_fed = false;
    bool grad_unused = false;  // nothing reads this node's gradient (a frozen input)
};
NodeExt& ext(const NodeBackProp* n);
void forget_ext(const NodeBackProp* n);
void node_born(const NodeBackProp* n);

// Decides the Linear -> activation bias-gradient fusion for a node list:
// an activation whose input is a biased Linear output consumed by nothing
// else adds that Linear's BCompress (column sums) to its own backward pass.
// Also finds gradients whose first writer in the backward walk (the
// consumer last in topological order) overwrites the whole buffer: a
// loss node, an activation, an Add, the token-major attention, a
// Convolute2D, or a Linear with a large input gradient.  That writer assigns (assign_inputs) and
// zero_grad leaves the buffer alone.
void prepare_fusions(const graph_tree& nodes);

// Whether forward fuses a residual Add with the LayerNorm that reads it
// (mle_set_add_norm_fusion).
bool add_norm_fusion();

// Base of the arena chunk (one device allocation) holding p, or nullptr.
const void* arena_chunk_of(const void* p);

// Gradient buffers zero_range skips (their first writer assigns them).
void set_preassigned_grads(const std::vector<const float*>& grads);
bool grad_preassigned(const float* grad);

}  // namespace mle
