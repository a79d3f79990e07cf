// Graph-op builders on the hot path.  Each keeps the reference builder's
// shape checks, allocation (output + grad at build time), and the exact
// forward/backward semantics of its lambdas (cited per builder), while the
// launches go through include/mle_kernels.h on mle::stream().
//
// Lambdas capture raw node pointers: a node is owned by whoever holds the
// graph (its consumers' `inputs`), and capturing the node's own shared_ptr
// inside its lambdas would keep it alive forever.
#include <math.h>
#include <stdio.h>

#include <unordered_map>
#include <unordered_set>

#include "engine.h"
#include "engine_internal.h"

using namespace mle;

namespace mle {

// Keyed by node address: a node drops its entry when it is constructed and
// destroyed, so a later node at a recycled address starts from defaults.
// Never destroyed, so nodes outliving static destruction can still erase.
static std::unordered_map<const NodeBackProp*, NodeExt>& ext_map() {
    static auto* m = new std::unordered_map<const NodeBackProp*, NodeExt>();
    return *m;
}
NodeExt& ext(const NodeBackProp* n) { return ext_map()[n]; }

// Every live node, so that a plan can see consumers outside its own graph.
static std::unordered_set<const NodeBackProp*>& live_nodes() {
    static auto* s = new std::unordered_set<const NodeBackProp*>();
    return *s;
}
void node_born(const NodeBackProp* n) {
    ext_map().erase(n);
    live_nodes().insert(n);
}
void forget_ext(const NodeBackProp* n) {
    ext_map().erase(n);
    live_nodes().erase(n);
}

void prepare_fusions(const graph_tree& nodes) {
    std::unordered_map<const NodeBackProp*, int> consumers;
    // the consumer of each node that runs first in the backward walk
    std::unordered_map<const NodeBackProp*, const NodeBackProp*> first_writer;
    for (auto& n : nodes)
        for (auto& in : n->inputs) {
            consumers[in.get()]++;
            first_writer[in.get()] = n.get();
        }
    // consumers anywhere: a node that another graph also reads may have its
    // gradient written by that graph's backward between this graph's
    // zero_grad and its first writer, so it is cleared and accumulated
    std::unordered_map<const NodeBackProp*, int> all_consumers;
    for (const NodeBackProp* n : live_nodes())
        for (auto& in : n->inputs) all_consumers[in.get()]++;
    for (auto& n : nodes) {
        NodeExt& e = ext(n.get());
        if (e.kind == OP_LINEAR) e.bias_grad_fused = false;
        if (e.kind == OP_ACTIVATION) e.fused_bias_target = nullptr;
        e.assign_inputs = 0;
        e.fused_norm = nullptr;
        e.norm_done = false;
    }
    // a residual Add whose sum a LayerNorm reads writes the norm's output in
    // the same pass (the norm's forward then has nothing left to do)
    if (add_norm_fusion()) {
        for (auto& n : nodes) {
            const NodeExt& le = ext(n.get());
            if (le.kind != OP_LAYERNORM || n->inputs.size() != 1) continue;
            const NodeBackProp* a = n->inputs[0].get();
            NodeExt& ae = ext(a);
            if (ae.kind != OP_ADD || ae.add_is_loss || ae.fused_norm) continue;
            ae.fused_norm = n.get();
        }
    }
    // first writers that overwrite the whole input gradient: the loss
    // (SoftMaxCrossEntropy assigns its prediction's gradient), an
    // activation, an Add, the token-major attention (dQ, dK, dV), a
    // Convolute2D (its input gradient), and a Linear whose input gradient
    // spans at least two waves of 128 x 128
    // tiles (its product then never splits K, so the assigned GEMM costs no
    // memset of its own).  The input must appear once among the writer's
    // inputs.
    std::vector<const float*> pre;
    if (first_write_assign()) {
        for (auto& n : nodes) {
            const NodeBackProp* x = n.get();
            auto it = first_writer.find(x);
            if (it == first_writer.end() || !x->grad) continue;
            if (all_consumers[x] != consumers[x]) continue;  // shared with another graph
            const NodeBackProp* w = it->second;
            NodeExt& we = ext(w);
            int pos = -1, seen = 0;
            for (size_t i = 0; i < w->inputs.size(); ++i)
                if (w->inputs[i].get() == x) {
                    pos = (int)i;
                    ++seen;
                }
            if (seen != 1) continue;
            bool ok = false;
            if (we.kind == OP_SMCE) ok = pos == 0;  // {prediction, target} or {prediction} (index labels)
            if (we.kind == OP_ACTIVATION) ok = pos == 0;
            if (we.kind == OP_ADD) ok = pos <= 1;
            if (we.kind == OP_ATTENTION) ok = pos <= 2;
            if (we.kind == OP_CONV) ok = pos == 0;
            if (we.kind == OP_LINEAR) ok = pos == 0 && (double)x->total >= 2.0 * 148 * 128.0 * 128.0;  // 148 SMs
            if (!ok) continue;
            if (we.kind != OP_SMCE) we.assign_inputs |= 1 << pos;
            pre.push_back(x->grad);
        }
    }
    set_preassigned_grads(pre);
    for (auto& n : nodes) {
        NodeExt& e = ext(n.get());
        if (e.kind != OP_ACTIVATION || n->inputs.size() != 1) continue;
        const NodeBackProp* L = n->inputs[0].get();
        NodeExt& le = ext(L);
        // (not when the Linear's weight-gradient product sums its dY's columns
        // itself: the activation backward then stays a plain elementwise pass)
        if (le.kind == OP_LINEAR && le.linear_bias_grad && consumers[L] == 1 && !mle_get_gemm_column_sums()) {
            e.fused_bias_target = le.linear_bias_grad;
            e.fused_rows = L->total / L->dim[3];
            e.fused_cols = L->dim[3];
            le.bias_grad_fused = true;
        }
    }
}

}  // namespace mle

static void dims_mismatch(const char* what, const graph& A, const graph& B) {
    std::cout << what << " \n";
    Dimension(A);
    Dimension(B);
    std::exit(1);
}

// ---------------------------------------------------------------- Copy (:683)
graph GraphOperations::Copy(const graph& X) {
    auto node = std::make_shared<NodeBackProp>("Copy of " + X->op_name, X->dim[0], X->dim[1], X->dim[2], X->dim[3], 1);
    node->inputs = {X};
    GB += (double)node->total * sizeof(float) / (1ULL << 30);
    NodeBackProp *nd = node.get(), *xp = X.get();
    node->forward = [nd, xp]() { check(mle_copy(xp->output, nd->output, nd->total, st()), "Copy forward"); };
    node->backward = [nd, xp]() {
        check(mle_accumulate(nd->grad, xp->grad, nd->total, 1.0, st()), "Copy backward");
    };
    node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

// ------------------------------------------------------------ identity (:701)
graph GraphOperations::identity(const graph& X) {
    auto node = std::make_shared<NodeBackProp>(X->op_name, X->dim[0], X->dim[1], X->dim[2], X->dim[3], 1);
    node->inputs = {X};
    GB += (double)node->total * sizeof(float) / (1ULL << 30);
    NodeBackProp *nd = node.get(), *xp = X.get();
    node->forward = [nd, xp]() { check(mle_copy(xp->output, nd->output, nd->total, st()), "identity forward"); };
    node->backward = [nd, xp]() { check(mle_copy(nd->grad, xp->grad, nd->total, st()), "identity backward"); };
    node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

graph GraphOperations::like(const graph& X, const str name) {
    auto node = std::make_shared<NodeBackProp>(name, X->dim[0], X->dim[1], X->dim[2], X->dim[3], 1);
    node->inputs = {X};
    GB += (double)node->total * sizeof(float) / (1ULL << 30);
    NodeBackProp* nd = node.get();
    node->forward = []() {};
    node->backward = []() {};
    node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

// ------------------------------------------ HeadifytoChannel/DeHeadify (:1143-1176)
graph GraphOperations::HeadifytoChannel(const graph& X, const int heads) {
    if (X->dim[1] != 1 || X->dim[3] % heads != 0) {
        std::cerr << "Headify: channel must be 1 and embed must be divisible by heads\n";
        Dimension(X);
        std::exit(1);
    }
    const int b = X->dim[0], seq = X->dim[2], embed = X->dim[3], hd = embed / heads;
    auto node = std::make_shared<NodeBackProp>("Headified " + X->op_name, b, heads, seq, hd, 1);
    node->inputs = {X};
    GB += (double)node->total * sizeof(float) / (1ULL << 30);
    NodeBackProp *nd = node.get(), *xp = X.get();
    node->forward = [=]() { check(mle_headify(xp->output, nd->output, b, heads, seq, hd, 0, st()), "Headify fwd"); };
    node->backward = [=]() { check(mle_headify(nd->grad, xp->grad, b, heads, seq, hd, 1, st()), "Headify bwd"); };
    node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

graph GraphOperations::DeHeadify(const graph& X) {
    const int b = X->dim[0], heads = X->dim[1], seq = X->dim[2], hd = X->dim[3];
    auto node = std::make_shared<NodeBackProp>("Deheadified " + X->op_name, b, 1, seq, heads * hd, 1);
    node->inputs = {X};
    GB += (double)node->total * sizeof(float) / (1ULL << 30);
    NodeBackProp *nd = node.get(), *xp = X.get();
    node->forward = [=]() { check(mle_headify(xp->output, nd->output, b, heads, seq, hd, 2, st()), "DeHeadify fwd"); };
    node->backward = [=]() { check(mle_headify(nd->grad, xp->grad, b, heads, seq, hd, 3, st()), "DeHeadify bwd"); };
    node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

// ------------------------------------------------- positional encodings (:1257-1295)
graph GraphOperations::PositionalEncoding(const int& t, const int d_model) {
    auto node = std::make_shared<NodeBackProp>("SinoSuodalPosEncoding", 1, 1, 1, d_model, 1);
    GB += (double)node->total * sizeof(float) / (1ULL << 30);
    NodeBackProp* nd = node.get();
    const int tt = t;
    node->forward = [nd, tt, d_model]() { check(mle_timestep_pe(nd->output, tt, d_model, st()), "PositionalEncoding"); };
    node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

graph GraphOperations::MatrixPositionalEncoding(const graph& X, const int start_idx) {
    if (X->dim[1] != 1) {
        std::cerr << "MatrixPositionalEncoding expects input with channel dimension of 1\n";
        Dimension(X);
        std::exit(1);
    }
    const int batch = X->dim[0], rows = X->dim[2], cols = X->dim[3];
    auto node = std::make_shared<NodeBackProp>("MatrixSinoSuodalPosEncoding", batch, 1, rows, cols, 1);
    node->inputs = {X};
    GB += (double)node->total * sizeof(float) / (1ULL << 30);
    NodeBackProp *nd = node.get(), *xp = X.get();
    // the positional term depends on (row, col) only: computed once here
    float* table = arena_alloc(ARENA_ACT, (int64_t)rows * cols, "MatPE table");
    check(mle_matpe_table(table, rows, cols, start_idx, st()), "MatPE table");
    const int64_t row_elems = (int64_t)rows * cols;
    ext(nd).pe_table = table;
    node->forward = [=]() {
        if (ext(nd).pe_fed) return;  // the gather feeding it added the table
        check(mle_rows_add_table(xp->output, table, nd->output, batch, row_elems, st()), "MatPE");
    };
    node->backward = [=]() {
        if (ext(xp).grad_unused) return;  // a frozen input: its gradient has no reader
        check(mle_accumulate(nd->grad, xp->grad, nd->total, 1.0, st()), "MatPE backward");
    };
    node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

// -------------------------------------------------------- Bias_Add (:1355-1395)
graph GraphOperations::Bias_Add(const graph& A, const graph& B) {
    if (B->dim[0] != 1 || B->dim[1] != 1 || B->dim[2] != 1 || B->dim[3] != A->dim[3]) {
        std::cout << "Dimension mismatch in Bias_Add.. Bias must be a 1D vector matching at dim[3] \n";
        Dimension(A);
        Dimension(B);
        std::exit(1);
    }
    const long long rows = (long long)A->dim[0] * A->dim[1] * A->dim[2], cols = A->dim[3];
    auto node = std::make_shared<NodeBackProp>("Bias Add", A->dim[0], A->dim[1], A->dim[2], A->dim[3], 1);
    node->inputs = {A, B};
    GB += (double)node->total * sizeof(float) / (1ULL << 30);
    NodeBackProp *nd = node.get(), *ap = A.get(), *bp = B.get();
    node->forward = [=]() { check(mle_bias_add_fwd(ap->output, bp->output, nd->output, rows, cols, st()), "Bias_Add"); };
    node->backward = [=]() {
        check(mle_accumulate(nd->grad, ap->grad, nd->total, 1.0, st()), "Bias_Add backward A");
        check(mle_bias_grad(nd->grad, bp->grad, rows, cols, 1.0f, st()), "Bias_Add backward B");
    };
    node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

// ----------------------------------------------- Broadcast_Channel (:1398-1444)
graph GraphOperations::Broadcast_Channel(const graph& A, const graph& B) {
    if (A->dim[1] != B->dim[3] || B->dim[1] != 1 || B->dim[2] != 1) {
        std::cout << "Channel mismatch in broadcast channel \n";
        Dimension(A);
        Dimension(B);
        std::exit(1);
    }
    const int batch = A->dim[0], channels = A->dim[1], a = A->dim[2], b = A->dim[3];
    auto node = std::make_shared<NodeBackProp>("Broadcast Channel", batch, channels, a, b, 1);
    node->inputs = {A, B};
    GB += (double)node->total * sizeof(float) / (1ULL << 30);
    NodeBackProp *nd = node.get(), *ap = A.get(), *bp = B.get();
    node->forward = [=]() {
        check(mle_channel_bias_fwd(ap->output, bp->output, nd->output, batch, channels, (int64_t)a * b, st()),
              "Broadcast_Channel");
    };
    // The reference reduces with Channel_Squeeze1D<<<b, tpb>>>: one block per
    // index of dim[3], i.e. the first min(b, channels) channels receive their
    // sums (Engine/engine.cu:1435).  The same channels are reduced here; the
    // out-of-range blocks the reference launches when b > channels are not.
    node->backward = [=]() {
        check(mle_accumulate(nd->grad, ap->grad, nd->total, 1.0, st()), "Broadcast_Channel backward A");
        const int reduced = b < channels ? b : channels;
        check(mle_channel_bias_bwd_first(nd->grad, bp->grad, batch, channels, reduced, (int64_t)a * b, st()),
              "Broadcast_Channel backward B");
    };
    node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

// -------------------------------------------------------------- Add (:1627-1670)
graph GraphOperations::Add(const graph& A, const graph& B, const bool last) {
    for (int i = 0; i < 4; ++i)
        if (A->dim[i] != B->dim[i]) dims_mismatch("Dimension mismatch in Add", A, B);
    auto node = std::make_shared<NodeBackProp>("Add", A->dim[0], A->dim[1], A->dim[2], A->dim[3], 1);
    node->inputs = {A, B};
    GB += (double)node->total * sizeof(float) / (1ULL << 30);
    NodeBackProp *nd = node.get(), *ap = A.get(), *bp = B.get();
    ext(nd).kind = OP_ADD;
    ext(nd).add_is_loss = last;
    node->forward = [=]() {
        if (const NodeBackProp* ln = ext(nd).fused_norm) {
            NodeExt& le = ext(ln);
            const int s = mle_add_layernorm_fwd(ap->output, bp->output, nd->output, ln->output, le.ln_mean, le.ln_sq,
                                                le.ln_dims[0], le.ln_dims[1], le.ln_dims[2], le.ln_dims[3], le.ln_eps,
                                                st());
            if (s != MLE_ERR_UNSUPPORTED) {
                check(s, "Add + LayerNorm forward");
                le.norm_done = true;
                return;
            }
        }
        check(mle_scale_add(ap->output, bp->output, nd->output, 1.0f, nd->total, st()), "Add forward");
        if (last && g_loss_readback) {
            check_cuda(cudaStreamSynchronize(stream()), "Add loss");
            check_cuda(cudaMemcpy(&loss, nd->output, sizeof(float), cudaMemcpyDeviceToHost), "Add loss");
        }
    };
    node->backward = [=]() {
        if (last) check(mle_fill(nd->grad, 1.0f, nd->total, st()), "Add backward fill");
        if (ap == bp) {  // x + x: two accumulations into the same gradient
            check(mle_accumulate(nd->grad, ap->grad, nd->total, 1.0, st()), "Add backward A");
            check(mle_accumulate(nd->grad, bp->grad, nd->total, 1.0, st()), "Add backward B");
        } else {
            check(mle_add_bwd_assign(nd->grad, ap->grad, bp->grad, nd->total, ext(nd).assign_inputs & 3, st()),
                  "Add backward");
        }
    };
    node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

// --------------------------------------------------------- Subtract (:1674-1718)
// A - B; backward dA += g, dB += -g (the reference's Accumulate with scale
// -1, in double as its kernel computes it).  With last, the upstream
// gradient is 1 and the output is the loss.
graph GraphOperations::Subtract(const graph& A, const graph& B, const bool last) {
    for (int i = 0; i < 4; ++i)
        if (A->dim[i] != B->dim[i]) dims_mismatch("Dimension mismatch in subtract", A, B);
    auto node = std::make_shared<NodeBackProp>(" Subtract", A->dim[0], A->dim[1], A->dim[2], A->dim[3], 1);
    node->inputs = {A, B};
    GB += (double)node->total * sizeof(float) / (1ULL << 30);
    NodeBackProp *nd = node.get(), *ap = A.get(), *bp = B.get();
    node->forward = [=]() {
        check(mle_scale_add(ap->output, bp->output, nd->output, -1.0f, nd->total, st()), "Subtract forward");
        if (last && g_loss_readback) {
            check_cuda(cudaStreamSynchronize(stream()), "Subtract loss");
            check_cuda(cudaMemcpy(&loss, nd->output, sizeof(float), cudaMemcpyDeviceToHost), "Subtract loss");
        }
    };
    node->backward = [=]() {
        if (last) check(mle_fill(nd->grad, 1.0f, nd->total, st()), "Subtract backward fill");
        check(mle_accumulate(nd->grad, ap->grad, nd->total, 1.0, st()), "Subtract backward - A grad");
        check(mle_accumulate(nd->grad, bp->grad, nd->total, -1.0, st()), "Subtract backward - B grad");
    };
    node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

// --------------------------------------------------------- Multiply (:1720-1763)
// Elementwise A * B; backward dA += g * B, dB += g * A.
graph GraphOperations::Multiply(const graph& A, const graph& B) {
    for (int i = 0; i < 4; ++i)
        if (A->dim[i] != B->dim[i]) dims_mismatch("Dimension mismatch in Multiply ", A, B);
    auto node = std::make_shared<NodeBackProp>("Multiply", A->dim[0], A->dim[1], A->dim[2], A->dim[3], 1);
    node->inputs = {A, B};
    GB += (double)node->total * sizeof(float) / (1ULL << 30);
    NodeBackProp *nd = node.get(), *ap = A.get(), *bp = B.get();
    node->forward = [=]() { check(mle_mul(ap->output, bp->output, nd->output, nd->total, 0, st()), "Multiply forward"); };
    node->backward = [=]() {
        check(mle_mul(nd->grad, bp->output, ap->grad, nd->total, 1, st()), "Multiply backward - A grad");
        check(mle_mul(nd->grad, ap->output, bp->grad, nd->total, 1, st()), "Multiply backward - B grad");
    };
    node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

// ------------------------------------------------------------ Scale (:2521-2549)
graph GraphOperations::Scale(const graph& input, const float scale, const bool last) {
    auto node =
        std::make_shared<NodeBackProp>("Scale", input->dim[0], input->dim[1], input->dim[2], input->dim[3], 1);
    node->inputs = {input};
    GB += (double)node->total * sizeof(float) / (1ULL << 30);
    NodeBackProp *nd = node.get(), *ip = input.get();
    node->forward = [=]() { check(mle_scale_write(ip->output, nd->output, nd->total, scale, st()), "Scale forward"); };
    node->backward = [=]() {
        if (last) check(mle_fill(nd->grad, 1.0f, nd->total, st()), "Scale backward fill");
        check(mle_accumulate(nd->grad, ip->grad, nd->total, (double)scale, st()), "Scale backward");
    };
    node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

// ------------------------------------------------ MeanSquaredError (:1895-1950)
graph GraphOperations::MeanSquaredError(const graph& prediction, const graph& target, const bool last) {
    for (int i = 0; i < 4; ++i)
        if (prediction->dim[i] != target->dim[i]) dims_mismatch("Dimension mismatch \n MSE dimensions are:", prediction, target);
    auto node = std::make_shared<NodeBackProp>("MSE", 1, 1, 1, 1, 1);
    node->inputs = {prediction, target};
    GB += (double)(prediction->total + target->total + 1) * sizeof(float) / (1ULL << 30);
    NodeBackProp *nd = node.get(), *pp = prediction.get(), *tp = target.get();
    node->forward = [=]() {
        if (calculate_loss || !last) {
            check(mle_mse_fwd(pp->output, tp->output, nd->output, pp->total, st()), "Scalar MSE in MSE forward");
            if (last && g_loss_readback) {
                check_cuda(cudaStreamSynchronize(stream()), "MSE loss");
                check_cuda(cudaMemcpy(&loss, nd->output, sizeof(float), cudaMemcpyDeviceToHost), "MSE loss");
            }
        }
    };
    node->backward = [=]() {
        check(mle_mse_bwd(pp->output, tp->output, last ? nullptr : nd->grad, pp->grad, tp->total, st()),
              "deriv_mse in MSE backward");
    };
    node->zero_grad = [nd]() { zero_range(nd->output, nd->total); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

// ------------------------------------------ SoftMaxCrossEntropy (:2063-2124)
// When `last`, the forward pass also writes the prediction gradient
// (p - t)/batch, which is exactly what the backward lambda assigns from the
// same probabilities; the backward then has nothing left to do.  A forward
// that skipped the softmax (calc_loss false) leaves the backward to assign
// from the kept probabilities, as the reference does with its stale buffer.
graph GraphOperations::SoftMaxCrossEntropy(const graph& prediction, const graph& target, const bool last) {
    for (int i = 0; i < 4; ++i)
        if (prediction->dim[i] != target->dim[i])
            dims_mismatch("Dimension mismatch \n CrossEntropy dimensions are:", prediction, target);
    const int batch = target->dim[0], channels = target->dim[1], c = target->dim[2], d = target->dim[3];
    auto node = std::make_shared<NodeBackProp>("SoftMaxCrossEntropy Loss", 1, 1, 1, 1, 1);
    node->inputs = {prediction, target};
    float* probs = arena_alloc(ARENA_ACT, prediction->total, "SoftMax");
    GB += (double)(target->total + 1) * sizeof(float) / (1ULL << 30);
    NodeBackProp *nd = node.get(), *pp = prediction.get(), *tp = target.get();
    ext(nd).kind = OP_SMCE;
    const long long rows = (long long)batch * channels * c;
    auto grad_written = std::make_shared<bool>(false);
    node->forward = [=]() {
        *grad_written = false;
        if (calculate_loss || !last) {
            float* gout = last ? pp->grad : nullptr;
            check(mle_softmax_ce_fwd(pp->output, tp->output, (g_keep_softmax || !last) ? probs : nullptr, nd->output,
                                     gout, (float)batch, rows, d, st()),
                  "SoftMaxCrossEntropy");
            *grad_written = (gout != nullptr);
            if (last && g_loss_readback) {
                check_cuda(cudaStreamSynchronize(stream()), "SMCE loss");
                check_cuda(cudaMemcpy(&loss, nd->output, sizeof(float), cudaMemcpyDeviceToHost), "SMCE loss");
            }
        }
    };
    node->backward = [=]() {
        if (*grad_written) return;
        check(mle_softmax_ce_bwd(probs, tp->output, last ? nullptr : nd->grad, pp->grad, (float)batch, tp->total, st()),
              "derivative of CE in CE backward");
    };
    node->zero_grad = [nd]() { zero_range(nd->output, 1); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

// SoftMaxCrossEntropy with index labels (extension): the same lambdas with
// the one-hot target replaced by its class indices.
graph GraphOperations::SoftMaxCrossEntropyIndex(const graph& prediction, const int32_t* labels, const bool last) {
    const int batch = prediction->dim[0], channels = prediction->dim[1], c = prediction->dim[2],
              d = prediction->dim[3];
    auto node = std::make_shared<NodeBackProp>("SoftMaxCrossEntropy Loss", 1, 1, 1, 1, 1);
    node->inputs = {prediction};
    float* probs = arena_alloc(ARENA_ACT, prediction->total, "SoftMax");
    GB += sizeof(float) / (double)(1ULL << 30);
    NodeBackProp *nd = node.get(), *pp = prediction.get();
    ext(nd).kind = OP_SMCE;
    const long long rows = (long long)batch * channels * c;
    auto grad_written = std::make_shared<bool>(false);
    node->forward = [=]() {
        *grad_written = false;
        if (calculate_loss || !last) {
            float* gout = last ? pp->grad : nullptr;
            check(mle_softmax_ce_index_fwd(pp->output, labels, (g_keep_softmax || !last) ? probs : nullptr,
                                           nd->output, gout, (float)batch, rows, d, st()),
                  "SoftMaxCrossEntropy (index labels)");
            *grad_written = (gout != nullptr);
            if (last && g_loss_readback) {
                check_cuda(cudaStreamSynchronize(stream()), "SMCE loss");
                check_cuda(cudaMemcpy(&loss, nd->output, sizeof(float), cudaMemcpyDeviceToHost), "SMCE loss");
            }
        }
    };
    node->backward = [=]() {
        if (*grad_written) return;
        check(mle_softmax_ce_index_bwd(probs, labels, last ? nullptr : nd->grad, pp->grad, (float)batch, rows, d,
                                       st()),
              "derivative of CE in CE backward (index labels)");
    };
    node->zero_grad = [nd]() { zero_range(nd->output, 1); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

// --------------------------------------------- BMM family (:2196-2428)
static int bcase(const graph& X) { return (X->dim[0] > 1) + 2 * (X->dim[1] > 1); }

static void check_bc(const char* op, const graph& A, const graph& B) {
    const bool bok = (A->dim[0] == B->dim[0]) || (A->dim[0] == 1) || (B->dim[0] == 1);
    const bool cok = (A->dim[1] == B->dim[1]) || (A->dim[1] == 1) || (B->dim[1] == 1);
    if (!(bok && cok)) {
        std::cout << "Batch and Channel mismatch in " << op << "...\n";
        Dimension(A);
        Dimension(B);
        std::exit(1);
    }
}

// variant: forward kernel; the two backward calls follow the reference:
//  BMM    : dA = bcmmABT(dZ, B), dB = bcmmATB(A, dZ)
//  BMMABT : dA = bcmm(dZ, B),    dB = bcmmT(A, dZ)
//  BMMATB : dA = bcmmT(dZ, B),   dB = bcmm(A, dZ)
//  BMMT   : dA = bcmmATB(dZ, B), dB = bcmmABT(A, dZ)
static graph bmm_node(const char* name, int variant, const graph& A, const graph& B, int m, int n, int p) {
    check_bc(name, A, B);
    const int Ac = bcase(A), Bc = bcase(B), Cc = Ac > Bc ? Ac : Bc;
    const int batch = A->dim[0], channels = A->dim[1];
    auto node = std::make_shared<NodeBackProp>(name, batch, channels, m, p, 1);
    node->inputs = {A, B};
    GraphOperations::GB += (double)node->total * sizeof(float) / (1ULL << 30);
    NodeBackProp *nd = node.get(), *ap = A.get(), *bp = B.get();
    node->forward = [=]() {
        check(mle_bcmm(variant, ap->output, bp->output, nd->output, batch, channels, m, n, p, 0, Ac, Bc, Cc, 1.0f,
                       st()),
              str(name) + " forward");
    };
    int va, vb;  // backward variants for dA and dB
    switch (variant) {
        case MLE_GEMM_AB: va = MLE_GEMM_ABT; vb = MLE_GEMM_ATB; break;
        case MLE_GEMM_ABT: va = MLE_GEMM_AB; vb = MLE_GEMM_ATBT; break;
        case MLE_GEMM_ATB: va = MLE_GEMM_ATBT; vb = MLE_GEMM_AB; break;
        default: va = MLE_GEMM_ATB; vb = MLE_GEMM_ABT; break;
    }
    node->backward = [=]() {
        check(mle_bcmm(va, nd->grad, bp->output, ap->grad, batch, channels, m, p, n, 1, Cc, Bc, Ac, 1.0f, st()),
              str(name) + " backward dA");
        check(mle_bcmm(vb, ap->output, nd->grad, bp->grad, batch, channels, n, m, p, 1, Ac, Cc, Bc, 1.0f, st()),
              str(name) + " backward dB");
    };
    node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

graph GraphOperations::BMM(const graph& A, const graph& B) {
    if (A->dim[3] != B->dim[2]) dims_mismatch("Dimension mismatch in BMM", A, B);
    return bmm_node("BMM", MLE_GEMM_AB, A, B, A->dim[2], A->dim[3], B->dim[3]);
}
graph GraphOperations::BMMABT(const graph& A, const graph& B) {
    if (A->dim[3] != B->dim[3]) dims_mismatch("Dimension mismatch in BMMABT", A, B);
    return bmm_node("BMMABT", MLE_GEMM_ABT, A, B, A->dim[2], A->dim[3], B->dim[2]);
}
graph GraphOperations::BMMATB(const graph& A, const graph& B) {
    if (A->dim[2] != B->dim[2]) dims_mismatch("Dimension mismatch in BMM", A, B);
    return bmm_node("BMMATB", MLE_GEMM_ATB, A, B, A->dim[3], A->dim[2], B->dim[3]);
}
graph GraphOperations::BMMT(const graph& A, const graph& B) {
    if (A->dim[2] != B->dim[3]) dims_mismatch("Dimension mismatch in BMMT", A, B);
    return bmm_node("BMMT", MLE_GEMM_ATBT, A, B, A->dim[3], A->dim[2], B->dim[2]);
}

// ------------------------------------------------ SOFTMAX / SOFTMASK (:2431-2497)
static graph softmax_node(const char* name, const graph& X, int type, int mask) {
    const int a = X->dim[0], b = X->dim[1], c = X->dim[2], d = X->dim[3];
    auto node = std::make_shared<NodeBackProp>(name, a, b, c, d, 1);
    node->inputs = {X};
    const int lines = (type == 0) ? a * b * c : a * b * d;
    GraphOperations::GB += (double)(node->total + 2 * lines) * sizeof(float) / (1ULL << 30);
    NodeBackProp *nd = node.get(), *xp = X.get();
    node->forward = [=]() {
        check(mle_softmax_fwd(xp->output, nd->output, (int64_t)a * b, c, d, type, mask, st()), str(name) + " forward");
    };
    node->backward = [=]() {
        check(mle_softmax_bwd(nd->output, nd->grad, xp->grad, (int64_t)a * b, c, d, type, st()),
              str(name) + " backward");
    };
    node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

graph GraphOperations::SOFTMAX(const graph& X, const int type) { return softmax_node("Softmax", X, type, 0); }
graph GraphOperations::SOFTMASK(const graph& X, const int type) { return softmax_node("Softmask", X, type, 1); }

// ---------------------------------------------------- activations (:2650-2850)
static graph act_node(const char* name, int kind, const graph& input) {
    auto node = std::make_shared<NodeBackProp>(name, input->dim[0], input->dim[1], input->dim[2], input->dim[3], 1);
    node->inputs = {input};
    GraphOperations::GB += (double)node->total * sizeof(float) / (1ULL << 30);
    NodeBackProp *nd = node.get(), *ip = input.get();
    ext(nd).kind = OP_ACTIVATION;
    node->forward = [=]() { check(mle_act_fwd(kind, ip->output, nd->output, nd->total, st()), str(name) + " forward"); };
    node->backward = [=]() {
        const NodeExt& e = ext(nd);
        check(((e.assign_inputs & 1) ? mle_act_bwd_assign : mle_act_bwd)(kind, ip->output, nd->grad, ip->grad,
                                                                        nd->total, e.fused_bias_target, e.fused_rows,
                                                                        e.fused_cols, st()),
              str(name) + " backward");
    };
    node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

graph GraphOperations::RELU(const graph& input) { return act_node("ReLU", MLE_ACT_RELU, input); }
graph GraphOperations::LeakyRELU(const graph& input) { return act_node("LeakyReLU", MLE_ACT_LEAKY_RELU, input); }
graph GraphOperations::SILU(const graph& input) { return act_node("SiLU", MLE_ACT_SILU, input); }
graph GraphOperations::TANH(const graph& input) { return act_node("TaNH", MLE_ACT_TANH, input); }
graph GraphOperations::GELU(const graph& input) { return act_node("GeLU", MLE_ACT_GELU, input); }
graph GraphOperations::SIGMOID(const graph& input) { return act_node("Sigmoid", MLE_ACT_SIGMOID, input); }

// ------------------------------------------------------- CopyCrop (:2855-2915)
// Channel concatenation when the spatial sizes agree.  With different sizes
// the reference crops input1 into a buffer sized for input2's channels and
// accumulates into a scratch gradient that is never cleared between steps
// (Engine/engine.cu:2873-2898); that branch is not reproduced.
graph GraphOperations::CopyCrop(const graph& input1, const graph& input2) {
    const int batch = input2->dim[0], depth = input2->dim[1], d1 = input1->dim[1];
    const int a = input2->dim[2], b = input2->dim[3];
    if (input1->dim[2] != a || input1->dim[3] != b) {
        std::cerr << "CopyCrop: cropping inputs of different spatial size is not supported by this runtime\n";
        std::exit(1);
    }
    auto node = std::make_shared<NodeBackProp>("CopyNCrop", batch, d1 + depth, a, b, 1);
    node->inputs = {input1, input2};
    GB += (double)node->total * sizeof(float) / (1ULL << 30);
    NodeBackProp *nd = node.get(), *p1 = input1.get(), *p2 = input2.get();
    node->forward = [=]() {
        check(mle_channel_concat(p1->output, p2->output, nd->output, batch, d1, depth, (int64_t)a * b, st()),
              "CopyCrop forward");
    };
    node->backward = [=]() {
        check(mle_channel_split(p1->grad, p2->grad, nd->grad, batch, d1, depth, (int64_t)a * b, st()),
              "CopyCrop backward");
    };
    node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

// -------------------------------------------------- LayerNorm (:3079-3135)
graph GraphOperations::LayerNorm(const graph& X) {
    const int a = X->dim[0], b = X->dim[1], c = X->dim[2], d = X->dim[3];
    const float eps = 1e-5f;
    auto node = std::make_shared<NodeBackProp>("LayerNorm", a, b, c, d, 1);
    float* mean = arena_alloc(ARENA_ACT, a, "LayerNorm mean");
    float* sq = arena_alloc(ARENA_ACT, a, "LayerNorm std");
    GB += (double)(node->total + 2 * a) * sizeof(float) / (1ULL << 30);
    node->inputs = {X};
    NodeBackProp *nd = node.get(), *xp = X.get();
    NodeExt& ne = ext(nd);
    ne.kind = OP_LAYERNORM;
    ne.ln_mean = mean;
    ne.ln_sq = sq;
    ne.ln_dims[0] = a;
    ne.ln_dims[1] = b;
    ne.ln_dims[2] = c;
    ne.ln_dims[3] = d;
    ne.ln_eps = eps;
    node->forward = [=]() {
        if (ext(nd).norm_done) {  // written by the Add it reads (one pass)
            ext(nd).norm_done = false;
            return;
        }
        check(mle_layernorm_fwd(xp->output, nd->output, mean, sq, a, b, c, d, eps, st()), "LayerNorm forward");
    };
    node->backward = [=]() {
        check(mle_layernorm_bwd(nd->output, nd->grad, sq, xp->grad, a, b, c, d, eps, st()), "LayerNorm backward");
    };
    node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

// -------------------------------------------------- GroupNorm (:3200-3275)
graph GraphOperations::GroupNorm(const graph& X, const int group) {
    const int a = X->dim[0], b = X->dim[1], c = X->dim[2], d = X->dim[3];
    if (b % group != 0) {
        std::cout << "Groups cannot be cleanly split \n";
        Dimension(X);
        std::exit(1);
    }
    const float eps = 1e-5f;
    auto node = std::make_shared<NodeBackProp>("GroupNorm", a, b, c, d, 1);
    float* mean = arena_alloc(ARENA_ACT, (int64_t)a * group, "GroupNorm mean");
    float* sq = arena_alloc(ARENA_ACT, (int64_t)a * group, "GroupNorm std");
    GB += (double)(node->total + 2 * a * group) * sizeof(float) / (1ULL << 30);
    node->inputs = {X};
    NodeBackProp *nd = node.get(), *xp = X.get();
    node->forward = [=]() {
        check(mle_groupnorm_fwd(xp->output, nd->output, mean, sq, a, b, group, c, d, eps, st()), "GroupNorm forward");
    };
    node->backward = [=]() {
        check(mle_groupnorm_bwd(nd->output, nd->grad, sq, xp->grad, a, b, group, c, d, eps, st()),
              "GroupNorm backward");
    };
    node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
    node->free = [nd]() { nd->clear(); };
    return node;
}

// -------------------------------------------- ScaledDotAttention (extension)
graph GraphOperations::ScaledDotAttention(const graph& Q, const graph& K, const graph& V, const int heads,
                                          const float scale, const bool mask, const int axis,
                                          const int key_grad_mode) {
    if (Q->dim[1] != 1 || K->dim[1] != 1 || V->dim[1] != 1 || Q->dim[3] % heads != 0 || K->dim[3] != Q->dim[3] ||
        V->dim[3] != Q->dim[3] || K->dim[2] != V->dim[2] || K->dim[0] != Q->dim[0] || V->dim[0] != Q->dim[0]) {
        std::cerr << "ScaledDotAttention: expects [B,1,S,H*hd] projections with matching shapes\n";
        Dimension(Q);
        Dimension(K);
        Dimension(V);
        std::exit(1);
    }
    const int B = Q->dim[0], Sq = Q->dim[2], Sk = K->dim[2], D = Q->dim[3], hd = D / heads;
    auto node = std::make_shared<NodeBackProp>("Attention", B, 1, Sq, D, 1);
    node->inputs = {Q, K, V};
    const int64_t nq = (int64_t)B * Sq * D, nk = (int64_t)B * Sk * D, ns = (int64_t)B * heads * Sq * Sk;
    NodeBackProp *nd = node.get(), *qp = Q.get(), *kp = K.get(), *vp = V.get();
    const int causal = (mask && Sq > 1) ? 1 : 0;
    if (mle_attention_flash_supported(Sq, Sk, hd, axis, key_grad_mode)) {
        // the scores stay on chip: two numbers per key (column max and
        // inverse sum) carry the softmax from the forward to the backward
        const int64_t nkeys = (int64_t)B * heads * Sk;
        float* stats = arena_alloc(ARENA_ACT, 2 * nkeys, "Attention column statistics");
        float* dvec = arena_alloc(ARENA_WS, nkeys, "Attention column dots");
        GB += (double)(3 * nkeys) * sizeof(float) / (1ULL << 30);
        node->forward = [=]() {
            check(mle_attention_flash_fwd(qp->output, kp->output, vp->output, nd->output, stats, B, heads, Sq, Sk,
                                          hd, scale, causal, MLE_ATTN_TOKEN_MAJOR, st()),
                  "Attention forward");
        };
        ext(nd).kind = OP_ATTENTION;
        node->backward = [=]() {
            check(mle_attention_flash_bwd(qp->output, kp->output, vp->output, nd->grad, stats, dvec, qp->grad,
                                          kp->grad, vp->grad, B, heads, Sq, Sk, hd, scale, causal, key_grad_mode,
                                          MLE_ATTN_TOKEN_MAJOR, ext(nd).assign_inputs & 7, st()),
                  "Attention backward");
        };
        node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
        node->free = [nd]() { nd->clear(); };
        return node;
    }
    if (mle_attention_fused_supported(Sq, Sk, hd, axis, key_grad_mode)) {
        // fused kernels read and write the Linear layout directly; only P is kept
        float* P = arena_alloc(ARENA_ACT, ns, "Attention P");
        float* ws = arena_alloc(ARENA_WS, ns, "Attention dScores");
        GB += (double)(2 * nq + 2 * ns) * sizeof(float) / (1ULL << 30);
        node->forward = [=]() {
            check(mle_attention_fwd(qp->output, kp->output, vp->output, P, nd->output, B, heads, Sq, Sk, hd, scale,
                                    causal, axis, MLE_ATTN_TOKEN_MAJOR, st()),
                  "Attention forward");
        };
        ext(nd).kind = OP_ATTENTION;
        node->backward = [=]() {
            check(mle_attention_bwd_assign(qp->output, kp->output, vp->output, P, nd->grad, qp->grad, kp->grad,
                                           vp->grad, nullptr, nullptr, ws, B, heads, Sq, Sk, hd, scale, causal, axis,
                                           key_grad_mode, MLE_ATTN_TOKEN_MAJOR, ext(nd).assign_inputs & 7, st()),
                  "Attention backward");
        };
        node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
        node->free = [nd]() { nd->clear(); };
        return node;
    }
    // composed path: headified operands and their gradients, P and the score gradients
    float* qh = arena_alloc(ARENA_ACT, nq, "Attention Qh");
    float* kh = arena_alloc(ARENA_ACT, nk, "Attention Kh");
    float* vh = arena_alloc(ARENA_ACT, nk, "Attention Vh");
    float* oh = arena_alloc(ARENA_ACT, nq, "Attention Oh");
    float* P = arena_alloc(ARENA_ACT, ns, "Attention P");
    float* gqh = arena_alloc(ARENA_GRAD, nq, "Attention dQh");
    float* gkh = arena_alloc(ARENA_GRAD, nk, "Attention dKh");
    float* gvh = arena_alloc(ARENA_GRAD, nk, "Attention dVh");
    float* goh = arena_alloc(ARENA_GRAD, nq, "Attention dOh");
    float* dP = arena_alloc(ARENA_GRAD, ns, "Attention dP");
    float* dS = arena_alloc(ARENA_GRAD, ns, "Attention dS");
    GB += (double)(2 * (2 * nq + 2 * nk + 2 * ns) + nq) * sizeof(float) / (1ULL << 30);
    node->forward = [=]() {
        check(mle_headify(qp->output, qh, B, heads, Sq, hd, 0, st()), "Attention headify Q");
        check(mle_headify(kp->output, kh, B, heads, Sk, hd, 0, st()), "Attention headify K");
        check(mle_headify(vp->output, vh, B, heads, Sk, hd, 0, st()), "Attention headify V");
        check(mle_attention_fwd(qh, kh, vh, P, oh, B, heads, Sq, Sk, hd, scale, causal, axis, MLE_ATTN_HEAD_MAJOR,
                                st()),
              "Attention forward");
        check(mle_headify(oh, nd->output, B, heads, Sq, hd, 2, st()), "Attention deheadify");
    };
    node->backward = [=]() {
        check(mle_headify(nd->grad, goh, B, heads, Sq, hd, 3, st()), "Attention dO");
        check(mle_attention_bwd(qh, kh, vh, P, goh, gqh, gkh, gvh, dP, dS, nullptr, B, heads, Sq, Sk, hd, scale,
                                causal, axis, key_grad_mode, MLE_ATTN_HEAD_MAJOR, st()),
              "Attention backward");
        check(mle_headify(gqh, qp->grad, B, heads, Sq, hd, 1, st()), "Attention dQ");
        check(mle_headify(gkh, kp->grad, B, heads, Sk, hd, 1, st()), "Attention dK");
        check(mle_headify(gvh, vp->grad, B, heads, Sk, hd, 1, st()), "Attention dV");
    };
    node->zero_grad = [=]() {
        zero_range(nd->grad, nd->total);
        zero_range(gqh, nq);
        zero_range(gkh, nk);
        zero_range(gvh, nk);
        zero_range(goh, nq);
        zero_range(dP, ns);
        zero_range(dS, ns);
    };
    node->free = [nd]() { nd->clear(); };
    return node;
}

// ===================================================== Linear (:3496-3606)
Linear::Linear(const int input, const int output, const str name, const bool bias)
    : in(input), out(output), bias(bias), W1(name + " W1", 1, 1, input, output), B1(name + " B1", 1, 1, 1, output) {
    if (name != "") op_name = name;
}

void Linear::save(std::ofstream& f) const {
    W1.save(f);
    if (bias) B1.save(f);
}
void Linear::load(std::ifstream& f) {
    W1.load(f);
    if (bias) B1.load(f);
}
void Linear::operator=(const Linear& other) {
    W1 = other.W1;
    if (bias) B1 = other.B1;
}

graph Linear::forward(const graph& X) {
    if (X->dim[3] != W1.dim[2]) {
        std::cout << "Shape Mismatch in Linear Layer of " << X->op_name << ": \n";
        std::exit(1);
    }
    const int batch = X->dim[0], channels = X->dim[1], m = X->dim[2], n = X->dim[3], p = out;
    auto node = std::make_shared<NodeBackProp>(op_name, batch, channels, m, p, 1);
    node->inputs = {X};
    const long long rows = (long long)batch * channels * m;
    NodeBackProp *nd = node.get(), *xp = X.get();
    AdamParameter* W = &W1;
    AdamParameter* Bp = bias ? &B1 : nullptr;
    NodeExt& e = ext(nd);
    e.kind = OP_LINEAR;
    e.linear_bias_grad = bias ? B1.grad : nullptr;
    e.param_grads = {W1.grad};
    if (bias) e.param_grads.push_back(B1.grad);
    node->forward = [=]() {
        check(mle_linear_fwd(xp->output, W->output, Bp ? Bp->output : nullptr, nd->output, rows, n, p, st()),
              "Linear forward");
    };
    node->backward = [=]() {
        const bool fused = ext(nd).bias_grad_fused;
        // dW and dB on the parameter-gradient stream, concurrent with dX
        void* ps = (void*)fork_param_stream();
        if (ext(nd).assign_inputs & 1)  // first writer of dX: dX = dY W^T
            check(mle_gemm(nd->grad, W->output, xp->grad, nullptr, 1, rows, n, p, p, p, n, 0, 0, 0, 0, 1, 1.0f, 0.0f,
                           st()),
                  "MatMul... in " + nd->op_name + " backward");
        else
            check(mle_linear_bwd(nullptr, W->output, nd->grad, xp->grad, nullptr, nullptr, rows, n, p, st()),
                  "MatMul... in " + nd->op_name + " backward");
        check(mle_linear_bwd(xp->output, W->output, nd->grad, nullptr, W->grad, (Bp && !fused) ? Bp->grad : nullptr,
                             rows, n, p, ps),
              "MatMul... in " + nd->op_name + " backward");
    };
    node->free = [nd]() { nd->clear(); };
    node->zero_grad = [=]() {
        zero_range(nd->grad, nd->total);
        zero_range(W->grad, W->total);
        if (Bp) zero_range(Bp->grad, Bp->total);
    };
    node->accumulate = [=](double* gs) {
        W->accumulate_grad(gs);
        if (Bp) Bp->accumulate_grad(gs);
    };
    node->clipnorm = [=](const double* gs) {
        W->gradnorm(gs);
        if (Bp) Bp->gradnorm(gs);
    };
    node->updateParams = [=](const float lr, const bool adamw) {
        W->update(lr, adamw);
        if (Bp) Bp->update(lr, adamw);
    };
    return node;
}

// --------------------------------------------- Convolute2D (Engine/engine.cu:3723-3817)
Convolute2D::Convolute2D(int Input, int Output, int C, int D, int stride_, int padding, str param)
    : inp(Input), out(Output), c(C), d(D), pad(padding), stride(stride_), name(param),
      W1(name + " Weight ", Output, Input, C, D), B1(name + " Bias ", 1, Output, 1, 1) {}

void Convolute2D::save(std::ofstream& f) const {
    W1.save(f);
    B1.save(f);
}
void Convolute2D::load(std::ifstream& f) {
    W1.load(f);
    B1.load(f);
}

namespace {
// the parameter-side lambdas every convolution layer shares with Linear
void conv_param_lambdas(const graph& node, AdamParameter* W, AdamParameter* B) {
    NodeBackProp* nd = node.get();
    node->zero_grad = [=]() {
        zero_range(nd->grad, nd->total);
        zero_range(W->grad, W->total);
        zero_range(B->grad, B->total);
    };
    node->free = [nd]() { nd->clear(); };
    node->accumulate = [=](double* gs) {
        W->accumulate_grad(gs);
        B->accumulate_grad(gs);
    };
    node->clipnorm = [=](const double* gs) {
        W->gradnorm(gs);
        B->gradnorm(gs);
    };
    node->updateParams = [=](const float lr, const bool adamw) {
        W->update(lr, adamw);
        B->update(lr, adamw);
    };
    ext(nd).param_grads = {W->grad, B->grad};
}
}  // namespace

graph Convolute2D::forward(const graph& X) {
    if (X->dim[1] != inp) {
        std::cout << "Dimension Mismatch! in " << name << ": \n";
        Dimension(X);
        std::cout << "Actual input (Batch x depth): (" << X->dim[0] << "x" << X->dim[1] << ") \n";
        std::cout << "Expected input (Batch x depth): (" << X->dim[0] << "x" << inp << ") \n";
        std::exit(1);
    }
    const int batch = X->dim[0], a = X->dim[2], b = X->dim[3];
    const int outR = mle_conv_out_size(a, c, pad, stride), outC = mle_conv_out_size(b, d, pad, stride);
    if (outR <= 0 || outC <= 0) {
        std::cout << "Kernel larger than the padded input in " << name << "\n";
        std::exit(1);
    }
    auto node = std::make_shared<NodeBackProp>(name, batch, out, outR, outC, 1);
    node->inputs = {X};
    GraphOperations::GB += (double)node->total * sizeof(float) / (1ULL << 30);
    const int64_t wsn = mle_conv2d_workspace_floats(batch, inp, a, b, out, c, d, pad, stride);
    float* ws = arena_alloc(ARENA_WS, wsn, name + " columns");
    NodeBackProp *nd = node.get(), *xp = X.get();
    ext(nd).kind = OP_CONV;
    AdamParameter *W = &W1, *B = &B1;
    const int ci = inp, co = out, kh = c, kw = d, p = pad, s = stride;
    node->forward = [=]() {
        check(mle_conv2d_fwd(xp->output, W->output, B->output, nd->output, ws, batch, ci, a, b, co, kh, kw, p, s, st()),
              "Forward Convolution in " + nd->op_name);
    };
    node->backward = [=]() {
        // dW assigned (GV2D) and dB += (Channel_Squeeze1D) on the parameter-
        // gradient stream, dX += (CV2D_GradInput) on the compute stream;
        // the two parts use disjoint workspace regions
        void* ps = (void*)fork_param_stream();
        if (xp->grad)
            check(mle_conv2d_bwd_assign(xp->output, W->output, nd->grad, xp->grad, nullptr, nullptr, ws, batch, ci, a,
                                        b, co, kh, kw, p, s, ext(nd).assign_inputs & 1, st()),
                  "Input Gradient in " + nd->op_name);
        check(mle_conv2d_bwd(xp->output, W->output, nd->grad, nullptr, W->grad, B->grad, ws, batch, ci, a, b, co, kh,
                             kw, p, s, ps),
              "Weight + Bias Gradient in " + nd->op_name);
    };
    conv_param_lambdas(node, W, B);
    return node;
}

// -------------------------------------------- Convolute2DT (Engine/engine.cu:3819-3912)
Convolute2DT::Convolute2DT(int Input, int Output, int C, int D, int stride_, int padding, str param)
    : inp(Input), out(Output), c(C), d(D), pad(padding), stride(stride_), name(param),
      W1(name + " Weight ", Output, Input, C, D), B1(name + " Bias ", 1, Output, 1, 1) {}

void Convolute2DT::save(std::ofstream& f) const {
    W1.save(f);
    B1.save(f);
}
void Convolute2DT::load(std::ifstream& f) {
    W1.load(f);
    B1.load(f);
}

graph Convolute2DT::forward(const graph& X) {
    if (X->dim[1] != inp) {
        std::cout << "Dimension Mismatch! in " << name << ": \n";
        Dimension(X);
        std::cout << "Actual input (Batch x depth): (" << X->dim[0] << "x" << X->dim[1] << ") \n";
        std::cout << "Expected input (Batch x depth): (" << X->dim[0] << "x" << inp << ") \n";
        std::exit(1);
    }
    const int batch = X->dim[0], ih = X->dim[2], iw = X->dim[3];
    const int oh = mle_convT_out_size(ih, c, pad, stride), ow = mle_convT_out_size(iw, d, pad, stride);
    auto node = std::make_shared<NodeBackProp>(name, batch, out, oh, ow, 1);
    node->inputs = {X};
    T_node = node;
    GraphOperations::GB += (double)(node->total + W1.total + B1.total) * sizeof(float) / (1ULL << 30);
    const int64_t wsn = mle_convT2d_workspace_floats(batch, inp, ih, iw, out, c, d, pad, stride);
    if (wsn < 0) {
        std::cout << "Unsupported transposed-convolution geometry in " << name << "\n";
        std::exit(1);
    }
    float* ws = arena_alloc(ARENA_WS, wsn, name + " workspace");
    NodeBackProp *nd = node.get(), *xp = X.get();
    AdamParameter *W = &W1, *B = &B1;
    const int ci = inp, co = out, kh = c, kw = d, p = pad, s = stride;
    node->forward = [=]() {
        check(mle_convT2d_fwd(xp->output, W->output, B->output, nd->output, ws, batch, ci, ih, iw, co, kh, kw, p, s,
                              st()),
              "ConvTranspose2D Forward Kernel");
    };
    node->backward = [=]() {
        // dW assigned (GVT2D), dB += (Channel_Squeeze1D), dX assigned (CVT2D_GradInput)
        check(mle_convT2d_bwd(xp->output, W->output, nd->grad, xp->grad, W->grad, B->grad, ws, batch, ci, ih, iw, co,
                              kh, kw, p, s, st()),
              "Gradient w.r.t W, B1 and input for ConvTranspose2D");
    };
    conv_param_lambdas(node, W, B);
    return node;
}

// ------------------------------------------- LinearGroup (extension)
std::vector<graph> GraphOperations::LinearGroup(const graph& X, const std::vector<Linear*>& layers) {
    const int n = (int)layers.size();
    if (n < 1 || n > 3) {
        std::cerr << "LinearGroup: 1 to 3 layers\n";
        std::exit(1);
    }
    const int batch = X->dim[0], channels = X->dim[1], m = X->dim[2], in = X->dim[3];
    const long long rows = (long long)batch * channels * m;
    struct Shared {
        const float* W[3];
        const float* bias[3];
        float* Y[3];
        const float* dY[3];
        float* dW[3];
        float* dB[3];
        int out[3];
        int n;
        int backward_seen = 0;
    };
    auto sh = std::make_shared<Shared>();
    sh->n = n;
    std::vector<graph> nodes;
    for (int i = 0; i < n; ++i) {
        Linear* L = layers[i];
        if (L->inputs() != in) {
            std::cout << "Shape Mismatch in Linear Layer of " << X->op_name << ": \n";
            std::exit(1);
        }
        auto node = std::make_shared<NodeBackProp>(L->op_name, batch, channels, m, L->outputs(), 1);
        node->inputs = {X};
        sh->W[i] = L->W1.output;
        sh->bias[i] = L->has_bias() ? L->B1.output : nullptr;
        sh->Y[i] = node->output;
        sh->dY[i] = node->grad;
        sh->dW[i] = L->W1.grad;
        sh->dB[i] = L->has_bias() ? L->B1.grad : nullptr;
        sh->out[i] = L->outputs();
        nodes.push_back(node);
    }
    NodeBackProp* xp = X.get();
    for (int i = 0; i < n; ++i) {
        NodeBackProp* nd = nodes[i].get();
        AdamParameter* W = &layers[i]->W1;
        AdamParameter* Bp = layers[i]->has_bias() ? &layers[i]->B1 : nullptr;
        if (i == 0) {
            nd->forward = [=]() {
                check(mle_linear_group_fwd(xp->output, sh->W, sh->bias, sh->Y, sh->n, rows, in, sh->out, st()),
                      "Linear group forward");
            };
        } else {
            nd->forward = []() {};  // computed with the first layer of the group
        }
        // the output gradients of all layers are complete once the reverse
        // walk has reached every one of them
        nd->backward = [=]() {
            // the node that issues the group's backward reports every
            // layer's parameter gradients (data-parallel buckets)
            std::vector<float*>& done = ext(nd).param_grads;
            done.clear();
            if (++sh->backward_seen < sh->n) return;
            sh->backward_seen = 0;
            // weight and bias gradients on the parameter-gradient stream
            void* ps = (void*)fork_param_stream();
            check(mle_linear_group_bwd(nullptr, sh->W, sh->dY, xp->grad, nullptr, nullptr, sh->n, rows, in, sh->out,
                                       st()),
                  "Linear group backward");
            check(mle_linear_group_bwd(xp->output, sh->W, sh->dY, nullptr, sh->dW, sh->dB, sh->n, rows, in, sh->out,
                                       ps),
                  "Linear group backward");
            for (int j = 0; j < sh->n; ++j) {
                done.push_back(sh->dW[j]);
                if (sh->dB[j]) done.push_back(sh->dB[j]);
            }
        };
        nd->free = [nd]() { nd->clear(); };
        nd->zero_grad = [=]() {
            zero_range(nd->grad, nd->total);
            zero_range(W->grad, W->total);
            if (Bp) zero_range(Bp->grad, Bp->total);
        };
        nd->accumulate = [=](double* gs) {
            W->accumulate_grad(gs);
            if (Bp) Bp->accumulate_grad(gs);
        };
        nd->clipnorm = [=](const double* gs) {
            W->gradnorm(gs);
            if (Bp) Bp->gradnorm(gs);
        };
        nd->updateParams = [=](const float lr, const bool adamw) {
            W->update(lr, adamw);
            if (Bp) Bp->update(lr, adamw);
        };
        ext(nd).param_grads.clear();
    }
    return nodes;
}
