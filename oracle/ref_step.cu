/*
 * The reference's own training step -- BASELINE MEASUREMENT AND TEST
 * INFRASTRUCTURE ONLY (the product never links this).
 *
 * Compiled by oracle/build.py together with the ML_Engine sources
 * Engine/{engine,kernels,debug,transformer}.cu, read where they lie in the
 * reference tree, into oracle/_ref/librefstep.so.  Everything below runs the
 * reference's own runtime: its NodeBackProp/GraphOperations/AdamParameter,
 * its Linear and MultiHeadAttention classes and op builders, its lambdas and
 * kernels on the legacy default stream, including the device synchronisations
 * its Linear backward performs (CheckError, Engine/engine.cu:3553,3556).
 *
 * Graphs (the BASELINE configurations, built the way the use cases build
 * them):
 *   MLP      Linear-ReLU-Linear-loss          (use_cases/mnist.cu)
 *   encoder  MatrixPositionalEncoding, pre-LN blocks of MultiHeadAttention::
 *            forward (Engine/transformer.cu:647-661) and a GELU FFN, the
 *            projection Linear, loss
 *   enc-dec  the same encoder, decoder blocks of masked self-attention,
 *            MultiHeadAttention::cross_forward (:662-675) and the FFN
 * LayerNorm runs per token through NodeBackProp::reshape to [B*S,1,1,D]
 * (Engine/engine.cu:82-124), as the reference's LayerNorm normalises a whole
 * dim0 slice.
 *
 * One deviation, forced: the reference's SoftMaxCrossEntropy allocates its
 * softmax buffer with the loss node's total (1 float, Engine/engine.cu:2074-
 * 2079) and then writes the whole prediction into it (:2094), an
 * out-of-bounds device write.  The loss node here issues the same kernels in
 * the same order (SoftMax, scalar_ce_kernel, then ScaleAdd and ScaleValue in
 * the backward, :2090-2111) on a buffer of the prediction's size.
 *
 * The step is the reference training loop body (Engine/transformer.cu:852-
 * 871): zero_grad, token gather (TextualEmbedding::forward,
 * Engine/transformer.cu:176-192), forward, backward, the private clip
 * GraphOperations::accumulate/clipNorm restated through the public per-node
 * lambdas (Engine/engine.cu:3362-3368), ParameterUpdate.
 *
 * One model per process; every entry point returns 0 or a CUDA error code.
 */
#include <cuda_runtime.h>

#include <memory>
#include <string>
#include <vector>

#include "engine.h"
#include "transformer.h"

namespace {

struct TokenInput {
    graph node;    // [B,1,S,D] gathered embeddings
    float* table;  // [vocab, D]
    int* keys;     // [B*S]
    int vocab;
    std::string name;
};

struct TargetInput {
    graph node;  // dense one-hot [rows_b,1,rows_s,classes]
    int classes;
    std::string name;
};

struct RefModel {
    int config = 0;
    int batch = 0, seq = 0, d_model = 0, heads = 0, ffn = 0, layers = 0, vocab = 0;
    GraphOperations go;
    graph loss;
    std::vector<std::unique_ptr<Linear>> linears;
    std::vector<std::unique_ptr<MultiHeadAttention>> mhas;
    std::vector<AdamParameter*> params;  // W1, B1 per Linear, construction order
    std::vector<TokenInput> tokens;
    std::vector<TargetInput> targets;
    graph x_input;  // MLP input
    double* clip_ws = nullptr;
    bool embed_update = false;  // TextualEmbedding::EmbeddingUpdate on the encoder-side tokens
    float embed_lr = LEARNING_RATE;
    float* softmax = nullptr;
    float* softmax_arr = nullptr;
    float* max_arr = nullptr;
};

RefModel* g_model = nullptr;

int last_error() { return (int)cudaGetLastError(); }

Linear* new_linear(RefModel& M, int in, int out, const std::string& name) {
    M.linears.emplace_back(new Linear(in, out, name));
    Linear* l = M.linears.back().get();
    M.params.push_back(&l->W1);
    M.params.push_back(&l->B1);
    return l;
}

MultiHeadAttention* new_mha(RefModel& M, const std::string& name) {
    M.mhas.emplace_back(new MultiHeadAttention(M.d_model, M.d_model, M.heads, name));
    MultiHeadAttention* a = M.mhas.back().get();
    for (Linear* l : {&a->q, &a->k, &a->v, &a->o}) {
        M.params.push_back(&l->W1);
        M.params.push_back(&l->B1);
    }
    return a;
}

// per-token LayerNorm of a [B,1,S,D] activation
graph ln_tokens(const graph& x, int B, int S, int D) {
    x->reshape(std::vector<int>{B * S, 1, 1, D});
    graph h = GraphOperations::LayerNorm(x);
    x->reshape(std::vector<int>{B, 1, S, D});
    h->reshape(std::vector<int>{B, 1, S, D});
    return h;
}

graph ffn(RefModel& M, const graph& h, const std::string& name) {
    Linear* l1 = new_linear(M, M.d_model, M.ffn, name + " FFN1");
    Linear* l2 = new_linear(M, M.ffn, M.d_model, name + " FFN2");
    return l2->forward(GraphOperations::GELU(l1->forward(h)));
}

graph encoder_block(RefModel& M, graph x, const std::string& name) {
    MultiHeadAttention* a = new_mha(M, name + " SelfAttn");
    graph h = ln_tokens(x, M.batch, M.seq, M.d_model);
    x = GraphOperations::Add(x, a->forward(h, false));
    graph h2 = ln_tokens(x, M.batch, M.seq, M.d_model);
    return GraphOperations::Add(x, ffn(M, h2, name));
}

graph decoder_block(RefModel& M, graph x, const graph& enc, const std::string& name) {
    MultiHeadAttention* self = new_mha(M, name + " MaskedSelfAttn");
    MultiHeadAttention* cross = new_mha(M, name + " CrossAttn");
    graph h = ln_tokens(x, M.batch, M.seq, M.d_model);
    x = GraphOperations::Add(x, self->forward(h, true));
    graph h2 = ln_tokens(x, M.batch, M.seq, M.d_model);
    x = GraphOperations::Add(x, cross->cross_forward(h2, enc));
    graph h3 = ln_tokens(x, M.batch, M.seq, M.d_model);
    return GraphOperations::Add(x, ffn(M, h3, name));
}

graph token_input(RefModel& M, const std::string& name) {
    TokenInput t;
    t.name = name;
    t.vocab = M.vocab;
    t.node = std::make_shared<NodeBackProp>(name + " Embeddings", M.batch, 1, M.seq, M.d_model, 1);
    SafeCudaMalloc(name + " table", t.table, (size_t)M.vocab * M.d_model);
    cudaMemset(t.table, 0, (size_t)M.vocab * M.d_model * sizeof(float));
    cudaMalloc((void**)&t.keys, (size_t)M.batch * M.seq * sizeof(int));
    cudaMemset(t.keys, 0, (size_t)M.batch * M.seq * sizeof(int));
    // the reference's embedding node clears its gradient with zero_grad
    // (DataLoading::forward, Engine/transformer.cu:547-548)
    NodeBackProp* nd = t.node.get();
    t.node->zero_grad = [nd]() {
        const int tpb = THREADSPERBLOCK;
        fillKernel<<<(int)((nd->total + tpb - 1) / tpb), tpb>>>(nd->grad, 0.0f, (unsigned long long)nd->total);
    };
    M.tokens.push_back(t);
    return t.node;
}

graph target_input(RefModel& M, const std::string& name, int rows_b, int rows_s, int classes) {
    TargetInput t;
    t.name = name;
    t.classes = classes;
    t.node = std::make_shared<NodeBackProp>(name, rows_b, 1, rows_s, classes, 1);
    cudaMemset(t.node->output, 0, (size_t)t.node->total * sizeof(float));
    M.targets.push_back(t);
    return t.node;
}

// SoftMaxCrossEntropy(prediction, target, last = true) with the softmax
// buffer sized to the prediction (see the header comment).
graph smce_loss(RefModel& M, const graph& prediction, const graph& target) {
    const int batch = target->dim[0], channels = target->dim[1], c = target->dim[2], d = target->dim[3];
    auto node = std::make_shared<NodeBackProp>("SoftMaxCrossEntropy Loss", 1, 1, 1, 1, 1);
    node->inputs = {prediction, target};
    SafeCudaMalloc("Softmax array", M.softmax_arr, (size_t)batch * channels * c);
    SafeCudaMalloc("Max array", M.max_arr, (size_t)batch * channels * c);
    SafeCudaMalloc("SoftMax", M.softmax, (size_t)prediction->total);
    float *softmax = M.softmax, *arr = M.softmax_arr, *max_arr = M.max_arr;
    const int tpb = THREADSPERBLOCK;
    const int bpg = (int)((prediction->total + tpb - 1) / tpb);
    NodeBackProp* nd = node.get();
    NodeBackProp* pred = prediction.get();
    NodeBackProp* tgt = target.get();
    node->forward = [=]() {
        SoftMax(pred->output, arr, softmax, max_arr, batch, channels, c, d, 0);
        static const float zero = 0.0f;  // WriteValueAt(node, 0.0f, 0)
        cudaMemcpy(nd->output, &zero, sizeof(float), cudaMemcpyHostToDevice);
        scalar_ce_kernel<<<bpg, tpb>>>(softmax, tgt->output, nd->output, pred->total);
        cudaMemcpy(&GraphOperations::loss, nd->output, sizeof(float), cudaMemcpyDeviceToHost);
    };
    node->backward = [=]() {
        ScaleAdd<<<bpg, tpb>>>(softmax, tgt->output, pred->grad, -1.0f, tgt->total);
        ScaleValue(pred->grad, (float)batch, pred->total, 1);
    };
    node->zero_grad = [=]() { Zerograd("Node", nd->output, 1); };
    return node;
}

void build(RefModel& M, int in_features, int hidden, int classes) {
    if (M.config == 1) {
        M.x_input = std::make_shared<NodeBackProp>("MNIST input", M.batch, 1, 1, in_features, 1);
        Linear* l1 = new_linear(M, in_features, hidden, "Linear1");
        Linear* l2 = new_linear(M, hidden, classes, "Linear2");
        graph logits = l2->forward(GraphOperations::RELU(l1->forward(M.x_input)));
        M.loss = smce_loss(M, logits, target_input(M, "labels", M.batch, 1, classes));
    } else if (M.config == 2) {
        graph x = GraphOperations::MatrixPositionalEncoding(token_input(M, "tokens"));
        for (int l = 0; l < M.layers; ++l) x = encoder_block(M, x, "Enc" + std::to_string(l));
        Linear* proj = new_linear(M, M.d_model, M.vocab, "Projection");
        M.loss = smce_loss(M, proj->forward(x), target_input(M, "targets", M.batch, M.seq, M.vocab));
    } else {
        graph e = GraphOperations::MatrixPositionalEncoding(token_input(M, "src"));
        for (int l = 0; l < M.layers; ++l) e = encoder_block(M, e, "Enc" + std::to_string(l));
        graph x = GraphOperations::MatrixPositionalEncoding(token_input(M, "tgt_in"));
        for (int l = 0; l < M.layers; ++l) x = decoder_block(M, x, e, "Dec" + std::to_string(l));
        Linear* proj = new_linear(M, M.d_model, M.vocab, "Projection");
        M.loss = smce_loss(M, proj->forward(x), target_input(M, "tgt_out", M.batch, M.seq, M.vocab));
    }
    M.go.nodes = topological_sort(M.loss);
    cudaMalloc((void**)&M.clip_ws, sizeof(double));
}

void gather_tokens(RefModel& M) {
    const int tpb = THREADSPERBLOCK;
    for (auto& t : M.tokens) {
        const unsigned long long total = (unsigned long long)t.node->total;
        GatherEmbeddings<<<(int)((total + tpb - 1) / tpb), tpb>>>(t.node->output, t.table, t.keys, M.seq, M.seq,
                                                                  M.d_model, total);
    }
}

void clip(RefModel& M, float max_norm) {
    cudaMemset(M.clip_ws, 0, sizeof(double));
    for (auto& n : M.go.nodes)
        if (n->accumulate) n->accumulate(M.clip_ws);
    Sqrt_Scale<<<1, 1>>>(M.clip_ws, (double)max_norm, 0);
    for (auto& n : M.go.nodes)
        if (n->clipnorm) n->clipnorm(M.clip_ws);
}

// phases: 0 zero_grad + gather + forward, 1 backward, 2 clip + update
void run_phase(RefModel& M, int phase, float lr, int adamw, float clip_norm) {
    if (phase == 0) {
        M.go.zero_grad();
        gather_tokens(M);
        M.go.forward(nullptr, true);
    } else if (phase == 1) {
        M.go.backward();
        if (M.embed_update && !M.tokens.empty()) {
            // embedder.EmbeddingUpdate(enc, "E") (Engine/transformer.cu:869,
            // 233-245): KeyUpdate with the encoder-side keys, at LEARNING_RATE
            // unless the caller set another rate
            TokenInput& t = M.tokens[0];
            const unsigned long long total = (unsigned long long)t.node->total;
            const int tpb = THREADSPERBLOCK;
            KeyUpdate<<<(int)((total + tpb - 1) / tpb), tpb>>>(t.table, t.node->grad, t.keys, M.seq, M.seq,
                                                               M.d_model, M.embed_lr, total);
        }
    } else {
        if (clip_norm > 0) clip(M, clip_norm);
        M.go.ParameterUpdate(nullptr, false, lr, adamw != 0);
    }
}

float* param_buffer(AdamParameter* p, int which) {
    switch (which) {
        case 0: return p->output;
        case 1: return p->grad;
        case 2: return p->m;
        default: return p->v;
    }
}

}  // namespace

extern "C" {

/* config: 1 MLP, 2 encoder, 3 encoder-decoder (the values of mle_config). */
int refstep_create(int config, int batch, int in_features, int hidden, int classes, int seq, int d_model, int heads,
                   int ffn_width, int layers, int vocab) {
    if (g_model || config < 1 || config > 3 || batch <= 0) return (int)cudaErrorInvalidValue;
    g_model = new RefModel();
    RefModel& M = *g_model;
    M.config = config;
    M.batch = batch;
    M.seq = seq;
    M.d_model = d_model;
    M.heads = heads;
    M.ffn = ffn_width;
    M.layers = layers;
    M.vocab = vocab;
    build(M, in_features, hidden, classes);
    cudaDeviceSynchronize();
    return last_error();
}

int refstep_destroy(void) {
    if (!g_model) return 0;
    RefModel& M = *g_model;
    cudaDeviceSynchronize();
    M.go.clean_clear_graph(M.loss);
    for (auto& t : M.tokens) {
        cudaFree(t.table);
        cudaFree(t.keys);
    }
    cudaFree(M.clip_ws);
    cudaFree(M.softmax);
    cudaFree(M.softmax_arr);
    cudaFree(M.max_arr);
    for (AdamParameter* p : M.params) {
        cudaFree(p->m);
        cudaFree(p->v);
    }
    delete g_model;
    g_model = nullptr;
    cudaDeviceSynchronize();
    return last_error();
}

int refstep_param_count(void) { return g_model ? (int)g_model->params.size() : 0; }

long long refstep_param_numel(int i) {
    if (!g_model || i < 0 || i >= (int)g_model->params.size()) return -1;
    return g_model->params[i]->total;
}

int refstep_param_step(int i) {
    if (!g_model || i < 0 || i >= (int)g_model->params.size()) return -1;
    return g_model->params[i]->t;
}

/* which: 0 weights, 1 gradient, 2 first moment, 3 second moment */
int refstep_param_write(int i, int which, const float* host) {
    if (!g_model || i < 0 || i >= (int)g_model->params.size()) return (int)cudaErrorInvalidValue;
    AdamParameter* p = g_model->params[i];
    return (int)cudaMemcpy(param_buffer(p, which), host, (size_t)p->total * sizeof(float), cudaMemcpyHostToDevice);
}

int refstep_param_read(int i, int which, float* host) {
    if (!g_model || i < 0 || i >= (int)g_model->params.size()) return (int)cudaErrorInvalidValue;
    AdamParameter* p = g_model->params[i];
    return (int)cudaMemcpy(host, param_buffer(p, which), (size_t)p->total * sizeof(float), cudaMemcpyDeviceToHost);
}

int refstep_embedding_count(void) { return g_model ? (int)g_model->tokens.size() : 0; }

/* on != 0: every step runs the reference's embedding update on the
 * encoder-side table after the backward pass, at rate lr (<= 0: the
 * reference's LEARNING_RATE). */
int refstep_set_embed_update(int on, float lr) {
    if (!g_model) return (int)cudaErrorInvalidValue;
    g_model->embed_update = on != 0;
    g_model->embed_lr = lr > 0 ? lr : LEARNING_RATE;
    return 0;
}

int refstep_embedding_read(int i, float* host, long long numel) {
    if (!g_model || i < 0 || i >= (int)g_model->tokens.size()) return (int)cudaErrorInvalidValue;
    TokenInput& t = g_model->tokens[i];
    if (numel != (long long)t.vocab * g_model->d_model) return (int)cudaErrorInvalidValue;
    return (int)cudaMemcpy(host, t.table, (size_t)numel * sizeof(float), cudaMemcpyDeviceToHost);
}

int refstep_embedding_write(int i, const float* host, long long numel) {
    if (!g_model || i < 0 || i >= (int)g_model->tokens.size()) return (int)cudaErrorInvalidValue;
    TokenInput& t = g_model->tokens[i];
    if (numel != (long long)t.vocab * g_model->d_model) return (int)cudaErrorInvalidValue;
    return (int)cudaMemcpy(t.table, host, (size_t)numel * sizeof(float), cudaMemcpyHostToDevice);
}

/* Inputs by the session's names: "x" (MLP, float32 [batch*in_features]);
 * token ids "tokens" / "src" / "tgt_in" (int32 [batch*seq]); class ids
 * "labels" / "targets" / "tgt_out" (int32), expanded here to the reference's
 * dense one-hot target. */
int refstep_input_write(const char* name, const void* host, long long numel) {
    if (!g_model || !name || !host) return (int)cudaErrorInvalidValue;
    RefModel& M = *g_model;
    const std::string n(name);
    if (n == "x" && M.x_input) {
        if (numel != M.x_input->total) return (int)cudaErrorInvalidValue;
        return (int)cudaMemcpy(M.x_input->output, host, (size_t)numel * sizeof(float), cudaMemcpyHostToDevice);
    }
    for (auto& t : M.tokens)
        if (t.name == n) {
            if (numel != (long long)M.batch * M.seq) return (int)cudaErrorInvalidValue;
            return (int)cudaMemcpy(t.keys, host, (size_t)numel * sizeof(int), cudaMemcpyHostToDevice);
        }
    for (auto& t : M.targets)
        if (t.name == n) {
            if (numel * t.classes != t.node->total) return (int)cudaErrorInvalidValue;
            std::vector<float> oh((size_t)t.node->total, 0.0f);
            const int* ids = static_cast<const int*>(host);
            for (long long r = 0; r < numel; ++r) {
                if (ids[r] < 0 || ids[r] >= t.classes) return (int)cudaErrorInvalidValue;
                oh[(size_t)r * t.classes + ids[r]] = 1.0f;
            }
            return (int)cudaMemcpy(t.node->output, oh.data(), oh.size() * sizeof(float), cudaMemcpyHostToDevice);
        }
    return (int)cudaErrorInvalidValue;
}

/* One training step; *loss (nullable) receives GraphOperations::loss. */
int refstep_step(float lr, int adamw, float clip_norm, float* loss) {
    if (!g_model) return (int)cudaErrorInvalidValue;
    for (int ph = 0; ph < 3; ++ph) run_phase(*g_model, ph, lr, adamw, clip_norm);
    const cudaError_t e = cudaDeviceSynchronize();
    if (loss) *loss = GraphOperations::loss;
    return e != cudaSuccess ? (int)e : last_error();
}

/* `warmup` untimed steps, then `steps` timed ones with CUDA events on the
 * legacy stream around each phase; ms[0..3] = mean forward (with zero_grad
 * and the token gather), backward, clip + update, whole step. */
int refstep_time(int warmup, int steps, float lr, int adamw, float clip_norm, double* ms) {
    if (!g_model || steps <= 0 || !ms) return (int)cudaErrorInvalidValue;
    RefModel& M = *g_model;
    for (int i = 0; i < warmup; ++i)
        for (int ph = 0; ph < 3; ++ph) run_phase(M, ph, lr, adamw, clip_norm);
    cudaEvent_t ev[4];
    for (auto& e : ev) cudaEventCreate(&e);
    double acc[4] = {0, 0, 0, 0};
    cudaDeviceSynchronize();
    for (int s = 0; s < steps; ++s) {
        cudaEventRecord(ev[0], 0);
        for (int ph = 0; ph < 3; ++ph) {
            run_phase(M, ph, lr, adamw, clip_norm);
            cudaEventRecord(ev[ph + 1], 0);
        }
        cudaEventSynchronize(ev[3]);
        for (int ph = 0; ph < 3; ++ph) {
            float t = 0;
            cudaEventElapsedTime(&t, ev[ph], ev[ph + 1]);
            acc[ph] += t;
        }
        float t = 0;
        cudaEventElapsedTime(&t, ev[0], ev[3]);
        acc[3] += t;
    }
    for (int i = 0; i < 4; ++i) ms[i] = acc[i] / steps;
    for (auto& e : ev) cudaEventDestroy(e);
    return last_error();
}

/* Device memory the graph build allocated, as the reference counts it. */
double refstep_graph_gb(void) { return GraphOperations::GB; }

}  // extern "C"
