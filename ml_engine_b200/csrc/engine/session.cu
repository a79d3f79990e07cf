// Benchmark/test sessions: the configuration graphs built with the
// reference-compatible API, their step, CUDA-graph capture and the C ABI of
// include/mle_engine.h.
//
// Graph shapes follow the benchmark configurations:
//   MLP      use_cases/mnist.cu:252-273 (Linear 784->256, ReLU, Linear 256->10,
//            SoftMaxCrossEntropy with a one-hot target built on the device)
//   ENCODER  embedding gather -> MatrixPositionalEncoding -> N x pre-LN blocks
//            [LayerNorm per token, MultiHeadAttention (column softmax, scale
//            1/sqrt(head_dim), Engine/transformer.cu:647-661), Add, LayerNorm,
//            Linear-GELU-Linear, Add] -> Linear projection -> SMCE
//   ENCDEC   encoder as above; decoder blocks add masked self-attention and
//            cross attention (scale 1/sqrt(d_model), masked whenever the query
//            length exceeds 1, Engine/transformer.cu:662-675)
// LayerNorm per token uses the reference's own mechanism: the token matrix
// is reshaped to [B*S,1,1,D] while the LayerNorm node is built
// (NodeBackProp::reshape, Engine/engine.cu:82-124).
#include <math.h>
#include <string.h>

#include <cstring>
#include <fstream>
#include <memory>
#include <random>
#include <string>
#include <vector>

#include "engine.h"
#include "engine_internal.h"
#include "mle_engine.h"
#include "session_dp.h"

using namespace mle;

namespace mle {
bool g_loss_readback = true;
}

namespace {

struct Input {
    std::string name;
    int dtype;  // 0 f32, 1 i32
    int64_t numel;
    void* host = nullptr;
    void* dev = nullptr;
};

struct Session {
    mle_session_desc d{};
    cudaStream_t stream = nullptr;
    GraphOperations go;
    graph loss;
    std::vector<std::unique_ptr<Linear>> linears;
    std::vector<std::unique_ptr<Convolute2D>> convs;
    std::vector<std::unique_ptr<Convolute2DT>> convts;
    // (weight, bias) of every layer in construction order: the parameter
    // order the session reports and the reference's layers update in
    std::vector<std::pair<AdamParameter*, AdamParameter*>> layer_params;
    std::vector<AdamParameter*> params;
    std::vector<Input> inputs;
    std::vector<std::function<void()>> prep;
    std::vector<std::pair<float*, int64_t>> emb;
    std::vector<int32_t*> emb_keys;  // the token ids each table gathers with (same order as emb)
    // token tables trained by the embedding SGD update (desc.embed_lr > 0)
    struct EmbTrain {
        int32_t* keys;
        float* table;
        NodeBackProp* node;   // gathered embeddings; its grad is the update's input
        float* gsum;          // [vocab, D]: the step's gradient per table row
        int64_t rows, table_n;
        int dim, row_len, vocab;
    };
    std::vector<EmbTrain> emb_train;
    float* loss_host = nullptr;
    // captured steps: [0] device-resident (no host copies), [1] with the
    // input upload and the loss download
    cudaGraph_t graph_[2] = {nullptr, nullptr};
    cudaGraphExec_t exec[2] = {nullptr, nullptr};
    // one captured graph per phase (device resident), for timing phases
    cudaGraphExec_t phase_exec[6] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
    std::unique_ptr<DataParallel> dp;
    size_t param_first = 0;
};

int status_of(cudaError_t e) {
    if (e != cudaSuccess) {
        fprintf(stderr, "mle_session: CUDA error %s\n", cudaGetErrorString(e));
        return MLE_ERR_CUDA;
    }
    return MLE_OK;
}

struct StreamScope {  // routes every op of this session to its stream and GEMM mode
    cudaStream_t prev;
    int prev_mode;
    explicit StreamScope(cudaStream_t s, int gemm_mode = -1) : prev(mle::stream()), prev_mode(mle_get_gemm_mode()) {
        mle::set_stream(s);
        if (gemm_mode >= 0) mle_set_gemm_mode(gemm_mode);
    }
    ~StreamScope() {
        mle::set_stream(prev);
        mle_set_gemm_mode(prev_mode);
    }
};

Linear* new_linear(Session& S, int in, int out, const std::string& name) {
    S.linears.emplace_back(new Linear(in, out, name));
    Linear* l = S.linears.back().get();
    S.layer_params.push_back({&l->W1, &l->B1});
    return l;
}

Convolute2D* new_conv(Session& S, int in, int out, int k, int stride, int pad, const std::string& name) {
    S.convs.emplace_back(new Convolute2D(in, out, k, k, stride, pad, name));
    Convolute2D* c = S.convs.back().get();
    S.layer_params.push_back({&c->W1, &c->B1});
    return c;
}

Convolute2DT* new_convT(Session& S, int in, int out, int k, int stride, int pad, const std::string& name) {
    S.convts.emplace_back(new Convolute2DT(in, out, k, k, stride, pad, name));
    Convolute2DT* c = S.convts.back().get();
    S.layer_params.push_back({&c->W1, &c->B1});
    return c;
}

// ResidualBlock::forward (Engine/diffusion.cu:109-137): conv-GroupNorm-SiLU,
// time MLP broadcast per channel, conv-GroupNorm, skip (a strided 1x1 conv
// when the shape changes), Add, SiLU.  The skip convolution is built only
// when it is used (the reference also constructs an unused one).
graph residual_block(Session& S, const graph& x, const graph& t, int in, int out, int stride, const std::string& name) {
    Convolute2D* c1 = new_conv(S, in, out, 3, stride, 1, name + " Conv1");
    Convolute2D* c2 = new_conv(S, out, out, 3, 1, 1, name + " Conv2");
    Linear* tm = new_linear(S, t->dim[3], out, name + " Time MLP");
    Convolute2D* sk = (in != out || stride != 1) ? new_conv(S, in, out, 1, stride, 0, name + " SkipConv") : nullptr;
    graph h = GraphOperations::SILU(GraphOperations::GroupNorm(c1->forward(x)));
    h = GraphOperations::Broadcast_Channel(h, tm->forward(t));
    h = GraphOperations::GroupNorm(c2->forward(h));
    graph skip = sk ? sk->forward(x) : x;
    return GraphOperations::SILU(GraphOperations::Add(h, skip));
}

Input& add_input(Session& S, const std::string& name, int dtype, int64_t numel, void* dev) {
    Input in;
    in.name = name;
    in.dtype = dtype;
    in.numel = numel;
    in.dev = dev;
    mle::check_cuda(cudaHostAlloc(&in.host, (size_t)numel * 4, cudaHostAllocDefault), "pinned input " + name);
    std::memset(in.host, 0, (size_t)numel * 4);
    S.inputs.push_back(in);
    return S.inputs.back();
}

// Token matrix [B,1,S,D] normalised per token.
graph ln_tokens(const graph& x, int B, int Sq, int D) {
    x->reshape({B * Sq, 1, 1, D});
    graph h = GraphOperations::LayerNorm(x);
    x->reshape({B, 1, Sq, D});
    h->reshape({B, 1, Sq, D});
    return h;
}

graph attention(Session& S, const graph& xq, const graph& xkv, bool mask, float scale, const std::string& name) {
    const int D = S.d.d_model, H = S.d.heads;
    Linear* q = new_linear(S, D, D, name + " Query");
    Linear* k = new_linear(S, D, D, name + " Key");
    Linear* v = new_linear(S, D, D, name + " Value");
    Linear* o = new_linear(S, D, D, name + " Output");
    graph Qp, Kp, Vp;
    if (S.d.fused_attention && xq.get() == xkv.get()) {
        // self-attention: the three projections read the same input
        std::vector<graph> p = GraphOperations::LinearGroup(xq, {q, k, v});
        Qp = p[0];
        Kp = p[1];
        Vp = p[2];
    } else if (S.d.fused_attention) {
        // cross-attention: keys and values read the encoder output
        Qp = q->forward(xq);
        std::vector<graph> p = GraphOperations::LinearGroup(xkv, {k, v});
        Kp = p[0];
        Vp = p[1];
    } else {
        Qp = q->forward(xq);
        Kp = k->forward(xkv);
        Vp = v->forward(xkv);
    }
    graph att;
    if (S.d.fused_attention) {
        att = GraphOperations::ScaledDotAttention(Qp, Kp, Vp, H, scale, mask, 1, S.d.key_grad_mode);
    } else {
        graph Q = GraphOperations::HeadifytoChannel(Qp, H);
        graph K = GraphOperations::HeadifytoChannel(Kp, H);
        graph V = GraphOperations::HeadifytoChannel(Vp, H);
        graph scores = GraphOperations::BMMABT(Q, K);
        graph scaled = GraphOperations::Scale(scores, scale);
        graph w = (mask && scaled->dim[2] > 1) ? GraphOperations::SOFTMASK(scaled, 1) : GraphOperations::SOFTMAX(scaled, 1);
        att = GraphOperations::DeHeadify(GraphOperations::BMM(w, V));
    }
    graph out = o->forward(att);
    out->op_name = name + " Output";
    return out;
}

graph ffn(Session& S, const graph& h, const std::string& name) {
    Linear* l1 = new_linear(S, S.d.d_model, S.d.ffn, name + " FFN1");
    Linear* l2 = new_linear(S, S.d.ffn, S.d.d_model, name + " FFN2");
    return l2->forward(GraphOperations::GELU(l1->forward(h)));
}

graph encoder_block(Session& S, graph x, int Sq, const std::string& name) {
    const int B = S.d.batch, D = S.d.d_model, hd = D / S.d.heads;
    graph h = ln_tokens(x, B, Sq, D);
    x = GraphOperations::Add(x, attention(S, h, h, false, 1.0f / sqrtf((float)hd), name + " SelfAttn"));
    graph h2 = ln_tokens(x, B, Sq, D);
    return GraphOperations::Add(x, ffn(S, h2, name));
}

graph decoder_block(Session& S, graph x, const graph& enc, int Sq, const std::string& name) {
    const int B = S.d.batch, D = S.d.d_model, hd = D / S.d.heads;
    graph h = ln_tokens(x, B, Sq, D);
    x = GraphOperations::Add(x, attention(S, h, h, true, 1.0f / sqrtf((float)hd), name + " MaskedSelfAttn"));
    graph h2 = ln_tokens(x, B, Sq, D);
    x = GraphOperations::Add(x, attention(S, h2, enc, true, 1.0f / sqrtf((float)D), name + " CrossAttn"));
    graph h3 = ln_tokens(x, B, Sq, D);
    return GraphOperations::Add(x, ffn(S, h3, name));
}

// token ids -> embedding node (gather) and target ids -> one-hot node
// token ids -> gathered embeddings (TextualEmbedding::forward,
// Engine/transformer.cu:176-192).  A trained table's node clears its
// gradient with the step's zero_grad, as the reference's embedding node does
// (DataLoading::forward, Engine/transformer.cu:547-548).
graph token_input(Session& S, const std::string& name, int vocab, bool train = false) {
    const int B = S.d.batch, Sq = S.d.seq_len, D = S.d.d_model;
    auto node = std::make_shared<NodeBackProp>(name + " Embeddings", B, 1, Sq, D, 1);
    float* table = arena_alloc(ARENA_PARAM, (int64_t)vocab * D, name + " embedding table");
    S.emb.push_back({table, (int64_t)vocab * D});
    int32_t* keys = (int32_t*)arena_alloc_bytes(ARENA_WS, (int64_t)B * Sq * 4, name + " keys");
    add_input(S, name, 1, (int64_t)B * Sq, keys);
    S.emb_keys.push_back(keys);
    NodeBackProp* nd = node.get();
    const int64_t nk = (int64_t)B * Sq;
    S.prep.push_back([=]() { check(mle_embedding_gather(keys, table, nd->output, nk, D, st()), "GatherEmbeddings"); });
    if (train) {
        node->zero_grad = [nd]() { zero_range(nd->grad, nd->total); };
        float* gsum = arena_alloc(ARENA_WS, (int64_t)vocab * D, name + " embedding gradient");
        S.emb_train.push_back({keys, table, nd, gsum, nk, (int64_t)vocab * D, D, Sq, vocab});
    }
    return node;
}

// token ids -> gathered embeddings -> MatrixPositionalEncoding, the gather
// and the positional add as one pass writing the positional node's output
// (the embedding node's own output then has no reader); a frozen table's
// node has no gradient reader either, so the positional backward skips it.
graph token_input_pe(Session& S, const std::string& name, int vocab, bool train = false) {
    graph e = token_input(S, name, vocab, train);
    graph pe = GraphOperations::MatrixPositionalEncoding(e);
    if (!train) ext(e.get()).grad_unused = true;
    const int Sq = S.d.seq_len, D = S.d.d_model;
    const int32_t* keys = S.emb_keys.back();
    const float* table = S.emb.back().first;
    NodeBackProp* pn = pe.get();
    const float* pet = ext(pn).pe_table;
    const int64_t nk = (int64_t)S.d.batch * Sq;
    auto gather = S.prep.back();
    S.prep.back() = [=]() {
        const int s = mle_embedding_gather_add(keys, table, pet, pn->output, nk, D, Sq, st());
        if (s == MLE_ERR_UNSUPPORTED) {  // the two launches
            ext(pn).pe_fed = false;
            gather();
            return;
        }
        check(s, "GatherEmbeddings + MatPE");
        ext(pn).pe_fed = true;
    };
    return pe;
}

// EmbeddingUpdate after the backward pass: the step's gradient rows summed
// per table row; on one GPU applied at once, under data parallelism summed
// over the ranks with the gradient buckets and applied in the update phase
// with the 1/world average.
void embedding_scatter(Session& S) {
    for (auto& e : S.emb_train) {
        if (!S.dp) {
            check(mle_embedding_update(e.keys, e.node->grad, e.table, e.gsum, e.vocab, e.rows, e.dim, e.row_len,
                                       e.row_len, S.d.embed_lr, st()),
                  "EmbeddingUpdate");
            continue;
        }
        check_cuda(cudaMemsetAsync(e.gsum, 0, (size_t)e.table_n * 4, stream()), "embedding gradient clear");
        check(mle_embedding_grad_scatter(e.keys, e.node->grad, e.gsum, e.rows, e.dim, e.row_len, e.row_len, st()),
              "EmbeddingUpdate (scatter)");
    }
}

void embedding_apply(Session& S) {
    if (!S.dp) return;
    for (auto& e : S.emb_train)
        check(mle_embedding_apply(e.table, e.gsum, e.table_n, -S.d.embed_lr / (float)S.dp->world(), st()),
              "EmbeddingUpdate (averaged)");
}

graph onehot_target(Session& S, const std::string& name, int rows_b, int rows_s, int classes) {
    auto node = std::make_shared<NodeBackProp>(name, rows_b, 1, rows_s, classes, 1);
    int32_t* keys = (int32_t*)arena_alloc_bytes(ARENA_WS, (int64_t)rows_b * rows_s * 4, name + " keys");
    add_input(S, name, 1, (int64_t)rows_b * rows_s, keys);
    NodeBackProp* nd = node.get();
    const int64_t nk = (int64_t)rows_b * rows_s;
    S.prep.push_back([=]() {
        check_cuda(cudaMemsetAsync(nd->output, 0, (size_t)nd->total * 4, stream()), "one-hot clear");
        check(mle_one_hot(keys, nd->output, nk, classes, st()), "OneHotEmbeddings");
    });
    return node;
}

// Loss over a classifier's logits and the int32 class ids of input `name`
// (rows_b x rows_s of them): the index-label softmax cross-entropy, or the
// reference's dense one-hot target when the session asks for it.
graph class_loss(Session& S, const graph& logits, const std::string& name, int rows_b, int rows_s, int classes) {
    // (the index kernel takes rows of a multiple of 4 classes, up to 8192)
    if (S.d.dense_targets || classes % 4 != 0 || classes > 8192)
        return GraphOperations::SoftMaxCrossEntropy(logits, onehot_target(S, name, rows_b, rows_s, classes), true);
    int32_t* keys = (int32_t*)arena_alloc_bytes(ARENA_WS, (int64_t)rows_b * rows_s * 4, name + " keys");
    add_input(S, name, 1, (int64_t)rows_b * rows_s, keys);
    return GraphOperations::SoftMaxCrossEntropyIndex(logits, keys, true);
}

void build(Session& S) {
    const mle_session_desc& d = S.d;
    if (d.config == MLE_CFG_MLP) {
        auto x = std::make_shared<NodeBackProp>("MNIST input", d.batch, 1, 1, d.in_features, 1);
        add_input(S, "x", 0, (int64_t)d.batch * d.in_features, x->output);
        Linear* l1 = new_linear(S, d.in_features, d.hidden, "Linear1");
        Linear* l2 = new_linear(S, d.hidden, d.classes, "Linear2");
        graph logits = l2->forward(GraphOperations::RELU(l1->forward(x)));
        S.loss = class_loss(S, logits, "labels", d.batch, 1, d.classes);
    } else if (d.config == MLE_CFG_ENCODER) {
        graph x = token_input_pe(S, "tokens", d.vocab, d.embed_lr > 0);
        for (int l = 0; l < d.layers; ++l) x = encoder_block(S, x, d.seq_len, "Enc" + std::to_string(l));
        Linear* proj = new_linear(S, d.d_model, d.vocab, "Projection");
        S.loss = class_loss(S, proj->forward(x), "targets", d.batch, d.seq_len, d.vocab);
    } else if (d.config == MLE_CFG_UNET) {
        // U_NET::build_train (Engine/diffusion.cu:271-294) with three levels
        const int B = d.batch, C = d.channels, HW = d.image_size, w = d.base_width;
        auto x = std::make_shared<NodeBackProp>("x_t", B, C, HW, HW, 1);
        add_input(S, "x_t", 0, (int64_t)B * C * HW * HW, x->output);
        auto target = std::make_shared<NodeBackProp>("noise", B, C, HW, HW, 1);
        add_input(S, "noise", 0, (int64_t)B * C * HW * HW, target->output);
        // TimeMLPBlock (Engine/engine.cu:3914-3922): Linear, SiLU, Linear
        graph t_emb = GraphOperations::PositionalEncoding(d.timestep, d.t_embed);
        Linear* t0 = new_linear(S, d.t_embed, d.t_embed / 2, "Time MLP L0");
        Linear* t1 = new_linear(S, d.t_embed / 2, d.t_embed / 2, "Time MLP L1");
        graph t = t1->forward(GraphOperations::SILU(t0->forward(t_emb)));
        graph e1 = residual_block(S, x, t, C, w, 1, "Enc1");
        graph e2 = residual_block(S, e1, t, w, 2 * w, 2, "Enc2");
        graph e3 = residual_block(S, e2, t, 2 * w, 4 * w, 2, "Enc3");
        graph b0 = residual_block(S, e3, t, 4 * w, 4 * w, 1, "Bottleneck0");
        graph b1 = residual_block(S, b0, t, 4 * w, 4 * w, 1, "Bottleneck1");
        graph u1 = new_convT(S, 4 * w, 4 * w, 2, 2, 0, "UpConv 1")->forward(b1);
        graph d1 = residual_block(S, GraphOperations::CopyCrop(u1, e2), t, 6 * w, 2 * w, 1, "Dec1");
        graph u2 = new_convT(S, 2 * w, 2 * w, 2, 2, 0, "UpConv 2")->forward(d1);
        graph d2 = residual_block(S, GraphOperations::CopyCrop(u2, e1), t, 3 * w, w, 1, "Dec2");
        graph y = new_conv(S, w, C, 1, 1, 0, "Output Convolution")->forward(d2);
        S.loss = GraphOperations::MeanSquaredError(y, target, true);
    } else if (d.config == MLE_CFG_ENCDEC) {
        graph e = token_input_pe(S, "src", d.vocab, d.embed_lr > 0);
        for (int l = 0; l < d.layers; ++l) e = encoder_block(S, e, d.seq_len, "Enc" + std::to_string(l));
        graph x = token_input_pe(S, "tgt_in", d.vocab);
        for (int l = 0; l < d.layers; ++l) x = decoder_block(S, x, e, d.seq_len, "Dec" + std::to_string(l));
        Linear* proj = new_linear(S, d.d_model, d.vocab, "Projection");
        S.loss = class_loss(S, proj->forward(x), "tgt_out", d.batch, d.seq_len, d.vocab);
    }
    S.go.nodes = topological_sort(S.loss);
}

// He init for the MLP (N(0, 2/fan_in)), N(0, 0.02) for transformers; biases 0.
void init_params(Session& S) {
    std::mt19937_64 gen(S.d.seed * 0x2545F4914F6CDD1Dull + 17);
    for (AdamParameter* p : S.params) {
        std::vector<float> h((size_t)p->total, 0.0f);
        const bool is_bias = p->dim[0] == 1 && p->dim[2] == 1;  // [1,1,1,out] or [1,out,1,1]
        if (!is_bias) {
            const double stdv = (S.d.config == MLE_CFG_MLP) ? sqrt(2.0 / p->dim[2]) : 0.02;
            std::normal_distribution<double> nd(0.0, stdv);
            for (auto& x : h) x = (float)nd(gen);
        }
        check_cuda(cudaMemcpy(p->output, h.data(), h.size() * 4, cudaMemcpyHostToDevice), "param init");
    }
    std::normal_distribution<double> ne(0.0, 0.02);
    for (auto& e : S.emb) {
        std::vector<float> h((size_t)e.second);
        for (auto& x : h) x = (float)ne(gen);
        check_cuda(cudaMemcpy(e.first, h.data(), h.size() * 4, cudaMemcpyHostToDevice), "embedding init");
    }
}

// Runs one phase of the step; returns MLE_OK or the data-parallel
// reduction's status (phase 3), after which the step must not update.
int run_phase(Session& S, int phase) {
    switch (phase) {
        case 0:
            S.go.zero_grad();
            break;
        case 1:
            for (auto& f : S.prep) f();
            S.go.forward(nullptr, true);
            break;
        case 2:
            if (S.dp) S.dp->begin_backward();
            S.go.backward();
            embedding_scatter(S);
            break;
        case 3:
            if (S.dp) return S.dp->reduce_remaining(stream());
            break;
        case 4:
            if (S.d.clip_norm > 0) S.go.clip_grad_norm(S.d.clip_norm);
            break;
        case 5:
            embedding_apply(S);
            S.go.ParameterUpdate(nullptr, false, S.d.lr, S.d.adamw != 0);
            break;
    }
    return MLE_OK;
}

int step_body(Session& S, int upload, int download) {
    if (upload)
        for (auto& in : S.inputs)
            check_cuda(cudaMemcpyAsync(in.dev, in.host, (size_t)in.numel * 4, cudaMemcpyHostToDevice, S.stream),
                       "input upload");
    for (int ph = 0; ph <= 5; ++ph) {
        const int st_ = run_phase(S, ph);
        if (st_ != MLE_OK) return st_;  // gradients not reduced: leave the parameters as they are
    }
    if (download)
        check_cuda(cudaMemcpyAsync(S.loss_host, S.loss->output, sizeof(float), cudaMemcpyDeviceToHost, S.stream),
                   "loss download");
    return MLE_OK;
}

void drop_graphs(Session& S) {
    for (int i = 0; i < 2; ++i) {
        if (S.exec[i]) cudaGraphExecDestroy(S.exec[i]);
        if (S.graph_[i]) cudaGraphDestroy(S.graph_[i]);
        S.exec[i] = nullptr;
        S.graph_[i] = nullptr;
    }
    for (auto& e : S.phase_exec) {
        if (e) cudaGraphExecDestroy(e);
        e = nullptr;
    }
}

Session* as_session(mle_session_t s) { return reinterpret_cast<Session*>(s); }

}  // namespace

extern "C" {

int mle_session_create(const mle_session_desc* desc, mle_session_t* out) {
    if (!desc || !out) return MLE_ERR_ARG;
    const mle_session_desc& d = *desc;
    if (d.batch <= 0 || (d.gemm_mode != MLE_GEMM_MODE_TF32 && d.gemm_mode != MLE_GEMM_MODE_FP32)) return MLE_ERR_ARG;
    if (d.config == MLE_CFG_MLP) {
        if (d.in_features <= 0 || d.hidden <= 0 || d.classes <= 0) return MLE_ERR_ARG;
    } else if (d.config == MLE_CFG_ENCODER || d.config == MLE_CFG_ENCDEC) {
        if (d.seq_len <= 0 || d.d_model <= 0 || d.heads <= 0 || d.d_model % d.heads || d.ffn <= 0 || d.layers <= 0 ||
            d.vocab <= 0)
            return MLE_ERR_ARG;
    } else if (d.config == MLE_CFG_UNET) {
        // widths w, 2w, 3w (a concatenation), 4w, 6w go through GroupNorm(8);
        // the image halves twice
        if (d.channels <= 0 || d.base_width <= 0 || d.base_width % 8 || d.image_size <= 0 || d.image_size % 4 ||
            d.t_embed < 2 || d.t_embed % 2 || d.timestep < 0)
            return MLE_ERR_ARG;
    } else {
        return MLE_ERR_ARG;
    }
    auto* S = new Session();
    S->d = d;
    if (cudaStreamCreateWithFlags(&S->stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete S;
        return MLE_ERR_CUDA;
    }
    mle::init_param_stream();  // before any capture of the step
    mle::set_seed(d.seed);
    mle::set_keep_softmax(false);
    mle::g_loss_readback = false;
    S->param_first = all_parameters().size();
    {
        StreamScope sc(S->stream, S->d.gemm_mode);
        build(*S);
    }
    // parameters in graph order (the order ParameterUpdate visits them)
    {
        std::vector<AdamParameter*> ordered;
        for (auto& wb : S->layer_params) {
            ordered.push_back(wb.first);
            ordered.push_back(wb.second);
        }
        S->params = ordered;
    }
    init_params(*S);
    mle::check_cuda(cudaHostAlloc((void**)&S->loss_host, sizeof(float) * 4, cudaHostAllocDefault), "pinned loss");
    mle::check_cuda(cudaDeviceSynchronize(), "session build");
    *out = S;
    return MLE_OK;
}

int mle_session_destroy(mle_session_t s) {
    Session* S = as_session(s);
    if (!S) return MLE_ERR_ARG;
    cudaStreamSynchronize(S->stream);
    drop_graphs(*S);
    S->dp.reset();
    for (auto& in : S->inputs) cudaFreeHost(in.host);
    cudaFreeHost(S->loss_host);
    cudaStreamDestroy(S->stream);
    // parameters are owned by the session's Linear layers
    auto& all = all_parameters();
    for (AdamParameter* p : S->params) all.erase(std::remove(all.begin(), all.end(), p), all.end());
    S->go.nodes.clear();
    S->loss.reset();
    delete S;
    return MLE_OK;
}

void* mle_session_stream(mle_session_t s) { return s ? (void*)as_session(s)->stream : nullptr; }

int mle_session_input_count(mle_session_t s) { return s ? (int)as_session(s)->inputs.size() : -1; }

int mle_session_input_info(mle_session_t s, int i, char* name, int name_len, int64_t* numel, int* dtype,
                           void** host_ptr, void** dev_ptr) {
    Session* S = as_session(s);
    if (!S || i < 0 || i >= (int)S->inputs.size()) return MLE_ERR_ARG;
    const Input& in = S->inputs[i];
    if (name && name_len > 0) {
        std::strncpy(name, in.name.c_str(), (size_t)name_len - 1);
        name[name_len - 1] = 0;
    }
    if (numel) *numel = in.numel;
    if (dtype) *dtype = in.dtype;
    if (host_ptr) *host_ptr = in.host;
    if (dev_ptr) *dev_ptr = in.dev;
    return MLE_OK;
}

int mle_session_step(mle_session_t s, int upload, float* loss_out) {
    Session* S = as_session(s);
    if (!S) return MLE_ERR_ARG;
    StreamScope sc(S->stream, S->d.gemm_mode);
    const int g = upload ? 1 : 0;
    if (S->exec[g]) {
        if (cudaGraphLaunch(S->exec[g], S->stream) != cudaSuccess) return status_of(cudaGetLastError());
        if (loss_out && !upload)
            check_cuda(cudaMemcpyAsync(S->loss_host, S->loss->output, sizeof(float), cudaMemcpyDeviceToHost,
                                       S->stream),
                       "loss download");
    } else {
        const int st_ = step_body(*S, upload, loss_out != nullptr || upload);
        if (st_ != MLE_OK) return st_;
    }
    if (loss_out) {
        const cudaError_t e = cudaStreamSynchronize(S->stream);
        if (e != cudaSuccess) return status_of(e);
        *loss_out = *S->loss_host;
    }
    return status_of(cudaGetLastError());
}

int mle_session_phase(mle_session_t s, int phase) {
    Session* S = as_session(s);
    if (!S || phase < 0 || phase > 5) return MLE_ERR_ARG;
    StreamScope sc(S->stream, S->d.gemm_mode);
    if (phase == 1)
        for (auto& in : S->inputs)
            check_cuda(cudaMemcpyAsync(in.dev, in.host, (size_t)in.numel * 4, cudaMemcpyHostToDevice, S->stream),
                       "input upload");
    const int st_ = run_phase(*S, phase);
    if (st_ != MLE_OK) return st_;
    if (phase == 1)
        check_cuda(cudaMemcpyAsync(S->loss_host, S->loss->output, sizeof(float), cudaMemcpyDeviceToHost, S->stream),
                   "loss download");
    return status_of(cudaGetLastError());
}

int mle_session_capture(mle_session_t s) {
    Session* S = as_session(s);
    if (!S) return MLE_ERR_ARG;
    StreamScope sc(S->stream, S->d.gemm_mode);
    drop_graphs(*S);
    cudaError_t e = cudaStreamSynchronize(S->stream);
    if (e != cudaSuccess) return status_of(e);
    for (int g = 0; g < 2; ++g) {
        e = cudaStreamBeginCapture(S->stream, cudaStreamCaptureModeThreadLocal);
        if (e != cudaSuccess) return status_of(e);
        const int st_ = step_body(*S, g, g);
        e = cudaStreamEndCapture(S->stream, &S->graph_[g]);
        if (st_ != MLE_OK) {
            drop_graphs(*S);
            return st_;
        }
        if (e != cudaSuccess) return status_of(e);
        e = cudaGraphInstantiate(&S->exec[g], S->graph_[g], 0);
        if (e != cudaSuccess) return status_of(e);
    }
    return MLE_OK;
}

int mle_session_capture_phases(mle_session_t s) {
    Session* S = as_session(s);
    if (!S) return MLE_ERR_ARG;
    StreamScope sc(S->stream, S->d.gemm_mode);
    for (auto& e : S->phase_exec) {
        if (e) cudaGraphExecDestroy(e);
        e = nullptr;
    }
    cudaError_t e = cudaStreamSynchronize(S->stream);
    if (e != cudaSuccess) return status_of(e);
    for (int ph = 0; ph < 6; ++ph) {
        // under data parallelism the backward issues bucket reductions on
        // the communication stream that only phase 3 joins: both phases
        // go into phase 2's graph, and phase 3's is empty
        if (ph == 3 && S->dp) continue;
        e = cudaStreamBeginCapture(S->stream, cudaStreamCaptureModeThreadLocal);
        if (e != cudaSuccess) return status_of(e);
        int st_ = run_phase(*S, ph);
        if (ph == 2 && S->dp && st_ == MLE_OK) st_ = run_phase(*S, 3);
        cudaGraph_t g = nullptr;
        e = cudaStreamEndCapture(S->stream, &g);
        if (st_ != MLE_OK || e != cudaSuccess) {
            if (g) cudaGraphDestroy(g);
            return st_ != MLE_OK ? st_ : status_of(e);
        }
        e = cudaGraphInstantiate(&S->phase_exec[ph], g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) return status_of(e);
    }
    return MLE_OK;
}

int mle_session_phase_replay(mle_session_t s, int phase) {
    Session* S = as_session(s);
    if (!S || phase < 0 || phase > 5) return MLE_ERR_ARG;
    if (phase == 3 && S->dp && S->phase_exec[2]) return MLE_OK;  // captured with phase 2
    if (!S->phase_exec[phase]) return MLE_ERR_ARG;
    return status_of(cudaGraphLaunch(S->phase_exec[phase], S->stream));
}

int mle_session_sync(mle_session_t s) {
    Session* S = as_session(s);
    if (!S) return MLE_ERR_ARG;
    return status_of(cudaStreamSynchronize(S->stream));
}

int mle_session_param_count(mle_session_t s) { return s ? (int)as_session(s)->params.size() : -1; }

int mle_session_param_info(mle_session_t s, int i, char* name, int name_len, int64_t* numel) {
    Session* S = as_session(s);
    if (!S || i < 0 || i >= (int)S->params.size()) return MLE_ERR_ARG;
    AdamParameter* p = S->params[i];
    if (name && name_len > 0) {
        std::strncpy(name, p->op_name.c_str(), (size_t)name_len - 1);
        name[name_len - 1] = 0;
    }
    if (numel) *numel = p->total;
    return MLE_OK;
}

static float* param_buf(AdamParameter* p, int which) {
    switch (which) {
        case 0: return p->output;
        case 1: return p->grad;
        case 2: return p->m;
        case 3: return p->v;
        default: return nullptr;
    }
}

int mle_session_param_read(mle_session_t s, int i, int which, float* host) {
    Session* S = as_session(s);
    if (!S || i < 0 || i >= (int)S->params.size() || !host) return MLE_ERR_ARG;
    float* src = param_buf(S->params[i], which);
    if (!src) return MLE_ERR_ARG;
    cudaError_t e = cudaStreamSynchronize(S->stream);
    if (e == cudaSuccess) e = cudaMemcpy(host, src, (size_t)S->params[i]->total * 4, cudaMemcpyDeviceToHost);
    return status_of(e);
}

int mle_session_param_write(mle_session_t s, int i, int which, const float* host) {
    Session* S = as_session(s);
    if (!S || i < 0 || i >= (int)S->params.size() || !host) return MLE_ERR_ARG;
    float* dst = param_buf(S->params[i], which);
    if (!dst) return MLE_ERR_ARG;
    cudaError_t e = cudaStreamSynchronize(S->stream);
    if (e == cudaSuccess) e = cudaMemcpy(dst, host, (size_t)S->params[i]->total * 4, cudaMemcpyHostToDevice);
    return status_of(e);
}

int mle_session_param_step(mle_session_t s, int i, int* t) {
    Session* S = as_session(s);
    if (!S || i < 0 || i >= (int)S->params.size() || !t) return MLE_ERR_ARG;
    StreamScope sc(S->stream, S->d.gemm_mode);
    S->params[i]->sync_step();
    *t = S->params[i]->t;
    return MLE_OK;
}

// Checkpoints: every parameter of the session in build order as the
// reference's AdamParameter::save records (u32 name length, name, i32 count,
// f32 weights, m, v; Engine/engine.cu:139-188), the file a use case gets
// from calling save() on its layers in the same order.  The reference does
// not save the Adam step t; `<path>.t` holds it (i32 count, then one i32 per
// parameter) so a resumed run continues the bias corrections.  Under data
// parallelism only rank 0 writes.  Loading checks every record's name and
// size before touching a parameter.
static bool read_record_header(std::ifstream& f, std::string& name, int& total) {
    uint32_t len = 0;
    if (!f.read(reinterpret_cast<char*>(&len), sizeof(len)) || len > (1u << 20)) return false;
    name.assign(len, '\0');
    if (len && !f.read(&name[0], len)) return false;
    return (bool)f.read(reinterpret_cast<char*>(&total), sizeof(int));
}

int mle_session_save(mle_session_t s, const char* path) {
    Session* S = as_session(s);
    if (!S || !path) return MLE_ERR_ARG;
    if (S->dp && S->dp->rank() != 0) return MLE_OK;
    StreamScope sc(S->stream, S->d.gemm_mode);
    if (cudaStreamSynchronize(S->stream) != cudaSuccess) return MLE_ERR_CUDA;
    {
        std::ofstream f(path, std::ios::binary | std::ios::trunc);
        if (!f) return MLE_ERR_ARG;
        for (AdamParameter* p : S->params) p->save(f);
        if (!f) return MLE_ERR_ARG;
    }
    std::ofstream t(std::string(path) + ".t", std::ios::binary | std::ios::trunc);
    if (!t) return MLE_ERR_ARG;
    const int n = (int)S->params.size();
    t.write(reinterpret_cast<const char*>(&n), sizeof(n));
    for (AdamParameter* p : S->params) {
        p->sync_step();
        const int32_t v = p->t;
        t.write(reinterpret_cast<const char*>(&v), sizeof(v));
    }
    return t ? MLE_OK : MLE_ERR_ARG;
}

int mle_session_load(mle_session_t s, const char* path) {
    Session* S = as_session(s);
    if (!S || !path) return MLE_ERR_ARG;
    StreamScope sc(S->stream, S->d.gemm_mode);
    {
        // names and sizes first, so a mismatched file changes nothing
        std::ifstream f(path, std::ios::binary);
        if (!f) return MLE_ERR_ARG;
        for (AdamParameter* p : S->params) {
            std::string name;
            int total = 0;
            if (!read_record_header(f, name, total) || name != p->op_name || total != (int)p->total)
                return MLE_ERR_ARG;
            if (!f.seekg((std::streamoff)total * 3 * (std::streamoff)sizeof(float), std::ios::cur)) return MLE_ERR_ARG;
        }
    }
    if (cudaStreamSynchronize(S->stream) != cudaSuccess) return MLE_ERR_CUDA;
    std::ifstream f(path, std::ios::binary);
    for (AdamParameter* p : S->params) p->load(f);
    std::ifstream t(std::string(path) + ".t", std::ios::binary);
    int n = 0;
    if (t && t.read(reinterpret_cast<char*>(&n), sizeof(n)) && n == (int)S->params.size()) {
        for (AdamParameter* p : S->params) {
            int32_t v = 0;
            if (!t.read(reinterpret_cast<char*>(&v), sizeof(v)) || v < 1) return MLE_ERR_ARG;
            p->t = v;
            if (cudaMemcpy(p->t_dev, &v, sizeof(v), cudaMemcpyHostToDevice) != cudaSuccess) return MLE_ERR_CUDA;
        }
    }
    return MLE_OK;
}

int mle_session_embedding_count(mle_session_t s) { return s ? (int)as_session(s)->emb.size() : -1; }

int mle_session_embedding_write(mle_session_t s, int i, const float* host, int64_t numel) {
    Session* S = as_session(s);
    if (!S || i < 0 || i >= (int)S->emb.size() || !host || numel != S->emb[i].second) return MLE_ERR_ARG;
    cudaError_t e = cudaStreamSynchronize(S->stream);
    if (e == cudaSuccess) e = cudaMemcpy(S->emb[i].first, host, (size_t)numel * 4, cudaMemcpyHostToDevice);
    return status_of(e);
}

int mle_session_embedding_read(mle_session_t s, int i, float* host, int64_t numel) {
    Session* S = as_session(s);
    if (!S || i < 0 || i >= (int)S->emb.size() || !host || numel != S->emb[i].second) return MLE_ERR_ARG;
    cudaError_t e = cudaStreamSynchronize(S->stream);
    if (e == cudaSuccess) e = cudaMemcpy(host, S->emb[i].first, (size_t)numel * 4, cudaMemcpyDeviceToHost);
    return status_of(e);
}

int mle_session_device_bytes(mle_session_t s, int64_t* bytes) {
    if (!s || !bytes) return MLE_ERR_ARG;
    double gib = 0;
    for (int a = 0; a < ARENA_COUNT; ++a) gib += arena_gib((Arena)a);
    *bytes = (int64_t)(gib * (double)(1ull << 30));
    return MLE_OK;
}

int mle_session_node_count(mle_session_t s) { return s ? (int)as_session(s)->go.nodes.size() : -1; }

int mle_set_param_grad_stream(int enable) {
    if (enable != 0 && enable != 1) return MLE_ERR_ARG;
    mle::set_param_stream_enabled(enable != 0);
    return MLE_OK;
}

int mle_get_param_grad_stream(void) { return mle::param_stream_enabled() ? 1 : 0; }

int mle_set_grad_first_write(int enable) {
    if (enable != 0 && enable != 1) return MLE_ERR_ARG;
    mle::set_first_write_assign(enable != 0);
    return MLE_OK;
}

int mle_get_grad_first_write(void) { return mle::first_write_assign() ? 1 : 0; }

int mle_session_graph_counts(mle_session_t s, int* kernels, int* memsets, int* copies) {
    Session* S = as_session(s);
    if (!S || !kernels || !memsets || !copies) return MLE_ERR_ARG;
    *kernels = *memsets = *copies = 0;
    if (!S->graph_[0]) return MLE_ERR_UNSUPPORTED;
    size_t n = 0;
    if (cudaGraphGetNodes(S->graph_[0], nullptr, &n) != cudaSuccess) return MLE_ERR_CUDA;
    std::vector<cudaGraphNode_t> nodes(n);
    if (cudaGraphGetNodes(S->graph_[0], nodes.data(), &n) != cudaSuccess) return MLE_ERR_CUDA;
    for (auto nd : nodes) {
        cudaGraphNodeType t;
        cudaGraphNodeGetType(nd, &t);
        if (t == cudaGraphNodeTypeKernel) ++*kernels;
        else if (t == cudaGraphNodeTypeMemset) ++*memsets;
        else if (t == cudaGraphNodeTypeMemcpy) ++*copies;
    }
    return MLE_OK;
}

int mle_session_graph_edges(mle_session_t s, int* edges, int* programmatic) {
    Session* S = as_session(s);
    if (!S || !edges || !programmatic) return MLE_ERR_ARG;
    *edges = *programmatic = 0;
    if (!S->graph_[0]) return MLE_ERR_UNSUPPORTED;
    size_t n = 0;
    if (cudaGraphGetEdges_v2(S->graph_[0], nullptr, nullptr, nullptr, &n) != cudaSuccess) return MLE_ERR_CUDA;
    std::vector<cudaGraphNode_t> from(n), to(n);
    std::vector<cudaGraphEdgeData> data(n);
    if (n && cudaGraphGetEdges_v2(S->graph_[0], from.data(), to.data(), data.data(), &n) != cudaSuccess)
        return MLE_ERR_CUDA;
    *edges = (int)n;
    for (size_t i = 0; i < n; ++i)
        if (data[i].type == cudaGraphDependencyTypeProgrammatic) ++*programmatic;
    return MLE_OK;
}

int mle_session_enable_dp(mle_session_t s, const uint8_t* id128, int rank, int world, int bucket_mb) {
    Session* S = as_session(s);
    if (!S || !id128 || world <= 0 || rank < 0 || rank >= world) return MLE_ERR_ARG;
    std::vector<GradSpan> grads;
    for (AdamParameter* p : S->params) grads.push_back({p->grad, p->total, arena_chunk_of(p->grad)});
    std::unique_ptr<DataParallel> dp(new DataParallel());
    const int st_ = dp->init(id128, rank, world, grads, bucket_mb, S->stream);
    if (st_ != MLE_OK) return st_;
    for (auto& e : S->emb_train)
        if (dp->add_dense(e.gsum, e.table_n) != MLE_OK) return MLE_ERR_CUDA;
    S->dp = std::move(dp);
    S->go.set_grad_prescale(1.0f / (float)world);
    DataParallel* d = S->dp.get();
    S->go.on_backward_done = [d](const NodeBackProp* n) {
        const std::vector<float*>& g = ext(n).param_grads;
        if (!g.empty()) d->grads_done(g, stream());
    };
    return MLE_OK;
}

}  // extern "C"
