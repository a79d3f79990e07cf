// engine.h -- B200-native replacement for ML_Engine's Includes/engine.h
// (training hot path).
//
// Declarations keep the reference's names, argument lists, default
// arguments and public fields (Includes/engine.h:33-213) so programs written
// against the reference compile and link unchanged for the ops on the path.
// What differs is underneath:
//   * every launch goes through the C ABI of include/mle_kernels.h on one
//     compute stream (mle::stream(); the legacy default stream unless a
//     session selects its own), with no device synchronisation in forward
//     or backward;
//   * node and parameter buffers are carved from static graph-build arenas
//     (still allocated once, when the graph is built), so zero_grad clears
//     coalesced ranges and the optimizer sees contiguous parameter storage;
//   * GraphOperations::ParameterUpdate, accumulate and clipNorm gather the
//     AdamParameters their lambdas touch and issue one fused multi-tensor
//     launch instead of one launch per tensor;
//   * AdamParameter::t is mirrored in device memory so a captured CUDA graph
//     replays the per-tensor step counter.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <fstream>
#include <functional>
#include <iostream>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include <type_traits>

#include "debugging_utils.h"
#include "kernels.h"
#include "mle_kernels.h"

struct NodeBackProp;
struct AdamParameter;
using graph = std::shared_ptr<NodeBackProp>;
using graph_tree = std::vector<graph>;
using graphFn = std::function<graph(graph)>;

namespace mle {

// Compute stream used by every op (default: legacy stream 0).
cudaStream_t stream();
void set_stream(cudaStream_t s);

// Parameter-gradient stream.  A backward lambda may put work that only
// parameter gradients depend on (a Linear layer's weight and bias
// gradients) on a second stream: fork_param_stream() makes that stream wait
// for everything issued on the compute stream so far and returns it (the
// compute stream itself when the feature is off), so the input-gradient
// chain goes on without waiting for those products.  GraphOperations::
// backward joins it back before returning (join_param_stream), so callers
// see every gradient complete on the compute stream, and a CUDA-graph
// capture of the backward holds both branches.
void init_param_stream();            // creates the stream (outside a capture)
cudaStream_t fork_param_stream();
void join_param_stream();
bool param_stream_pending();         // forked since the last join
cudaStream_t param_stream();         // the second stream (nullptr before init)
void set_param_stream_enabled(bool on);
bool param_stream_enabled();

// First-writer assignment: a gradient whose first writer in the backward
// walk overwrites all of it (see prepare_fusions) is not cleared by
// zero_grad, and that writer assigns instead of adding.  The results are
// those of adding into a cleared buffer, bit for bit.  On by default.
void set_first_write_assign(bool on);
bool first_write_assign();

// Maps a non-zero mle_status onto the reference's behaviour: print the
// reason and exit(1) (Engine/debug.cu:15-25).
void check(int status, const str& what);

// Static graph-build arenas.  Memory is handed out in 256-byte aligned
// slices of large cudaMalloc'ed chunks and only returned by release_all().
enum Arena { ARENA_ACT = 0, ARENA_GRAD = 1, ARENA_PARAM = 2, ARENA_PARAM_GRAD = 3, ARENA_WS = 4, ARENA_COUNT = 5 };
float* arena_alloc(Arena a, int64_t n_floats, const str& name);
void* arena_alloc_bytes(Arena a, int64_t bytes, const str& name);
double arena_gib(Arena a);
void release_all_arenas();

// Zeroing of many small ranges, coalesced into as few memsets as possible
// while a ZeroBatch is alive (GraphOperations::zero_grad keeps one open).
void zero_range(float* p, int64_t n);
struct ZeroBatch {
    ZeroBatch();
    ~ZeroBatch();
};

// Every AdamParameter ever constructed, in construction order.
std::vector<AdamParameter*>& all_parameters();

// Seed for parameter initialisation (Standard_Weights draws from
// std::random_device in the reference; a fixed seed makes runs repeatable).
void set_seed(uint64_t seed);

// Global gradient-norm workspace (one double) used by clip_grad_norm.
double* clip_workspace();

}  // namespace mle

struct NodeBackProp {
    str op_name;
    graph_tree inputs;
    float* output;
    float* grad;
    int dim[4];
    long long total;
    bool forward_called = false;
    std::function<void()> forward;
    std::function<void()> backward;
    std::function<void()> free;
    std::function<void()> zero_grad;
    std::function<void()> serious_free;
    std::function<void(const float lr, const bool adamw)> updateParams;
    std::function<void(const double*)> clipnorm;
    std::function<void(double*)> accumulate;
    std::function<void(const bool full)> printparams;
    virtual void update(const float lr = LEARNING_RATE, const bool W = ADAMW) {}
    NodeBackProp(str name, int batch, int d1, int d2, int d3, int allocation);
    virtual ~NodeBackProp();
    void clear();
    void reshape(std::vector<int> new_dims);
    void reshape(int arr[], const int size = 4);
};

float ReadValueAt(const graph& X, const int& idx, const bool flag = false);
void WriteValueAt(const graph& X, const float value, const int& idx, const bool flag = false);

struct AdamParameter : public NodeBackProp {
    float *m, *v;
    int t;
    float b1, b2, epsilon;
    int batch_size;
    float group_norm;
    float weight_decay;
    int32_t* t_dev;  // device mirror of t, read and advanced by the fused update

    AdamParameter(str n, int out, int in, int row, int col, double norm = NORM);
    void save(std::ofstream& f) const;
    void load(std::ifstream& f);
    void update(const float lr = LEARNING_RATE, const bool W = ADAMW) override;
    void accumulate_grad(double* global_scale);
    void gradnorm(const double* global_scale);
    void operator=(const AdamParameter& other);
    // copies the device step counter back into t
    void sync_step();
};

void Dimension(graph X);
void Dimension(AdamParameter X);
void Zerograd(AdamParameter X);
void Zerograd(graph X);
graph_tree topological_sort(const graph& root);

namespace mle {
// Counts the NaNs of a device array on the compute stream and waits; on any
// prints `what` and exits(1).  The reference's ISNAN kernel traps the GPU
// instead (Includes/kernels.h:381-391), which this never does.
void nan_check(const str& what, const float* x, long long n);
}  // namespace mle

// NaN checks (Includes/engine.h:20-29, Engine/engine.cu:328-348): type 0
// the output, otherwise the gradient.
template <typename numeric>
void isNan(const str name, const numeric* X, const long long total) {
    static_assert(std::is_same<numeric, float>::value, "isNan checks float tensors");
    mle::nan_check(name + "   has nan value", X, total);
}
void isNan(graph X, const int type = 0);
void isNan(AdamParameter X, const int type = 0);

// Host prints of a node's output (type 0) or gradient: every element per
// batch and channel, or the top-left 3 x 5 x 5 corner (Engine/engine.cu:
// 350-474).
void printGPU(const graph X, const int type = 0);
void printGPU(AdamParameter X, const int type = 0);
void printHeadGPU(const graph X, const int type = 0);
void printHeadGPU(AdamParameter X, const int type = 0);

// Index of the largest element of a [1, 1, 1, D] node (the first on ties),
// or a sample from its k largest entries taken in proportion to their values
// (Engine/engine.cu:564-646); the overloads with X use that int of device
// memory as the result slot, the others a slot of their own.
int ArgMaxToCPU(const graph& input, int* X);
int TopKSampleToCPU(const graph& input, int* X, const int k);
int ArgMaxToCPU(const graph& input);
int TopKSampleToCPU(const graph& input, const int k);

// Fills a node's output with Gaussian ("gaussian") or uniform ("uniform")
// noise of the given mean and spread (Engine/engine.cu:3936-3944).
void Noise(const graph& input, const float mean = 0.f, const float std = 1.f, const str type = "gaussian");

class Linear;

class GraphOperations {
   private:
    static bool calculate_loss;
    void clipNorm(double* global_scale);
    void accumulate(double* global_scale);

   public:
    graph_tree nodes;

    static double GB;
    static float loss;

    void ParameterUpdate(const graph& X = nullptr, const bool show = false, const float lr = LEARNING_RATE,
                         const bool adamw = ADAMW);
    void forward(const graph& X = nullptr, const bool calc_loss = false, const bool show = false,
                 const bool time = false, const bool check_nan = false);
    void backward(const graph& X = nullptr, const bool show = false, const bool time = false,
                  const bool check_nan = false);
    void zero_grad(const graph& X = nullptr, const bool show = false);
    void printParams(const graph& X = nullptr, const bool show = false);
    void printNodes(const graph& X = nullptr, const int show = 0);
    void clear_graph(const graph& X = nullptr, const bool show = false);
    void clean_clear_graph(const graph& X = nullptr, const bool show = false);

    // Public gradient-norm clip (the reference keeps accumulate/clipNorm
    // private and never calls them, Includes/engine.h:112-113).  Computes
    // s = max(||g||_2 / max_norm, 1) over every parameter of `nodes`; the
    // division g /= s is applied by the next ParameterUpdate inside the
    // fused update (and written back to the gradients), or immediately by
    // apply_clip().
    void clip_grad_norm(const float max_norm = NORM);
    void apply_clip();
    // Multiplies every gradient by `scale` inside the next update and
    // before the norm (data-parallel averaging).
    void set_grad_prescale(float scale) { grad_prescale_ = scale; }
    // Called after each node's backward lambda has been issued (data
    // parallelism starts a bucket's reduction as soon as its last gradient
    // is complete).
    std::function<void(const NodeBackProp*)> on_backward_done;

    static graph Copy(const graph& X);
    static graph identity(const graph& X);
    static graph like(const graph& X, const str name = "");
    static graph MatrixPositionalEncoding(const graph& X, const int start_idx = 0);
    static graph PositionalEncoding(const int& t, const int d_model);
    static graph HeadifytoChannel(const graph& X, const int new_channels);
    static graph DeHeadify(const graph& X);
    static graph Bias_Add(const graph& A, const graph& B);
    static graph Broadcast_Channel(const graph& A, const graph& B);
    static graph Scale(const graph& input, const float scale, const bool last = false);
    static graph Add(const graph& A, const graph& B, const bool last = false);
    static graph Subtract(const graph& A, const graph& B, const bool last = false);
    static graph Multiply(const graph& A, const graph& B);

    static graph MeanSquaredError(const graph& prediction, const graph& target, const bool last);
    static graph SoftMaxCrossEntropy(const graph& prediction, const graph& target, const bool last);
    // Extension: the target as one int32 class index per row of `prediction`
    // (device memory, rows = dim0*dim1*dim2), same loss and gradient as the
    // dense one-hot target without building it.
    static graph SoftMaxCrossEntropyIndex(const graph& prediction, const int32_t* labels, const bool last);

    static graph BMM(const graph& A, const graph& B);     // m x n, n x p = m x p
    static graph BMMABT(const graph& A, const graph& B);  // m x n, p x n = m x p
    static graph BMMATB(const graph& A, const graph& B);  // n x m, n x p = m x p
    static graph BMMT(const graph& A, const graph& B);    // n x m, p x n = m x p

    static graph SOFTMAX(const graph& X, const int type = 0);
    static graph SOFTMASK(const graph& X, const int type = 0);

    static graph RELU(const graph& input);
    static graph SILU(const graph& input);
    static graph TANH(const graph& input);
    static graph GELU(const graph& input);
    static graph SIGMOID(const graph& input);
    static graph LeakyRELU(const graph& input);

    static graph CopyCrop(const graph& input1, const graph& input2);

    static graph LayerNorm(const graph& X);
    static graph GroupNorm(const graph& X, const int group = 8);

    // Extension: the whole attention sub-graph of MultiHeadAttention
    // (Headify x3, BMMABT, Scale, SOFTMAX/SOFTMASK type `axis`, BMM,
    // DeHeadify; Engine/transformer.cu:647-675) as one node over the flat
    // [B,1,S,H*hd] projections, forward on the tensor cores and backward
    // through mle_attention_flash_bwd (the scores never in HBM) where it
    // applies, else mle_attention_bwd.  key_grad_mode selects the
    // reference's BMMABT key gradient (default) or the mathematical one.
    static graph ScaledDotAttention(const graph& Q, const graph& K, const graph& V, const int heads, const float scale,
                                    const bool mask, const int axis = 1,
                                    const int key_grad_mode = MLE_KEYGRAD_REFERENCE);

    // Extension: several Linear layers that read the same input X (the
    // query/key/value projections of MultiHeadAttention) with one tensor-core
    // launch for their forward and one each for their dX and dW; returns one
    // node per layer with Linear::forward's semantics.
    static std::vector<graph> LinearGroup(const graph& X, const std::vector<Linear*>& layers);

   private:
    float grad_prescale_ = 1.0f;
    bool clip_pending_ = false;
    // clip_grad_norm left to the update's single launch (norm, clip,
    // Adam/AdamW, step counters), whose tensor table lives in fused_ws_
    bool clip_deferred_ = false;
    float clip_max_norm_ = 0.0f;
    void* fused_ws_ = nullptr;
    int64_t fused_ws_bytes_ = 0;
    std::vector<mle_param_view> fused_views_;
    void flush_deferred_clip();
    bool fused_update(const std::vector<AdamParameter*>& ps, float lr, bool adamw);
    void collect_params(std::vector<AdamParameter*>& out);
};

inline graph operator+(const graph& A, const graph& B) { return GraphOperations::Add(A, B); }
inline graph operator-(const graph& A, const graph& B) { return GraphOperations::Subtract(A, B); }
inline graph operator*(const graph& A, const graph& B) { return GraphOperations::Multiply(A, B); }

class Linear {
   private:
    int in, out;
    const bool bias;

   public:
    AdamParameter W1;
    AdamParameter B1;
    str op_name = "Linear Layer";
    Linear(const int input, const int output, const str name = "", const bool bias = true);
    graph forward(const graph& X);
    void save(std::ofstream& f) const;
    void load(std::ifstream& f);
    void operator=(const Linear& other);
    int inputs() const { return in; }
    int outputs() const { return out; }
    bool has_bias() const { return bias; }
};

// Convolute2D (Includes/engine.h:235-255): weights [out][inp][C][D], NCHW.
class Convolute2D {
   public:
    int inp, out, c, d, pad, stride;
    str name;
    AdamParameter W1, B1;
    Convolute2D(int Input, int Output, int C = 3, int D = 3, int stride = 1, int padding = 1, str param = "");
    void save(std::ofstream& f) const;
    void load(std::ifstream& f);
    graph forward(const graph& X);
};

// Convolute2DT (Includes/engine.h:257-280): weights [out][inp][C][D].
class Convolute2DT {
   private:
    graph T_node;
    int inp, out, c, d, pad, stride;

   public:
    str name;
    AdamParameter W1, B1;
    Convolute2DT(int Input, int Output, int C = 2, int D = 2, int stride = 2, int padding = 0, str param = "");
    void save(std::ofstream& f) const;
    void load(std::ifstream& f);
    graph forward(const graph& X);
};

// TimeMLPBlock (Includes/engine.h:282-290, Engine/engine.cu:3914-3924):
// Linear, SiLU, Linear.
class TimeMLPBlock {
   public:
    Linear L0, L1;
    TimeMLPBlock(const int t_embed_dim, const int t_hidden);
    graph forward(const graph& X);
    void save(std::ofstream& f) const;
    void load(std::ifstream& f);
};

// Multi_Linear_Residual_Block (Includes/engine.h:292-319, Engine/engine.cu:
// 3926-3934): an input Linear, `num_residuals` residual groups of `layers`
// hidden Linears with the caller's activation, each group added back and
// normalised with the caller's norm, and an output Linear.
class Multi_Linear_Residual_Block {
   public:
    const int input_dim, output_dim, residuals, hidden_dim, layers;
    std::vector<Linear*> sequence;
    Multi_Linear_Residual_Block(const int input, const int output, const int num_residuals, const int layers,
                                const int hidden_size);
    template <typename ActFn, typename NormFn>
    graph forward(const graph& X, ActFn activation, NormFn norm) {
        graph H = sequence[0]->forward(X);
        for (int r = 0; r < residuals; ++r) {
            graph A = H;
            for (int j = 0; j < layers; ++j) {
                const int idx = r * layers + j + 1;
                if (idx < residuals * layers) A = activation(sequence[idx]->forward(A));
            }
            H = norm(H + A);
        }
        return sequence[residuals * layers]->forward(H);
    }
    void save(std::ofstream& f) const;
    void load(std::ifstream& f);
};
