// Host-side utilities of the reference's engine API that use cases call
// around the training step: NaN checks, prints, arg-max / top-k sampling to
// the host, noise fills, the Timing helper, and two layer classes built
// from Linear (TimeMLPBlock, Multi_Linear_Residual_Block).  Each keeps the
// reference's signature and observable behaviour (cited per function); the
// device work goes through include/mle_kernels.h on the compute stream.
#include <stdio.h>

#include <algorithm>
#include <random>
#include <vector>

#include "engine.h"
#include "engine_internal.h"

using namespace mle;

namespace mle {

void nan_check(const str& what, const float* x, long long n) {
    if (!x || n <= 0) return;
    static unsigned long long* d_count = nullptr;  // one slot per process, made on first use
    if (!d_count) check_cuda(cudaMalloc((void**)&d_count, sizeof(unsigned long long)), "isNan counter");
    check(mle_count_nan(x, n, d_count, stream()), what);
    unsigned long long h = 0;
    check_cuda(cudaStreamSynchronize(stream()), what);
    check_cuda(cudaMemcpy(&h, d_count, sizeof(h), cudaMemcpyDeviceToHost), what);
    if (h) {
        printf("%llu NaN value(s)\\n", h);
        std::cerr << "Runtime error in " << what << std::endl;
        std::exit(1);
    }
}

}  // namespace mle

// --------------------------------------------------- isNan (:328-348)
void isNan(graph X, const int type) {
    mle::nan_check(X->op_name + (type == 0 ? "output" : "grad") + " has nan value", type == 0 ? X->output : X->grad,
                   X->total);
}

void isNan(AdamParameter X, const int type) {
    mle::nan_check(X.op_name + (type == 0 ? "output" : "grad") + " has nan value", type == 0 ? X.output : X.grad,
                   X.total);
}

// --------------------------------------------- printGPU (:350-418)
static std::vector<float> to_host(const float* p, long long n) {
    std::vector<float> h((size_t)std::max<long long>(n, 0));
    check_cuda(cudaStreamSynchronize(stream()), "print");
    if (n > 0) check_cuda(cudaMemcpy(h.data(), p, (size_t)n * sizeof(float), cudaMemcpyDeviceToHost), "print");
    return h;
}

static void print_all(const str& name, const float* p, const int* dim, long long total, int type) {
    const std::vector<float> h = to_host(p, total);
    std::cout << "Printing dimensions for node " << name << (type == 0 ? "->output \n" : "->grad \n");
    for (int b = 0; b < dim[0]; ++b) {
        std::cout << "_____________________________________ \n";
        std::cout << " -----BATCH " << b << "-----  \n";
        for (int c = 0; c < dim[1]; ++c) {
            std::cout << "Channel " << c << ":\n";
            for (int r = 0; r < dim[2]; ++r) {
                for (int k = 0; k < dim[3]; ++k)
                    std::cout << h[(size_t)(((long long)b * dim[1] + c) * dim[2] + r) * dim[3] + k] << "\t";
                std::cout << "\n";
            }
            std::cout << "------------------------------\n";
        }
        std::cout << "_____________________________________ \n \n \n";
    }
}

void printGPU(const graph X, const int type) { print_all(X->op_name, type == 0 ? X->output : X->grad, X->dim, X->total, type); }
void printGPU(AdamParameter X, const int type) { print_all(X.op_name, type == 0 ? X.output : X.grad, X.dim, X.total, type); }

// ------------------------------------------ printHeadGPU (:420-474)
void printHeadGPU(const graph X, const int type) {
    check_cuda(cudaStreamSynchronize(stream()), "printHeadGPU");
    if (type == 0) printHeadGPU(X->op_name, X->output, X->dim[1], X->dim[2], X->dim[3], (int)X->total);
    else printHeadGrad(X->op_name, X->grad, X->dim[1], X->dim[2], X->dim[3], (int)X->total);
}

void printHeadGPU(AdamParameter X, const int type) {
    check_cuda(cudaStreamSynchronize(stream()), "printHeadGPU");
    if (type == 0) printHeadGPU(X.op_name, X.output, X.dim[1], X.dim[2], X.dim[3], (int)X.total);
    else printHeadGrad(X.op_name, X.grad, X.dim[1], X.dim[2], X.dim[3], (int)X.total);
}

// ------------------------------ ArgMaxToCPU / TopKSampleToCPU (:564-646)
static void require_row(const graph& input, const char* what) {
    for (int i = 0; i < 3; ++i)
        if (input->dim[i] != 1) {
            printf("%s: dimension does not match the required (1 x 1 x 1 x D)\n", what);
            Dimension(input);
            std::exit(1);
        }
}

int ArgMaxToCPU(const graph& input, int* X) {
    require_row(input, "ArgMaxToCPU");
    check(mle_argmax(input->output, input->total, X, st()), "ArgMax");
    int id = 0;
    check_cuda(cudaStreamSynchronize(stream()), "ArgMaxToCPU");
    check_cuda(cudaMemcpy(&id, X, sizeof(int), cudaMemcpyDeviceToHost), "ArgMaxToCPU");
    return id;
}

int ArgMaxToCPU(const graph& input) {
    int* X = nullptr;
    SafeCudaMalloc("X", X, 1);
    const int id = ArgMaxToCPU(input, X);
    cudaFree(X);
    return id;
}

// The k largest entries in the reference's order (descending; of equal
// values the earlier index first), normalised by their sum (1 if the sum is
// below 1e-8), and the first whose running sum reaches a uniform draw in
// (1e-7, 1 - 1e-7); the last of the k if none does (TopKSampleKernel,
// Engine/kernels.cu:2298-2351).  The k values are selected on the host from
// the row the call copies back, since the result goes to the host anyway.
static int topk_sample(const std::vector<float>& row, int k, float rand_val) {
    const int n = (int)row.size();
    k = std::min(k, n);
    std::vector<int> idx((size_t)n);
    for (int i = 0; i < n; ++i) idx[(size_t)i] = i;
    std::partial_sort(idx.begin(), idx.begin() + k, idx.end(), [&](int a, int b) {
        return row[(size_t)a] > row[(size_t)b] || (row[(size_t)a] == row[(size_t)b] && a < b);
    });
    float sum = 0.f;
    for (int i = 0; i < k; ++i) sum += row[(size_t)idx[(size_t)i]];
    if (sum < 1e-8f) sum = 1.0f;
    float left = rand_val;
    for (int i = 0; i < k; ++i) {
        left -= row[(size_t)idx[(size_t)i]] / sum;
        if (left <= 0.0f) return idx[(size_t)i];
    }
    return idx[(size_t)(k - 1)];
}

int TopKSampleToCPU(const graph& input, int* X, const int k) {
    require_row(input, "TopKSample");
    if (k > THREADSPERBLOCK || k < 1) {
        printf("TopKSample: k must be in [1, %d], got %d\n", THREADSPERBLOCK, k);
        std::exit(1);
    }
    static std::mt19937 gen(std::random_device{}());
    static std::uniform_real_distribution<float> dist(1e-7f, 1.0f - 1e-7f);
    const int id = topk_sample(to_host(input->output, input->total), k, dist(gen));
    if (X) check_cuda(cudaMemcpy(X, &id, sizeof(int), cudaMemcpyHostToDevice), "TopKSampleToCPU");
    return id;
}

int TopKSampleToCPU(const graph& input, const int k) { return TopKSampleToCPU(input, nullptr, k); }

// --------------------------------------------------- Noise (:3936-3944)
void Noise(const graph& input, const float mean, const float std_, const str type) {
    std::random_device rd;
    const uint64_t seed = ((uint64_t)rd() << 32) | rd();
    if (type == "gaussian") check(mle_fill_noise(input->output, input->total, mean, std_, 0, seed, st()), "Noise");
    if (type == "uniform") check(mle_fill_noise(input->output, input->total, mean, std_, 1, seed, st()), "Noise");
}

// ---------------------------------------------------------------- Timing
Timing::Timing(const str reason) : what_(reason) {}
Timing::~Timing() {}
void Timing::start() {
    beg_ = std::chrono::high_resolution_clock::now();
    running_ = true;
}
void Timing::end() {
    if (!running_) return;
    running_ = false;
    const auto t = std::chrono::high_resolution_clock::now();
    std::cout << "Time elapsed for " << what_ << ": " << std::chrono::duration<double, std::milli>(t - beg_).count()
              << "ms \n";
}

// ---------------------------------------------- TimeMLPBlock (:3914-3924)
TimeMLPBlock::TimeMLPBlock(const int t_embed_dim, const int t_hidden)
    : L0(t_embed_dim, t_hidden, "Time MLP L0"), L1(t_hidden, t_hidden, "Time MLP L1") {}

graph TimeMLPBlock::forward(const graph& X) { return L1.forward(GraphOperations::SILU(L0.forward(X))); }
void TimeMLPBlock::save(std::ofstream& f) const {
    L0.save(f);
    L1.save(f);
}
void TimeMLPBlock::load(std::ifstream& f) {
    L0.load(f);
    L1.load(f);
}

// ------------------------------- Multi_Linear_Residual_Block (:3926-3934)
Multi_Linear_Residual_Block::Multi_Linear_Residual_Block(const int input, const int output, const int num_residuals,
                                                         const int layers_, const int hidden_size)
    : input_dim(input), output_dim(output), residuals(num_residuals), hidden_dim(hidden_size), layers(layers_) {
    sequence.push_back(new Linear(input, hidden_size));
    for (int i = 1; i < num_residuals * layers_; ++i) sequence.push_back(new Linear(hidden_size, hidden_size));
    sequence.push_back(new Linear(hidden_size, output));
}

void Multi_Linear_Residual_Block::save(std::ofstream& f) const {
    for (const Linear* p : sequence) p->save(f);
}
void Multi_Linear_Residual_Block::load(std::ifstream& f) {
    for (Linear* p : sequence) p->load(f);
}
