// A training program written against the reference's C++ API the way its
// use cases are (use_cases/mnist.cu's convolutional classifier, minus the
// OpenCV image loader; plus the other layer classes and helpers use cases
// reach for), compiled and linked against this repository's engine.h,
// transformer.h and libmle_engine.so with no change to the program text a
// reference build would need.  Exit status 0 when every part trained:
// finite losses that fall, arg-max and sampling in range.
#include <cmath>
#include <cstdio>

#include "engine.h"
#include "transformer.h"

// output size of a stack of convolutions (use_cases/mnist.cu's FOD)
static int FOD(const int row, const int col, const std::vector<Convolute2D>& vecs) {
    int r = row, c = col;
    for (const auto& p : vecs) {
        r = ((r - p.c + 2 * p.pad) / p.stride) + 1;
        c = ((c - p.d + 2 * p.pad) / p.stride) + 1;
    }
    return vecs.back().out * r * c;
}

class Model {
   private:
    Convolute2D conv1, conv2;
    Linear fc1, fc2;
    Multi_Linear_Residual_Block head;

   public:
    Model()
        : conv1(1, 8, 5, 5, 1, 0, "Conv1"),
          conv2(8, 8, 5, 5, 1, 0, "Conv2"),
          fc1(FOD(28, 28, {conv1, conv2}), 64, "First Linear"),
          fc2(64, 10, "Projection"),
          head(64, 10, 2, 2, 32) {}
    template <typename NormFn, typename ActFn>
    graph forward(const graph& Xm, NormFn norm, ActFn act) {
        auto A1 = act(norm(conv1.forward(Xm)));
        auto A2 = act(norm(conv2.forward(A1)));
        auto A3 = GraphOperations::Copy(A2);
        A3->reshape({A2->dim[0], 1, 1, (int)A2->total / A2->dim[0]});
        auto L1 = act(fc1.forward(A3));
        auto out = fc2.forward(L1) + head.forward(L1, GraphOperations::GELU, GraphOperations::LayerNorm);
        out->op_name = "Prediction";
        return out;
    }
};

static int fail(const char* what) {
    printf("FAILED: %s\n", what);
    return 1;
}

int main() {
    GraphOperations go;
    const int B = 16;
    // ---------------------------------------------------- classifier
    auto data = std::make_shared<NodeBackProp>("Data", B, 1, 28, 28, 1);
    auto labels = std::make_shared<NodeBackProp>("Labels", B, 1, 1, 10, 1);
    Noise(data, 0.f, 1.f, "gaussian");
    fillKernel<<<(B * 10 + THREADSPERBLOCK - 1) / THREADSPERBLOCK, THREADSPERBLOCK>>>(labels->output, 0.f,
                                                                                      (unsigned long long)B * 10);
    for (int b = 0; b < B; ++b) WriteValueAt(labels, 1.0f, b * 10 + (b * 7) % 10);
    CheckError("inputs");
    Model model;
    auto prediction = model.forward(data, go.LayerNorm, go.GELU);
    auto loss = go.SoftMaxCrossEntropy(prediction, labels, true);
    go.nodes = topological_sort(loss);
    float first = 0.f, last = 0.f;
    for (int i = 0; i < 40; i++) {
        go.zero_grad();
        go.forward(nullptr, true);
        CheckError("Forward");
        go.backward();
        go.ParameterUpdate(nullptr, false, 1e-3f);
        if (i == 0) first = go.loss;
        last = go.loss;
        if (i % 10 == 0) printf("%i: loss: %f \n", i, go.loss);
    }
    isNan(prediction);
    isNan(prediction, 1);
    if (!(std::isfinite(first) && std::isfinite(last) && last < first)) return fail("classifier loss did not fall");
    printHeadGPU(prediction);

    // arg-max and top-k sampling of one row of probabilities
    auto row = std::make_shared<NodeBackProp>("Row", 1, 1, 1, 10, 1);
    for (int c = 0; c < 10; ++c) WriteValueAt(row, (c == 6) ? 0.55f : 0.05f, c);
    if (ArgMaxToCPU(row) != 6) return fail("ArgMaxToCPU");
    int* slot = nullptr;
    SafeCudaMalloc("slot", slot, 1);
    if (ArgMaxToCPU(row, slot) != 6) return fail("ArgMaxToCPU (slot)");
    if (TopKSampleToCPU(row, slot, 1) != 6) return fail("TopKSampleToCPU k=1");
    const int s3 = TopKSampleToCPU(row, 3);
    if (s3 < 0 || s3 >= 10) return fail("TopKSampleToCPU k=3");
    cudaFree(slot);
    go.clear_graph();

    // ---------------- time MLP, elementwise ops and attention, MSE loss
    GraphOperations go2;
    auto x = std::make_shared<NodeBackProp>("Tokens", 2, 1, 16, 32, 1);
    auto target = std::make_shared<NodeBackProp>("Target", 2, 1, 16, 32, 1);
    Noise(x, 0.f, 1.f, "gaussian");
    Noise(target, 0.f, 0.5f, "uniform");
    MultiHeadAttention self_attn(32, 32, 4, "Self");
    MultiHeadAttention cross(32, 32, 4, "Cross");
    TimeMLPBlock tmlp(32, 32);
    auto h = x + self_attn.forward(GraphOperations::LayerNorm(x), true);
    auto c = h + cross.cross_forward(GraphOperations::LayerNorm(h), x);
    auto y = tmlp.forward(c) * GraphOperations::SIGMOID(c) - GraphOperations::Scale(c, 0.5f);
    auto mse = go2.MeanSquaredError(y, target, true);
    go2.nodes = topological_sort(mse);
    first = last = 0.f;
    for (int i = 0; i < 60; i++) {
        go2.zero_grad();
        go2.forward(nullptr, true);
        go2.backward();
        go2.ParameterUpdate(nullptr, false, 1e-3f);
        if (i == 0) first = go2.loss;
        last = go2.loss;
    }
    printf("attention block loss %f -> %f\n", first, last);
    CheckError("attention block");
    if (!(std::isfinite(first) && std::isfinite(last) && last < first)) return fail("attention loss did not fall");
    go2.clear_graph();
    printf("usecase ok\n");
    return 0;
}
