// Two graphs that share a node, driven through the reference's C++ API in
// the order a multi-loss program may use: both zero_grads, both forwards,
// then graph B's backward before graph A's.  The shared node's gradient
// must end as the sum of what the two backward passes contribute, as the
// reference's clear-then-accumulate gives it; in graph A the shared node's
// first writer (an activation) could overwrite its gradient, in graph B a
// Scale adds to it.  Exit status 0 when the sum holds.
#include <cmath>
#include <cstdio>
#include <vector>

#include "engine.h"

static std::vector<float> grad_of(const graph& g) {
    std::vector<float> h(g->total);
    cudaDeviceSynchronize();
    cudaMemcpy(h.data(), g->grad, g->total * sizeof(float), cudaMemcpyDeviceToHost);
    return h;
}

int main() {
    auto x = std::make_shared<NodeBackProp>("X", 64, 1, 1, 48, 1);
    auto ta = std::make_shared<NodeBackProp>("Target A", 64, 1, 1, 32, 1);
    auto tb = std::make_shared<NodeBackProp>("Target B", 64, 1, 1, 32, 1);
    Noise(x, 0.f, 1.f, "gaussian");
    Noise(ta, 0.f, 1.f, "gaussian");
    Noise(tb, 0.f, 1.f, "gaussian");
    Linear lin(48, 32, "Shared");
    graph s = lin.forward(x);                                     // the shared node
    GraphOperations A, B;
    graph la = A.MeanSquaredError(GraphOperations::GELU(s), ta, true);       // A: GELU first writes s.grad
    graph lb = B.MeanSquaredError(GraphOperations::Scale(s, 0.5f), tb, true);  // B: Scale adds to it
    A.nodes = topological_sort(la);
    B.nodes = topological_sort(lb);

    // each graph's contribution alone
    A.zero_grad();
    A.forward(nullptr, true);
    A.backward();
    const std::vector<float> ga = grad_of(s);
    B.zero_grad();
    B.forward(nullptr, true);
    B.backward();
    const std::vector<float> gb = grad_of(s);

    // interleaved: both cleared, B's backward, then A's
    A.zero_grad();
    B.zero_grad();
    A.forward(nullptr, true);
    B.forward(nullptr, true);
    B.backward();
    A.backward();
    const std::vector<float> both = grad_of(s);
    CheckError("two graphs");

    double num = 0.0, den = 0.0;
    for (size_t i = 0; i < both.size(); ++i) {
        const double want = (double)ga[i] + (double)gb[i];
        num = std::fmax(num, std::fabs((double)both[i] - want));
        den = std::fmax(den, std::fabs(want));
    }
    const double rel = num / (den > 0 ? den : 1.0);
    printf("shared gradient: max |got - (gA + gB)| / max |gA + gB| = %.3g\n", rel);
    A.clear_graph();
    B.clear_graph();
    if (!(rel <= 1e-6)) {
        printf("FAILED: the shared node's gradient is not the sum of both graphs' contributions\n");
        return 1;
    }
    printf("two graphs ok\n");
    return 0;
}
