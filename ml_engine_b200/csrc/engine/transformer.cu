// MultiHeadAttention (Includes/transformer.h:106-118, Engine/transformer.cu:
// 634-675) on the engine's fused attention node.
#include <math.h>

#include "transformer.h"

MultiHeadAttention::MultiHeadAttention(const int embed_dim_, const int hidden_, const int num_heads_, const str& name_)
    : embed_dim(embed_dim_),
      hidden(hidden_),
      num_heads(num_heads_),
      name(name_),
      q(embed_dim_, hidden_, name_ + " Query"),
      k(embed_dim_, hidden_, name_ + " Key"),
      v(embed_dim_, hidden_, name_ + " Value"),
      o(hidden_, embed_dim_, name_ + " Output") {
    if (hidden % num_heads != 0)
        printf("Cannot Split MHA because hidden dim: %i is not divisible by num heads: %i", hidden, num_heads);
    head_dim = hidden / num_heads;
}

void MultiHeadAttention::save(std::ofstream& f) const {
    q.save(f);
    k.save(f);
    v.save(f);
    o.save(f);
}

void MultiHeadAttention::load(std::ifstream& f) {
    q.load(f);
    k.load(f);
    v.load(f);
    o.load(f);
}

graph MultiHeadAttention::forward(const graph& X, const bool mask) {
    std::vector<graph> p = GraphOperations::LinearGroup(X, {&q, &k, &v});
    graph att = GraphOperations::ScaledDotAttention(p[0], p[1], p[2], num_heads, 1.0f / sqrtf((float)head_dim),
                                                    mask && X->dim[2] > 1);
    graph out = o.forward(att);
    out->op_name = "Multi Head Attention Output";
    return out;
}

graph MultiHeadAttention::cross_forward(const graph& X, const graph& Y) {
    graph Q = q.forward(X);
    std::vector<graph> p = GraphOperations::LinearGroup(Y, {&k, &v});
    graph att = GraphOperations::ScaledDotAttention(Q, p[0], p[1], num_heads, 1.0f / sqrtf((float)embed_dim),
                                                    X->dim[2] > 1);
    graph out = o.forward(att);
    out->op_name = " Cross MHA Block Output";
    return out;
}
