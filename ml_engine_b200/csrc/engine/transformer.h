// transformer.h -- MultiHeadAttention of ML_Engine's Includes/transformer.h
// (:106-118) with the same members, constructor and forward signatures, so
// encoder/decoder code written against the reference compiles unchanged.
//
// forward / cross_forward build the same computation as the reference's
// Headify x3 -> BMMABT -> Scale -> SOFTMAX/SOFTMASK(type 1) -> BMM ->
// DeHeadify chain (Engine/transformer.cu:647-675), as one attention node
// (GraphOperations::ScaledDotAttention) fed by the projections of one grouped
// Linear launch.  The KV-cached generation forwards, the tokenizer
// (TextualEmbedding), the data loader and the LLM driver are not part of
// the training path and are not provided.
#pragma once

#include "engine.h"

class MultiHeadAttention {
   public:
    const int embed_dim;
    const int hidden;
    const int num_heads;
    int head_dim;
    str name;
    Linear q, k, v, o;

    MultiHeadAttention(const int embed_dim, const int hidden, const int num_heads,
                       const str& name = "MultiHeadAttention");
    void save(std::ofstream& f) const;
    void load(std::ifstream& f);

    // self-attention over X [B, 1, S, embed_dim]; scores scaled by
    // 1/sqrt(head_dim); `mask` hides later queries from each key column
    graph forward(const graph& X, const bool mask = false);
    // queries from X, keys and values from Y; scaled by 1/sqrt(embed_dim)
    // and masked, as the reference's cross_forward does
    graph cross_forward(const graph& X, const graph& Y);
};
