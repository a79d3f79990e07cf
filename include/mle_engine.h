/*
 * mle_engine.h -- C ABI of the B200 host runtime (libmle_engine.so).
 *
 * A "session" owns one training graph built with the reference-compatible
 * C++ API (NodeBackProp / GraphOperations / AdamParameter / Linear, the
 * replacement of Includes/engine.h) for one of the benchmark configurations,
 * with its static graph-build allocation, a compute stream, pinned host
 * staging buffers for the step's inputs and loss, an optional captured CUDA
 * graph of the whole step, and an optional data-parallel NCCL communicator.
 *
 * One step is the reference training loop body
 *   go.zero_grad(); go.forward(nullptr, true); go.backward();
 *   [clip]; go.ParameterUpdate(nullptr, false, lr, adamw);
 * (use_cases/mnist.cu:284-293, Engine/transformer.cu:852-871), with the clip
 * being the reference's private accumulate/Sqrt_Scale/clipNorm sequence
 * (Engine/engine.cu:3362-3368) generalised to a max norm.
 *
 * All functions return 0 or an mle_status code (include/mle_kernels.h).
 */
#ifndef MLE_ENGINE_H
#define MLE_ENGINE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* mle_session_t;

enum mle_config {
    MLE_CFG_MLP = 1,      /* Linear-ReLU-Linear + SoftMaxCrossEntropy (use_cases/mnist.cu:252-273) */
    MLE_CFG_ENCODER = 2,  /* pre-LN transformer encoder stack + projection + SMCE */
    MLE_CFG_ENCDEC = 3,   /* encoder-decoder (self, masked self, cross attention) + SMCE */
    MLE_CFG_UNET = 4      /* DDPM noise-prediction U-Net (ResidualBlocks, Conv2D/Conv2DT, GroupNorm, MSE) */
};

typedef struct mle_session_desc {
    int config;          /* enum mle_config */
    int batch;           /* local (per-rank) batch */
    /* MLP */
    int in_features, hidden, classes;
    /* transformer */
    int seq_len, d_model, heads, ffn, layers, vocab;
    int fused_attention; /* 1: ScaledDotAttention node, 0: the reference's graph ops */
    int key_grad_mode;   /* MLE_KEYGRAD_REFERENCE or MLE_KEYGRAD_TRUE */
    /* optimizer */
    float lr;
    int adamw;
    float clip_norm;     /* <= 0 disables the clip */
    uint64_t seed;
    int gemm_mode;       /* MLE_GEMM_MODE_TF32 or MLE_GEMM_MODE_FP32 for every GEMM of the step */
    /* U-Net: images [batch, channels, image_size, image_size]; levels of
     * base_width, 2x and 4x channels; sinusoidal time embedding of t_embed
     * features for the timestep `timestep` (fixed when the graph is built,
     * as the reference's PositionalEncoding node captures it) */
    int channels, image_size, base_width, t_embed, timestep;
    /* classifier targets: 0 = class indices fed straight to the index-label
     * softmax cross-entropy; 1 = the reference's dense one-hot tensor built
     * each step by OneHotEmbeddings.  Same loss and gradients, bit for bit;
     * the input is the int32 class ids either way. */
    int dense_targets;
    /* embedding training: > 0 runs TextualEmbedding::EmbeddingUpdate
     * (Engine/transformer.cu:233-245) on the encoder-side token table
     * ("tokens" / "src") after each backward pass, an SGD step of this
     * learning rate (the reference's LLM::train uses LEARNING_RATE = 1e-4,
     * Engine/transformer.cu:869); 0 keeps every table frozen.  Under data
     * parallelism each rank scatters its rows into a dense [vocab, d_model]
     * delta, the deltas are summed with the gradient buckets and applied
     * with the same 1/world average, so every rank keeps the same table. */
    float embed_lr;
} mle_session_desc;

/* Builds the graph and allocates everything the step needs. */
int mle_session_create(const mle_session_desc* desc, mle_session_t* out);
int mle_session_destroy(mle_session_t s);

/* The session's compute stream (cudaStream_t as void*). */
void* mle_session_stream(mle_session_t s);

/* Step inputs.  Each input has a pinned host staging buffer (host_ptr) the
 * caller fills before mle_session_step(..., upload=1, ...), and a device
 * buffer (dev_ptr).  dtype: 0 = float32, 1 = int32. */
int mle_session_input_count(mle_session_t s);
int mle_session_input_info(mle_session_t s, int i, char* name, int name_len, int64_t* numel, int* dtype,
                           void** host_ptr, void** dev_ptr);

/* One training step on the session stream.  upload != 0 copies every input
 * host -> device first (cudaMemcpyAsync from pinned memory); if loss_out is
 * non-NULL the loss is copied device -> pinned host and the call waits for
 * the stream.  Replays the captured graph when one was captured. */
int mle_session_step(mle_session_t s, int upload, float* loss_out);

/* Runs one phase of the step: 0 zero_grad, 1 forward (calc_loss),
 * 2 backward, 3 data-parallel gradient reduction, 4 clip, 5 update. */
int mle_session_phase(mle_session_t s, int phase);

/* Captures the whole step into two CUDA graphs, one device-resident and one
 * that also uploads the inputs and downloads the loss; later
 * mle_session_step calls replay the one matching `upload`. */
int mle_session_capture(mle_session_t s);

/* Whether backward puts the Linear layers' weight and bias gradients on a
 * second stream (forked from the compute stream where the layer's output
 * gradient is complete, joined back at the end of the backward), so they
 * run concurrently with the input-gradient chain.  1 (default) on, 0 all on
 * the compute stream.  Process-wide; takes effect for steps issued (or
 * captured) afterwards. */
int mle_set_param_grad_stream(int enable);
int mle_get_param_grad_stream(void);

/* First-writer assignment of activation gradients: when the first node to
 * write a gradient in the backward walk overwrites all of it (the loss,
 * an activation, or a Linear whose input gradient spans at least two waves
 * of 128 x 128 tiles), zero_grad leaves that buffer alone and the writer
 * assigns instead of adding, with bit-identical results.  1 (default) on,
 * 0 every gradient cleared and accumulated.  Process-wide; decided when a
 * backward pass starts, so it applies from the next zero_grad on. */
int mle_set_grad_first_write(int enable);
int mle_get_grad_first_write(void);

/* One launch for the optimizer: when ParameterUpdate covers exactly the
 * parameters clip_grad_norm collected (each once, one learning rate and one
 * rule), the gradient norm, the clip, Adam/AdamW and the step counters run
 * as the single cooperative kernel of mle_clip_adam_run instead of the
 * sum-of-squares, finalize and update launches; clip_grad_norm then only
 * records max_norm, and the norm is taken of the gradients as they are when
 * the update runs.  The norm's summation order differs (per-block partials
 * in block order), so the clip coefficient agrees to rounding; the
 * per-element update is the same arithmetic.  The tensor table is copied to
 * the device by the first such update outside stream capture; an update
 * captured before that takes the separate launches.  1 (default) on, 0 the
 * separate launches.  Process-wide; takes effect at the next
 * clip_grad_norm. */
int mle_set_fused_optimizer(int enable);
int mle_get_fused_optimizer(void);

/* Forward: a residual Add whose sum a LayerNorm reads runs as one pass that
 * writes the sum and the norm's output and statistics
 * (mle_add_layernorm_fwd), the norm's own launch dropped; both outputs are
 * bitwise those of the two launches.  1 (default) on, 0 off.
 * Process-wide; decided when a forward pass starts. */
int mle_set_add_norm_fusion(int enable);
int mle_get_add_norm_fusion(void);

/* Captures each phase of the step (the numbering of mle_session_phase,
 * device resident: no upload, no loss download) as its own CUDA graph, so a
 * caller can time phases on the device; mle_session_phase_replay(s, ph)
 * launches phase ph's graph on the session stream.  Replaying phases 0..5 in
 * order is one training step.  Under data parallelism phase 2's graph also
 * holds phase 3 (the bucket reductions the backward starts on the
 * communication stream are joined there), and replaying phase 3 does
 * nothing. */
int mle_session_capture_phases(mle_session_t s);
int mle_session_phase_replay(mle_session_t s, int phase);

/* Kernel, memset and memcpy nodes of the captured device-resident step
 * (the launches one replay issues). */
int mle_session_graph_counts(mle_session_t s, int* kernels, int* memsets, int* copies);

/* Dependency edges of the same graph: all of them, and those of the
 * programmatic kind (a kernel that may start its prologue while the
 * previous kernel finishes). */
int mle_session_graph_edges(mle_session_t s, int* edges, int* programmatic);

int mle_session_sync(mle_session_t s);

/* Parameters in graph order (W1 then B1 per Linear). */
int mle_session_param_count(mle_session_t s);
int mle_session_param_info(mle_session_t s, int i, char* name, int name_len, int64_t* numel);
/* which: 0 weights, 1 gradient, 2 first moment, 3 second moment. */
int mle_session_param_read(mle_session_t s, int i, int which, float* host);
int mle_session_param_write(mle_session_t s, int i, int which, const float* host);
/* Step counter t of parameter i, read from its device mirror. */
int mle_session_param_step(mle_session_t s, int i, int* t);

/* Checkpoint of every parameter (weights, Adam m and v) in build order as
 * the reference's AdamParameter::save records (Engine/engine.cu:139-188),
 * plus `<path>.t` with the Adam step of each parameter, which the reference
 * does not save.  Under data parallelism only rank 0 writes.  Load checks
 * every record's name and size first (MLE_ERR_ARG and nothing changed on a
 * mismatch), then reads the records (Engine/engine.cu:190-268) and, when
 * the sidecar is present, the steps. */
int mle_session_save(mle_session_t s, const char* path);
int mle_session_load(mle_session_t s, const char* path);

/* Embedding tables (transformer configs, in input order; trained only when
 * desc.embed_lr > 0, the encoder-side one). */
int mle_session_embedding_count(mle_session_t s);
int mle_session_embedding_write(mle_session_t s, int i, const float* host, int64_t numel);
int mle_session_embedding_read(mle_session_t s, int i, float* host, int64_t numel);

/* Total device bytes held by the session's arenas. */
int mle_session_device_bytes(mle_session_t s, int64_t* bytes);

/* Number of graph nodes and launches of the last non-captured step. */
int mle_session_node_count(mle_session_t s);

/* ---- data parallelism (one process per GPU, NCCL over NVLink) ---- */

/* Writes a fresh NCCL unique id (128 bytes) for rank 0 to distribute. */
int mle_dp_unique_id(uint8_t* out128);

/* Host-side bucket plan of data parallelism (what mle_session_enable_dp
 * uses): gradient tensors (device addresses and float counts) sorted by
 * address and merged while contiguous (gaps up to 64 floats bridged), inside
 * one allocation and within bucket_mb MiB (bucket_mb <= 0: the size
 * mle_dp_auto_bucket_mb gives for the total).  `chunks` (nullable: all in
 * one allocation) names the allocation each tensor lies in, by any id, such
 * as its base address; tensors of different allocations never share a
 * bucket, even when their addresses touch.  Writes up to max_out buckets
 * (base address, float count) and their number to *out_n; MLE_ERR_ARG if
 * more than max_out are needed.  Touches no device. */
int mle_dp_plan_buckets(const uint64_t* addrs, const int64_t* counts, const uint64_t* chunks, int n, int bucket_mb,
                        uint64_t* out_base, int64_t* out_count, int max_out, int* out_n);

/* The automatic bucket size for `total_floats` of gradients: the smallest
 * power of two of MiB, from 1 to 32, that splits them into at most four
 * buckets (configs[1]'s 10.5 MB -> 4 MiB, configs[2]'s 193 MB -> 32 MiB). */
int mle_dp_auto_bucket_mb(int64_t total_floats);

/* Joins a communicator of `world` ranks.  After backward, the parameter
 * gradients are summed over ranks in buckets of `bucket_mb` MiB (<= 0:
 * automatic, as above) on a second stream, each bucket as soon as the
 * backward pass has produced every gradient in it, and the update averages
 * them (scale 1/world) before the clip norm and AdamW.  A step whose
 * all-reduce NCCL refuses returns MLE_ERR_CUDA without updating any
 * parameter. */
int mle_session_enable_dp(mle_session_t s, const uint8_t* id128, int rank, int world, int bucket_mb);

#ifdef __cplusplus
}
#endif

#endif /* MLE_ENGINE_H */
