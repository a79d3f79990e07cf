/*
 * mle_kernels.h -- C ABI of the B200 (sm_100a) kernels behind ML_Engine's
 * training hot path.
 *
 * Every entry point replaces one group of `<<<>>>` launches that the
 * reference issues from the backward lambdas in Engine/engine.cu, from the
 * AdamParameter methods, or from the forward lambdas that produce the
 * tensors those backward lambdas read.  Each declaration names the
 * reference code it stands in for (path:line inside the ML_Engine tree).
 *
 * Conventions shared by all entry points
 *   - pointers are device pointers to fp32 unless stated otherwise;
 *   - sizes are int64_t element counts; shapes follow the reference's
 *     [dim0, dim1, dim2, dim3] row-major layout;
 *   - `stream` is a cudaStream_t passed as void*; NULL is the legacy default
 *     stream, which keeps the reference's implicit ordering;
 *   - the return value is 0 (MLE_OK) or an mle_status code; nothing here
 *     allocates device memory, synchronises the device, or exits the
 *     process -- the C++ shim maps a non-zero status onto the reference's
 *     print-and-exit behaviour;
 *   - "accumulate" outputs are `+=` exactly where the reference's kernel
 *     uses `+=`/atomicAdd, and "assign" outputs are `=` where it assigns.
 */
#ifndef MLE_KERNELS_H
#define MLE_KERNELS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* mle_stream_t;

enum mle_status {
    MLE_OK = 0,
    MLE_ERR_ARG = 1,          /* invalid size, pointer or flag */
    MLE_ERR_CUDA = 2,         /* a CUDA runtime call or launch failed */
    MLE_ERR_UNSUPPORTED = 3,  /* shape/flag combination not implemented */
    MLE_ERR_TIMEOUT = 4       /* a bounded wait gave up (a device-side wait, or the host waiting for other ranks) */
};

enum mle_activation {
    MLE_ACT_RELU = 0,
    MLE_ACT_LEAKY_RELU = 1,
    MLE_ACT_SILU = 2,
    MLE_ACT_TANH = 3,
    MLE_ACT_GELU = 4,
    MLE_ACT_SIGMOID = 5
};

/* GEMM variants, named after the reference kernels they replace
 * (Engine/kernels.cu:387-539):
 *   MLE_GEMM_AB   bcmm     C[m,p] (op) A[m,n]   * B[n,p]
 *   MLE_GEMM_ABT  bcmmABT  C[m,p] (op) A[m,n]   * B[p,n]^T
 *   MLE_GEMM_ATB  bcmmATB  C[m,p] (op) A[n,m]^T * B[n,p]
 *   MLE_GEMM_ATBT bcmmT    C[m,p] (op) A[n,m]^T * B[p,n]^T               */
enum mle_gemm_variant {
    MLE_GEMM_AB = 0,
    MLE_GEMM_ABT = 1,
    MLE_GEMM_ATB = 2,
    MLE_GEMM_ATBT = 3
};

/* ------------------------------------------------------------------ */
/* library / status                                                    */
/* ------------------------------------------------------------------ */

/* Human readable name of an mle_status value. */
const char* mle_status_string(int status);

/* Last CUDA error code recorded by a failing entry point (0 if none). */
int mle_last_cuda_error(void);

/* Reads and clears the device watchdog word that bounded waits inside the
 * tensor-core kernels set when they give up (0 = no timeout).  Synchronises
 * `stream`; call it outside the timed region. */
int mle_watchdog_read(int* out_flag, mle_stream_t stream);

/* Version of this ABI (incremented on incompatible change). */
int mle_abi_version(void);

/* ------------------------------------------------------------------ */
/* elementwise glue (graph-op forward/backward lambdas)                */
/* ------------------------------------------------------------------ */

/* x[i] = value.  Replaces fillKernel (Includes/kernels.h:13-19) as launched
 * by Zerograd (Engine/engine.cu:312-326). */
int mle_fill(float* x, float value, int64_t n, mle_stream_t stream);

/* y[i] = x[i].  Replaces Write (Engine/kernels.cu:1670-1675). */
int mle_copy(const float* x, float* y, int64_t n, mle_stream_t stream);

/* y[i] = (float)((double)y[i] + scale * x[i]) (the sum in double).  Replaces
 * Accumulate (Engine/kernels.cu:1702-1708), the backward of Copy, Scale,
 * MatrixPositionalEncoding, Bias_Add/Broadcast_Channel input A
 * (Engine/engine.cu:696,2543,1287,1388,1433). */
int mle_accumulate(const float* x, float* y, int64_t n, double scale, mle_stream_t stream);

/* ga += g; gb += g in one pass.  Replaces the two Accumulate launches of
 * GraphOperations::Add backward (Engine/engine.cu:1659-1667). */
int mle_add_bwd(const float* g, float* ga, float* gb, int64_t n, mle_stream_t stream);
/* The same with ga (assign_mask bit 0) and/or gb (bit 1) written instead of
 * accumulated: bitwise what mle_add_bwd leaves in cleared buffers.  For the
 * first writer of a gradient buffer that is not cleared between steps;
 * ga == gb with an assign bit is MLE_ERR_ARG. */
int mle_add_bwd_assign(const float* g, float* ga, float* gb, int64_t n, int assign_mask, mle_stream_t stream);

/* y[i] = scale * x[i].  Replaces Scale_Write (Engine/kernels.cu:1677-1682),
 * the forward of Scale (Engine/engine.cu:2533-2538). */
int mle_scale_write(const float* x, float* y, int64_t n, float scale, mle_stream_t stream);

/* z[i] = x[i] + scale * y[i].  Replaces ScaleAdd (Engine/kernels.cu:1718-1724),
 * the forward of Add (Engine/engine.cu:1650-1655). */
int mle_scale_add(const float* x, const float* y, float* z, float scale, int64_t n, mle_stream_t stream);

/* Activation forward y = f(x).  Replaces ReLU/LeakyReLU/SiLU/TaNH/GeLU/Sigmoid
 * (Engine/kernels.cu:1214-1319). */
int mle_act_fwd(int kind, const float* x, float* y, int64_t n, mle_stream_t stream);

/* Activation backward gx[i] += gy[i] * f'(x[i]) with x the activation INPUT,
 * using the reference's derivative formulas (deriv_* in
 * Engine/kernels.cu:1223-1328, lambdas Engine/engine.cu:2666-2842).
 * If bias_grad is non-NULL the same pass also adds the column sums of the
 * updated gx (a [rows, cols] matrix, rows*cols == n) into bias_grad[cols]; this fuses the BCompress launch of the producing Linear
 * (Engine/kernels.cu:1562-1584) when the activation is that Linear's only
 * consumer. */
int mle_act_bwd(int kind, const float* x, const float* gy, float* gx, int64_t n,
                float* bias_grad, int64_t rows, int64_t cols, mle_stream_t stream);
/* The same with gx's previous contents taken as zero: gx is written, not
 * read, and equals bit for bit what mle_act_bwd leaves in a cleared gx.
 * For the first writer of a gradient buffer that is not cleared between
 * steps. */
int mle_act_bwd_assign(int kind, const float* x, const float* gy, float* gx, int64_t n,
                       float* bias_grad, int64_t rows, int64_t cols, mle_stream_t stream);

/* y[r, c] = x[r, c] + bias[c].  Replaces BCumAdd (Engine/kernels.cu:1586-1592)
 * as launched by Linear/Bias_Add forward.  y may alias x. */
int mle_bias_add_fwd(const float* x, const float* bias, float* y, int64_t rows, int64_t cols,
                     mle_stream_t stream);

/* bias_grad[c] += scale * sum_r g[r, c].  Replaces BCompress
 * (Engine/kernels.cu:1562-1584) in Linear and Bias_Add backward. */
int mle_bias_grad(const float* g, float* bias_grad, int64_t rows, int64_t cols, float scale,
                  mle_stream_t stream);

/* Per-channel broadcast of a [1,1,1,C] vector over [B,C,H,W]:
 * y = x + b[c].  Replaces broadcast_add (Engine/kernels.cu:1661-1668). */
int mle_channel_bias_fwd(const float* x, const float* b, float* y, int batch, int channels,
                         int64_t spatial, mle_stream_t stream);

/* gb[c] += sum_{n,s} g[n,c,s]; if gx != NULL also gx += g.  Replaces
 * Channel_Squeeze1D (Engine/kernels.cu:1734-1761) plus the Accumulate of
 * Broadcast_Channel backward (Engine/engine.cu:1430-1438) and the dB part
 * of Convolute2D/2DT backward (Engine/engine.cu:3768,3868). */
int mle_channel_bias_bwd(const float* g, float* gx, float* gb, int batch, int channels,
                         int64_t spatial, mle_stream_t stream);
/* The same sums for the first `first` channels only: Broadcast_Channel's
 * backward launches Channel_Squeeze1D with one block per index of dim[3],
 * so only channels [0, min(dim[3], C)) receive their sums
 * (Engine/engine.cu:1435). */
int mle_channel_bias_bwd_first(const float* g, float* gb, int batch, int channels, int first,
                               int64_t spatial, mle_stream_t stream);

/* Sinusoidal matrix positional encoding, y = x + PE (sin even / cos odd
 * columns).  Replaces MatPEncoding (Engine/kernels.cu:166-185). */
int mle_matpe_fwd(const float* x, float* y, int batch, int rows, int cols, int start_idx,
                  mle_stream_t stream);

/* Timestep encoding (cos first half, sin second half).  Replaces PEncoding
 * (Engine/kernels.cu:147-164). */
int mle_timestep_pe(float* y, int t, int dim, mle_stream_t stream);

/* Head split/merge between [B,1,S,H*hd] and [B,H,S,hd].  flag follows
 * HeadifyColChannel (Engine/kernels.cu:1371-1406):
 *   0: out[headified] = in[flat]      (Headify forward)
 *   1: out[flat]     += in[headified] (Headify backward)
 *   2: out[flat]      = in[headified] (DeHeadify forward)
 *   3: out[headified]+= in[flat]      (DeHeadify backward)               */
int mle_headify(const float* in, float* out, int batch, int heads, int seq, int head_dim,
                int flag, mle_stream_t stream);

/* Channel concat / split: Channel_Concat and Channel_Split
 * (Engine/kernels.cu:1408-1432).  split accumulates (+=). */
int mle_channel_concat(const float* a, const float* b, float* c, int batch, int c1, int c2,
                       int64_t spatial, mle_stream_t stream);
int mle_channel_split(float* ga, float* gb, const float* gc, int batch, int c1, int c2,
                      int64_t spatial, mle_stream_t stream);

/* Centre crop (a,b)->(c,d) and its adjoint (CopynCrop / PaddingCrop,
 * Engine/kernels.cu:1330-1369).  pad_crop accumulates. */
int mle_center_crop(const float* x, float* y, int batch, int depth, int a, int b, int c, int d,
                    mle_stream_t stream);
int mle_pad_crop(const float* x, float* y, int batch, int depth, int a, int b, int c, int d,
                 mle_stream_t stream);

/* Embedding gather out[i, :] = table[keys[i], :] (GatherEmbeddings,
 * Engine/kernels.cu:2279-2296); a key < 0 (masked) gives a zero row.
 * one_hot writes out[i, keys[i]] = 1 into a zeroed [n, vocab] matrix
 * (OneHotEmbeddings, Engine/kernels.cu:1551-1560). */
int mle_embedding_gather(const int32_t* keys, const float* table, float* out, int64_t n_keys,
                         int dim, mle_stream_t stream);
/* The gather followed by the positional table's broadcast add
 * (MatrixPositionalEncoding forward, Engine/engine.cu:1272-1290, over the
 * gathered rows): out[i, :] = table[keys[i], :] + pe[i % seq, :], bitwise
 * mle_embedding_gather then mle_rows_add_table.  dim a multiple of 4 and
 * 16-byte aligned table, pe and out (else MLE_ERR_UNSUPPORTED). */
int mle_embedding_gather_add(const int32_t* keys, const float* table, const float* pe, float* out, int64_t n_keys,
                             int dim, int seq, mle_stream_t stream);
int mle_one_hot(const int32_t* keys, float* out, int64_t n_keys, int vocab, mle_stream_t stream);

/* z = x * y (accumulate = 0) or z += x * y (1), elementwise: mulKernel
 * (Engine/kernels.cu:139-145) as Multiply's forward and backward launch it. */
int mle_mul(const float* x, const float* y, float* z, int64_t n, int accumulate, mle_stream_t stream);

/* *count (device) = the number of NaN elements of x.  The reference's ISNAN
 * (Includes/kernels.h:381-391) traps the GPU on the first NaN; this counts
 * them and leaves the decision to the host (isNan prints and exits). */
int mle_count_nan(const float* x, int64_t n, unsigned long long* count, mle_stream_t stream);

/* *out (device) = the first index of the largest of x[0..n) (ArgMax,
 * Engine/kernels.cu:2353-2366, one block instead of one thread). */
int mle_argmax(const float* x, int64_t n, int* out, mle_stream_t stream);

/* x = mean + std * N(0,1) (kind 0) or mean + std * U[0,1) (kind 1) from a
 * counter-based generator keyed by `seed` (Noise / GaussianNoise /
 * UnifNoise, Engine/engine.cu:3936-3944; the reference draws from cuRAND, so
 * the values differ and the distributions agree). */
int mle_fill_noise(float* x, int64_t n, float mean, float stdv, int kind, uint64_t seed, mle_stream_t stream);

/* Embedding SGD update, the replacement of KeyUpdate (Engine/kernels.cu:
 * 1536-1549) as TextualEmbedding::EmbeddingUpdate launches it
 * (Engine/transformer.cu:233-245; key_stride = MAX_CONTEXT_LEN there):
 *   grad_scatter  gsum[key, :] += grad[r, :] for each of the `rows` gradient
 *                 rows (grad [rows, dim], rows = batch * row_len tokens; the
 *                 key of token t of batch b at keys[b * key_stride + t];
 *                 keys < 0, masked tokens, skipped);
 *   apply         table = fma(neg_lr, gsum, table) over n = vocab * dim;
 *   update        both, with gsum (vocab * dim floats, caller-owned) cleared
 *                 first: table[key] -= lr * (sum of its rows' gradients).
 * For a key that occurs once this is the reference's own arithmetic (one
 * fused multiply-add per element), bit for bit.  The reference adds repeated
 * keys' rows without atomics, so they race and its result is undefined;
 * here their gradients are summed first (atomically, in no fixed order). */
int mle_embedding_grad_scatter(const int32_t* keys, const float* grad, float* gsum, int64_t rows, int dim,
                               int row_len, int key_stride, mle_stream_t stream);
int mle_embedding_apply(float* table, const float* gsum, int64_t n, float neg_lr, mle_stream_t stream);
int mle_embedding_update(const int32_t* keys, const float* grad, float* table, float* gsum, int vocab, int64_t rows,
                         int dim, int row_len, int key_stride, float lr, mle_stream_t stream);

/* ------------------------------------------------------------------ */
/* normalisation                                                        */
/* ------------------------------------------------------------------ */

/* LayerNorm over each dim0 index (N = channels*row*col elements), gamma=1,
 * beta=0: writes y, mean[batch] and sqdev[batch] = sum (x-mean)^2.
 * Replaces LayerMean+LayerStd+LNorm (Engine/kernels.cu:541-572,670-699,
 * 794-804) as launched by LayerNorm forward (Engine/engine.cu:3099-3113). */
int mle_layernorm_fwd(const float* x, float* y, float* mean, float* sqdev, int batch,
                      int channels, int row, int col, float eps, mle_stream_t stream);

/* The residual Add and the LayerNorm that reads its sum, in one pass:
 * xr = x + r (GraphOperations::Add forward, Engine/engine.cu:1650-1655, as
 * ScaleAdd with scale 1) and then mle_layernorm_fwd of xr into y, mean and
 * sqdev -- both outputs bitwise those of the two launches.  Segments of up
 * to 1024 elements (a multiple of 4) with 16-byte aligned x, r, xr and y;
 * other shapes return MLE_ERR_UNSUPPORTED with nothing written (the caller
 * then launches the two apart). */
int mle_add_layernorm_fwd(const float* x, const float* r, float* xr, float* y, float* mean, float* sqdev, int batch,
                          int channels, int row, int col, float eps, mle_stream_t stream);

/* LayerNorm backward gx += rstd*(gy - sum(gy)/N - y*sum(gy*y)/N), with the
 * reference's index map (only the first batch*row*col elements, correct for
 * channels == 1).  Replaces Scale_Write+mulKernel+2xLayerMean+LayerBackward
 * (Engine/engine.cu:3116-3130, Engine/kernels.cu:849-862). */
int mle_layernorm_bwd(const float* y, const float* gy, const float* sqdev, float* gx, int batch,
                      int channels, int row, int col, float eps, mle_stream_t stream);

/* GroupNorm forward/backward over (sample, group) blocks of
 * (channels/groups)*row*col elements.  Replaces GroupMean/GroupStd/GNorm and
 * GroupBackward (Engine/kernels.cu:607-639,732-763,818-834,877-896) as used by
 * GroupNorm (Engine/engine.cu:3232-3270). */
int mle_groupnorm_fwd(const float* x, float* y, float* mean, float* sqdev, int batch,
                      int channels, int groups, int row, int col, float eps, mle_stream_t stream);
int mle_groupnorm_bwd(const float* y, const float* gy, const float* sqdev, float* gx, int batch,
                      int channels, int groups, int row, int col, float eps, mle_stream_t stream);

/* ------------------------------------------------------------------ */
/* softmax and losses                                                   */
/* ------------------------------------------------------------------ */

/* Softmax over [bc, rows, cols].  axis 0 normalises each row over its
 * columns, axis 1 normalises each column over its rows (the reference's
 * "type 1", used by attention).  causal != 0 zeroes entries with col > row
 * before normalising (SoftMask).  An all-zero line is divided by 1 as in
 * SumRows/SumCols.  Replaces SoftMax/SoftMask (Engine/kernels.cu:2183-2235). */
int mle_softmax_fwd(const float* x, float* y, int64_t bc, int rows, int cols, int axis,
                    int causal, mle_stream_t stream);

/* gx += y * (gy - sum_axis(gy*y)).  Replaces deriv_softmax
 * (Engine/kernels.cu:2149-2181). */
int mle_softmax_bwd(const float* y, const float* gy, float* gx, int64_t bc, int rows, int cols,
                    int axis, mle_stream_t stream);

/* Softmax cross-entropy forward over rows of `cols` logits with a dense
 * target: probs = softmax_row(logits); *loss = sum(-t*log(p+1e-27)) / (rows*cols)
 * (assigned).  If grad != NULL the same pass also writes the `last=true`
 * backward grad[r,c] = (p - t) / batch_div (assign), which is what
 * SoftMaxCrossEntropy backward computes (Engine/engine.cu:2090-2111,
 * Engine/kernels.cu:1818-1826).  probs may be NULL when not needed. */
int mle_softmax_ce_fwd(const float* logits, const float* target, float* probs, float* loss,
                       float* grad, float batch_div, int64_t rows, int cols, mle_stream_t stream);

/* SoftMaxCrossEntropy backward from stored probabilities:
 * grad = (probs - target) [* upstream[0]] / batch_div (assign). */
int mle_softmax_ce_bwd(const float* probs, const float* target, const float* upstream,
                       float* grad, float batch_div, int64_t n, mle_stream_t stream);

/* The same two entry points with the target as one int32 class index per
 * row instead of the dense one-hot tensor the reference builds with
 * OneHotEmbeddings (no counterpart in the reference: an index-label
 * variant that skips building the one-hot tensor).  Loss, probs and grad
 * equal the dense entry points' on the one-hot target of `labels`, bit for
 * bit; a label outside [0, cols) is a row of zeros.  The forward needs cols % 4 == 0, cols <= 8192 and 16-byte
 * aligned logits/probs/grad (else MLE_ERR_UNSUPPORTED). */
int mle_softmax_ce_index_fwd(const float* logits, const int32_t* labels, float* probs, float* loss,
                             float* grad, float batch_div, int64_t rows, int cols,
                             mle_stream_t stream);
int mle_softmax_ce_index_bwd(const float* probs, const int32_t* labels, const float* upstream,
                             float* grad, float batch_div, int64_t rows, int cols,
                             mle_stream_t stream);

/* Mean squared error: *loss = sum (t-x)^2 / n (assigned);
 * backward gx += 2 (x-t)/n [* upstream[0]].  Replaces scalar_mse_kernel and
 * deriv_mse_kernel (Engine/kernels.cu:1808-1848). */
int mle_mse_fwd(const float* x, const float* target, float* loss, int64_t n, mle_stream_t stream);
int mle_mse_bwd(const float* x, const float* target, const float* upstream, float* gx, int64_t n,
                mle_stream_t stream);

/* ------------------------------------------------------------------ */
/* tensor-core GEMM (tcgen05 kind::tf32, TMEM accumulator, TMA operands) */
/* ------------------------------------------------------------------ */

/* How the GEMM entry points below multiply, per host thread:
 *   MLE_GEMM_MODE_TF32: tcgen05 kind::tf32 tensor cores with fp32
 *     accumulation wherever TMA can describe the operands (default);
 *   MLE_GEMM_MODE_FP32: CUDA-core fp32 FMA chains in k order, the
 *     reference's own product arithmetic (for graphs whose forward feeds a
 *     discontinuous derivative, e.g. ReLU masks, where TF32 rounding of a
 *     pre-activation near zero flips the mask). */
enum mle_gemm_mode { MLE_GEMM_MODE_TF32 = 0, MLE_GEMM_MODE_FP32 = 1 };
int mle_set_gemm_mode(int mode);
int mle_get_gemm_mode(void);

/* Whether the tensor-core GEMM may compute large products (at least two
 * waves of 128 x 128 tiles) on CTA pairs: 2-CTA clusters whose 256 x 256
 * tiles issue cta_group::2 MMAs, each SM staging half of the tile's B, so
 * a pair fills shared memory with a third fewer bytes per FLOP.  0 off,
 * 1 (default) where the tile model prefers them, 2 wherever the shapes
 * allow (a measurement aid).  Per host thread; no counterpart in the
 * reference. */
int mle_set_gemm_pairs(int enable);
int mle_get_gemm_pairs(void);
/* k-blocks (32 fp32 of K) per pipeline stage of the tensor-core GEMM: 2
 * (default) stages two k-blocks of each operand with ONE tiled copy, where
 * both operands' contiguous extents (K for a K-major operand, M or N for
 * an MN-major one) are multiples of 32, else one; 1 forces one k-block
 * per stage.  A copy engine serves few large copies faster than many
 * small ones (measured on B200: 30 B/clk per SM for 16 KB boxes, 47 for
 * 32 KB, 59 for 64 KB).  mle_gemm_last_stage_kblocks() reports the value
 * this thread's last product ran with (0 after an mle_gemm call that did
 * not run on the tensor cores).  Per host thread; no counterpart in the
 * reference. */
int mle_set_gemm_stage_kblocks(int kblocks);
int mle_get_gemm_stage_kblocks(void);
int mle_gemm_last_stage_kblocks(void);
/* Element type of the tensor-core GEMM's operand loads: 0 fp32 (the MMA
 * uses the TF32 part of each value: its low 13 mantissa bits are dropped),
 * 1 (default) TF32 (tensor maps of TF32 element type: the copy engine
 * rounds each fp32 value to the nearest TF32, ties to even, as it lands in
 * shared memory).  Outputs and accumulation are fp32 either way.  Per host
 * thread; no counterpart in the reference. */
int mle_set_gemm_operand_rounding(int mode);
int mle_get_gemm_operand_rounding(void);
/* Where a Linear's bias gradient comes from when its weight gradient is
 * taken too (mle_linear_bwd, mle_linear_group_bwd with dW and dB): 1
 * (default) the epilogue warps of the dW product sum dY's columns from the
 * dY tiles as they pass through shared memory (in a CTA pair each CTA the
 * columns it staged; launches of at most one tile per CTA, else a separate
 * column sum follows), so dB uses the operand values the product uses --
 * TF32-rounded under operand rounding 1, the fp32 values under 0; 0 a
 * separate column-sum launch of the fp32 dY (BCompress,
 * Engine/kernels.cu:1562-1584).  Per host thread. */
int mle_set_gemm_column_sums(int enable);
int mle_get_gemm_column_sums(void);
/* 1 when the calling thread's last product took its column sums in its
 * epilogue warps, 0 when a separate column-sum launch followed (or none was
 * asked for).  The epilogue takes them only for launches of at most one
 * tile per CTA: a CTA with several tiles would lose the overlap of one
 * tile's epilogue with the next tile's mainloop. */
int mle_gemm_last_column_sums(void);
/* Forces the tile width (64, 128 or 256), the split-K count (1..64, as
 * many as the k-blocks allow) and CTA pairs (0/1) of this thread's plain
 * and grouped tensor-core products (convolutions keep the tile model);
 * bn = 0 returns to the tile model.  A measurement aid for tuning the
 * model; no counterpart in the reference. */
int mle_set_gemm_tiles(int bn, int splits, int pair);
/* out3 = {tile width, split-K count, 1 if CTA pairs} of this thread's last
 * single tensor-core product (diagnostics for tests and benchmarks). */
int mle_gemm_last_choice(int* out3);
/* How the tensor-core GEMM writes assigned outputs on this host thread:
 * 0 bulk tensor (TMA) stores of staged 32 x 32 blocks, 1 (default) the
 * epilogue warps' own row-contiguous 16-byte stores, measured faster on
 * B200 for every shape tried.  Accumulated outputs always use bulk tensor
 * reduce-adds.  No counterpart in the reference. */
int mle_set_gemm_store_path(int path);

/* Batched GEMM with the reference's broadcast flags.  Same argument meaning
 * as bcmm/bcmmABT/bcmmATB/bcmmT (Engine/kernels.cu:387-539): `backward`!=0
 * adds scale*product into C (the reference's atomicAdd), 0 assigns it.
 * Flags A_case/B_case/C_case in {0,1,2,3}: bit 0 = has batch, bit 1 = has
 * channel.  Whenever several (batch, channel) products map onto one C
 * matrix they are summed, exactly as the reference's atomics do. */
int mle_bcmm(int variant, const float* A, const float* B, float* C, int batch, int channels,
             int m, int n, int p, int backward, int A_case, int B_case, int C_case, float scale,
             mle_stream_t stream);

/* Plain strided GEMM  C = alpha * op(A) * op(B) + beta * C  (+ bias[col]),
 * row-major, op(A) is [M,K], op(B) is [K,N].  beta must be 0 or 1.
 * trans_a: A stored [K,M]; trans_b: B stored [N,K].  lda/ldb/ldc are row
 * strides in elements; batch strides may be 0 (broadcast). */
int mle_gemm(const float* A, const float* B, float* C, const float* bias, int batch, int64_t M,
             int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc, int64_t stride_a,
             int64_t stride_b, int64_t stride_c, int trans_a, int trans_b, float alpha, float beta,
             mle_stream_t stream);

/* Linear layer forward Y = X*W (+ bias), X [rows, in], W [in, out] ([1,1,in,out]
 * AdamParameter), Y [rows, out].  Replaces bcmm(...,0,3,0,3) + BCumAdd in
 * Linear::forward (Engine/engine.cu:3536-3548), with the batch*channel*m
 * rows flattened into one GEMM. */
int mle_linear_fwd(const float* X, const float* W, const float* bias, float* Y, int64_t rows,
                   int in_features, int out_features, mle_stream_t stream);

/* Linear layer backward: dX += dY*W^T (if dX != NULL), dW += X^T*dY as one
 * GEMM with K = rows (if dW != NULL), dB += column sums of dY (if dB !=
 * NULL); X is read only for dW.  The parts may run on different streams as
 * separate calls (input gradient on one, parameter gradients on another).
 * Replaces
 * bcmmABT + bcmmATB + BCompress of the Linear backward lambda
 * (Engine/engine.cu:3550-3563) without its two device synchronisations. */
int mle_linear_bwd(const float* X, const float* W, const float* dY, float* dX, float* dW,
                   float* dB, int64_t rows, int in_features, int out_features,
                   mle_stream_t stream);

/* ------------------------------------------------------------------ */
/* fused attention backward                                             */
/* Up to three Linear layers that read the same input X -- the query, key
 * and value projections of MultiHeadAttention::forward
 * (Engine/transformer.cu:647-650) -- in one persistent tensor-core launch
 * each way, with the semantics of n separate mle_linear_fwd / _bwd calls:
 *   forward : Y_i = X W_i (+ b_i) (assigned), W_i [in, out_i];
 *   backward: dX += sum_i dY_i W_i^T (one launch, reduce-added), dW_i +=
 *             X^T dY_i (one launch), dB_i += column sums of dY_i;
 *             dX, dW (all weight gradients skipped), bias and dB (or any
 *             dB[i]) may be NULL.
 * Pointer arrays are HOST arrays of n device pointers. */
int mle_linear_group_fwd(const float* X, const float* const* W, const float* const* bias, float* const* Y,
                         int n, int64_t rows, int in_features, const int* out_features,
                         mle_stream_t stream);
int mle_linear_group_bwd(const float* X, const float* const* W, const float* const* dY, float* dX,
                         float* const* dW, float* const* dB, int n, int64_t rows, int in_features,
                         const int* out_features, mle_stream_t stream);

/* ------------------------------------------------------------------ */

/* Key-gradient semantics of mle_attention_bwd.
 *   MLE_KEYGRAD_REFERENCE: what the reference's BMMABT backward computes,
 *     bcmmT(Q, dScores, K.grad, n, m, p) (Engine/engine.cu:2307): dScores'
 *     memory is read as a [Sk, Sq] matrix M and K.grad's memory receives
 *     (M Q)^T laid out [hd, Sk].  This equals dScores^T Q only when
 *     Sq == Sk == hd; it is the drop-in default because it is the
 *     reference's result.
 *   MLE_KEYGRAD_TRUE: dK += scale * dS^T Q, the mathematical gradient. */
enum mle_keygrad_mode { MLE_KEYGRAD_REFERENCE = 0, MLE_KEYGRAD_TRUE = 1 };

/* Layout of Q, K, V, O and their gradients in the attention entry points:
 *   MLE_ATTN_HEAD_MAJOR : [B, H, S, hd] (the Headify nodes' tensors);
 *   MLE_ATTN_TOKEN_MAJOR: [B, S, H*hd] (the q/k/v Linear outputs and the
 *                         DeHeadify output), so no head copies are needed.
 * P and the score gradients are always [B, H, Sq, Sk]. */
enum mle_attn_layout { MLE_ATTN_HEAD_MAJOR = 0, MLE_ATTN_TOKEN_MAJOR = 1 };

/* Forward of the attention sub-graph built by MultiHeadAttention::forward /
 * cross_forward (Engine/transformer.cu:647-675): P = softmax_axis(scale *
 * Q K^T) [causal: entries with key > query zeroed before normalising],
 * O = P V (assigned).  Replaces bcmmABT (BMMABT), Scale_Write, SoftMax /
 * SoftMask and bcmm (BMM) plus the Headify/DeHeadify copies.  The column-
 * wise softmax (axis 1) runs as two fused kernels (P by key blocks, O by
 * query blocks) whose sums follow the reference kernels' order, so P and O
 * are bitwise the reference's; other shapes run the composed path
 * (head-major only).  Q, K, V, O (and, backward, dO, dQ, dK, dV) must be
 * 16-byte aligned for the fused path. */
int mle_attention_fwd(const float* Q, const float* K, const float* V, float* P, float* O,
                      int batch, int heads, int seq_q, int seq_k, int head_dim, float scale,
                      int causal, int softmax_axis, int layout, mle_stream_t stream);

/* Backward of the same sub-graph.  Inputs Q, K, V, dO in `layout`, P as
 * written by the forward.  Accumulates dQ, dK, dV (+=) in `layout`; if
 * dP_out / dS_out are non-NULL they receive (+=) the softmax node's
 * gradient dO V^T and the Scale node's gradient (the softmax backward), as
 * the reference keeps them in node->grad.  The fused path needs
 * `workspace`, batch*heads*seq_q*seq_k floats of scratch (left holding
 * the score gradients); the composed path ignores it and needs dP_out and
 * dS_out instead.  Replaces bcmmABT/bcmmATB (BMM bwd), deriv_softmax,
 * Accumulate (Scale bwd), bcmm/bcmmT (BMMABT bwd) and the Headify backward
 * copies (Engine/engine.cu:2246-2253,2302-2309,2450-2455,2488-2493,
 * 2540-2546).  The fused kernels keep the reference's summation order for
 * every product. */
int mle_attention_bwd(const float* Q, const float* K, const float* V, const float* P,
                      const float* dO, float* dQ, float* dK, float* dV, float* dP_out,
                      float* dS_out, float* workspace, int batch, int heads, int seq_q, int seq_k,
                      int head_dim, float scale, int causal, int softmax_axis, int key_grad_mode,
                      int layout, mle_stream_t stream);
/* The same with dQ (assign_mask bit 0), dK (bit 1) and/or dV (bit 2)
 * written instead of accumulated: the tensor-core path writes them with
 * beta = 0 products, the other paths clear them and accumulate.  For the
 * first writer of gradient buffers that are not cleared between steps;
 * an assigned gradient may not alias another one (MLE_ERR_ARG). */
int mle_attention_bwd_assign(const float* Q, const float* K, const float* V, const float* P,
                             const float* dO, float* dQ, float* dK, float* dV, float* dP_out, float* dS_out,
                             float* workspace, int batch, int heads, int seq_q, int seq_k, int head_dim,
                             float scale, int causal, int softmax_axis, int key_grad_mode, int layout,
                             int assign_mask, mle_stream_t stream);

/* 1 if mle_attention_fwd/bwd take the fused path for these sizes (any
 * layout), 0 if they need the head-major composed path. */
int mle_attention_fused_supported(int seq_q, int seq_k, int head_dim, int softmax_axis, int key_grad_mode);

/* Which implementation mle_attention_fwd/bwd use for the column softmax on
 * this host thread (no counterpart in the reference):
 *   MLE_ATTN_PATH_AUTO  : tensor cores in TF32 GEMM mode when the heads are
 *                         not tiny (Sq*Sk*hd >= 2^18, e.g. 128 x 128 x 32),
 *                         the CUDA-core kernels in the reference's summation
 *                         order otherwise and in FP32 GEMM mode;
 *   MLE_ATTN_PATH_FUSED : always the CUDA-core kernels where they apply;
 *   MLE_ATTN_PATH_TENSOR: tensor cores wherever the sizes allow (TF32 GEMM
 *                         mode, Sq, Sk, hd multiples of 4; the
 *                         reference key gradient also needs Sq == Sk, hd a
 *                         multiple of 32 dividing Sk).
 * The tensor-core backward writes its score gradients to `workspace`. */
enum mle_attn_path { MLE_ATTN_PATH_AUTO = 0, MLE_ATTN_PATH_FUSED = 1, MLE_ATTN_PATH_TENSOR = 2 };
int mle_set_attention_path(int path);
int mle_get_attention_path(void);

/* On the tensor-core path (softmax axis 1): 1 (default) computes P =
 * softmax(scale Q K^T) over each key column, and the score gradient
 * P (dP - column sums of P dP) with dP = dO V^T, each in one kernel that
 * holds one key per TMEM lane and all its queries in the lane's columns
 * (Sq <= 256, head_dim 32, 64 or 128), so the scores and dP never reach
 * HBM; 0 writes the product to HBM and runs the column softmax (or its
 * backward) over it.  Process-wide per host thread. */
int mle_set_attention_keys_kernel(int enable);
int mle_get_attention_keys_kernel(void);

/* Attention with the column softmax (softmax axis 1) whose score matrices
 * never reach HBM (no counterpart in the reference, whose MultiHeadAttention
 * writes scale*QK^T, P, dP and dS as [B, H, Sq, Sk] tensors,
 * Engine/transformer.cu:647-675).  The forward writes O and two numbers per
 * key, stats = [column max m (B*H*Sk floats), inverse column sum 1/l
 * (B*H*Sk floats)]; P = exp(scale QK^T - m) / l (0 where causal masks key >
 * query) equals the P of mle_attention_fwd to rounding.  The backward
 * recomputes P from Q, K and stats and writes dQ, dK, dV (bits of
 * assign_mask as in mle_attention_bwd_assign), using dvec (B*H*Sk floats)
 * as workspace for the per-key dot products sum_q P dP.  key_grad_mode as
 * for mle_attention_bwd (the reference's BMMABT key gradient or the true
 * one).  Tensor cores (TF32 GEMM mode) only: *_supported returns 1 for
 * softmax_axis 1, seq_q <= 256, seq_k <= 512, head_dim 32 or 64 (the
 * reference key gradient also needs seq_q == seq_k, seq_k % head_dim == 0)
 * while mle_set_attention_flash(1) (the default) holds; otherwise the entry
 * points return MLE_ERR_UNSUPPORTED with nothing written.  Pointers 16-byte
 * aligned. */
int mle_attention_flash_supported(int seq_q, int seq_k, int head_dim, int softmax_axis, int key_grad_mode);
int mle_attention_flash_fwd(const float* Q, const float* K, const float* V, float* O, float* stats, int batch,
                            int heads, int seq_q, int seq_k, int head_dim, float scale, int causal, int layout,
                            mle_stream_t stream);
int mle_attention_flash_bwd(const float* Q, const float* K, const float* V, const float* dO, const float* stats,
                            float* dvec, float* dQ, float* dK, float* dV, int batch, int heads, int seq_q,
                            int seq_k, int head_dim, float scale, int causal, int key_grad_mode, int layout,
                            int assign_mask, mle_stream_t stream);
/* 1 (default): graph attention nodes take the entry points above where
 * they are supported; 0: mle_attention_fwd/bwd.  Per host thread. */
int mle_set_attention_flash(int enable);
int mle_get_attention_flash(void);

/* Positional table of MatPEncoding alone, table[r, c] = (float)sin/cos of
 * the angle for position r + start_idx (Engine/kernels.cu:166-185), and its
 * broadcast add y[b, i] = x[b, i] + table[i]: together bitwise equal to
 * mle_matpe_fwd, with the trigonometry done once at graph build. */
int mle_matpe_table(float* table, int rows, int cols, int start_idx, mle_stream_t stream);
int mle_rows_add_table(const float* x, const float* table, float* y, int64_t batch, int64_t row_elems,
                       mle_stream_t stream);

/* ------------------------------------------------------------------ */
/* 2-D convolution and transposed convolution (NCHW, fp32)              */
/* ------------------------------------------------------------------ */

/* Output size of Convolute2D, (in + 2*pad - k)/stride + 1 (-1 if the
 * kernel does not fit), and of Convolute2DT, (in - 1)*stride - 2*pad + k
 * (Engine/engine.cu:3744-3745,3842-3843). */
int mle_conv_out_size(int in, int k, int pad, int stride);
int mle_convT_out_size(int in, int k, int pad, int stride);

/* cols[n][(c*kh + i)*kw + j][oy*OW + ox] = x[n][c][oy*stride - pad + i][ox*stride - pad + j]
 * (0 outside the image), OH/OW from mle_conv_out_size; and the gather
 * adjoint x[n][c][y][x] (= or +=) sum of the columns entries that read it. */
int mle_im2col(const float* x, float* cols, int batch, int channels, int h, int w, int kh, int kw,
               int pad, int stride, mle_stream_t stream);
int mle_col2im(const float* cols, float* x, int batch, int channels, int h, int w, int kh, int kw,
               int pad, int stride, int accumulate, mle_stream_t stream);
/* out = in with two of its three dimensions exchanged: mode 0
 * [a][b][c] -> [b][a][c], mode 1 [a][b][c] -> [a][c][b]. */
int mle_swap_dims(const float* in, float* out, int a, int b, int c, int mode, mle_stream_t stream);

/* Stride-2 convolutions (mle_conv2d_fwd / _bwd) in tensor-core mode as the
 * stride-1 implicit GEMM over the input's polyphase sub-images -- phase
 * (py, px) = x[2Y + py][2X + px] becomes a block of channels, each tap
 * (kh, kw) a tap of a kernel of ceil-half size with top/left padding only
 * -- with a one-pass phase split (and a phase merge of dx); the weights are
 * expanded to and dW folded back from that kernel.  2: always; 1: where
 * that kernel has no empty taps (1x1 and 2x2 kernels: a pure re-layout; a
 * 3x3 kernel runs 16 products per output for 9); 0 (default): never
 * (im2col + GEMM + col2im, which measured faster on the U-Net step: 5.07 ms
 * against 5.11 ms with 1 and 5.24 ms with 2).  Shapes the implicit path
 * cannot take fall
 * back to im2col.  Per host thread; the forward and the backward of one
 * convolution must see the same setting (they share the workspace layout).
 * No counterpart in the reference. */
int mle_set_conv_phase(int enable);
int mle_get_conv_phase(void);

/* Convolute2D (Engine/engine.cu:3732-3817): weights [cout][cin][kh][kw],
 * x [batch][cin][h][w], y [batch][cout][OH][OW].
 *   forward : y = conv(x) (+ bias) (assigned, CV2D Engine/kernels.cu:985-1019);
 *             ws (mle_conv2d_workspace_floats floats) receives what the
 *             backward reads of x (shifted copies of x for the stride-1
 *             implicit GEMM, else its im2col columns) and must still hold
 *             it when the backward runs;
 *   backward: dw = sum over the batch (assigned, GV2D :1021-1051), db +=
 *             channel sums (Channel_Squeeze1D :1734-1761), dx += (CV2D_GradInput
 *             :1053-1089); x is the forward's input; any of dx, dw, db may be
 *             NULL.  The dx part and the dw/db part touch disjoint regions of
 *             ws, so they may be issued as two calls on two streams (each
 *             after the forward); either part may run once per forward. */
int64_t mle_conv2d_workspace_floats(int batch, int cin, int h, int w, int cout, int kh, int kw, int pad,
                                    int stride);
int mle_conv2d_fwd(const float* x, const float* wgt, const float* bias, float* y, float* ws, int batch,
                   int cin, int h, int w, int cout, int kh, int kw, int pad, int stride,
                   mle_stream_t stream);
int mle_conv2d_bwd(const float* x, const float* wgt, const float* dy, float* dx, float* dw, float* db,
                   float* ws, int batch, int cin, int h, int w, int cout, int kh, int kw, int pad,
                   int stride, mle_stream_t stream);
/* The same with dx written instead of accumulated when assign_dx is 1 (dx's
 * previous contents are not read): for the first writer of an input
 * gradient that is not cleared between steps. */
int mle_conv2d_bwd_assign(const float* x, const float* wgt, const float* dy, float* dx, float* dw, float* db,
                          float* ws, int batch, int cin, int h, int w, int cout, int kh, int kw, int pad,
                          int stride, int assign_dx, mle_stream_t stream);

/* Convolute2DT (Engine/engine.cu:3828-3912): weights [cout][cin][kh][kw],
 * x [batch][cin][h][w], y [batch][cout][OH][OW] with OH from
 * mle_convT_out_size.  forward y = (assigned, CVT2D :1091-1135) (+ bias);
 * backward dw = (assigned, GVT2D :1137-1176), db += , dx = (assigned,
 * CVT2D_GradInput :1178-1212).  ws: mle_convT2d_workspace_floats floats,
 * scratch for each call. */
int64_t mle_convT2d_workspace_floats(int batch, int cin, int h, int w, int cout, int kh, int kw, int pad,
                                     int stride);
int mle_convT2d_fwd(const float* x, const float* wgt, const float* bias, float* y, float* ws, int batch,
                    int cin, int h, int w, int cout, int kh, int kw, int pad, int stride,
                    mle_stream_t stream);
int mle_convT2d_bwd(const float* x, const float* wgt, const float* dy, float* dx, float* dw, float* db,
                    float* ws, int batch, int cin, int h, int w, int cout, int kh, int kw, int pad,
                    int stride, mle_stream_t stream);

/* ------------------------------------------------------------------ */
/* gradient-norm clip + Adam/AdamW                                      */
/* ------------------------------------------------------------------ */

/* One parameter tensor as seen by the optimizer.  t points at the tensor's
 * step counter in DEVICE memory (AdamParameter::t, Includes/engine.h:64);
 * the update reads it and the same launch increments it, so a captured
 * CUDA graph replays the reference's per-tensor t++ (Engine/engine.cu:291). */
typedef struct mle_param_view {
    float* w;
    float* g;
    float* m;
    float* v;
    int64_t n;
    int32_t* t;
    float b1, b2, eps, weight_decay;
} mle_param_view;

/* *norm_ws += scale^2 * sum over all tensors of g^2, accumulated in double.
 * Replaces one SumSquared launch per tensor (AdamParameter::accumulate_grad,
 * Engine/engine.cu:294-300; Engine/kernels.cu:1486-1506).  `params` is a
 * HOST array; its contents travel as kernel parameters (no allocation). */
int mle_grad_sumsq(const mle_param_view* params, int n_tensors, double* norm_ws, double scale,
                   mle_stream_t stream);

/* *norm_ws = max(sqrt(*norm_ws), max_norm) (a NaN is left unchanged).
 * Replaces Sqrt_Scale<<<1,1>>>(ws, 1.0, 0) (Engine/kernels.cu:1763-1773)
 * for max_norm = 1, as called by GraphOperations::accumulate
 * (Engine/engine.cu:3364-3368). */
int mle_clip_finalize(double* norm_ws, double max_norm, mle_stream_t stream);

/* g /= (float)(*norm_ws) in place for every tensor.  Replaces the per-tensor
 * SP launches of GraphOperations::clipNorm (Engine/engine.cu:3362,302). */
int mle_clip_apply(const mle_param_view* params, int n_tensors, const double* norm_ws,
                   mle_stream_t stream);

/* Fused multi-tensor update.  For every tensor: g' = g * pre_scale, then if
 * clip_ws != NULL g' = g' / (float)(*clip_ws) (written back to g when
 * write_back_grad != 0), then AdamW (adamw != 0) or Adam with the
 * reference's arithmetic (AdamWUpdate/AdamUpdate, Engine/kernels.cu:1508-1534),
 * then *t += 1.  One launch replaces the per-tensor AdamParameter::update
 * loop (Engine/engine.cu:283-292, 3370-3384). */
int mle_adam_update(const mle_param_view* params, int n_tensors, const double* clip_ws,
                    float pre_scale, float lr, int adamw, int write_back_grad,
                    mle_stream_t stream);

/* Norm, clip and update as ONE launch.  Replaces, together, the per-tensor
 * SumSquared launches, Sqrt_Scale, the SP launches and the AdamWUpdate loop
 * of GraphOperations::accumulate / clipNorm / ParameterUpdate
 * (Engine/engine.cu:283-302, 3362-3384; Engine/kernels.cu:1486-1534,
 * 1763-1773).  A cooperative kernel (every block resident) gives each block
 * a contiguous range of 4096-element chunks over all tensors; each block
 * sums g^2 over its range into the workspace, passes a grid barrier, adds
 * all partials in block order (times pre_scale^2) and forms
 * c = max(||g||, max_norm)/max_norm (max_norm <= 0: no clip and no barrier;
 * a NaN norm stays NaN); it then walks its range again, backwards, applying
 * g' = g * pre_scale / (float)c and the same per-element Adam/AdamW
 * arithmetic as mle_adam_update.  The last block to finish adds 1 to every
 * tensor's t.  g' is written back when write_back_grad != 0.
 *
 * Workspace: mle_clip_adam_ws_bytes(n) bytes of device memory, 16-byte
 * aligned, owned by the caller.  mle_clip_adam_prepare copies the tensor
 * table and zeroed counters into it (stream ordered; MLE_ERR_UNSUPPORTED
 * while the stream is being captured, since the table is a host array);
 * every later run reuses it with no further copy or memset, so runs of a
 * prepared workspace may be replayed inside a CUDA graph.  Runs on one
 * workspace must not overlap on the device.  The grid barrier waits at most
 * two seconds; a wait that gives up sets a status word and ends the kernel
 * early (the update then incomplete), and every later run returns at once
 * until the workspace is prepared again.  mle_clip_adam_status reads the
 * word (synchronizing the stream) and returns MLE_ERR_TIMEOUT when it is
 * set.  The clip coefficient's summation order differs from
 * mle_grad_sumsq's (per-block partials instead of atomics), so it agrees to
 * rounding; with no clip the result is bit-identical to mle_adam_update. */
int64_t mle_clip_adam_ws_bytes(int n_tensors);
int mle_clip_adam_prepare(const mle_param_view* params, int n_tensors, void* ws, int64_t ws_bytes,
                          mle_stream_t stream);
int mle_clip_adam_run(void* ws, float max_norm, float pre_scale, float lr, int adamw, int write_back_grad,
                      mle_stream_t stream);
int mle_clip_adam_status(void* ws, int* out_status, mle_stream_t stream);

/* No counterpart in the reference: a gradient-norm clip that needs no
 * workspace from the caller.  It computes what mle_grad_sumsq (scale 1),
 * mle_clip_finalize and mle_clip_apply compute together -- g /= c with
 * c = max(||g||, max_norm) / max_norm over all tensors -- but keeps its
 * scratch (one double per 4096-element block of gradients plus the
 * coefficient) in a static device array of the library, so a caller that
 * owns no device memory of its own (a host binding only this C ABI, or a
 * training loop whose memory is planned once at graph build and must not
 * call cudaMalloc, which can synchronise the device, in the middle of a
 * step) can still clip.  The per-block sums are added in a fixed order,
 * so the coefficient does not depend on block scheduling.
 *   - Limit: the tensors may span at most MLE_CLIP_STATIC_MAX_BLOCKS blocks
 *     of 4096 elements (each tensor rounded up to whole blocks, an empty
 *     tensor counting as one), about 33.5 million gradient elements; larger
 *     sets return MLE_ERR_ARG before anything is launched.
 *   - If coef_out != NULL (device pointer) it receives c, the value
 *     mle_clip_finalize leaves in norm_ws.
 *   - Nothing in the scratch has to start at zero: every slot read is
 *     written earlier in the same call.
 *   - The scratch is one array per device: calls that overlap in time
 *     (several streams or host threads on one device) race on it.
 *   - The first call on each device resolves the scratch's address with
 *     cudaGetSymbolAddress (with that device current); make that first
 *     call before any stream capture on the device. */
#define MLE_CLIP_STATIC_MAX_BLOCKS 8192
int mle_clip_grad_norm_static(const mle_param_view* params, int n_tensors, double max_norm,
                              double* coef_out, mle_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MLE_KERNELS_H */
