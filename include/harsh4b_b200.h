/*
 * harsh4b_b200 -- C ABI of the B200 (sm_100a) decode backend for the
 * Qwen3-4B packed int4 model.
 *
 * Conventions (following the reference's native ABI,
 * cpu_kernels/litespark_int4.cpp:78-81): extern "C", raw pointers and int
 * sizes, the caller owns every buffer, outputs land in caller memory, and
 * nothing allocates on the hot path. Unlike the reference (which returns
 * void), every entry point returns an int status: 0 on success, a positive
 * cudaError_t value for a CUDA failure, or a negative H4B_E* code for a
 * rejected argument. All data pointers are DEVICE pointers unless named
 * host_*; `stream` is a cudaStream_t (NULL = legacy default stream).
 *
 * Weight layout (the reference's packed cache, cpu_lightspark.py:139-146,
 * :571-676): uint8[rows, width/2], row-major, two signed int4 codes per
 * byte, low nibble = even column, codes in [-7, +7]; float32 row scales.
 */
#ifndef HARSH4B_B200_H
#define HARSH4B_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define H4B_EINVAL (-1)       /* bad size, alignment or pointer */
#define H4B_EUNSUPPORTED (-2) /* shape outside what the kernels implement */
#define H4B_ETOOBIG (-3)      /* request exceeds the library's static scratch */

/* Device-side status word (bit 1: a bounded wait gave up; bit 2: token id
 * out of range; bit 4: position beyond capacity). Reads and clears it; the
 * read synchronises with the device. */
int h4b_get_status(int *host_status);

/* One-time set-up of the current device (kernel shared-memory limits).
 * Call it before capturing any graph; other entry points call it lazily. */
int h4b_prepare(void);

/* Number of SMs and the device's compute capability (for tests). */
int h4b_device_info(int *host_sm_count, int *host_cc_major, int *host_cc_minor);

/* ---- operator level ------------------------------------------------------ */

/* Replaces litespark_int4_i8_gemv (cpu_kernels/litespark_int4.cpp:78-84):
 *   output[r] = float(sum_k w[r,k] * x[k]) * activation_scale * scales[r]
 * evaluated left to right as the reference does (litespark_int4.cpp:73-74).
 * x: int8[width]; width a positive multiple of 32, weights 16-byte aligned.
 * acc (may be NULL) receives the int32 accumulators. */
int h4b_int4_i8_gemv(const int8_t *x, const uint8_t *weights, const float *scales,
                     float activation_scale, float *output, int32_t *acc,
                     int rows, int width, void *stream);

/* Replaces the pair kernel.quantize_activation + litespark_int4_i8_gemv that
 * cpu_lightspark.LiteSparkQwen._projection runs (cpu_lightspark.py:433-434,
 * :351-371), fused: the fp32 input is absmax-quantised to int8 inside the
 * kernel. act_scale_out (may be NULL) receives the dequant scale. */
int h4b_int4_gemv_fused_quant(const float *values, const uint8_t *weights, const float *scales,
                              float *output, int32_t *acc, float *act_scale_out,
                              int rows, int width, void *stream);

/* Launch flag: programmatic dependent launch. The kernel may start while
 * the previous kernel on the stream is still running; it streams its weights
 * into shared memory at once and waits for the previous kernel's writes
 * (griddepcontrol.wait) before it reads activations or writes anything. */
#define H4B_LAUNCH_PDL 1

/* h4b_int4_gemv_fused_quant with launch flags (H4B_LAUNCH_PDL). */
int h4b_int4_gemv_fused_quant_ex(const float *values, const uint8_t *weights, const float *scales,
                                 float *output, int32_t *acc, float *act_scale_out,
                                 int rows, int width, int flags, void *stream);

/* Replaces kernel.quantize_activation (third-party, called at
 * cpu_lightspark.py:433): q = clamp(rint(v * 127/m), -127, 127) with
 * m = max(absmax(v), 1e-5); *scale_out = m / 127. */
int h4b_quantize_activation(const float *values, int8_t *quantized, float *scale_out, int n,
                            void *stream);

/* Replaces kernel.rmsnorm_into (third-party, cpu_lightspark.py:431):
 * out = (x * (1 / sqrt(mean(x^2) + eps))) * weight. */
int h4b_rmsnorm(const float *x, const float *weight, float *out, int n, float eps, void *stream);

/* Replaces kernel.add_inplace (third-party, cpu_lightspark.py:445): x += y. */
int h4b_add_inplace(float *x, const float *y, int n, void *stream);

/* Replaces litespark_gqa_decode (cpu_kernels/litespark_int4.cpp:160-171):
 * single-token grouped-query attention, fp32, keys/values laid out
 * [time, kv_heads, head_dim], query/output heads [kv_head, group, head_dim].
 * scores: caller scratch of q_heads * score_stride floats (as in the
 * reference); the kernel keeps its split partials there. head_dim = 128. */
int h4b_gqa_decode(const float *query, const float *keys, const float *values, float *scores,
                   float *output, int context, int kv_heads, int groups, int head_dim,
                   int score_stride, void *stream);

/* No counterpart in the reference. The same attention as h4b_gqa_decode for
 * callers that cannot allocate device memory when they run it: for example
 * a serving process that reserved nearly all HBM for its own pool up front
 * (a fresh cudaMalloc would fail or fragment that reservation), or a plugin
 * whose host application owns the device allocator and forbids side
 * allocations. It takes no scratch argument and allocates nothing: the
 * split partials live in a 1 MiB array inside the library (256K floats,
 * held on every GPU that loads the library until the process exits). It
 * needs kv_heads * groups * (head_dim + 4) <= 262144 floats and returns
 * H4B_ETOOBIG beyond that. The first call on each device looks up the
 * array's device address (cudaGetSymbolAddress); make that first call
 * before any stream capture. All calls share the one array: calls that
 * overlap on the GPU (other streams, other host threads) race on it. No
 * state carries over between calls -- every slot a call reads, it wrote. */
int h4b_gqa_decode_noalloc(const float *query, const float *keys, const float *values, float *output,
                           int context, int kv_heads, int groups, int head_dim, void *stream);

/* Replaces LiteSparkQwen._embedding_into (cpu_lightspark.py:341-349):
 * out[k] = int4(embedding[token, k]) * scales[token]. The token id is read
 * from device memory; an out-of-range id sets status bit 2 and writes 0. */
int h4b_embedding(const int32_t *token, const uint8_t *embedding, const float *scales,
                  float *out, int vocab, int hidden, void *stream);

/* Greedy selection (cpu_lightspark.py:704-705): first index of the maximum
 * of logits[n], written to *token_out (device int32). */
int h4b_argmax(const float *logits, int n, int32_t *token_out, void *stream);

/* Stochastic sampling of one token (inference_runtime.sample_numpy,
 * inference_runtime.py:144-163; cpu_lightspark.sample_logits,
 * cpu_lightspark.py:700-726): repetition penalty on the `n_generated`
 * DISTINCT ids in `generated` (applied to `logits` in place), then greedy if
 * temperature <= 0.01, else top-k (top_k <= 64; <= 0 means 50) of
 * logits / temperature, softmax, top-p cut, and the token whose float64 CDF
 * interval holds `uniform` (a draw in [0, 1) from the caller's generator --
 * numpy's Generator.choice does the same search). Optional outputs: the k
 * candidate ids (descending) and their final probabilities. `scratch` holds
 * h4b_sample_scratch_bytes(vocab, top_k) bytes. */
int h4b_sample(float *logits, int vocab, const int32_t *generated, int n_generated, float temperature, int top_k,
               float top_p, float repetition_penalty, double uniform, int32_t *token_out, int32_t *topk_ids_out,
               float *topk_probs_out, void *scratch, void *stream);
long long h4b_sample_scratch_bytes(int vocab, int top_k);

/* ---- tensor parallelism (o and down split along K across ranks) ------------
 * Quantise `values` with the given device absmax (the max over the ranks),
 * then litespark_int4_i8_gemv over the local K slice: int32 row sums into
 * `acc` (to be summed across ranks), fp32 rows into `output` if not null. */
int h4b_int4_gemv_absmax(const float *values, const float *absmax, const uint8_t *weights, const float *scales,
                         float *output, int32_t *acc, int rows, int width, void *stream);
/* x[r] += float(acc[r]) * (max(*absmax, 1e-5) / 127) * w_scales[r] -- the
 * residual epilogue of the reduced sums. */
int h4b_residual_acc(float *x, const int32_t *acc, const float *absmax, const float *w_scales, int n, void *stream);

/* ---- batched (M > 1 tokens): batched decode and prefill ---------------------
 * Per-token quantisation of `rows` activations of `width` floats (the
 * quantize_activation contract applied to each row), also returning each
 * row's int8 sum. */
int h4b_quantize_rows(const float *values, int8_t *quantized, float *scales, int32_t *sums, int rows, int width,
                      void *stream);

/* out[m][n] = float(sum_k w[n][k] * x8[m][k]) * act_scales[m] * scales[n] for
 * m < tokens, n < rows: litespark_int4_i8_gemv (litespark_int4.cpp:78-84)
 * applied to `tokens` activations at once on the tensor cores; row m equals
 * the single-token GEMV of token m bit for bit. act_sums[m] = sum_k x8[m][k]
 * (from h4b_quantize_rows). rows % 128 == 0 and width % 64 == 0; with
 * width % 128 == 0 the tcgen05 kernel (TMA-fed, accumulators in tensor
 * memory) runs, otherwise the mma.sync kernel. */
int h4b_int4_gemm(const int8_t *x8, const float *act_scales, const int32_t *act_sums, const uint8_t *weights,
                  const float *scales, float *output, int tokens, int rows, int width, void *stream);

/* h4b_int4_gemm with an explicit kernel: 0 = as h4b_int4_gemm, 1 = tcgen05
 * only (H4B_EUNSUPPORTED when the shape does not allow it), 2 = mma.sync
 * only. Both give the same bits. */
int h4b_int4_gemm_ex(const int8_t *x8, const float *act_scales, const int32_t *act_sums, const uint8_t *weights,
                     const float *scales, float *output, int tokens, int rows, int width, int kernel, void *stream);

/* h4b_int4_gemm through a caller's int32 buffer acc [tokens][rows], zero on
 * entry and left zero: the kernel may split the K sum over several CTAs
 * (few tokens: one CTA per SM over the (128-row tile, 128-k step) units, or
 * K slices when the row tiles are few), adding the exact int32 partial sums
 * in acc, then applies the same epilogue -- the same bits as h4b_int4_gemm.
 * residual != 0: output[m][n] = output[m][n] + value (x + proj) instead of
 * value. The batched decode runs its projections this way. */
int h4b_int4_gemm_acc(const int8_t *x8, const float *act_scales, const int32_t *act_sums, const uint8_t *weights,
                      const float *scales, float *output, int32_t *acc, int tokens, int rows, int width, int residual,
                      void *stream);

/* ---- model level ----------------------------------------------------------- */

/* Device-resident Qwen3 model. Every weight kind is one buffer covering all
 * layers: w_qkv [L][q+2kv][H/2] (q, k, v rows concatenated as
 * cpu_lightspark.py:638-661 combines them); w_o [L][H][q/2]; w_gate_up
 * [L][2I][H/2] with gate and up rows interleaved in blocks of 4 (rows
 * 8b..8b+3 = gate 4b..4b+3, rows 8b+4..8b+7 = up 4b..4b+3); w_down
 * [L][H][I/2]; scales alongside. Norm vectors: norm_in/norm_post [L][H],
 * norm_q/norm_k [L][head_dim]. rope_cos/rope_sin: [max_pos][head_dim/2] fp32
 * tables (cpu_lightspark.py:329-336). */
typedef struct h4b_model {
    int layers, hidden, intermediate, heads, kv_heads, head_dim, vocab, max_pos;
    float eps;
    const uint8_t *w_qkv;     const float *s_qkv;
    const uint8_t *w_o;       const float *s_o;
    const uint8_t *w_gate_up; const float *s_gate_up;
    const uint8_t *w_down;    const float *s_down;
    const uint8_t *w_embed;   const float *s_embed;
    const float *norm_in, *norm_post, *norm_q, *norm_k, *norm_final;
    const float *rope_cos, *rope_sin;
} h4b_model;

/* One decode session (QwenDecodeState, cpu_lightspark.py:275-309), all
 * buffers caller-allocated on the device. k_cache/v_cache:
 * [L][kv_heads][capacity][head_dim] in kv_dtype (0 = fp32, 1 = fp16).
 * position/token/next_token: device int32 scalars; the step reads token and
 * position, writes next_token (greedy) and advances position by one.
 * Scratch: x[H], qkv[q+2kv], attended[q], act[I], logits[V]; absmax[2L]
 * floats and argmax_key[1] are rewritten every step; attn_partials holds
 * kv_heads * max(attn_splits, persistent splits) * groups * (head_dim + 4)
 * floats (the persistent step uses up to 148 / kv_heads splits); attn_counters
 * holds kv_heads ints and must be zero when the session is created. */
typedef struct h4b_state {
    int capacity, kv_dtype, attn_splits;
    void *k_cache, *v_cache;
    int32_t *position, *token, *next_token;
    float *x, *qkv, *attended, *act, *logits;
    float *absmax;
    unsigned long long *argmax_key;
    float *attn_partials;
    int *attn_counters;
    /* Persistent decode only: h4b_persistent_exchange_words(model) 64-bit
     * words, 16-byte aligned, zeroed when the session is created and never
     * cleared afterwards (they carry their own tags). */
    unsigned long long *exchange;
} h4b_state;

/* Checks the shapes/pointers of a model + state pair against what the
 * kernels implement. */
int h4b_validate(const h4b_model *model, const h4b_state *state);

/* One full decode token (LiteSparkQwen.forward_token,
 * cpu_lightspark.py:424-468) as a chain of kernel launches on `stream`:
 * embedding, 36 x (qkv GEMV, attention, o GEMV, gate/up GEMV, down GEMV),
 * LM head + argmax, position += 1. Capturable in a CUDA graph. */
int h4b_decode_step(const h4b_model *model, const h4b_state *state, void *stream);

/* Launches one stage of h4b_decode_step without programmatic launch, for
 * per-category timing (LiteSparkQwen.profile_forward_token,
 * cpu_lightspark.py:470-553). stage: 0 embedding, 1 qkv GEMV, 2 attention,
 * 3 o GEMV, 4 gate/up GEMV, 5 down GEMV (1-5 take `layer`), 6 LM head +
 * argmax, 7 finalize (next_token, position += 1). */
int h4b_decode_stage(const h4b_model *model, const h4b_state *state, int stage, int layer, void *stream);

/* The same token as ONE cooperative kernel, one CTA per SM, with no other
 * launch or memset. A producer warp per SM streams that SM's rows of every
 * weight matrix for the whole token through a shared-memory ring with bulk
 * copies, never waiting on activations. Consumer warps hand activations to
 * each other through state->exchange: every value is a 64-bit word
 * {tag, fp32} stored without a fence, and readers poll the words until the
 * tag of this launch and phase appears (bounded: a timeout sets status bit 1
 * and every CTA stops; after a failed step re-zero the exchange). Attention
 * splits merge the same way. Capturable in a CUDA graph. */
int h4b_decode_persistent(const h4b_model *model, const h4b_state *state, void *stream);

/* Size in 64-bit words of state->exchange for h4b_decode_persistent
 * (< 0: H4B_EINVAL for an inconsistent model). */
long long h4b_persistent_exchange_words(const h4b_model *model);

/* Captures h4b_decode_step into a CUDA graph bound to (model, state) and
 * instantiates it; *graph_out is an opaque handle. */
int h4b_graph_create(const h4b_model *model, const h4b_state *state, void *stream, void **graph_out);
/* Same, capturing h4b_decode_persistent. */
int h4b_graph_create_persistent(const h4b_model *model, const h4b_state *state, void *stream,
                                void **graph_out);
int h4b_graph_launch(void *graph, void *stream);
/* One greedy token with a host round trip, for a caller that feeds each
 * token from the host (forward_token + argmax, cpu_lightspark.py:424-468,
 * 704-705): copies the token id from token_host (pinned) to token_dev, launches
 * the graph, copies the graph's greedy token from next_dev to next_host
 * (pinned) and waits for the stream. */
int h4b_graph_token(void *graph, const int32_t *token_host, int32_t *token_dev, const int32_t *next_dev,
                    int32_t *next_host, void *stream);
int h4b_graph_destroy(void *graph);

/* ---- batched decode (B sequences, one token each per call) ----------------
 * All buffers caller-allocated on the device, 16-byte aligned.
 * k_cache/v_cache: [B][L][kv_heads][capacity][head_dim] in kv_dtype.
 * positions/tokens/next_tokens: int32[B]; the step reads tokens and
 * positions, writes next_tokens (greedy), copies them to tokens and advances
 * every position by one. Scratch: x[B][H], x8 int8[B][max(H, q, I)],
 * act_scale[B], act_sum[B], qkv[B][q + 2kv], attended[B][q], proj[B][H],
 * gate_up[B][2I], act[B][I], logits[B][V]; attn_partials holds
 * B * kv_heads * attn_splits * groups * (head_dim + 4) floats and
 * attn_counters B * kv_heads ints, zero when the session is created. */
typedef struct h4b_batch_state {
    int batch, capacity, kv_dtype, attn_splits;
    void *k_cache, *v_cache;
    int32_t *positions, *tokens, *next_tokens;
    float *x;
    int8_t *x8;
    float *act_scale;
    int32_t *act_sum;
    float *qkv, *attended, *proj, *gate_up, *act, *logits;
    float *attn_partials;
    int *attn_counters;
    int32_t *gemm_acc;  /* optional: [batch][gemm_acc_width] int32 zeros for split-K / stream-K GEMMs
                           (every projection with at most gemm_acc_width rows, at small batch); left zero
                           after every step */
    /* H4B_BATCH_ATTN_EXACT (0): the fp32 split kernel, each row bit-identical
     * to a decode step. H4B_BATCH_ATTN_TENSOR (1): tcgen05 attention with
     * split-fp16 operands (fp32 outputs within the 1e-3 relative tolerance)
     * over splits of whole 128-key tiles (one wave of CTAs for small batches,
     * about two per SM otherwise, at most
     * attn_splits), where the cache is fp16, head_dim 128 and 4 q heads share
     * a kv head; else as 0. */
    int attn_kernel;
    /* int32 row width of gemm_acc; 0 = max((heads + 2 kv_heads) * head_dim, hidden). 2 * intermediate
     * lets the gate/up projection use it as well. */
    int gemm_acc_width;
} h4b_batch_state;

#define H4B_BATCH_ATTN_EXACT 0
#define H4B_BATCH_ATTN_TENSOR 1

int h4b_validate_batch(const h4b_model *model, const h4b_batch_state *state);

/* One decode token for each of the B sequences (forward_token per sequence):
 * tensor-core GEMMs over the batch for every projection and the LM head,
 * batched split-K attention, per-row RMSNorm / quantisation / SwiGLU with the
 * single-token arithmetic, so row b equals the one-token step of sequence b.
 * Capturable in a CUDA graph. */
int h4b_decode_batch(const h4b_model *model, const h4b_batch_state *state, void *stream);

/* Layer `layer`'s attention step of h4b_decode_batch alone (reads state->qkv,
 * appends each sequence's k/v at its position, writes state->attended), for
 * per-kernel timing. */
int h4b_batch_attention(const h4b_model *model, const h4b_batch_state *state, int layer, void *stream);

/* ---- tensor-parallel exchanges over NVLink peer memory ------------------------
 * One receive buffer per rank, mapped by every rank (CUDA IPC); values travel
 * as {tag, payload} words stored into the peers' buffers and polled in one's
 * own (bounded polls: a timeout sets status bit 1). generation is a device
 * counter, zero at creation, advanced by every exchange; all ranks must run
 * the same exchanges in the same order. */
#define H4B_TP_MAX_RANKS 8
typedef struct h4b_tp_group {
    int world, rank, capacity;                        /* capacity: words per source slot */
    unsigned long long *buffers[H4B_TP_MAX_RANKS];    /* rank r's receive buffer, as mapped here */
    unsigned int *generation;
} h4b_tp_group;

/* Bytes of one receive buffer (two parities x world slots x capacity words). */
long long h4b_tp_buffer_bytes(int world, int capacity);
/* Zeroed device allocation shareable with other processes; handle receives
 * the 64-byte cudaIpcMemHandle_t. */
int h4b_ipc_alloc(long long bytes, void **ptr, void *handle);
int h4b_ipc_open(const void *handle, void **ptr);
int h4b_ipc_close(void *ptr);
int h4b_ipc_free(void *ptr);
/* value[0] <- max over ranks (the o / down quantisation absmax;
 * replaces an all-reduce MAX). */
int h4b_tp_allreduce_max(const h4b_tp_group *group, float *value, void *stream);
/* x[i] += float(sum over ranks acc[i]) * dequant(absmax) * w_scales[i], i < n:
 * the exact int32 all-reduce of a K-split projection fused with its residual
 * epilogue (replaces all-reduce SUM + h4b_residual_acc). */
int h4b_tp_allreduce_sum_residual(const h4b_tp_group *group, const int32_t *acc, float *x, const float *absmax,
                                  const float *w_scales, int n, void *stream);
/* pairs[2r] = rank r's logits[local_index], pairs[2r+1] = its local_index +
 * vocab_offset (as doubles): the greedy candidates of every rank. */
int h4b_tp_gather_best(const h4b_tp_group *group, const float *logits, const int32_t *local_index,
                       int vocab_offset, double *pairs, void *stream);

/* ---- prefill ----------------------------------------------------------------
 * Scratch for h4b_prefill, owned by the caller: buffers for up to max_tokens
 * prompt rows (16-byte aligned). attn_splits is the number of context splits
 * of every prompt query's attention (1..64; 1 = each query walks its whole
 * context in one CTA, no merge). With attn_splits > 1, attn_partials holds
 * attn_queries * kv_heads * attn_splits * groups * (head_dim + 4) floats and
 * attn_counters attn_queries * kv_heads ints (zero at creation; the kernels
 * leave them zero). */
typedef struct h4b_prefill_scratch {
    int max_tokens, attn_queries, attn_splits;
    float *x;           /* [max_tokens][hidden] */
    int8_t *x8;         /* [max_tokens][max(hidden, heads*head_dim, intermediate)] */
    float *act_scale;   /* [max_tokens] */
    int32_t *act_sum;   /* [max_tokens] */
    float *qkv;         /* [max_tokens][(heads + 2 kv_heads) * head_dim] */
    float *attended;    /* [max_tokens][heads * head_dim] */
    float *gate_up;     /* [max_tokens][2 intermediate] */
    float *act;         /* [max_tokens][intermediate] */
    float *proj;        /* [max_tokens][hidden] */
    int32_t *tokens;    /* [max_tokens] prompt token ids, filled by the caller */
    int32_t *positions; /* [max_tokens] */
    float *attn_partials;
    int *attn_counters;
    /* H4B_PREFILL_ATTN_EXACT (0): fp32 attention in the decode kernel's
     * order, every row bit-identical to a decode step. H4B_PREFILL_ATTN_TENSOR
     * (1): tcgen05 tensor-core attention with split fp16 operands (fp32
     * outputs within the 1e-3 relative tolerance, not bit-identical) where
     * the cache is fp16, head_dim 128 and 4 q heads share a kv head, else as
     * 0. Used when attn_splits == 1. */
    int attn_kernel;
} h4b_prefill_scratch;

#define H4B_PREFILL_ATTN_EXACT 0
#define H4B_PREFILL_ATTN_TENSOR 1

/* Feeds scratch->tokens[0, count) to the session at positions *position ..
 * *position + count - 1 (LiteSparkQwen.forward_token called count times,
 * cpu_lightspark.py:424-468, as the reference's prefill loop does,
 * cpu_lightspark.py:809-810), with the body projections as tensor-core GEMMs
 * over all prompt rows. Afterwards state->logits holds the last row's
 * logits, next_token/token its greedy token and *position has advanced by
 * count -- bit for bit what count h4b_decode_step calls leave when the
 * session's attention splits equal scratch->attn_splits and
 * scratch->attn_kernel is H4B_PREFILL_ATTN_EXACT (with the tensor-core
 * attention, within its tolerance). */
int h4b_prefill(const h4b_model *model, const h4b_state *state, const h4b_prefill_scratch *scratch, int count,
                void *stream);

/* The prompt attention of one layer alone, for timing: the `count` q rows
 * left in scratch->qkv by an h4b_prefill of `count` tokens (normalised and
 * rotated; the last layer's) against the session's cache for `layer`, with
 * scratch->positions and scratch->attn_kernel, into scratch->attended. */
int h4b_prefill_attention(const h4b_model *model, const h4b_state *state, const h4b_prefill_scratch *scratch,
                          int count, int layer, void *stream);

/* One stage of a tensor-parallel prefill on this rank's slice of the model
 * (its q/k/v heads, its MLP units, K-slices of o_proj and down_proj, its
 * vocabulary rows; x replicated): the reference's prefill loop
 * (cpu_lightspark.py:809-810) over `count` prompt rows, as h4b_prefill, with
 * the o and down projections split along K. Stages, per layer in order:
 *   0 (once, layer ignored): positions, embedding of scratch->tokens from the
 *     full table `table` / `table_scales` (table_vocab rows);
 *   1: attention block (RMSNorm, quantisation, qkv GEMM, q/k norm, RoPE,
 *      K/V append, attention); absmax[i] = max |attended row i| here;
 *   2: attended rows quantised with the scale of absmax[i] (the maximum over
 *      all ranks after a MAX reduction), o GEMM: acc[i][r] = exact int32 sum
 *      over this rank's K slice;
 *   3: x += float(acc) * act_scale * w_scale (acc summed over the ranks),
 *      then the MLP block (RMSNorm, quantisation, gate/up GEMM, SwiGLU);
 *      absmax[i] = max |act row i| here;
 *   4: act quantised with absmax (the global maximum), down GEMM into acc;
 *   5: x += float(acc) * act_scale * w_scale (acc summed over the ranks);
 *   6 (once): last row through the final RMSNorm and this rank's LM-head rows;
 *      state->logits, argmax key, next_token (a local index) and position.
 * The caller reduces absmax with MAX after stages 1 and 3 and acc with an
 * int32 SUM after stages 2 and 4. absmax: float[count], acc: int32[count][hidden]. */
int h4b_prefill_tp_stage(const h4b_model *model, const h4b_state *state, const h4b_prefill_scratch *scratch,
                         int count, int layer, int stage, const uint8_t *table, const float *table_scales,
                         int table_vocab, float *absmax, int32_t *acc, void *stream);

/* ---- format producer: LATTICE checkpoint -> packed int4 cache ------------- */

/* One LATTICE projection as stored in the checkpoint (all pointers are
 * device pointers; the reference reads the same fields in
 * cpu_lightspark._convert_projection, cpu_lightspark.py:149-201):
 * maskid / t0: uint8[rows][ceil(width/4)], four 2-bit codes per byte (code j
 * of a row in bits 2(j%4)..2(j%4)+1 of byte j/4); t1c: the compact T1 codes
 * of every column whose mode id is 0 or 1, row-major over the whole matrix,
 * n_t1 codes in t1c_bytes bytes (MLX/lattice_model.py:160-185 expands them);
 * mu, a0: [4][rows][nblocks], a1: [n_o2][rows][nblocks], float32
 * (param_dtype 0) or float16 (param_dtype 1); o2_idx: the mode id each a1
 * plane applies to; left: float32[dim_l][dim_l], right: float32[dim_r][dim_r]
 * with dim_l * dim_r == width. */
typedef struct h4b_lattice_projection {
    int rows, width, blocksize, nblocks;
    const uint8_t *maskid, *t0, *t1c;
    long long n_t1, t1c_bytes;
    const void *mu, *a0, *a1;
    int param_dtype, n_o2;
    int o2_idx[4];
    const float *left, *right;
    int dim_l, dim_r;
} h4b_lattice_projection;

/* Bytes of caller scratch h4b_lattice_to_int4 needs for `rows` rows. */
long long h4b_lattice_scratch_bytes(int rows);

/* Replaces cpu_lightspark._convert_projection (cpu_lightspark.py:149-201)
 * with expand_t1 (MLX/lattice_model.py:160-185): reconstructs the fp32
 * weights, absorbs the rotation (W_r -> left^T W_r right^T per row, fp64
 * accumulation rounded once to fp32), and writes the row-int4 cache form:
 * packed uint8[rows][width/2] and float32 scales[rows] with
 * scale = max(max|w|, 1e-8) / 7 and codes clip(rint(w / scale), -7, 7).
 * Checks, as expand_t1 does, that the mode ids select exactly n_t1 codes
 * (*host_error = 1 and H4B_EINVAL otherwise). Synchronises `stream`. */
int h4b_lattice_to_int4(const h4b_lattice_projection *projection, uint8_t *packed, float *scales,
                        void *scratch, int *host_error, void *stream);

/* Replaces cpu_lightspark._convert_embedding (cpu_lightspark.py:204-229):
 * per-row symmetric int4 of a dense matrix source[rows][width] (float32 when
 * source_dtype is 0, float16 when 1), same scale and code rule as above;
 * bit-exact with the reference. */
int h4b_rows_to_int4(const void *source, int source_dtype, int rows, int width, uint8_t *packed,
                     float *scales, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* HARSH4B_B200_H */
