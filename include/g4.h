/*
 * g4.h -- C ABI of libg4b200: B200 (sm_100a) kernels for gemma4.kt's two hot
 * paths, the quantized matrix-vector product and the mixture-of-experts layer.
 *
 * The Kotlin host binds these with java.lang.foreign (FFM) downcalls.  Every
 * reference interface below is cited by its file:line under
 * lib/src/main/kotlin/io/github/lbenedetto/internal/.
 *
 * Conventions
 *  - Every entry point returns 0 on success and a negative G4_E* code on
 *    failure; g4_last_error() then describes the failure.  No C++ exception and
 *    no abort ever crosses this boundary (the reference throws
 *    UnsupportedOperationException / IllegalArgumentException instead:
 *    FloatTensorFactory.kt:21, Q8_0FloatTensor.kt:130).
 *  - A g4_ctx is bound to one CUDA device and is not thread-safe; use one per
 *    host thread / LlamaState, as the reference uses one LlamaState per thread.
 *  - Pointers named *_dev are device pointers; *_host are host pointers.
 *    `stream` is a cudaStream_t (NULL = legacy default stream).  Device-pointer
 *    calls are asynchronous on that stream; *_host calls are synchronous.
 *  - Weights are uploaded once in their on-disk GGUF block layout (no
 *    dequantization on load) and live until g4_tensor_free.
 */
#ifndef G4_H
#define G4_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define G4_OK 0
#define G4_E_ARG -1        /* bad argument (IllegalArgumentException) */
#define G4_E_TYPE -2       /* unsupported GGML type (UnsupportedOperationException) */
#define G4_E_CUDA -3       /* CUDA runtime error */
#define G4_E_NOMEM -4      /* device allocation failed */
#define G4_E_DEVICE -5     /* a kernel reported an error status (e.g. bounded wait expired) */
#define G4_E_DIST -6       /* NCCL / multi-GPU error */

/* GGML type ids accepted by g4_tensor_upload (GGMLType.kt:16-46) */
#define G4_TYPE_F32 0
#define G4_TYPE_F16 1
#define G4_TYPE_Q4_0 2
#define G4_TYPE_Q4_1 3
#define G4_TYPE_Q5_1 7
#define G4_TYPE_Q8_0 8
#define G4_TYPE_Q4_K 12
#define G4_TYPE_Q5_K 13
#define G4_TYPE_Q6_K 14
#define G4_TYPE_BF16 30
#define G4_TYPE_MXFP4 39

typedef struct g4_ctx g4_ctx;
typedef struct g4_tensor g4_tensor;

/* Create a context on CUDA device `device`.  (No reference counterpart: the
 * reference's "device" is the JVM heap plus an mmap, GGUF.kt:195-212.) */
int g4_init(int device, g4_ctx **out);
int g4_destroy(g4_ctx *ctx);

/* Description of the last failure on this context ("" if none).  A NULL ctx
 * returns the last failure of g4_init on this thread. */
const char *g4_last_error(const g4_ctx *ctx);

/* Upload a tensor's raw block stream (`nbytes` bytes holding `n_elems`
 * elements of GGML type `ggml_type`) to HBM unchanged.
 * Replaces FloatTensorFactory.create (FloatTensorFactory.kt:7-23) reached from
 * ModelLoader.loadQuantized (ModelLoader.kt:268-271); `host_blocks` is the
 * address of the tensor's mmap slice (GGUF.kt:195-212, GGMLTensorEntry.kt:5-11).
 * nbytes must equal GGMLType.byteSizeFor(n_elems) (GGMLType.kt:58-62). */
int g4_tensor_upload(g4_ctx *ctx, int ggml_type, const void *host_blocks, uint64_t nbytes,
                     uint64_t n_elems, g4_tensor **out);

/* Upload rows [row_begin, row_begin+row_count) of a row-major [rows, cols]
 * tensor (one output-row shard).  `host_blocks` points at the FULL tensor;
 * the shard's rows must start and end on block boundaries. */
int g4_tensor_upload_rows(g4_ctx *ctx, int ggml_type, const void *host_blocks, uint64_t cols,
                          uint64_t row_begin, uint64_t row_count, g4_tensor **out);
int g4_tensor_free(g4_tensor *t);
/* Device address of the tensor's block stream (for callers composing kernels). */
const void *g4_tensor_device_ptr(const g4_tensor *t);
uint64_t g4_tensor_nbytes(const g4_tensor *t);
uint64_t g4_tensor_n_elems(const g4_tensor *t);
int g4_tensor_type(const g4_tensor *t);

/* out_dev[i] = dot(W[this_offset + i*dim1 ...], x_dev[0..dim1)), i < dim0.
 * Replaces FloatTensor.matmul(that, out, dim0, dim1, thisOffset)
 * (FloatTensor.kt:25-29) and matmul(that, out, dim0, dim1) (FloatTensor.kt:18-22,
 * this_offset = 0), i.e. every XFloatTensor.vectorDot it fans out to
 * (Q8_0FloatTensor.kt:39-142, Q4_KFloatTensor.kt:86-207,
 * Q6_KFloatTensor.kt:111-250, BF16FloatTensor.kt:35-74, F32FloatTensor.kt:37-66).
 * x_dev must hold dim1 floats, out_dev dim0 floats. */
int g4_matmul(g4_ctx *ctx, const g4_tensor *w, int64_t this_offset, const float *x_dev, float *out_dev,
              int dim0, int dim1, void *stream);

/* Same with host arrays (the Kotlin heap FloatArrays ArrayFloatTensor.values,
 * ArrayFloatTensor.kt:12-28): copies x in, runs, copies out, synchronizes. */
int g4_matmul_host(g4_ctx *ctx, const g4_tensor *w, int64_t this_offset, const float *x_host,
                   float *out_host, int dim0, int dim1);

/* out_dev[i] = W.get(offset + i), i < n: the reference's element decoder
 * (Q8_0FloatTensor.kt:21-28, Q4_KFloatTensor.kt:23-55, Q6_KFloatTensor.kt:26-73,
 * BF16FloatTensor.kt:20-24, F32FloatTensor.kt:18-20), bit-exact. */
int g4_dequant(g4_ctx *ctx, const g4_tensor *w, int64_t offset, int64_t n, float *out_dev, void *stream);

/* Wait for all work issued through this context on `stream` and report any
 * error status a kernel recorded (bounded waits that expired). */
int g4_sync(g4_ctx *ctx, void *stream);

/* ---------------- mixture-of-experts layer (Llama.kt:247-346) ----------------
 * Weights of one MoE layer, all uploaded with g4_tensor_upload:
 *   gate_inp        F32  [dim, n_expert]     blk.N.ffn_gate_inp.weight
 *   gate_inp_scale  F32  [dim]               blk.N.ffn_gate_inp.scale
 *   gate_up_exps    Q4_K/Q8_0/Q6_K/BF16/F32 [dim, 2*ff, n_expert] blk.N.ffn_gate_up_exps.weight
 *   down_exps       same types [ff, dim, n_expert]              blk.N.ffn_down_exps.weight
 *   down_exps_scale F32  [n_expert]          blk.N.ffn_down_exps.scale
 *   pre_ffw_norm_2  F32  [dim]               blk.N.pre_ffw_norm_2.weight
 *   post_ffw_norm_2 F32  [dim] or NULL       blk.N.post_ffw_norm_2.weight
 * (tensor names: ModelLoader.kt:223-232; shapes: LlamaWeights.kt:50-65). */
typedef struct {
  int dim;        /* gemma4.embedding_length (2816) */
  int n_expert;   /* gemma4.expert_count (128) */
  int n_used;     /* gemma4.expert_used_count (8) */
  int expert_ff;  /* gemma4.expert_feed_forward_length (704) */
  float eps;      /* gemma4.attention.layer_norm_rms_epsilon */
  const g4_tensor *gate_inp;
  const g4_tensor *gate_inp_scale;
  const g4_tensor *gate_up_exps;
  const g4_tensor *down_exps;
  const g4_tensor *down_exps_scale;
  const g4_tensor *pre_ffw_norm_2;
  const g4_tensor *post_ffw_norm_2;
} g4_moe_weights;

/* Expert half of the MoE block for n_tokens independent tokens
 * (Llama.kt:247-346): moeInput = rmsnorm(x, pre_ffw_norm_2); router
 * rms(x)/sqrt(dim)*gate_inp_scale -> gate_inp matmul -> softmax -> top-n_used
 * (ties to the lowest index, probabilities not renormalised); per selected
 * expert gate_up matmul -> gelu(gate)*up -> down matmul -> accumulate with
 * weight prob*down_exps_scale[e] in selection order; then
 * rmsnorm(post_ffw_norm_2) when given.
 * x_dev: [n_tokens, dim] residual stream (state.x); out_dev: [n_tokens, dim].
 * topk_idx_dev / topk_prob_dev: [n_tokens, n_used] or NULL. */
int g4_moe_layer(g4_ctx *ctx, const g4_moe_weights *w, const float *x_dev, float *out_dev, int n_tokens,
                 int32_t *topk_idx_dev, float *topk_prob_dev, void *stream);

/* Host-buffer variant (synchronous), for the Kotlin heap arrays. */
int g4_moe_layer_host(g4_ctx *ctx, const g4_moe_weights *w, const float *x_host, float *out_host,
                      int n_tokens, int32_t *topk_idx_host, float *topk_prob_host);

/* Allocation-free variant of g4_moe_layer (no counterpart in the reference).
 * For hosts that cannot let the library allocate device memory while they run:
 * e.g. a host that hands all free HBM to its own pool at start-up, or a decode
 * loop that must not stall on the device-wide synchronisation a cudaMalloc or
 * cudaFree can cause.  Same kernels and results as g4_moe_layer; the work
 * buffers live in one fixed array of G4_MOE_NOALLOC_SCRATCH_BYTES bytes that
 * the library image reserves on every GPU it is used on, held until exit.
 *  - A call needs 4*n_tokens*(2*dim + dim/16 + n_expert + 3*n_used
 *    + n_used*(ff + ff/16 + dim)) + 4*(n_expert + 1) bytes (each buffer rounded
 *    up to 256 bytes; about 138 KB per token for dim 2816, 128 experts, top-8,
 *    ff 704, so up to 60 tokens).  Larger
 *    batches are rejected with G4_E_ARG and a message; split them.
 *  - g4_init creates the array on its device and resolves its address (under
 *    CUDA's lazy module loading it would otherwise only appear at first use):
 *    create the context before the host reserves the free HBM for its own
 *    pool.  If that failed, the first call on the device retries it; make
 *    that call before any stream capture.
 *  - All calls on a device share the array: calls that can overlap on the GPU
 *    (different streams, or several contexts on one device) race.  Nothing in
 *    it needs to start at zero: each call writes every buffer before reading.
 *  - Never calls cudaMalloc, cudaFree or any allocating library routine. */
#define G4_MOE_NOALLOC_SCRATCH_BYTES (8u << 20)
int g4_moe_layer_noalloc(g4_ctx *ctx, const g4_moe_weights *w, const float *x_dev, float *out_dev,
                         int n_tokens, int32_t *topk_idx_dev, float *topk_prob_dev, void *stream);

/* Expert-parallel variant of g4_moe_layer for one process per GPU (no
 * counterpart in the reference, which runs in one process).  After
 * g4_dist_init, rank r of world W holds experts [r*E/W, (r+1)*E/W): its
 * gate_up_exps / down_exps tensors contain only those experts, in the same
 * per-expert layout; gate_inp, gate_inp_scale, down_exps_scale (all E) and
 * the norms are replicated.  Every rank calls this with its own n_tokens
 * tokens (0 allowed) at the same time: each routed slot's row travels to the
 * rank owning its expert (NCCL send/recv), the products come back and are
 * combined on the owning rank exactly as g4_moe_layer combines them.
 * topk_* report global expert ids.  Synchronises the stream once (the row
 * counts are exchanged through the host).  Q4_K experts only. */
int g4_moe_layer_ep(g4_ctx *ctx, const g4_moe_weights *w_local, const float *x_dev, float *out_dev,
                    int n_tokens, int32_t *topk_idx_dev, float *topk_prob_dev, void *stream);

/* ---------------- MoE FFN block (Llama.kt:226-353) ----------------
 * The whole FFN half of a MoE layer, in place on n_tokens rows of the
 * residual stream x (state.x after the attention residual):
 *   shared MLP   h = rmsnorm(x, ffn_norm); xb = ffn_down . (gelu(ffn_gate . h) * (ffn_up . h));
 *                xb = rmsnorm(xb, post_ffw_norm_1)                        Llama.kt:231-243
 *   experts      moeOutput = g4_moe_layer(x) (pre_ffw_norm_2 ... post_ffw_norm_2)  Llama.kt:247-346
 *   merge        xb += moeOutput; x += rmsnorm(xb, post_ffw_norm)          Llama.kt:349-353
 *   layer scale  x *= layer_output_scale when it is not 1                  Llama.kt:393-397
 * Pass layer_output_scale = 1 when the model has a per-layer-embedding step
 * (Llama.kt:366-391) between the merge and the scale.  The shared MLP
 * tensors take any format g4_matmul takes; the norms are F32 [dim]. */
typedef struct {
  const g4_moe_weights *moe;       /* the expert half; its dim and eps serve the whole block */
  int ff;                          /* gemma4.feed_forward_length of the layer */
  const g4_tensor *ffn_gate;       /* blk.N.ffn_gate.weight [dim, ff] */
  const g4_tensor *ffn_up;         /* blk.N.ffn_up.weight   [dim, ff] */
  const g4_tensor *ffn_down;       /* blk.N.ffn_down.weight [ff, dim] */
  const g4_tensor *ffn_norm;       /* blk.N.ffn_norm.weight */
  const g4_tensor *post_ffw_norm_1; /* blk.N.post_ffw_norm_1.weight */
  const g4_tensor *post_ffw_norm;  /* blk.N.post_ffw_norm.weight */
  float layer_output_scale;        /* blk.N.layer_output_scale.weight[0], or 1 */
} g4_ffn_moe_weights;

/* x_dev: [n_tokens, dim], updated in place, on `stream`. */
int g4_ffn_moe_block(g4_ctx *ctx, const g4_ffn_moe_weights *w, float *x_dev, int n_tokens, void *stream);
/* Host-buffer variant (synchronous): x_host updated in place. */
int g4_ffn_moe_block_host(g4_ctx *ctx, const g4_ffn_moe_weights *w, float *x_host, int n_tokens);

/* ---------------- whole-model decode (Llama.kt:105-477) ----------------
 * A GPU-resident Llama.forward: the residual stream, the KV cache and the
 * greedy sampler stay in HBM; one decode step is one CUDA graph.
 *
 * Model configuration, as LlamaConfiguration (LlamaConfiguration.kt:3-55) is
 * derived by ModelLoader.loadModel (ModelLoader.kt:39-139).  The arrays are
 * copied by g4_model_create.  Per-layer embeddings (embedding_length_per_layer
 * > 0, Llama.kt:115-143,366-391) are not supported. */
typedef struct {
  int dim;                   /* gemma4.embedding_length */
  int n_layers;              /* gemma4.block_count */
  int n_heads;               /* gemma4.attention.head_count */
  int vocab;                 /* size of tokenizer.ggml.tokens */
  int ctx_len;               /* context length (KV cache positions) */
  int head_size_full;        /* gemma4.attention.key_length */
  int head_size_swa;         /* gemma4.attention.key_length_swa */
  int sliding_window;        /* gemma4.attention.sliding_window */
  int n_layer_kv_from_start; /* block_count - gemma4.attention.shared_kv_layers */
  float eps;                 /* gemma4.attention.layer_norm_rms_epsilon */
  float rope_theta;          /* gemma4.rope.freq_base */
  float rope_theta_swa;      /* gemma4.rope.freq_base_swa */
  float logit_softcap;       /* gemma4.final_logit_softcapping (0: none) */
  int n_expert;              /* gemma4.expert_count (0: dense model) */
  int n_expert_used;         /* gemma4.expert_used_count */
  int expert_ff;             /* gemma4.expert_feed_forward_length */
  const int *n_kv_heads;     /* [n_layers] KV heads (attn_k rows / head size) */
  const int *ff;             /* [n_layers] gemma4.feed_forward_length */
  const unsigned char *is_swa; /* [n_layers] gemma4.attention.sliding_window_pattern */
} g4_model_config;

typedef struct g4_model g4_model;
typedef struct g4_state g4_state;

/* Replaces ModelLoader.loadWeights (ModelLoader.kt:154-261) for the decoder:
 * create, hand over every tensor by its GGUF name (raw blocks, no dequant:
 * token_embd, output (optional: tied), output_norm, rope_freqs and the blk.N.*
 * tensors of ModelLoader.kt:179-248), then finalize.  Finalize fuses q|k|v
 * and gate/up of each layer into one tensor each (same GGML type required,
 * rows of whole blocks) and builds the RoPE tables (RotaryPositionEmbeddings.kt).
 * set_tensor copies the data; the host buffer may be released afterwards.
 * Unknown tensors (per-layer embeddings) are rejected with G4_E_TYPE. */
int g4_model_create(g4_ctx *ctx, const g4_model_config *cfg, g4_model **out);
int g4_model_set_tensor(g4_model *model, const char *gguf_name, int ggml_type, const void *host_blocks,
                        uint64_t nbytes, uint64_t n_elems);
int g4_model_finalize(g4_model *model);
int g4_model_free(g4_model *model);

/* LlamaState (LlamaState.kt:38-77) on the device: activations, fp32 KV cache
 * [ctx_len][kv_dim] per KV layer, step control.  One per sequence; not
 * thread-safe.  Its work runs on a stream of its own. */
int g4_state_create(g4_model *model, g4_state **out);
int g4_state_free(g4_state *state);

/* Llama.forward(model, state, token, position) (Llama.kt:105-408): one step.
 * logits_host (vocab floats, after softcapping) and next_token_host (the
 * argmax, FloatTensor.argmax: first maximum) may be NULL.  Synchronous. */
int g4_decode_step(g4_state *state, int token, int position, float *logits_host, int *next_token_host);

/* Llama.generateTokens with the ARGMAX sampler (Llama.kt:413-458), stop tokens
 * not checked: tokens[i] is fed at position start_position + i (tokens[0] is
 * normally <bos>), then n_generate greedy tokens, each fed back on the device
 * (n_tokens + n_generate - 1 steps, no host round trip between them).
 * out_tokens[n_generate] receives the generated ids.  Synchronous. */
int g4_decode_greedy(g4_state *state, const int *tokens, int n_tokens, int start_position, int n_generate,
                     int *out_tokens);

/* Building blocks of g4_decode_greedy for callers that time or pipeline the
 * steps: stage the inputs of steps [0, n_steps) (token, or -1 for the previous
 * step's argmax; position) and reset the step counter; enqueue n_steps steps
 * on the state's stream (asynchronous); read the argmax of steps
 * [first_step, first_step + n) (synchronous). */
int g4_decode_stage(g4_state *state, const int *tokens, const int *positions, int n_steps);
int g4_decode_enqueue(g4_state *state, int n_steps);
int g4_decode_read_tokens(g4_state *state, int first_step, int n, int *out);
/* The state's cudaStream_t. */
void *g4_state_stream(g4_state *state);

/* Batched decode: many sequences, one position each per step.  The reference
 * runs one LlamaState per sequence and Llama.forward per token (Llama.kt:105-408,
 * GemmaModel.kt:73); a g4_batch holds n_max <= 64 sequences (KV cache of
 * max_positions positions each, slot i = sequence i) and advances n of them
 * per g4_batch_step, every weight read shared by the n tokens.  Needs every
 * projection and the output matrix in Q8_0 (G4_E_TYPE otherwise); the model
 * keeps a repacked copy of them.  Not thread-safe; its own stream. */
typedef struct g4_batch g4_batch;
int g4_batch_create(g4_model *model, int n_max, int max_positions, g4_batch **out);
int g4_batch_free(g4_batch *batch);
/* Llama.forward for n rows at once: row i feeds tokens[i] at positions[i] of
 * the sequence in KV slot slots[i] (slots NULL: slot i).  Several rows may
 * belong to one slot at distinct positions (a prompt chunk, prefilled in one
 * step: every row's K/V row is written before any row attends); every
 * earlier position of a slot must have been fed before, as generateTokens
 * does.  logits_host [n][vocab] (after softcapping) and next_tokens_host [n]
 * (argmax, first maximum) may be NULL.  Synchronous. */
int g4_batch_step(g4_batch *batch, const int *tokens, const int *positions, const int *slots, int n,
                  float *logits_host, int *next_tokens_host);
/* The batch's cudaStream_t. */
void *g4_batch_stream(g4_batch *batch);
/* Expert parallelism for a batch (no counterpart in the reference, which runs
 * in one process): after g4_dist_init on W >= 2 ranks, rank r computes experts
 * [r*E/W, (r+1)*E/W) of every MoE layer for all ranks' tokens (the layer runs
 * as g4_moe_layer_ep); attention and the dense layers stay with the rank's
 * own sequences.  Every rank then calls g4_batch_step together, each with its
 * own sequences.  Q4_K experts; E divisible by W. */
int g4_batch_expert_parallel(g4_batch *batch);

/* Router top-k alone on given logits (Llama.kt:273-293 + softmaxInPlace,
 * MutableFloatTensor.kt:54-59): probs_dev/idx_dev [n_tokens, k]. */
int g4_moe_topk(g4_ctx *ctx, const float *logits_dev, int n_tokens, int n_expert, int k,
                int32_t *idx_dev, float *prob_dev, void *stream);

/* ---------------- multi-GPU (one process per GPU, NCCL over NVLink) ----------------
 * No reference counterpart: the reference is single-process (no distributed code). */
#define G4_NCCL_ID_BYTES 128
int g4_dist_unique_id(void *id_out /* G4_NCCL_ID_BYTES */);
/* Join the communicator of `world` ranks.  The communicator is created
 * non-blocking and every wait on peers is bounded: if the other ranks do not
 * all join within timeout_ms, or a later collective of this context does not
 * complete within it, the communicator is aborted and the call returns
 * G4_E_DIST (the context is then single-rank again).  g4_dist_init uses the
 * G4_DIST_TIMEOUT_MS environment variable, else 120 s. */
int g4_dist_init_timeout(g4_ctx *ctx, int rank, int world, const void *id, int timeout_ms);
int g4_dist_init(g4_ctx *ctx, int rank, int world, const void *id /* G4_NCCL_ID_BYTES */);
/* Abort the context's communicator (for a host watchdog that gave up on a
 * peer); the context stays usable for single-GPU calls. */
int g4_dist_abort(g4_ctx *ctx);
int g4_dist_rank(const g4_ctx *ctx);
int g4_dist_world(const g4_ctx *ctx);

/* Row-sharded matmul: this rank holds rows [rank*rows/world, (rank+1)*rows/world)
 * of a [rows, cols] weight (uploaded with g4_tensor_upload_rows); computes
 * them and all-gathers into out_dev[rows] on every rank. rows % world == 0. */
int g4_matmul_sharded(g4_ctx *ctx, const g4_tensor *w_shard, const float *x_dev, float *out_dev, int rows,
                      int cols, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* G4_H */
