/*
 * g4_oracle.h -- CPU restatement of gemma4.kt's quantized matrix-vector
 * kernels and its mixture-of-experts block.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg /
 * `--impl reference` arm may load it.  The product library never links it.
 *
 * Every function cites the reference source it restates (paths relative to
 * lib/src/main/kotlin/io/github/lbenedetto/internal/).  The file is compiled
 * with -ffp-contract=off because Java float arithmetic is never contracted:
 * a*b+c rounds twice unless the Kotlin source calls .fma() explicitly.
 *
 * Parity pin: the block decoders (o_get) are checked bit-for-bit against
 * gguf-py 0.19.0's numpy dequantizers (tests/golden/make_golden.py), which
 * evaluate the same expressions in the same order.  The 16-lane dot-product
 * structure follows the 512-bit branch of each vectorDot; the JVM's
 * reduceLanes(ADD) order is unspecified, so the oracle fixes a pairwise tree
 * (lanes i and i+8, then +4, +2, +1) and GEMV results are compared within a
 * relative-L2 tolerance, never bitwise.
 */
#ifndef G4_ORACLE_H
#define G4_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type ids, GGMLType.kt:16-46 */
enum {
  O_F32 = 0,
  O_F16 = 1,
  O_Q4_0 = 2,
  O_Q4_1 = 3,
  O_Q5_1 = 7,
  O_Q8_0 = 8,
  O_Q4_K = 12,
  O_Q5_K = 13,
  O_Q6_K = 14,
  O_BF16 = 30,
  O_MXFP4 = 39
};

int o_block_size(int type);  /* elements per block, GGMLType.kt:12-56 */
int o_type_size(int type);   /* bytes per block */

/* IEEE binary16 -> binary32, exact (Float.float16ToFloat,
 * FloatTensorHelpers.kt:39-41; Q6_KFloatTensor.kt:87-109) */
float o_f16_to_f32(uint16_t h);

/* FloatTensor.get(index) for one element of a flat block stream */
float o_get(int type, const uint8_t *base, int64_t index);
/* out[i] = get(offset + i), i < n */
void o_dequant(int type, const uint8_t *base, int64_t offset, int64_t n, float *out);

/* FloatTensorHelpers.scalarDot (FloatTensorHelpers.kt:65-71) */
float o_scalar_dot(int type, const uint8_t *base, int64_t this_offset, const float *x, int size);
/* XFloatTensor.dot with the Vector API enabled at 512 bits */
float o_vector_dot(int type, const uint8_t *base, int64_t this_offset, const float *x, int size);

/* FloatTensor.matmul(that, out, dim0, dim1, thisOffset) (FloatTensor.kt:18-29):
 * out[i] = dot(thisOffset + i*dim1, x, 0, dim1), rows split across nthreads
 * (IntStream.parallel in Parallel.kt:5-7). vector=0 selects scalarDot. */
void o_matmul(int type, const uint8_t *base, int64_t this_offset, const float *x, float *out,
              int dim0, int dim1, int nthreads, int vector);

/* Llama.kt:23-25 */
float o_gelu(float x);
/* Llama.kt:27-37 */
void o_rmsnorm(float *out, const float *x, const float *w, int size, float eps);
/* MutableFloatTensor.kt:54-59 */
void o_softmax(float *x, int n);
/* Llama.kt:276-293: iterative argmax, strict '>', lowest index wins ties.
 * probs is modified (picked entries set to -inf). */
void o_topk(float *probs, int n, int k, int32_t *idx, float *val);
/* Routing margin (test infrastructure): smallest gap between the k-th and
 * (k+1)-th router probability over the o_moe_token calls since the reset. */
void o_note_topk_margin(const float *probs, int n, int k);
void o_reset_topk_margin(void);
double o_topk_margin(void);

/* The expert half of the MoE block for one token, Llama.kt:248-346.
 * x is the residual stream state.x (dim floats).  Writes the rms-normalised
 * expert output (after post_ffw_norm_2) to out[dim] and the selection to
 * topk_idx/topk_prob (in selection order, raw softmax probabilities). */
typedef struct {
  int dim;            /* hidden size, 2816 */
  int n_expert;       /* 128 */
  int n_used;         /* 8 */
  int expert_ff;      /* 704 */
  float eps;          /* rms_norm eps */
  int gate_up_type;   /* ggml type of ffn_gate_up_exps (Q4_K) */
  int down_type;      /* ggml type of ffn_down_exps (Q4_K) */
  const uint8_t *gate_inp;        /* F32 [dim, n_expert]: n_expert rows of dim */
  const float *gate_inp_scale;    /* F32 [dim] */
  const uint8_t *gate_up_exps;    /* [dim, 2*ff, n_expert] */
  const uint8_t *down_exps;       /* [ff, dim, n_expert] */
  const float *down_exps_scale;   /* F32 [n_expert] */
  const float *pre_ffw_norm_2;    /* F32 [dim] */
  const float *post_ffw_norm_2;   /* F32 [dim] (NULL: skip the post-norm) */
} o_moe_weights;

void o_moe_token(const o_moe_weights *w, const float *x, float *out, int32_t *topk_idx,
                 float *topk_prob, float *router_logits_out, int nthreads);

/* Router stage only (Llama.kt:257-270): logits[n_expert] before softmax */
void o_moe_router_logits(const o_moe_weights *w, const float *x, float *logits);

/* ---------------- whole-model forward (Llama.kt:105-408) ----------------
 * One token at one position through every layer, exactly as Llama.forward:
 * embedding x sqrt(dim), per layer attention (RMSNorm, Q/K/V projections,
 * per-head Q/K norms and bare V norm, NeoX RoPE from the precomputed tables,
 * GQA attention with scale 1.0 over [attStart, position], shared KV for the
 * layers past n_layer_kv_from_start), output projection, post-attention
 * norm + residual, then the dense GELU FFN or the MoE block (shared MLP +
 * experts + merge), layer output scale; final norm, logits, softcapping.
 * Per-layer embeddings (Llama.kt:115-143,366-391) are not restated: the
 * synthetic models of the benchmark have none. */
typedef struct {
  int type;             /* GGML type id */
  const uint8_t *data;  /* block stream */
} o_tensor;

typedef struct {
  const float *attn_norm, *attn_q_norm, *attn_k_norm, *post_attention_norm, *ffn_norm, *post_ffw_norm;
  o_tensor wq, wk, wv, wo; /* wv.data == NULL: V = K (Llama.kt:176-181) */
  o_tensor w1, w2, w3;     /* ffn_gate, ffn_down, ffn_up */
  /* MoE layers only (Llama.kt:226-353) */
  const float *post_ffw_norm_1, *pre_ffw_norm_2, *post_ffw_norm_2, *gate_inp_scale, *down_exps_scale;
  o_tensor gate_inp, gate_up_exps, down_exps;
} o_layer;

typedef struct {
  int dim, n_layers, n_heads, vocab, ctx_len;
  int head_size_full, head_size_swa, sliding_window, n_layer_kv_from_start;
  float eps, rope_theta, rope_theta_swa, logit_softcap;
  int n_expert, n_expert_used, expert_ff; /* n_expert == 0: dense model */
  const int *n_kv_heads;     /* [n_layers] */
  const int *ff;             /* [n_layers] feed_forward_length */
  const uint8_t *is_swa;     /* [n_layers] */
  const float *layer_scale;  /* [n_layers] */
  const float *rope_freqs;   /* [head_size_full/2] rope_freqs.weight */
  o_tensor tok_embd, output; /* output.data == NULL: tied to tok_embd */
  const float *output_norm;
  const o_layer *layers;
} o_model;

typedef struct o_state o_state;

/* RotaryPositionEmbeddings.precomputeFreqsCis (RotaryPositionEmbeddings.kt:8-27)
 * and precomputeFreqsCisFromFreqs (:29-53): cr/ci [ctx * head/2]. */
void o_rope_table(int ctx_len, int head_size, double theta, const float *freq_factors, float *cr, float *ci);

o_state *o_state_new(const o_model *m);
void o_state_free(o_state *s);
/* Llama.forward(model, state, token, position); returns state.logits (vocab floats). */
const float *o_forward(const o_model *m, o_state *s, int token, int position, int nthreads);
/* FloatTensor.argmax (FloatTensor.kt:120-133): first index of the maximum. */
int o_argmax(const float *v, int n);
/* 1 (default): the Vector API dot products (512-bit branch); 0: scalarDot
 * everywhere, the reference's llama.VectorBitSize=0 mode. */
void o_set_vector_api(int on);

#ifdef __cplusplus
}
#endif
#endif
