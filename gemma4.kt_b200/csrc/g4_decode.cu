// g4_decode.cu -- GPU-resident Llama.forward (Llama.kt:105-408) and the greedy
// decode loop of Llama.generateTokens (Llama.kt:413-477), on sm_100a.
//
// One decode step (one token at one position) is one CUDA graph of, per layer:
//
//   qkv GEMV     prologue: previous layer's residual + post-FFN norm + layer
//                scale (or the embedding x sqrt(dim) at layer 0), then
//                rmsnorm(attn_norm); rows q | k | v of one fused tensor
//   attention    per (KV head, position chunk) CTA: the chunk's K/V rows bulk-
//                copied to shared memory, Q/K norms, NeoX RoPE, the new K/V row
//                into the cache, scores (scale 1.0), softmax partials and V sums
//   wo GEMV      prologue: the chunks combined into the attention output
//   gate/up GEMV prologue: residual + post-attention norm, rmsnorm(ffn_norm);
//                rows interleaved gate_i, up_i; epilogue gelu(gate) * up
//   down GEMV    plain (the shared MLP of a MoE layer)
//   [MoE layers: the expert half (g4_moe.cu kernels) on the residual stream;
//    the next layer's qkv prologue merges shared + expert outputs]
//
// then the logits GEMV (final residual, output_norm, softcapping, argmax as
// an atomicMax key) and a one-thread sampling kernel that records the argmax
// and feeds it to the next step.  Every kernel after the first is launched
// with programmatic stream serialization: a GEMV streams its first weight
// stages before waiting for its predecessor.  The step index, the input token
// and the position live in device memory, so a greedy generation of N tokens
// is N graph launches with no host round trip.  The GEMVs use fp32-level
// activations (three int8 limbs on the Q8_0 tensor-core tiles, two-part int16
// on the CUDA-core decoders): with attention scale 1.0 on normalised q and k,
// activation errors of a few 1e-5 visibly move the attention weights.
//
// The second half of the file is the batched decoder (g4_batch_*): up to 64
// rows per step, each a (token, position, KV slot), so many sequences advance
// together (configuration 5) or one sequence's prompt is prefilled in chunks;
// per layer a per-token prologue into int8 limbs, the T-token GEMM on the
// repacked Q8_0 tiles (g4_gemv_mma.cu), a K/V-row pre-pass, the attention
// kernel with a row grid axis, and the MoE layer on the step's tokens (across
// GPUs: expert-parallel, g4_batch_expert_parallel).
#include "g4.h"
#include "g4_ctx.h"
#include "g4_gemv.cuh"
#include "g4_internal.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <initializer_list>
#include <map>
#include <new>
#include <string>
#include <vector>

namespace g4 {

constexpr int kAttnThreads = 256;
constexpr int kMaxKvHeads = 64;      // KV heads per layer
constexpr size_t kAttnTileBudget = 160 * 1024;  // shared memory for a chunk's K and V rows

// Position chunks of the decoder's attention: at most kAttnMaxChunks per
// KV head, about len / target positions each, a multiple of 16, at most
// ch_max (the shared-memory tile).
constexpr int kAttnMaxChunks = 128;
constexpr int kAttnMaxHs = 512;     // head size
constexpr int kAttnMaxGroup = 16;   // query heads per KV head
__host__ __device__ __forceinline__ int attn_chunk(int len, int ch_max, int target) {
  int ch = ((len + target - 1) / target + 15) / 16 * 16;
  return ch < 16 ? 16 : ch > ch_max ? ch_max : ch;
}

struct AttnArgs {
  const float* qkv;        // raw projections: q [n_heads*hs] | k [n_kv*hs] | v [n_kv*hs]
  int hs, kv_mul, kvdim;
  int k_off, v_off;        // offsets of k and v in qkv (v_off == k_off when V = K)
  const float* q_norm;     // [hs]
  const float* k_norm;     // [hs]
  float eps;
  const float* cr;         // rope tables [ctx][hs/2] of this layer's attention type
  const float* ci;
  float* kc;               // KV cache of the layer's KV source layer [ctx][kvdim]
  float* vc;
  int write_kv;            // the layer has its own KV (Llama.kt:174)
  int window;              // sliding window (0: full attention)
  const int* step;
  const int* in_pos;
  float* part;             // [n_heads][kAttnMaxChunks][hs + 2]: (max, sum, acc[hs]) per chunk
  unsigned* tickets;       // [n_heads] chunks finished; the last one combines and resets it
  float* out;              // [n_heads * hs] attention output
  int ch_max;              // positions per chunk that fit the shared-memory tiles (multiple of 16)
  unsigned* status;
  // Batched decode (g4_batch_step): sequence blockIdx.y at position pos_arr[y]
  // with its own rows of qkv / cache / partials / tickets / out (strides in
  // elements); chunk_stride CTAs per query head along x.  Single-sequence
  // decode: pos_arr == nullptr, strides 0, chunk_stride kAttnMaxChunks.
  const int* pos_arr;
  const int* slot_arr;     // batched: KV-cache slot of each grid row (nullptr: slot = row)
  long long qkv_stride, kv_stride, part_stride, out_stride;
  int tick_stride, chunk_stride;
  int target_chunks;       // chunks per KV head aimed at (attn_chunk)
  int heads_per_cta;       // query heads of a KV group served by one CTA (divides kv_mul)
};

// Llama.kt:39-59 per-head rmsnorm, (w * ss) * x left to right (w == nullptr:
// the bare norm of Llama.kt:62-81); one warp per head vector in shared memory.
__device__ __forceinline__ void head_rmsnorm(float* v, const float* w, int hs, float eps, int lane) {
  float ss = 0.f;
  for (int i = lane; i < hs; i += 32) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
  const float s = rms_scale(warp_sum(ss), hs, eps);
  __syncwarp();
  for (int i = lane; i < hs; i += 32) v[i] = w ? __fmul_rn(__fmul_rn(w[i], s), v[i]) : __fmul_rn(s, v[i]);
  __syncwarp();
}

// Llama.kt:83-103: pairs (ic, ic + hs/2)
__device__ __forceinline__ void head_rope(float* v, const float* fr, const float* fi, int hs, int lane) {
  const int half = hs / 2;
  for (int ic = lane; ic < half; ic += 32) {
    const float fcr = fr[ic], fci = fi[ic];
    const float v0 = v[ic], v1 = v[ic + half];
    v[ic] = __fsub_rn(__fmul_rn(v0, fcr), __fmul_rn(v1, fci));
    v[ic + half] = __fadd_rn(__fmul_rn(v0, fci), __fmul_rn(v1, fcr));
  }
  __syncwarp();
}

// Attention of one layer (Llama.kt:157-218) for KV head g and position chunk
// c of this CTA: every query head of the group (kv_mul of them, Llama.kt:200)
// reads the same K and V rows, so the CTA stages the chunk's rows once and
// serves all of them.  The chunk's rows of earlier positions are final before
// the step starts, so their bulk copies into shared memory (and the RoPE row
// of the position) are issued before waiting for the q/k/v projection.  Each
// (query head, chunk) leaves (max, sum, acc) partials; the group's last chunk
// to finish (a ticket counter) combines them into the heads' outputs.
template <int HMAX>  // heads_per_cta <= HMAX
__global__ void __launch_bounds__(kAttnThreads, HMAX == 1 ? 1 : 3) dec_attention_kernel(const __grid_constant__ AttnArgs a) {
  extern __shared__ __align__(128) uint8_t smraw[];
  const int hs = a.hs, half = hs / 2, H = a.heads_per_cta, nsub = a.kv_mul / H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, NW = kAttnThreads / 32;
  // the step's position is staged by the host before the step's first kernel
  const int sq = blockIdx.y;
  const int pos = a.pos_arr ? a.pos_arr[sq] : a.in_pos[*a.step];
  const int start = a.window > 0 ? max(0, pos - a.window + 1) : 0;
  const int len = pos - start + 1;
  const int ch = attn_chunk(len, a.ch_max, a.target_chunks);
  const int nch = (len + ch - 1) / ch;
  // CTA x index: (KV head g, subset hsub of its query heads, chunk c)
  const int gs = blockIdx.x / a.chunk_stride, c = blockIdx.x % a.chunk_stride;
  const int g = gs / nsub, hq0 = g * a.kv_mul + (gs % nsub) * H;  // first query head of this CTA
  const float* qkv = a.qkv + sq * a.qkv_stride;
  const long long slot = a.slot_arr ? a.slot_arr[sq] : sq;
  float* kc = a.kc + slot * a.kv_stride;
  float* vc = a.vc + slot * a.kv_stride;
  float* part_base = a.part + sq * a.part_stride;
  unsigned* tickets = a.tickets + sq * a.tick_stride;
  float* out = a.out + sq * a.out_stride;
  if (c >= nch) return;
  const int t0 = start + c * ch, t1 = min(t0 + ch, pos + 1), n = t1 - t0;
  float* kt = reinterpret_cast<float*>(smraw);        // [ch_max][hs]
  float* vt = kt + (size_t)a.ch_max * hs;             // [ch_max][hs]
  float* qs = vt + (size_t)a.ch_max * hs;             // [H][hs]
  float* fr = qs + (size_t)H * hs;                    // [hs/2] RoPE row of pos
  float* fi = fr + half;
  float* sc = fi + half;                              // [H][ch_max] scores, then exp
  float* wc = sc + (size_t)H * a.ch_max;              // [H][kAttnMaxChunks] combine weights
  float* st = wc + (size_t)H * kAttnMaxChunks;        // [H][4]: max, sum, denominator; [4H] last flag
  uint64_t* bar = reinterpret_cast<uint64_t*>(st + ((4 * H + 2) & ~1));

  // rows t < pos of the chunk: bulk copies before the wait
  const int n_pre = max(0, min(t1, pos) - t0);
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (warp == 0) {
    const uint32_t row_bytes = (uint32_t)hs * 4u;
    if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)n_pre * row_bytes * 2u);
    __syncwarp();
    for (int j = lane; j < n_pre; j += 32) {
      const size_t src = (size_t)(t0 + j) * a.kvdim + (size_t)g * hs;
      bulk_g2s(kt + (size_t)j * hs, kc + src, row_bytes, bar);
      bulk_g2s(vt + (size_t)j * hs, vc + src, row_bytes, bar);
    }
  }
  const bool has_pos = t1 == pos + 1;
  for (int i = tid; i < half; i += kAttnThreads) {
    fr[i] = a.cr[(size_t)pos * half + i];
    fi[i] = a.ci[(size_t)pos * half + i];
  }
  grid_dep_wait();
  grid_dep_launch();
  float* kp = kt + (size_t)(pos - t0) * hs;  // the row of this position (when has_pos)
  float* vp = vt + (size_t)(pos - t0) * hs;
  // q of the group's heads (Llama.kt:158-168) and, in the chunk holding the
  // position, its K/V row: computed (Llama.kt:174-195) or, for a layer that
  // shares an earlier layer's cache, read from it
  for (int i = tid; i < H * hs; i += kAttnThreads) qs[i] = qkv[(size_t)hq0 * hs + i];
  if (has_pos) {
    const size_t row = (size_t)pos * a.kvdim + (size_t)g * hs;
    for (int i = tid; i < hs; i += kAttnThreads) {
      kp[i] = a.write_kv ? qkv[a.k_off + (size_t)g * hs + i] : kc[row + i];
      vp[i] = a.write_kv ? qkv[a.v_off + (size_t)g * hs + i] : vc[row + i];
    }
  }
  __syncthreads();
  // per warp: query heads, then (own row) K: learned norm and RoPE, V: bare norm (Llama.kt:183-195)
  for (int j = warp; j < H + 2; j += NW) {
    if (j < H) {
      head_rmsnorm(qs + (size_t)j * hs, a.q_norm, hs, a.eps, lane);
      head_rope(qs + (size_t)j * hs, fr, fi, hs, lane);
    } else if (has_pos && a.write_kv) {
      if (j == H) {
        head_rmsnorm(kp, a.k_norm, hs, a.eps, lane);
        head_rope(kp, fr, fi, hs, lane);
      } else {
        head_rmsnorm(vp, nullptr, hs, a.eps, lane);
      }
    }
  }
  __syncthreads();
  if (has_pos && a.write_kv && gs % nsub == 0) {
    const size_t row = (size_t)pos * a.kvdim + (size_t)g * hs;
    for (int i = tid; i < hs; i += kAttnThreads) {
      kc[row + i] = kp[i];
      vc[row + i] = vp[i];
    }
  }
  if (!mbar_wait_bounded(bar, 0)) {
    record_error(a.status, ERR_TIMEOUT_FULL);
    // give the copies still in flight one more bounded wait before the CTA leaves
    if (!mbar_wait_bounded(bar, 0)) record_error(a.status, ERR_TIMEOUT_DRAIN);
    return;
  }

  // scores q_j . k_t (Llama.kt:204-208): a warp per position, the K row in
  // registers, every head of the group against it
  for (int p = warp; p < n; p += NW) {
    const float* kr = kt + (size_t)p * hs;
    float kreg[kAttnMaxHs / 32];
#pragma unroll
    for (int u = 0; u < kAttnMaxHs / 32; ++u) kreg[u] = lane + 32 * u < hs ? kr[lane + 32 * u] : 0.f;
    for (int j = 0; j < H; ++j) {
      const float* qj = qs + (size_t)j * hs;
      float acc = 0.f;
#pragma unroll
      for (int u = 0; u < kAttnMaxHs / 32; ++u)
        if (lane + 32 * u < hs) acc = fmaf(qj[lane + 32 * u], kreg[u], acc);
      acc = warp_sum(acc);
      if (lane == 0) sc[(size_t)j * a.ch_max + p] = acc;
    }
  }
  __syncthreads();
  // chunk softmax statistics per head: exp((s - m) as double), as softmaxInPlace (MutableFloatTensor.kt:54-59)
  for (int j = warp; j < H; j += NW) {
    float* sj = sc + (size_t)j * a.ch_max;
    float m = -INFINITY;
    for (int p = lane; p < n; p += 32) m = fmaxf(m, sj[p]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int p = lane; p < n; p += 32) {
      const float e = (float)exp((double)__fsub_rn(sj[p], m));
      sj[p] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      st[4 * j] = m;
      st[4 * j + 1] = l;
    }
  }
  __syncthreads();
  // partial V sums per head (Llama.kt:211-217): each V element read once for all heads
  for (int d = tid; d < hs; d += kAttnThreads) {
    float acc[HMAX];
#pragma unroll
    for (int j = 0; j < HMAX; ++j) acc[j] = 0.f;
    for (int p = 0; p < n; ++p) {
      const float v = vt[(size_t)p * hs + d];
#pragma unroll
      for (int j = 0; j < HMAX; ++j)
        if (j < H) acc[j] = fmaf(sc[(size_t)j * a.ch_max + p], v, acc[j]);
    }
#pragma unroll
    for (int j = 0; j < HMAX; ++j)
      if (j < H) part_base[((size_t)(hq0 + j) * kAttnMaxChunks + c) * (hs + 2) + 2 + d] = acc[j];
  }
  if (tid < H) {
    float* pj = part_base + ((size_t)(hq0 + tid) * kAttnMaxChunks + c) * (hs + 2);
    pj[0] = st[4 * tid];
    pj[1] = st[4 * tid + 1];
  }
  // the group's last chunk to finish combines the partials (release: fence, then the ticket)
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const unsigned done = atomicAdd(tickets + gs, 1u);
    st[4 * H] = done + 1 == (unsigned)nch ? 1.f : 0.f;
  }
  __syncthreads();
  if (st[4 * H] == 0.f) return;
  __threadfence();  // acquire: the other chunks' partials are visible
  // out_j = sum_c w_c acc_c / sum_c w_c l_c, w_c = exp(m_c - max m) (Llama.kt:201-218 over the chunks)
  for (int j = warp; j < H; j += NW) {
    const float* ph = part_base + (size_t)(hq0 + j) * kAttnMaxChunks * (hs + 2);
    float* wj = wc + (size_t)j * kAttnMaxChunks;
    float mc[kAttnMaxChunks / 32], lc[kAttnMaxChunks / 32];
#pragma unroll
    for (int u = 0; u < kAttnMaxChunks / 32; ++u) {
      const int k = lane + 32 * u;
      mc[u] = k < nch ? __ldcg(ph + (size_t)k * (hs + 2)) : -INFINITY;
      lc[u] = k < nch ? __ldcg(ph + (size_t)k * (hs + 2) + 1) : 0.f;
    }
    float M = -INFINITY;
#pragma unroll
    for (int u = 0; u < kAttnMaxChunks / 32; ++u) M = fmaxf(M, mc[u]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float dsum = 0.f;
#pragma unroll
    for (int u = 0; u < kAttnMaxChunks / 32; ++u) {
      const int k = lane + 32 * u;
      if (k < nch) {
        const float w = (float)exp((double)__fsub_rn(mc[u], M));
        wj[k] = w;
        dsum = fmaf(w, lc[u], dsum);
      }
    }
    dsum = warp_sum(dsum);
    if (lane == 0) st[4 * j + 2] = dsum;
  }
  __syncthreads();
  // every output of this thread (up to kEl) and kCh chunks per round: one
  // round of memory latency for up to kCh chunks
  constexpr int kCh = 8, kEl = HMAX < 4 ? HMAX : 4;
  for (int e0 = tid; e0 < H * hs; e0 += kEl * kAttnThreads) {
    float num[kEl];
#pragma unroll
    for (int i = 0; i < kEl; ++i) num[i] = 0.f;
    for (int k0 = 0; k0 < nch; k0 += kCh) {
      float v[kEl][kCh];
#pragma unroll
      for (int i = 0; i < kEl; ++i) {
        const int e = e0 + i * kAttnThreads, j = e / hs, d = e - j * hs;
        const float* ph = part_base + (size_t)(hq0 + j) * kAttnMaxChunks * (hs + 2) + 2 + d;
#pragma unroll
        for (int u = 0; u < kCh; ++u)
          v[i][u] = (e < H * hs && k0 + u < nch) ? __ldcg(ph + (size_t)(k0 + u) * (hs + 2)) : 0.f;
      }
#pragma unroll
      for (int i = 0; i < kEl; ++i) {
        const int e = e0 + i * kAttnThreads, j = e / hs;
#pragma unroll
        for (int u = 0; u < kCh; ++u)
          if (e < H * hs && k0 + u < nch) num[i] = fmaf(wc[(size_t)j * kAttnMaxChunks + k0 + u], v[i][u], num[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < kEl; ++i) {
      const int e = e0 + i * kAttnThreads, j = e / hs, d = e - j * hs;
      if (e < H * hs) out[(size_t)(hq0 + j) * hs + d] = __fdiv_rn(num[i], st[4 * j + 2]);
    }
  }
  if (tid == 0) tickets[gs] = 0u;  // every chunk has arrived: ready for the next launch
}

// Batched steps: the K/V rows of every token of the step (Llama.kt:174-195:
// K learned norm then RoPE, V bare norm) written to its sequence's cache
// before any attention of the step reads them, so that tokens of one
// sequence at consecutive positions (a prompt chunk) see each other's rows.
// Grid (KV head, token); warp 0 K, warp 1 V.
__global__ void __launch_bounds__(64) batch_kv_write_kernel(const __grid_constant__ AttnArgs a) {
  extern __shared__ __align__(16) float kvrow[];  // [2][hs]
  const int g = blockIdx.x, sq = blockIdx.y, hs = a.hs, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = a.pos_arr[sq];
  const long long slot = a.slot_arr ? a.slot_arr[sq] : sq;
  const float* qkv = a.qkv + sq * a.qkv_stride;
  float* v = kvrow + warp * hs;
  const float* src = qkv + (warp == 0 ? a.k_off : a.v_off) + (size_t)g * hs;
  for (int i = lane; i < hs; i += 32) v[i] = src[i];
  __syncwarp();
  if (warp == 0) {
    head_rmsnorm(v, a.k_norm, hs, a.eps, lane);
    head_rope(v, a.cr + (size_t)pos * (hs / 2), a.ci + (size_t)pos * (hs / 2), hs, lane);
  } else {
    head_rmsnorm(v, nullptr, hs, a.eps, lane);
  }
  float* dst = (warp == 0 ? a.kc : a.vc) + slot * a.kv_stride + (size_t)pos * a.kvdim + (size_t)g * hs;
  for (int i = lane; i < hs; i += 32) dst[i] = v[i];
}

// Greedy sampling (Sampler.ARGMAX, FloatTensor.argmax): the logits GEMV left
// the maximum's key; record the token, feed it to the next step, reset.
__global__ void dec_sample_kernel(int* ctl, int* out_tok, unsigned long long* argmax) {
  grid_dep_wait();
  if (threadIdx.x == 0) {
    const int s = ctl[0];
    const unsigned long long k = *argmax;
    const int tok = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
    out_tok[s] = tok;
    ctl[1] = tok;
    ctl[0] = s + 1;
    *argmax = 0ull;
  }
}

}  // namespace g4

using namespace g4;

// ---------------------------------------------------------------- host side
namespace {

struct LayerDev {
  int hs = 0, qdim = 0, kvdim = 0, n_kv = 0, ff = 0, has_v = 0, swa = 0, kv_src = 0;
  float scale = 1.f;
  g4_tensor* qkv = nullptr;      // rows q | k | v
  g4_tensor* wo = nullptr;
  g4_tensor* gate_up = nullptr;  // rows interleaved gate_i, up_i
  g4_tensor* down = nullptr;
  const float *attn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr, *post_attn_norm = nullptr;
  const float *ffn_norm = nullptr, *post_ffw_norm = nullptr, *post_ffw_norm_1 = nullptr;
  g4_moe_weights moe{};
  GemvPlan p_qkv{}, p_wo{}, p_gu{}, p_down{};        // general GEMV plans (BF16 / F32 and other layouts)
  DecGemvPlan d_qkv{}, d_wo{}, d_gu{}, d_down{};     // decoder GEMV (Q8_0 / Q4_K / Q6_K), used when fast
  MmaGemvPlan m_qkv{}, m_wo{}, m_gu{}, m_down{};     // Q8_0 on the tensor cores, used when fast
  uint8_t *k_qkv = nullptr, *k_wo = nullptr, *k_gu = nullptr, *k_down = nullptr;  // their repacked weights
};

// One of a layer's projections: the tensor-core Q8_0 GEMV (repacked weights),
// else the decoder GEMV when it applies, else the general one.
static int launch_proj(const MmaGemvPlan& mm, const uint8_t* packed, const DecGemvPlan& d, const GemvPlan& g,
                       const g4_tensor* w, const float* x, float* y, const GemvFuse& f, unsigned* status,
                       cudaStream_t st, bool pdl) {
  if (mm.fast && packed) return launch_gemv_mma(mm, packed, x, y, f, status, st, pdl);
  if (d.fast) return launch_gemv_dec(d, (const uint8_t*)w->d, x, y, f, status, st, pdl);
  return launch_gemv_fused(g, (const uint8_t*)w->d, x, y, f, status, st, pdl);
}

const char* kLayerNames[] = {
    "attn_norm.weight", "attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_output.weight",
    "attn_q_norm.weight", "attn_k_norm.weight", "post_attention_norm.weight", "ffn_norm.weight",
    "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight", "post_ffw_norm.weight", "layer_output_scale.weight",
    "post_ffw_norm_1.weight", "pre_ffw_norm_2.weight", "post_ffw_norm_2.weight", "ffn_gate_inp.weight",
    "ffn_gate_inp.scale", "ffn_gate_up_exps.weight", "ffn_down_exps.weight", "ffn_down_exps.scale"};

}  // namespace

struct g4_model {
  g4_ctx* ctx = nullptr;
  g4_model_config cfg{};
  std::vector<int> n_kv, ff;
  std::vector<unsigned char> is_swa;
  std::map<std::string, g4_tensor*> t;  // uploaded tensors by GGUF name
  std::vector<float> layer_scale;
  std::vector<float> rope_freqs;
  std::vector<LayerDev> L;
  const g4_tensor* wcls = nullptr;
  GemvPlan p_logits{};
  MmaGemvPlan m_logits{};    // the output projection on the tensor-core tiles (Q8_0), used when fast
  uint8_t* k_cls = nullptr;  // the output matrix repacked (the decoder's logits, the batched decoder)
  float *cr_full = nullptr, *ci_full = nullptr, *cr_swa = nullptr, *ci_swa = nullptr;
  bool finalized = false;
  int max_q = 0, max_kv = 0, max_ff = 0, max_hs = 0;

  const g4_tensor* get(const std::string& n) const {
    auto it = t.find(n);
    return it == t.end() ? nullptr : it->second;
  }
  const float* f32(const std::string& n) const {
    const g4_tensor* x = get(n);
    return x ? static_cast<const float*>(x->d) : nullptr;
  }
};

struct g4_state {
  g4_model* m = nullptr;
  cudaStream_t st = nullptr;
  float* buf = nullptr;  // one allocation for the activations and the KV cache
  float *x[2] = {nullptr, nullptr}, *qkv = nullptr, *xbk = nullptr, *xb2 = nullptr, *hb = nullptr, *sh = nullptr;
  float *moe_out = nullptr, *logits = nullptr, *part = nullptr;
  std::vector<float*> kc, vc;
  uint8_t* small = nullptr;     // argmax key, step control
  unsigned long long* argmax = nullptr;
  int* ctl = nullptr;     // [0] step, [1] next token, then in_tok[ctx], in_pos[ctx], out_tok[ctx]
  unsigned* tickets = nullptr;  // attention: chunks finished per query head (zero between launches)
  int* h_ctl = nullptr;   // pinned staging of the same layout
  cudaGraphExec_t graph = nullptr;
  int* in_tok() const { return ctl + 4; }
  int* in_pos() const { return ctl + 4 + m->cfg.ctx_len; }
  int* out_tok() const { return ctl + 4 + 2 * m->cfg.ctx_len; }
};

static int tensor_ok_n(const g4_tensor* t, int type, uint64_t n) {
  return t && (type < 0 || t->type == type) && t->n_elems == n;
}

extern "C" {

int g4_model_create(g4_ctx* c, const g4_model_config* cfg, g4_model** out) {
  if (!c) return G4_E_ARG;
  if (!cfg || !out || !cfg->n_kv_heads || !cfg->ff || !cfg->is_swa) {
    c->set_err("g4_model_create: NULL argument");
    return G4_E_ARG;
  }
  const g4_model_config& k = *cfg;
  if (k.dim <= 0 || k.dim % 32 || k.n_layers <= 0 || k.n_heads <= 0 || k.vocab <= 0 || k.ctx_len <= 0 ||
      k.head_size_full <= 0 || k.head_size_swa <= 0 || k.head_size_full % 2 || k.head_size_swa % 2 ||
      k.n_layer_kv_from_start < 1 || k.n_layer_kv_from_start > k.n_layers || k.dim > 16384) {
    c->set_err("g4_model_create: unsupported configuration");
    return G4_E_ARG;
  }
  g4_model* m = new (std::nothrow) g4_model();
  if (!m) return G4_E_NOMEM;
  m->ctx = c;
  m->cfg = k;
  m->n_kv.assign(k.n_kv_heads, k.n_kv_heads + k.n_layers);
  m->ff.assign(k.ff, k.ff + k.n_layers);
  m->is_swa.assign(k.is_swa, k.is_swa + k.n_layers);
  m->cfg.n_kv_heads = m->n_kv.data();
  m->cfg.ff = m->ff.data();
  m->cfg.is_swa = m->is_swa.data();
  m->layer_scale.assign(k.n_layers, 1.f);
  for (int l = 0; l < k.n_layers; ++l) {
    const int hs = m->is_swa[l] ? k.head_size_swa : k.head_size_full;
    if (m->n_kv[l] <= 0 || m->n_kv[l] > kMaxKvHeads || k.n_heads % m->n_kv[l] || m->ff[l] <= 0) {
      delete m;
      c->set_err("g4_model_create: layer %d: bad KV head count (1..%d dividing the heads) or FFN width", l,
                 kMaxKvHeads);
      return G4_E_ARG;
    }
    const int chm = (int)std::min<size_t>(256, kAttnTileBudget / ((size_t)hs * 8) / 16 * 16);
    if (chm < 16 || k.ctx_len > kAttnMaxChunks * chm) {
      delete m;
      c->set_err("g4_model_create: context %d too long for head size %d (at most %d positions)", k.ctx_len, hs,
                 kAttnMaxChunks * chm);
      return G4_E_ARG;
    }
    m->max_q = std::max(m->max_q, k.n_heads * hs);
    m->max_kv = std::max(m->max_kv, m->n_kv[l] * hs);
    m->max_ff = std::max(m->max_ff, m->ff[l]);
    m->max_hs = std::max(m->max_hs, hs);
  }
  *out = m;
  return 0;
}

int g4_model_set_tensor(g4_model* m, const char* name, int ggml_type, const void* host, uint64_t nbytes,
                        uint64_t n_elems) {
  if (!m) return G4_E_ARG;
  g4_ctx* c = m->ctx;
  if (!name || !host) {
    c->set_err("g4_model_set_tensor: NULL argument");
    return G4_E_ARG;
  }
  if (m->finalized) {
    c->set_err("g4_model_set_tensor: the model is already finalized");
    return G4_E_ARG;
  }
  const std::string n(name);
  bool known = n == "token_embd.weight" || n == "output.weight" || n == "output_norm.weight" ||
               n == "rope_freqs.weight";
  if (!known && n.rfind("blk.", 0) == 0) {
    const size_t dot = n.find('.', 4);
    if (dot != std::string::npos) {
      const std::string suffix = n.substr(dot + 1);
      for (const char* s : kLayerNames) known = known || suffix == s;
      const int l = atoi(n.substr(4, dot - 4).c_str());
      known = known && l >= 0 && l < m->cfg.n_layers;
    }
  }
  if (!known) {
    // per-layer embeddings (Llama.kt:115-143,366-391) and anything else the
    // decoder does not compute
    c->set_err("g4_model_set_tensor: tensor %s is not used by this decoder", name);
    return G4_E_TYPE;
  }
  static const std::string kScale = "layer_output_scale.weight";
  if (n.size() > kScale.size() && n.compare(n.size() - kScale.size(), kScale.size(), kScale) == 0) {
    if (ggml_type != G4_TYPE_F32 || n_elems < 1) {
      c->set_err("g4_model_set_tensor: %s must be F32", name);
      return G4_E_TYPE;
    }
    const int l = atoi(n.c_str() + 4);
    memcpy(&m->layer_scale[l], host, 4);  // ModelLoader.kt:179-188
    return 0;
  }
  if (n == "rope_freqs.weight") {
    if (ggml_type != G4_TYPE_F32 || n_elems != (uint64_t)m->cfg.head_size_full / 2) {
      c->set_err("g4_model_set_tensor: rope_freqs.weight must be F32[%d]", m->cfg.head_size_full / 2);
      return G4_E_ARG;
    }
    m->rope_freqs.assign((const float*)host, (const float*)host + n_elems);
    return 0;
  }
  auto it = m->t.find(n);
  if (it != m->t.end()) {
    g4_tensor_free(it->second);
    m->t.erase(it);
  }
  g4_tensor* t = nullptr;
  if (int r = g4_tensor_upload(c, ggml_type, host, nbytes, n_elems, &t)) return r;
  m->t[n] = t;
  return 0;
}

}  // extern "C"

// RotaryPositionEmbeddings.kt:8-53 (ff == nullptr: precomputeFreqsCis)
static void rope_table(int ctx, int hs, double theta, const float* ff, std::vector<float>& cr,
                       std::vector<float>& ci) {
  const int half = hs / 2;
  cr.resize((size_t)ctx * half);
  ci.resize((size_t)ctx * half);
  size_t n = 0;
  for (int pos = 0; pos < ctx; ++pos)
    for (int i = 0; i < half; ++i) {
      float value;
      if (ff) {
        const float base = (float)(1.0 / pow(theta, (2.0 * i) / hs));
        value = (float)pos * base;
        value = value / ff[i];
      } else {
        const float freq = (float)(1.0 / pow(theta, (double)(2 * i) / (double)hs));
        value = (float)pos * freq;
      }
      cr[n] = (float)cos((double)value);
      ci[n] = (float)sin((double)value);
      ++n;
    }
}

static int upload_f32(g4_ctx* c, const std::vector<float>& v, float** out) {
  if (cudaMalloc(out, v.size() * 4 + 256) != cudaSuccess) {
    cudaGetLastError();
    *out = nullptr;
    c->set_err("decoder: cannot allocate %zu bytes", v.size() * 4);
    return G4_E_NOMEM;
  }
  if (cudaError_t e = cudaMemcpy(*out, v.data(), v.size() * 4, cudaMemcpyHostToDevice))
    return c->cuda_fail(e, "decoder upload");
  return 0;
}

// A device tensor holding the rows of several same-type tensors: rows of
// `parts` one after the other (interleave false), or row i of every part in
// turn (interleave true: gate_0, up_0, gate_1, up_1, ...).
static int fuse_rows(g4_ctx* c, const std::vector<const g4_tensor*>& parts, int cols, bool interleave,
                     g4_tensor** out) {
  const int type = parts[0]->type;
  const uint64_t BS = block_size(type), TS = type_size(type);
  if (cols % BS) {
    c->set_err("decoder: rows of %d elements do not hold whole %llu-element blocks", cols, (unsigned long long)BS);
    return G4_E_TYPE;
  }
  const size_t row_bytes = (size_t)cols / BS * TS;
  uint64_t n = 0, bytes = 0;
  for (const g4_tensor* p : parts) {
    if (p->type != type) {
      c->set_err("decoder: fused projections need one GGML type (got %d and %d)", type, p->type);
      return G4_E_TYPE;
    }
    n += p->n_elems;
    bytes += p->nbytes;
  }
  g4_tensor* t = new (std::nothrow) g4_tensor();
  if (!t) return G4_E_NOMEM;
  const size_t alloc = (bytes + 255) / 256 * 256 + 256;
  if (cudaMalloc(&t->d, alloc) != cudaSuccess) {
    cudaGetLastError();
    delete t;
    c->set_err("decoder: cannot allocate %zu bytes", alloc);
    return G4_E_NOMEM;
  }
  cudaMemset(t->d, 0, alloc);
  uint8_t* dst = (uint8_t*)t->d;
  cudaError_t e = cudaSuccess;
  if (!interleave) {
    size_t o = 0;
    for (const g4_tensor* p : parts) {
      e = cudaMemcpy(dst + o, p->d, p->nbytes, cudaMemcpyDeviceToDevice);
      o += p->nbytes;
      if (e) break;
    }
  } else {
    const size_t k = parts.size();
    for (size_t i = 0; i < k && !e; ++i)
      e = cudaMemcpy2D(dst + i * row_bytes, k * row_bytes, parts[i]->d, row_bytes, row_bytes,
                       parts[i]->nbytes / row_bytes, cudaMemcpyDeviceToDevice);
  }
  if (e) {
    cudaFree(t->d);
    delete t;
    return c->cuda_fail(e, "decoder: fusing projections");
  }
  t->ctx = c;
  t->type = type;
  t->nbytes = bytes;
  t->n_elems = n;
  *out = t;
  return 0;
}

static void drop(g4_model* m, const std::string& n) {
  auto it = m->t.find(n);
  if (it != m->t.end()) {
    g4_tensor_free(it->second);
    m->t.erase(it);
  }
}

// The tensor-core Q8_0 GEMV (g4_gemv_mma.cu) is the decoder's Q8_0 path
// unless G4_DEC_MMA=0 selects the CUDA-core decoder GEMV.
static bool mma_wanted() {
  const char* e = getenv("G4_DEC_MMA");
  return !(e && e[0] == '0');
}

// A Q8_0 projection's copy in the tensor-core tile layout, and its plan;
// other types (or shapes the plan rejects) keep plan.fast == 0.
static int make_mma(g4_ctx* c, const g4_tensor* w, int rows, int cols, bool pair, bool fused, MmaGemvPlan& plan,
                    uint8_t*& packed) {
  if (!w || w->type != G4_TYPE_Q8_0 || w->n_elems != (uint64_t)rows * (uint64_t)cols) return 0;
  MmaGemvPlan p = plan_gemv_mma(c->dev, rows, cols, pair, fused);
  if (!p.fast) return 0;
  const size_t bytes = mma_packed_bytes(rows, cols);
  if (cudaMalloc(&packed, bytes) != cudaSuccess) {
    cudaGetLastError();
    packed = nullptr;
    c->set_err("g4_model_finalize: cannot allocate %zu bytes of repacked Q8_0 weights", bytes);
    return G4_E_NOMEM;
  }
  cudaError_t e = (cudaError_t)repack_q8_0_mma((const uint8_t*)w->d, rows, cols, packed, nullptr);
  if (!e) e = cudaStreamSynchronize(nullptr);
  if (e) return c->cuda_fail(e, "g4_model_finalize: Q8_0 repack");
  plan = p;
  return 0;
}

extern "C" int g4_model_finalize(g4_model* m) {
  if (!m) return G4_E_ARG;
  g4_ctx* c = m->ctx;
  if (m->finalized) return 0;
  if (int r = c->bind()) return r;
  const g4_model_config& k = m->cfg;
  const int dim = k.dim;
  auto need = [&](const std::string& n, int type, uint64_t elems) -> bool {
    if (!tensor_ok_n(m->get(n), type, elems)) {
      c->set_err("g4_model_finalize: tensor %s missing or of the wrong type/size (%llu elements expected)", n.c_str(),
                 (unsigned long long)elems);
      return false;
    }
    return true;
  };
  if (!need("token_embd.weight", -1, (uint64_t)dim * k.vocab) || !need("output_norm.weight", G4_TYPE_F32, dim))
    return G4_E_ARG;
  m->wcls = m->get("output.weight") ? m->get("output.weight") : m->get("token_embd.weight");
  if (m->wcls->n_elems != (uint64_t)dim * k.vocab) {
    c->set_err("g4_model_finalize: output.weight has the wrong size");
    return G4_E_ARG;
  }
  if ((int)m->rope_freqs.size() != k.head_size_full / 2) {
    c->set_err("g4_model_finalize: rope_freqs.weight missing (ModelLoader.kt:156)");
    return G4_E_ARG;
  }
  m->L.resize(k.n_layers);
  for (int l = 0; l < k.n_layers; ++l) {
    LayerDev& L = m->L[l];
    const std::string p = "blk." + std::to_string(l) + ".";
    L.swa = m->is_swa[l] != 0;
    L.hs = L.swa ? k.head_size_swa : k.head_size_full;
    L.n_kv = m->n_kv[l];
    L.qdim = k.n_heads * L.hs;
    L.kvdim = L.n_kv * L.hs;
    L.ff = m->ff[l];
    L.kv_src = l < k.n_layer_kv_from_start ? l : k.n_layer_kv_from_start - (L.swa ? 2 : 1);  // kvSourceLayer
    if (L.kv_src < 0) {
      c->set_err("g4_model_finalize: layer %d has no KV source layer", l);
      return G4_E_ARG;
    }
    if (L.hs > kAttnMaxHs || L.hs % 4 || k.n_heads / L.n_kv > kAttnMaxGroup) {
      c->set_err("g4_model_finalize: layer %d: head size %d (at most %d, a multiple of 4) or %d query heads per "
                 "KV head (at most %d) not supported", l, L.hs, kAttnMaxHs, k.n_heads / L.n_kv, kAttnMaxGroup);
      return G4_E_ARG;
    }
    L.scale = m->layer_scale[l];
    const bool own_kv = l < k.n_layer_kv_from_start;
    if (!need(p + "attn_norm.weight", G4_TYPE_F32, dim) || !need(p + "attn_q_norm.weight", G4_TYPE_F32, L.hs) ||
        !need(p + "post_attention_norm.weight", G4_TYPE_F32, dim) || !need(p + "ffn_norm.weight", G4_TYPE_F32, dim) ||
        !need(p + "post_ffw_norm.weight", G4_TYPE_F32, dim) ||
        !need(p + "attn_q.weight", -1, (uint64_t)dim * L.qdim) ||
        !need(p + "attn_output.weight", -1, (uint64_t)dim * L.qdim) ||
        !need(p + "ffn_gate.weight", -1, (uint64_t)dim * L.ff) ||
        !need(p + "ffn_up.weight", -1, (uint64_t)dim * L.ff) || !need(p + "ffn_down.weight", -1, (uint64_t)dim * L.ff))
      return G4_E_ARG;
    if (own_kv && (!need(p + "attn_k.weight", -1, (uint64_t)dim * L.kvdim) ||
                   !need(p + "attn_k_norm.weight", G4_TYPE_F32, L.hs)))
      return G4_E_ARG;
    L.has_v = m->get(p + "attn_v.weight") != nullptr;
    if (own_kv && L.has_v && !need(p + "attn_v.weight", -1, (uint64_t)dim * L.kvdim)) return G4_E_ARG;
    if (k.n_expert > 0) {
      const int E = k.n_expert, eff = k.expert_ff;
      if (!need(p + "post_ffw_norm_1.weight", G4_TYPE_F32, dim) ||
          !need(p + "pre_ffw_norm_2.weight", G4_TYPE_F32, dim) ||
          !need(p + "post_ffw_norm_2.weight", G4_TYPE_F32, dim) ||
          !need(p + "ffn_gate_inp.weight", G4_TYPE_F32, (uint64_t)dim * E) ||
          !need(p + "ffn_gate_inp.scale", G4_TYPE_F32, dim) || !need(p + "ffn_down_exps.scale", G4_TYPE_F32, E) ||
          !need(p + "ffn_gate_up_exps.weight", -1, (uint64_t)dim * 2 * eff * E) ||
          !need(p + "ffn_down_exps.weight", -1, (uint64_t)eff * dim * E))
        return G4_E_ARG;
      L.moe = g4_moe_weights{dim, E, k.n_expert_used, eff, k.eps, m->get(p + "ffn_gate_inp.weight"),
                             m->get(p + "ffn_gate_inp.scale"), m->get(p + "ffn_gate_up_exps.weight"),
                             m->get(p + "ffn_down_exps.weight"), m->get(p + "ffn_down_exps.scale"),
                             m->get(p + "pre_ffw_norm_2.weight"), m->get(p + "post_ffw_norm_2.weight")};
      L.post_ffw_norm_1 = m->f32(p + "post_ffw_norm_1.weight");
    }
    // fused projections: q | k | v and interleaved gate / up
    std::vector<const g4_tensor*> qkv = {m->get(p + "attn_q.weight")};
    if (own_kv) {
      qkv.push_back(m->get(p + "attn_k.weight"));
      if (L.has_v) qkv.push_back(m->get(p + "attn_v.weight"));
    }
    if (int r = fuse_rows(c, qkv, dim, false, &L.qkv)) return r;
    if (int r = fuse_rows(c, {m->get(p + "ffn_gate.weight"), m->get(p + "ffn_up.weight")}, dim, true, &L.gate_up))
      return r;
    drop(m, p + "attn_q.weight");
    drop(m, p + "attn_k.weight");
    drop(m, p + "attn_v.weight");
    drop(m, p + "ffn_gate.weight");
    drop(m, p + "ffn_up.weight");
    L.wo = m->t[p + "attn_output.weight"];
    L.down = m->t[p + "ffn_down.weight"];
    L.attn_norm = m->f32(p + "attn_norm.weight");
    L.q_norm = m->f32(p + "attn_q_norm.weight");
    L.k_norm = m->f32(p + "attn_k_norm.weight");
    L.post_attn_norm = m->f32(p + "post_attention_norm.weight");
    L.ffn_norm = m->f32(p + "ffn_norm.weight");
    L.post_ffw_norm = m->f32(p + "post_ffw_norm.weight");
    const int qkv_rows = (int)(L.qkv->n_elems / dim);
    // two-part activations everywhere: fp32-level products (plan_gemv exact_x)
    GemvOpts o;
    o.exact_x = true;
    o.latency = true;
    o.fused = true;
    L.p_qkv = plan_gemv(c->dev, L.qkv->type, 0, qkv_rows, dim, o);
    GemvOpts oc = o;  // the attention output is final: no prologue
    oc.fused = false;
    L.p_wo = plan_gemv(c->dev, L.wo->type, 0, dim, L.qdim, oc);
    GemvOpts op = o;
    op.pair_rows = true;
    L.p_gu = plan_gemv(c->dev, L.gate_up->type, 0, 2 * L.ff, dim, op);
    GemvOpts od = o;
    od.fused = false;
    L.p_down = plan_gemv(c->dev, L.down->type, 0, dim, L.ff, od);
    L.d_qkv = plan_gemv_dec(c->dev, L.qkv->type, qkv_rows, dim, false, true);
    L.d_wo = plan_gemv_dec(c->dev, L.wo->type, dim, L.qdim, false, false);
    L.d_gu = plan_gemv_dec(c->dev, L.gate_up->type, 2 * L.ff, dim, true, true);
    L.d_down = plan_gemv_dec(c->dev, L.down->type, dim, L.ff, false, false);
    if (mma_wanted()) {
      if (int r = make_mma(c, L.qkv, qkv_rows, dim, false, true, L.m_qkv, L.k_qkv)) return r;
      if (int r = make_mma(c, L.wo, dim, L.qdim, false, false, L.m_wo, L.k_wo)) return r;
      if (int r = make_mma(c, L.gate_up, 2 * L.ff, dim, true, true, L.m_gu, L.k_gu)) return r;
      if (int r = make_mma(c, L.down, dim, L.ff, false, false, L.m_down, L.k_down)) return r;
    }
    if ((!L.p_qkv.fast && !L.d_qkv.fast) || (!L.p_gu.fast && !L.d_gu.fast) || (!L.p_wo.fast && !L.d_wo.fast) ||
        (!L.p_down.fast && !L.d_down.fast)) {
      c->set_err("g4_model_finalize: layer %d: the projections need a streaming-kernel format "
                 "(Q8_0 / Q4_K / Q6_K / BF16 / F32, rows of whole blocks)", l);
      return G4_E_TYPE;
    }
  }
  GemvOpts ol;
  ol.fused = true;
  ol.exact_x = true;
  m->p_logits = plan_gemv(c->dev, m->wcls->type, 0, k.vocab, dim, ol);
  if (!m->p_logits.fast || m->p_logits.pr != 1) {
    c->set_err("g4_model_finalize: the output projection needs a streaming-kernel format");
    return G4_E_TYPE;
  }
  if (mma_wanted())  // a Q8_0 output matrix also runs on the tensor-core tiles
    if (int r = make_mma(c, m->wcls, k.vocab, dim, false, true, m->m_logits, m->k_cls)) return r;
  // ModelLoader.loadWeights (ModelLoader.kt:154-166): SWA tables from theta_swa, full from rope_freqs
  std::vector<float> cr, ci;
  rope_table(k.ctx_len, k.head_size_swa, (double)k.rope_theta_swa, nullptr, cr, ci);
  if (int r = upload_f32(c, cr, &m->cr_swa)) return r;
  if (int r = upload_f32(c, ci, &m->ci_swa)) return r;
  rope_table(k.ctx_len, k.head_size_full, (double)k.rope_theta, m->rope_freqs.data(), cr, ci);
  if (int r = upload_f32(c, cr, &m->cr_full)) return r;
  if (int r = upload_f32(c, ci, &m->ci_full)) return r;
  m->finalized = true;
  return 0;
}

extern "C" int g4_model_free(g4_model* m) {
  if (!m) return G4_E_ARG;
  cudaSetDevice(m->ctx->dev.device);
  for (auto& kv : m->t) g4_tensor_free(kv.second);
  for (LayerDev& L : m->L) {
    if (L.qkv) g4_tensor_free(L.qkv);
    if (L.gate_up) g4_tensor_free(L.gate_up);
    for (uint8_t* p : {L.k_qkv, L.k_wo, L.k_gu, L.k_down})
      if (p) cudaFree(p);
  }
  if (m->k_cls) cudaFree(m->k_cls);
  for (float* p : {m->cr_full, m->ci_full, m->cr_swa, m->ci_swa})
    if (p) cudaFree(p);
  delete m;
  return 0;
}

extern "C" int g4_state_free(g4_state* s);

extern "C" int g4_state_create(g4_model* m, g4_state** out) {
  if (!m) return G4_E_ARG;
  g4_ctx* c = m->ctx;
  if (!out || !m->finalized) {
    c->set_err("g4_state_create: %s", out ? "finalize the model first" : "NULL argument");
    return G4_E_ARG;
  }
  if (int r = c->bind()) return r;
  const g4_model_config& k = m->cfg;
  g4_state* s = new (std::nothrow) g4_state();
  if (!s) return G4_E_NOMEM;
  s->m = m;
  auto al = [](size_t n) { return (n + 63) / 64 * 64; };  // floats, 256-byte multiples
  const size_t dim = k.dim;
  size_t off = 0;
  const size_t o_x0 = off; off += al(dim);
  const size_t o_x1 = off; off += al(dim);
  const size_t o_qkv = off; off += al(m->max_q + 2 * m->max_kv);
  const size_t o_xbk = off; off += al(m->max_q);
  const size_t o_xb2 = off; off += al(dim);
  const size_t o_hb = off; off += al(m->max_ff);
  const size_t o_sh = off; off += al(dim);
  const size_t o_moe = off; off += al(dim);
  const size_t o_log = off; off += al(k.vocab);
  const size_t o_part = off; off += al((size_t)k.n_heads * kAttnMaxChunks * (m->max_hs + 2));
  std::vector<size_t> o_kc, o_vc;
  for (int l = 0; l < k.n_layer_kv_from_start; ++l) {
    const int hs = m->is_swa[l] ? k.head_size_swa : k.head_size_full;
    const size_t n = al((size_t)k.ctx_len * m->n_kv[l] * hs);
    o_kc.push_back(off);
    off += n;
    o_vc.push_back(off);
    off += n;
  }
  if (cudaMalloc(&s->buf, off * 4) != cudaSuccess) {
    cudaGetLastError();
    delete s;
    c->set_err("g4_state_create: cannot allocate %zu bytes of activations and KV cache", off * 4);
    return G4_E_NOMEM;
  }
  cudaMemset(s->buf, 0, off * 4);
  s->x[0] = s->buf + o_x0;
  s->x[1] = s->buf + o_x1;
  s->qkv = s->buf + o_qkv;
  s->xbk = s->buf + o_xbk;
  s->xb2 = s->buf + o_xb2;
  s->hb = s->buf + o_hb;
  s->sh = s->buf + o_sh;
  s->moe_out = s->buf + o_moe;
  s->logits = s->buf + o_log;
  s->part = s->buf + o_part;
  for (int l = 0; l < k.n_layer_kv_from_start; ++l) {
    s->kc.push_back(s->buf + o_kc[l]);
    s->vc.push_back(s->buf + o_vc[l]);
  }
  const size_t ctl_ints = 4 + 3 * (size_t)k.ctx_len;
  const size_t tickets_off = 256 + (ctl_ints * 4 + 255) / 256 * 256;
  const size_t small = tickets_off + (size_t)k.n_heads * 4;
  if (cudaMalloc(&s->small, small) != cudaSuccess || cudaMallocHost(&s->h_ctl, ctl_ints * 4) != cudaSuccess ||
      cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking) != cudaSuccess) {
    cudaGetLastError();
    g4_state_free(s);
    c->set_err("g4_state_create: cannot allocate control buffers");
    return G4_E_NOMEM;
  }
  cudaMemset(s->small, 0, small);
  s->argmax = reinterpret_cast<unsigned long long*>(s->small);
  s->ctl = reinterpret_cast<int*>(s->small + 256);
  s->tickets = reinterpret_cast<unsigned*>(s->small + tickets_off);
  // The MoE layers take their work buffers from the context's arena: size it
  // (and set the kernels up) now, outside any stream capture.
  if (k.n_expert > 0) {
    int r = g4_moe_layer(c, &m->L[0].moe, s->x[0], s->moe_out, 1, nullptr, nullptr, s->st);
    if (!r) r = c->check_status(s->st);
    if (r) {
      g4_state_free(s);
      return r;
    }
  }
  if (cudaError_t e = cudaStreamSynchronize(s->st)) {
    g4_state_free(s);
    return c->cuda_fail(e, "g4_state_create");
  }
  *out = s;
  return 0;
}

extern "C" int g4_state_free(g4_state* s) {
  if (!s) return G4_E_ARG;
  cudaSetDevice(s->m->ctx->dev.device);
  if (s->st) cudaStreamSynchronize(s->st);
  if (s->graph) cudaGraphExecDestroy(s->graph);
  if (s->small) cudaFree(s->small);
  if (s->h_ctl) cudaFreeHost(s->h_ctl);
  if (s->buf) cudaFree(s->buf);
  if (s->st) cudaStreamDestroy(s->st);
  delete s;
  return 0;
}

// Query heads per attention CTA of the single-sequence decoder: G4_ATTN_HEADS
// (a divisor of the group size; default 1).
static int attn_heads_per_cta(int kv_mul) {
  const char* e = getenv("G4_ATTN_HEADS");
  int h = e ? atoi(e) : 1;
  if (h < 1 || h > kv_mul || kv_mul % h) h = 1;
  return h;
}

// The attention kernel compiled for at least `heads` query heads per CTA.
using AttnFn = void (*)(const AttnArgs);
static AttnFn attn_fn(int heads) {
  return heads <= 1 ? dec_attention_kernel<1> : heads <= 2 ? dec_attention_kernel<2> : heads <= 4 ? dec_attention_kernel<4>
       : heads <= 8 ? dec_attention_kernel<8> : dec_attention_kernel<16>;
}

// Positions per attention chunk that fit kAttnTileBudget (K and V rows), a multiple of 16.
static int attn_ch_max(int hs) { return (int)std::min<size_t>(256, kAttnTileBudget / ((size_t)hs * 8) / 16 * 16); }
// K and V tiles, the group's q rows, the RoPE row, scores and combine weights
// per head, 4 statistics per head and a flag, the mbarrier
static size_t attn_smem(int hs, int group, int ch_max) {
  const size_t ch = (size_t)ch_max, H = (size_t)group;
  return ((2 * ch * hs + H * hs + (size_t)hs + H * ch + H * kAttnMaxChunks + ((4 * H + 2) & ~(size_t)1)) * 4 + 7) /
             8 * 8 + 8;
}

template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl_k(void (*kern)(KArgs...), int grid, int block, size_t smem, cudaStream_t st,
                                Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// A projection's weights as a kernel streams them: the repacked tensor-core
// copy when there is one, else the GGUF blocks.
struct ProjW {
  const g4_tensor* t;
  const uint8_t* packed;
  size_t packed_bytes;
};

static ProjW proj_w(const g4_tensor* t, const uint8_t* packed, const MmaGemvPlan& p) {
  return ProjW{t, packed, packed && p.fast ? mma_packed_bytes(p.rows, p.cols) : 0};
}

static void set_prefetch(GemvFuse& f, std::initializer_list<ProjW> ts) {
  int k = 0;
  for (const ProjW& w : ts)
    if (w.t && k < GemvFuse::kPrefetch) {
      f.pf[k] = w.packed_bytes ? w.packed : (const uint8_t*)w.t->d;
      f.pf_bytes[k] = w.packed_bytes ? (long long)w.packed_bytes : (long long)w.t->nbytes;
      ++k;
    }
}

// Enqueue one decode step on s->st (captured into the graph).
static int enqueue_step(g4_state* s) {
  g4_model* m = s->m;
  g4_ctx* c = m->ctx;
  const g4_model_config& k = m->cfg;
  const int dim = k.dim;
  cudaStream_t st = s->st;
  int cur = 0;
  const int* step = s->ctl;
  const float* branch = nullptr;     // output of the previous residual branch (FFN)
  const float* branch_w = nullptr;   // its post-norm weight
  float branch_scale = 1.f;          // layer output scale of the previous layer
  const float* moe_prev = nullptr;   // previous layer's expert output (MoE merge)
  const float* moe_w = nullptr;
  for (int l = 0; l < k.n_layers; ++l) {
    const LayerDev& L = m->L[l];
    // ---- q | k | v, prologue: previous layer's residual (or embedding) + rmsnorm(attn_norm)
    GemvFuse f;
    f.eps = k.eps;
    f.w_in = L.attn_norm;
    f.x_out = s->x[cur ^ 1];
    if (l == 0) {
      f.in_mode = IN_EMBED_NORM;
      const g4_tensor* emb = m->get("token_embd.weight");
      f.emb = (const uint8_t*)emb->d;
      f.emb_type = emb->type;
      f.sqrt_dim = (float)sqrt((double)dim);
      f.step = step;
      f.in_tok = s->in_tok();
      f.next_tok = s->ctl + 1;
    } else if (moe_prev) {
      f.in_mode = IN_MOE_MERGE;
      f.r = branch;
      f.w_r = branch_w;
      f.m = moe_prev;
      f.w_m = moe_w;
      f.scale = branch_scale;
    } else {
      f.in_mode = IN_RESID_NORM;
      f.r = branch;
      f.w_r = branch_w;
      f.scale = branch_scale;
    }
    // this layer's remaining projections stream into L2 during q|k|v and the attention
    set_prefetch(f, {proj_w(L.wo, L.k_wo, L.m_wo), proj_w(L.gate_up, L.k_gu, L.m_gu), proj_w(L.down, L.k_down, L.m_down)});
    int e = launch_proj(L.m_qkv, L.k_qkv, L.d_qkv, L.p_qkv, L.qkv, s->x[cur], s->qkv, f, c->status, st, l > 0);
    if (e) return c->cuda_fail((cudaError_t)e, "decode: qkv projection");
    cur ^= 1;
    // ---- attention
    AttnArgs aa{};
    aa.qkv = s->qkv;
    aa.hs = L.hs;
    aa.kv_mul = k.n_heads / L.n_kv;
    aa.kvdim = L.kvdim;
    const bool own = l < k.n_layer_kv_from_start;
    aa.k_off = L.qdim;
    aa.v_off = L.has_v ? L.qdim + L.kvdim : L.qdim;
    aa.q_norm = L.q_norm;
    aa.k_norm = L.k_norm;
    aa.eps = k.eps;
    aa.cr = L.swa ? m->cr_swa : m->cr_full;
    aa.ci = L.swa ? m->ci_swa : m->ci_full;
    aa.kc = s->kc[L.kv_src];
    aa.vc = s->vc[L.kv_src];
    aa.write_kv = own ? 1 : 0;
    aa.window = L.swa ? k.sliding_window : 0;
    aa.step = step;
    aa.in_pos = s->in_pos();
    aa.part = s->part;
    aa.tickets = s->tickets;
    aa.out = s->xbk;
    aa.ch_max = attn_ch_max(L.hs);
    aa.status = c->status;
    aa.chunk_stride = kAttnMaxChunks;
    aa.target_chunks = 8;
    aa.heads_per_cta = attn_heads_per_cta(aa.kv_mul);  // one sequence: keep the grid wide
    const size_t asmem = attn_smem(L.hs, aa.heads_per_cta, aa.ch_max);
    // the attribute is a cap shared by every user of the kernel (single and batched decode): the device's limit
    if (asmem > (size_t)c->dev.smem_optin ||
        cudaFuncSetAttribute(attn_fn(aa.heads_per_cta), cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)c->dev.smem_optin))
      return c->cuda_fail(cudaGetLastError(), "decode: attention set-up");
    cudaError_t ce = launch_pdl_k(attn_fn(aa.heads_per_cta), k.n_heads / aa.heads_per_cta * kAttnMaxChunks,
                                  kAttnThreads, asmem, st, aa);
    if (ce) return c->cuda_fail(ce, "decode: attention");
    // ---- output projection of the attention output
    e = launch_proj(L.m_wo, L.k_wo, L.d_wo, L.p_wo, L.wo, s->xbk, s->xb2, GemvFuse{}, c->status, st, true);
    if (e) return c->cuda_fail((cudaError_t)e, "decode: output projection");
    // ---- gate / up, prologue: x += rmsnorm(xb2, post_attention_norm); rmsnorm(x, ffn_norm)
    GemvFuse g;
    g.in_mode = IN_RESID_NORM;
    g.out_mode = OUT_GELU_PAIR;
    g.eps = k.eps;
    g.r = s->xb2;
    g.w_r = L.post_attn_norm;
    g.w_in = L.ffn_norm;
    g.x_out = s->x[cur ^ 1];
    if (l + 1 < k.n_layers) {
      const LayerDev& N = m->L[l + 1];
      set_prefetch(g, {proj_w(N.qkv, N.k_qkv, N.m_qkv)});
    }  // the next layer's first projection
    e = launch_proj(L.m_gu, L.k_gu, L.d_gu, L.p_gu, L.gate_up, s->x[cur], s->hb, g, c->status, st, true);
    if (e) return c->cuda_fail((cudaError_t)e, "decode: gate/up projection");
    cur ^= 1;
    e = launch_proj(L.m_down, L.k_down, L.d_down, L.p_down, L.down, s->hb, s->sh, GemvFuse{}, c->status, st, true);
    if (e) return c->cuda_fail((cudaError_t)e, "decode: down projection");
    branch = s->sh;
    branch_scale = L.scale;
    if (k.n_expert > 0) {
      // expert half on the residual stream after attention (Llama.kt:247-346)
      if (int r = g4_moe_layer(c, &L.moe, s->x[cur], s->moe_out, 1, nullptr, nullptr, st)) return r;
      branch_w = L.post_ffw_norm_1;
      moe_prev = s->moe_out;
      moe_w = L.post_ffw_norm;
    } else {
      branch_w = L.post_ffw_norm;
      moe_prev = nullptr;
    }
  }
  // ---- logits: last residual, rmsnorm(output_norm), projection, softcap, argmax
  GemvFuse f;
  f.in_mode = moe_prev ? IN_MOE_MERGE : IN_RESID_NORM;
  f.out_mode = OUT_SOFTCAP_ARGMAX;
  f.eps = k.eps;
  f.r = branch;
  f.w_r = branch_w;
  f.m = moe_prev;
  f.w_m = moe_w;
  f.scale = branch_scale;
  f.w_in = m->f32("output_norm.weight");
  f.softcap = k.logit_softcap;
  f.argmax = s->argmax;
  set_prefetch(f, {proj_w(m->L[0].qkv, m->L[0].k_qkv, m->L[0].m_qkv)});  // the next step's first projection
  int e = m->m_logits.fast && m->k_cls
              ? launch_gemv_mma(m->m_logits, m->k_cls, s->x[cur], s->logits, f, c->status, st, true)
              : launch_gemv_fused(m->p_logits, (const uint8_t*)m->wcls->d, s->x[cur], s->logits, f, c->status, st,
                                  true);
  if (e) return c->cuda_fail((cudaError_t)e, "decode: logits");
  cudaError_t ce = launch_pdl_k(dec_sample_kernel, 1, 32, 0, st, s->ctl, s->out_tok(), s->argmax);
  if (ce) return c->cuda_fail(ce, "decode: sampling");
  return 0;
}

static int build_graph(g4_state* s) {
  g4_ctx* c = s->m->ctx;
  if (s->graph) return 0;
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal);
  if (e) return c->cuda_fail(e, "decode: begin capture");
  const int r = enqueue_step(s);
  e = cudaStreamEndCapture(s->st, &g);
  if (r) {
    if (g) cudaGraphDestroy(g);
    cudaGetLastError();
    return r;
  }
  if (e) return c->cuda_fail(e, "decode: end capture");
  e = cudaGraphInstantiate(&s->graph, g, 0);
  cudaGraphDestroy(g);
  if (e) {
    s->graph = nullptr;
    return c->cuda_fail(e, "decode: graph instantiation");
  }
  return 0;
}

// Stage steps [0, n) (input token or -1, position, in h_ctl) and reset the step counter.
static int stage_steps(g4_state* s, int n) {
  g4_ctx* c = s->m->ctx;
  const int ctx = s->m->cfg.ctx_len;
  s->h_ctl[0] = 0;
  s->h_ctl[1] = 0;
  cudaError_t e = cudaMemcpyAsync(s->ctl, s->h_ctl, 8, cudaMemcpyHostToDevice, s->st);
  if (!e) e = cudaMemcpyAsync(s->in_tok(), s->h_ctl + 4, (size_t)n * 4, cudaMemcpyHostToDevice, s->st);
  if (!e) e = cudaMemcpyAsync(s->in_pos(), s->h_ctl + 4 + ctx, (size_t)n * 4, cudaMemcpyHostToDevice, s->st);
  return e ? c->cuda_fail(e, "decode: staging") : 0;
}

extern "C" {

int g4_decode_step(g4_state* s, int token, int position, float* logits_host, int* next_token_host) {
  if (!s) return G4_E_ARG;
  g4_model* m = s->m;
  g4_ctx* c = m->ctx;
  if (token < 0 || token >= m->cfg.vocab || position < 0 || position >= m->cfg.ctx_len) {
    c->set_err("g4_decode_step: token %d / position %d out of range (vocab %d, context %d)", token, position,
               m->cfg.vocab, m->cfg.ctx_len);
    return G4_E_ARG;
  }
  if (int r = c->bind()) return r;
  if (int r = build_graph(s)) return r;
  if (cudaError_t e = cudaStreamSynchronize(s->st)) return c->cuda_fail(e, "g4_decode_step");
  s->h_ctl[4] = token;
  s->h_ctl[4 + m->cfg.ctx_len] = position;
  if (int r = stage_steps(s, 1)) return r;
  cudaError_t e = cudaGraphLaunch(s->graph, s->st);
  if (e) return c->cuda_fail(e, "g4_decode_step: graph launch");
  if (logits_host) e = cudaMemcpyAsync(logits_host, s->logits, (size_t)m->cfg.vocab * 4, cudaMemcpyDeviceToHost, s->st);
  if (!e && next_token_host) e = cudaMemcpyAsync(next_token_host, s->out_tok(), 4, cudaMemcpyDeviceToHost, s->st);
  if (e) return c->cuda_fail(e, "g4_decode_step: read back");
  return c->check_status(s->st);
}

int g4_decode_greedy(g4_state* s, const int* tokens, int n_tokens, int start_position, int n_generate,
                     int* out_tokens) {
  if (!s) return G4_E_ARG;
  g4_model* m = s->m;
  g4_ctx* c = m->ctx;
  const int ctx = m->cfg.ctx_len;
  if (!tokens || n_tokens < 1 || n_generate < 0 || (n_generate > 0 && !out_tokens) || start_position < 0 ||
      (long long)start_position + n_tokens + std::max(n_generate, 1) - 1 > ctx) {
    c->set_err("g4_decode_greedy: bad arguments (%d tokens from position %d, %d to generate, context %d)", n_tokens,
               start_position, n_generate, ctx);
    return G4_E_ARG;
  }
  for (int i = 0; i < n_tokens; ++i)
    if (tokens[i] < 0 || tokens[i] >= m->cfg.vocab) {
      c->set_err("g4_decode_greedy: token %d out of range", tokens[i]);
      return G4_E_ARG;
    }
  if (int r = c->bind()) return r;
  if (int r = build_graph(s)) return r;
  if (cudaError_t e = cudaStreamSynchronize(s->st)) return c->cuda_fail(e, "g4_decode_greedy");
  const int steps = n_tokens + std::max(n_generate, 1) - 1;
  for (int i = 0; i < steps; ++i) {
    s->h_ctl[4 + i] = i < n_tokens ? tokens[i] : -1;
    s->h_ctl[4 + ctx + i] = start_position + i;
  }
  if (int r = stage_steps(s, steps)) return r;
  for (int i = 0; i < steps; ++i)
    if (cudaError_t e = cudaGraphLaunch(s->graph, s->st)) return c->cuda_fail(e, "g4_decode_greedy: graph launch");
  if (n_generate > 0) {
    cudaError_t e = cudaMemcpyAsync(out_tokens, s->out_tok() + (n_tokens - 1), (size_t)n_generate * 4,
                                    cudaMemcpyDeviceToHost, s->st);
    if (e) return c->cuda_fail(e, "g4_decode_greedy: read back");
  }
  return c->check_status(s->st);
}

int g4_decode_stage(g4_state* s, const int* tokens, const int* positions, int n_steps) {
  if (!s) return G4_E_ARG;
  g4_ctx* c = s->m->ctx;
  const int ctx = s->m->cfg.ctx_len;
  if (!tokens || !positions || n_steps < 1 || n_steps > ctx) {
    c->set_err("g4_decode_stage: bad arguments (%d steps, context %d)", n_steps, ctx);
    return G4_E_ARG;
  }
  if (int r = c->bind()) return r;
  if (cudaError_t e = cudaStreamSynchronize(s->st)) return c->cuda_fail(e, "g4_decode_stage");
  for (int i = 0; i < n_steps; ++i) {
    if (positions[i] < 0 || positions[i] >= ctx || tokens[i] >= s->m->cfg.vocab || (i == 0 && tokens[i] < 0)) {
      c->set_err("g4_decode_stage: step %d: token %d / position %d out of range", i, tokens[i], positions[i]);
      return G4_E_ARG;
    }
    s->h_ctl[4 + i] = tokens[i];
    s->h_ctl[4 + ctx + i] = positions[i];
  }
  return stage_steps(s, n_steps);
}

int g4_decode_enqueue(g4_state* s, int n_steps) {
  if (!s || n_steps < 0) return G4_E_ARG;
  g4_ctx* c = s->m->ctx;
  if (int r = c->bind()) return r;
  if (int r = build_graph(s)) return r;
  for (int i = 0; i < n_steps; ++i)
    if (cudaError_t e = cudaGraphLaunch(s->graph, s->st)) return c->cuda_fail(e, "g4_decode_enqueue");
  return 0;
}

int g4_decode_read_tokens(g4_state* s, int first_step, int n, int* out) {
  if (!s) return G4_E_ARG;
  g4_ctx* c = s->m->ctx;
  if (!out || first_step < 0 || n < 0 || first_step + n > s->m->cfg.ctx_len) {
    c->set_err("g4_decode_read_tokens: bad arguments");
    return G4_E_ARG;
  }
  cudaError_t e = cudaMemcpyAsync(out, s->out_tok() + first_step, (size_t)n * 4, cudaMemcpyDeviceToHost, s->st);
  if (e) return c->cuda_fail(e, "g4_decode_read_tokens");
  return c->check_status(s->st);
}

void* g4_state_stream(g4_state* s) { return s ? (void*)s->st : nullptr; }

}  // extern "C"

// ---------------------------------------------------------------- batched decode
// Many sequences advanced one position each per call (
// 64 concurrent sequences).  The reference runs one LlamaState per sequence
// (Llama.kt:105-408 per token); here the n sequences of a step share each
// weight read: per layer a per-token prologue kernel, the T-token int8 mma GEMM
// on the repacked Q8_0 tiles, the attention kernel with a sequence grid axis,
// and g4_moe_layer on the n tokens.  Sequence i owns KV-cache slot i.

struct g4_batch {
  g4_model* m = nullptr;
  int n_max = 0, max_pos = 0;
  cudaStream_t st = nullptr;
  float* buf = nullptr;  // activations, attention partials, KV caches
  float *x[2] = {nullptr, nullptr}, *qkv = nullptr, *xbk = nullptr, *xb2 = nullptr, *hb = nullptr, *sh = nullptr;
  float *moe_out = nullptr, *logits = nullptr, *part = nullptr;
  std::vector<float*> kc, vc;   // per KV-owning layer: [n_max][max_pos][kvdim]
  size_t part_stride = 0;       // floats of one sequence's attention partials
  uint8_t* small = nullptr;     // limbs, scales, keys, tokens, positions, tickets
  int8_t* lim = nullptr;
  float* lsc = nullptr;
  unsigned long long* keys = nullptr;
  int *d_tok = nullptr, *d_pos = nullptr, *d_slot = nullptr;
  unsigned* tickets = nullptr;
  float* gemm_part = nullptr;   // split-K partial sums of the batched GEMMs
  unsigned* gemm_tickets = nullptr;
  int* h_io = nullptr;          // pinned: tokens [n_max], positions [n_max], slots [n_max]
  unsigned long long* h_keys = nullptr;  // pinned [n_max]
  std::map<std::tuple<int, int, int>, MmaBatchPlan> plans;
  // expert parallelism (g4_batch_expert_parallel): per layer, this rank's experts
  // as views into the model's expert tensors
  bool ep = false;
  std::vector<g4_tensor> ep_views;  // [layer][gate_up, down]
  std::vector<g4_moe_weights> ep_moe;

  const MmaBatchPlan* plan(int rows, int cols, int T) {
    const int ng = T <= 8 ? 1 : T <= 16 ? 2 : T <= 32 ? 4 : 8;
    auto key = std::make_tuple(rows, cols, ng);
    auto it = plans.find(key);
    if (it == plans.end()) it = plans.emplace(key, plan_gemm_mma_batch(m->ctx->dev, rows, cols, 8 * ng)).first;
    return it->second.fast ? &it->second : nullptr;
  }
};

extern "C" int g4_batch_free(g4_batch* b);

// Batched attention: chunks of at most 32 positions, so that a few CTAs (their
// K/V tiles) are resident per SM while the sequences fill the grid.
static int batch_ch_max(int hs) { return std::min(32, attn_ch_max(hs)); }


// The Q8_0 projections of every layer and the output matrix in the tile layout
// of the tensor-core GEMMs (kept by the model; the single-sequence decoder uses
// the layer copies only when it planned them itself).
static int batch_repack(g4_model* m) {
  g4_ctx* c = m->ctx;
  auto pack = [&](const g4_tensor* w, int rows, int cols, uint8_t*& packed) -> int {
    if (packed) return 0;
    if (!w || w->type != G4_TYPE_Q8_0 || w->n_elems != (uint64_t)rows * (uint64_t)cols || cols % 32) {
      c->set_err("g4_batch_create: batched decode needs every projection and the output matrix in Q8_0");
      return G4_E_TYPE;
    }
    const size_t bytes = mma_packed_bytes(rows, cols);
    if (cudaMalloc(&packed, bytes) != cudaSuccess) {
      cudaGetLastError();
      packed = nullptr;
      c->set_err("g4_batch_create: cannot allocate %zu bytes of repacked weights", bytes);
      return G4_E_NOMEM;
    }
    cudaError_t e = (cudaError_t)repack_q8_0_mma((const uint8_t*)w->d, rows, cols, packed, nullptr);
    if (!e) e = cudaStreamSynchronize(nullptr);
    return e ? c->cuda_fail(e, "g4_batch_create: repack") : 0;
  };
  const int dim = m->cfg.dim;
  for (LayerDev& L : m->L) {
    const int qkv_rows = (int)(L.qkv->n_elems / dim);
    if (int r = pack(L.qkv, qkv_rows, dim, L.k_qkv)) return r;
    if (int r = pack(L.wo, dim, L.qdim, L.k_wo)) return r;
    if (int r = pack(L.gate_up, 2 * L.ff, dim, L.k_gu)) return r;
    if (int r = pack(L.down, dim, L.ff, L.k_down)) return r;
  }
  return pack(m->wcls, m->cfg.vocab, dim, m->k_cls);
}

extern "C" int g4_batch_create(g4_model* m, int n_max, int max_positions, g4_batch** out) {
  if (!m) return G4_E_ARG;
  g4_ctx* c = m->ctx;
  const g4_model_config& k = m->cfg;
  if (!out || !m->finalized || n_max < 1 || n_max > kBatchMaxT || max_positions < 1 || max_positions > k.ctx_len) {
    c->set_err("g4_batch_create: bad arguments (finalized model, 1..%d sequences, 1..%d positions)", kBatchMaxT,
               k.ctx_len);
    return G4_E_ARG;
  }
  if (int r = c->bind()) return r;
  if (int r = batch_repack(m)) return r;
  g4_batch* b = new (std::nothrow) g4_batch();
  if (!b) return G4_E_NOMEM;
  b->m = m;
  b->n_max = n_max;
  b->max_pos = max_positions;
  auto al = [](size_t n) { return (n + 63) / 64 * 64; };  // floats, 256-byte multiples
  const size_t N = n_max, dim = k.dim;
  const size_t qkv_w = m->max_q + 2 * m->max_kv;
  b->part_stride = al((size_t)k.n_heads * kAttnMaxChunks * (m->max_hs + 2));
  size_t off = 0;
  const size_t o_x0 = off; off += al(N * dim);
  const size_t o_x1 = off; off += al(N * dim);
  const size_t o_qkv = off; off += al(N * qkv_w);
  const size_t o_xbk = off; off += al(N * m->max_q);
  const size_t o_xb2 = off; off += al(N * dim);
  const size_t o_hb = off; off += al(N * m->max_ff);
  const size_t o_sh = off; off += al(N * dim);
  const size_t o_moe = off; off += al(N * dim);
  const size_t o_log = off; off += al(N * k.vocab);
  const size_t o_part = off; off += N * b->part_stride;
  std::vector<size_t> o_kc, o_vc;
  for (int l = 0; l < k.n_layer_kv_from_start; ++l) {
    const int hs = m->is_swa[l] ? k.head_size_swa : k.head_size_full;
    const size_t n = al(N * max_positions * m->n_kv[l] * hs);
    o_kc.push_back(off);
    off += n;
    o_vc.push_back(off);
    off += n;
  }
  const size_t widest = std::max<size_t>(dim, std::max<size_t>(m->max_q, m->max_ff));
  const size_t lim_bytes = (N * (widest / 32) * 96 + 255) / 256 * 256;
  const size_t lsc_bytes = (N * (widest / 32) * 4 + 255) / 256 * 256;
  const size_t small = lim_bytes + lsc_bytes + 256 + 4 * ((N * 8 + 255) / 256 * 256) + N * k.n_heads * 4;
  if (cudaMalloc(&b->buf, off * 4) != cudaSuccess || cudaMalloc(&b->small, small) != cudaSuccess ||
      cudaMallocHost(&b->h_io, N * 12) != cudaSuccess || cudaMallocHost(&b->h_keys, N * 8) != cudaSuccess ||
      cudaStreamCreateWithFlags(&b->st, cudaStreamNonBlocking) != cudaSuccess) {
    cudaGetLastError();
    g4_batch_free(b);
    c->set_err("g4_batch_create: cannot allocate %zu bytes of activations and KV cache", off * 4);
    return G4_E_NOMEM;
  }
  cudaMemset(b->buf, 0, off * 4);
  cudaMemset(b->small, 0, small);
  b->x[0] = b->buf + o_x0;
  b->x[1] = b->buf + o_x1;
  b->qkv = b->buf + o_qkv;
  b->xbk = b->buf + o_xbk;
  b->xb2 = b->buf + o_xb2;
  b->hb = b->buf + o_hb;
  b->sh = b->buf + o_sh;
  b->moe_out = b->buf + o_moe;
  b->logits = b->buf + o_log;
  b->part = b->buf + o_part;
  for (int l = 0; l < k.n_layer_kv_from_start; ++l) {
    b->kc.push_back(b->buf + o_kc[l]);
    b->vc.push_back(b->buf + o_vc[l]);
  }
  uint8_t* p = b->small;
  b->lim = reinterpret_cast<int8_t*>(p);
  p += lim_bytes;
  b->lsc = reinterpret_cast<float*>(p);
  p += lsc_bytes + 256;
  b->keys = reinterpret_cast<unsigned long long*>(p);
  p += (N * 8 + 255) / 256 * 256;
  b->d_tok = reinterpret_cast<int*>(p);
  p += (N * 8 + 255) / 256 * 256;
  b->d_pos = reinterpret_cast<int*>(p);
  p += (N * 8 + 255) / 256 * 256;
  b->d_slot = reinterpret_cast<int*>(p);
  p += (N * 8 + 255) / 256 * 256;
  b->tickets = reinterpret_cast<unsigned*>(p);
  // split-K scratch of the batched GEMMs (plans at the widest batch)
  size_t part_floats = 0;
  int max_nrb = 0;
  auto need = [&](int rows, int cols) -> bool {
    const MmaBatchPlan* p = b->plan(rows, cols, n_max);
    if (!p) return false;
    part_floats = std::max(part_floats, mma_batch_partials(*p, n_max));
    max_nrb = std::max(max_nrb, p->nrb);
    return true;
  };
  bool ok = need(k.vocab, (int)dim);
  for (const LayerDev& L : m->L)
    ok = ok && need((int)(L.qkv->n_elems / dim), (int)dim) && need((int)dim, L.qdim) && need(2 * L.ff, (int)dim) &&
         need((int)dim, L.ff);
  if (!ok) {
    g4_batch_free(b);
    c->set_err("g4_batch_create: no batched GEMM plan for the model's projections");
    return G4_E_DEVICE;
  }
  if (cudaMalloc(&b->gemm_part, part_floats * 4 + (size_t)max_nrb * 4 + 256) != cudaSuccess) {
    cudaGetLastError();
    g4_batch_free(b);
    c->set_err("g4_batch_create: cannot allocate the GEMM partial sums");
    return G4_E_NOMEM;
  }
  b->gemm_tickets = reinterpret_cast<unsigned*>(b->gemm_part + (part_floats + 63) / 64 * 64);
  cudaMemset(b->gemm_tickets, 0, (size_t)max_nrb * 4);
  // attention kernel set-up, and the MoE layers' work buffers at the widest batch
  for (const LayerDev& L : m->L) {
    const int grp = k.n_heads / L.n_kv;
    if (attn_smem(L.hs, grp, batch_ch_max(L.hs)) > (size_t)c->dev.smem_optin ||
        cudaFuncSetAttribute(attn_fn(grp), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c->dev.smem_optin)) {
      g4_batch_free(b);
      return c->cuda_fail(cudaGetLastError(), "g4_batch_create: attention set-up");
    }
  }
  if (k.n_expert > 0) {
    int r = g4_moe_layer(c, &m->L[0].moe, b->x[0], b->moe_out, n_max, nullptr, nullptr, b->st);
    if (!r) r = c->check_status(b->st);
    if (r) {
      g4_batch_free(b);
      return r;
    }
  }
  if (cudaError_t e = cudaStreamSynchronize(b->st)) {
    g4_batch_free(b);
    return c->cuda_fail(e, "g4_batch_create");
  }
  *out = b;
  return 0;
}

extern "C" int g4_batch_free(g4_batch* b) {
  if (!b) return G4_E_ARG;
  cudaSetDevice(b->m->ctx->dev.device);
  if (b->st) cudaStreamSynchronize(b->st);
  if (b->buf) cudaFree(b->buf);
  if (b->small) cudaFree(b->small);
  if (b->gemm_part) cudaFree(b->gemm_part);
  if (b->h_io) cudaFreeHost(b->h_io);
  if (b->h_keys) cudaFreeHost(b->h_keys);
  if (b->st) cudaStreamDestroy(b->st);
  delete b;
  return 0;
}

// One projection of the batch: activation limbs already in b->lim / b->lsc.
static int batch_gemm(g4_batch* b, const uint8_t* packed, int rows, int cols, int n, float* y, int ldy, int out_mode,
                      float softcap, unsigned long long* keys, const char* what) {
  g4_ctx* c = b->m->ctx;
  const MmaBatchPlan* p = b->plan(rows, cols, n);
  if (!p) {
    c->set_err("g4_batch_step: no GEMM plan for %s (%d x %d)", what, rows, cols);
    return G4_E_DEVICE;
  }
  const int e = launch_gemm_mma_batch(*p, packed, b->lim, b->lsc, n, y, ldy, out_mode, softcap, keys, b->gemm_part,
                                      b->gemm_tickets, b->st);
  return e ? c->cuda_fail((cudaError_t)e, what) : 0;
}

static int batch_prologue(g4_batch* b, const GemvFuse& f, const float* x, int dim, int n, const char* what) {
  const int e = launch_batch_prologue(f, x, dim, n, b->lim, b->lsc, b->st);
  return e ? b->m->ctx->cuda_fail((cudaError_t)e, what) : 0;
}

extern "C" int g4_batch_step(g4_batch* b, const int* tokens, const int* positions, const int* slots, int n,
                             float* logits_host, int* next_tokens_host) {
  if (!b) return G4_E_ARG;
  g4_model* m = b->m;
  g4_ctx* c = m->ctx;
  const g4_model_config& k = m->cfg;
  if (!tokens || !positions || n < 1 || n > b->n_max) {
    c->set_err("g4_batch_step: bad arguments (%d sequences, at most %d)", n, b->n_max);
    return G4_E_ARG;
  }
  for (int i = 0; i < n; ++i) {
    const int sl = slots ? slots[i] : i;
    if (tokens[i] < 0 || tokens[i] >= k.vocab || positions[i] < 0 || positions[i] >= b->max_pos || sl < 0 ||
        sl >= b->n_max) {
      c->set_err("g4_batch_step: row %d: token %d / position %d / slot %d out of range (vocab %d, %d positions, "
                 "%d slots)", i, tokens[i], positions[i], sl, k.vocab, b->max_pos, b->n_max);
      return G4_E_ARG;
    }
    if (slots)
      for (int j = 0; j < i; ++j)
        if (slots[j] == sl && positions[j] == positions[i]) {
          c->set_err("g4_batch_step: rows %d and %d both write position %d of slot %d", j, i, positions[i], sl);
          return G4_E_ARG;
        }
  }
  if (int r = c->bind()) return r;
  cudaStream_t st = b->st;
  if (cudaError_t e = cudaStreamSynchronize(st)) return c->cuda_fail(e, "g4_batch_step");
  std::memcpy(b->h_io, tokens, (size_t)n * 4);
  std::memcpy(b->h_io + b->n_max, positions, (size_t)n * 4);
  for (int i = 0; i < n; ++i) b->h_io[2 * b->n_max + i] = slots ? slots[i] : i;
  cudaError_t ce = cudaMemcpyAsync(b->d_tok, b->h_io, (size_t)n * 4, cudaMemcpyHostToDevice, st);
  if (!ce) ce = cudaMemcpyAsync(b->d_pos, b->h_io + b->n_max, (size_t)n * 4, cudaMemcpyHostToDevice, st);
  if (!ce) ce = cudaMemcpyAsync(b->d_slot, b->h_io + 2 * b->n_max, (size_t)n * 4, cudaMemcpyHostToDevice, st);
  if (ce) return c->cuda_fail(ce, "g4_batch_step: staging");
  const int dim = k.dim;
  int cur = 0;
  const float* branch = nullptr;
  const float* branch_w = nullptr;
  float branch_scale = 1.f;
  const float* moe_prev = nullptr;
  const float* moe_w = nullptr;
  for (int l = 0; l < k.n_layers; ++l) {
    const LayerDev& L = m->L[l];
    const int qkv_n = (int)(L.qkv->n_elems / dim);  // rows of q | k | v (no v rows without attn_v)
    // ---- q | k | v, prologue as the single-sequence decoder's (enqueue_step)
    GemvFuse f;
    f.eps = k.eps;
    f.w_in = L.attn_norm;
    f.x_out = b->x[cur ^ 1];
    if (l == 0) {
      f.in_mode = IN_EMBED_NORM;
      const g4_tensor* emb = m->get("token_embd.weight");
      f.emb = (const uint8_t*)emb->d;
      f.emb_type = emb->type;
      f.sqrt_dim = (float)sqrt((double)dim);
      f.in_tok = b->d_tok;
    } else if (moe_prev) {
      f.in_mode = IN_MOE_MERGE;
      f.r = branch;
      f.w_r = branch_w;
      f.m = moe_prev;
      f.w_m = moe_w;
      f.scale = branch_scale;
    } else {
      f.in_mode = IN_RESID_NORM;
      f.r = branch;
      f.w_r = branch_w;
      f.scale = branch_scale;
    }
    if (int r = batch_prologue(b, f, l == 0 ? nullptr : b->x[cur], dim, n, "batch: qkv prologue")) return r;
    if (int r = batch_gemm(b, L.k_qkv, qkv_n, dim, n, b->qkv, qkv_n, OUT_PLAIN, 0.f, nullptr, "batch: qkv")) return r;
    cur ^= 1;
    // ---- attention, one grid row per sequence
    AttnArgs aa{};
    aa.qkv = b->qkv;
    aa.hs = L.hs;
    aa.kv_mul = k.n_heads / L.n_kv;
    aa.kvdim = L.kvdim;
    const bool own = l < k.n_layer_kv_from_start;
    aa.k_off = L.qdim;
    aa.v_off = L.has_v ? L.qdim + L.kvdim : L.qdim;
    aa.q_norm = L.q_norm;
    aa.k_norm = L.k_norm;
    aa.eps = k.eps;
    aa.cr = L.swa ? m->cr_swa : m->cr_full;
    aa.ci = L.swa ? m->ci_swa : m->ci_full;
    aa.kc = b->kc[L.kv_src];
    aa.vc = b->vc[L.kv_src];
    aa.write_kv = 0;  // the step's K/V rows are written first, by batch_kv_write_kernel
    aa.window = L.swa ? k.sliding_window : 0;
    aa.part = b->part;
    aa.tickets = b->tickets;
    aa.out = b->xbk;
    aa.ch_max = batch_ch_max(L.hs);
    aa.status = c->status;
    aa.pos_arr = b->d_pos;
    aa.slot_arr = b->d_slot;
    aa.qkv_stride = qkv_n;
    aa.kv_stride = (long long)b->max_pos * L.kvdim;
    aa.part_stride = (long long)b->part_stride;
    aa.out_stride = L.qdim;
    aa.tick_stride = k.n_heads;
    aa.target_chunks = 8;  // the sequences give the grid its width
    aa.heads_per_cta = aa.kv_mul;  // K/V rows staged once for the whole group
    int nch_max = 1;
    for (int i = 0; i < n; ++i) {
      const int pos = positions[i];
      const int start = aa.window > 0 ? std::max(0, pos - aa.window + 1) : 0;
      const int len = pos - start + 1;
      const int ch = attn_chunk(len, aa.ch_max, aa.target_chunks);
      nch_max = std::max(nch_max, (len + ch - 1) / ch);
    }
    aa.chunk_stride = nch_max;
    if (own) {
      batch_kv_write_kernel<<<dim3(L.n_kv, n), 64, (size_t)2 * L.hs * 4, st>>>(aa);
      if (cudaError_t e = cudaGetLastError()) return c->cuda_fail(e, "batch: K/V rows");
    }
    attn_fn(aa.kv_mul)<<<dim3(L.n_kv * nch_max, n), kAttnThreads, attn_smem(L.hs, aa.kv_mul, aa.ch_max), st>>>(aa);
    if (cudaError_t e = cudaGetLastError()) return c->cuda_fail(e, "batch: attention");
    // ---- output projection
    GemvFuse plain;
    if (int r = batch_prologue(b, plain, b->xbk, L.qdim, n, "batch: o prologue")) return r;
    if (int r = batch_gemm(b, L.k_wo, dim, L.qdim, n, b->xb2, dim, OUT_PLAIN, 0.f, nullptr, "batch: o")) return r;
    // ---- gate / up: x += rmsnorm(xb2, post_attention_norm); rmsnorm(x, ffn_norm); gelu(gate) * up
    GemvFuse g;
    g.in_mode = IN_RESID_NORM;
    g.eps = k.eps;
    g.r = b->xb2;
    g.w_r = L.post_attn_norm;
    g.w_in = L.ffn_norm;
    g.x_out = b->x[cur ^ 1];
    if (int r = batch_prologue(b, g, b->x[cur], dim, n, "batch: gate/up prologue")) return r;
    if (int r = batch_gemm(b, L.k_gu, 2 * L.ff, dim, n, b->hb, L.ff, OUT_GELU_PAIR, 0.f, nullptr, "batch: gate/up"))
      return r;
    cur ^= 1;
    if (int r = batch_prologue(b, plain, b->hb, L.ff, n, "batch: down prologue")) return r;
    if (int r = batch_gemm(b, L.k_down, dim, L.ff, n, b->sh, dim, OUT_PLAIN, 0.f, nullptr, "batch: down")) return r;
    branch = b->sh;
    branch_scale = L.scale;
    if (k.n_expert > 0) {
      const int r = b->ep ? g4_moe_layer_ep(c, &b->ep_moe[l], b->x[cur], b->moe_out, n, nullptr, nullptr, st)
                          : g4_moe_layer(c, &L.moe, b->x[cur], b->moe_out, n, nullptr, nullptr, st);
      if (r) return r;
      branch_w = L.post_ffw_norm_1;
      moe_prev = b->moe_out;
      moe_w = L.post_ffw_norm;
    } else {
      branch_w = L.post_ffw_norm;
      moe_prev = nullptr;
    }
  }
  // ---- logits: last residual, rmsnorm(output_norm), projection, softcap, arg-max per sequence
  GemvFuse f;
  f.in_mode = moe_prev ? IN_MOE_MERGE : IN_RESID_NORM;
  f.eps = k.eps;
  f.r = branch;
  f.w_r = branch_w;
  f.m = moe_prev;
  f.w_m = moe_w;
  f.scale = branch_scale;
  f.w_in = m->f32("output_norm.weight");
  if (int r = batch_prologue(b, f, b->x[cur], dim, n, "batch: logits prologue")) return r;
  if (cudaError_t e = cudaMemsetAsync(b->keys, 0, (size_t)n * 8, st)) return c->cuda_fail(e, "batch: keys");
  if (int r = batch_gemm(b, m->k_cls, k.vocab, dim, n, b->logits, k.vocab, OUT_SOFTCAP_ARGMAX, k.logit_softcap,
                         b->keys, "batch: logits"))
    return r;
  ce = cudaMemcpyAsync(b->h_keys, b->keys, (size_t)n * 8, cudaMemcpyDeviceToHost, st);
  if (!ce && logits_host)
    ce = cudaMemcpyAsync(logits_host, b->logits, (size_t)n * k.vocab * 4, cudaMemcpyDeviceToHost, st);
  if (ce) return c->cuda_fail(ce, "g4_batch_step: read back");
  if (int r = c->check_status(st)) return r;  // synchronises the stream
  if (next_tokens_host)
    for (int i = 0; i < n; ++i) next_tokens_host[i] = (int)(0xFFFFFFFFu - (uint32_t)(b->h_keys[i] & 0xFFFFFFFFull));
  return 0;
}

extern "C" void* g4_batch_stream(g4_batch* b) { return b ? (void*)b->st : nullptr; }

// Expert parallelism for a batch: rank r of the context's communicator
// (g4_dist_init) computes experts [r*E/W, (r+1)*E/W) of every MoE layer for
// all ranks' tokens, through g4_moe_layer_ep; attention and the dense layers
// stay with the rank's own sequences (data parallel).  The expert tensors are
// not re-uploaded: each layer's local experts are a view into the model's
// tensors.  From this call on every rank must run g4_batch_step together.
extern "C" int g4_batch_expert_parallel(g4_batch* b) {
  if (!b) return G4_E_ARG;
  g4_model* m = b->m;
  g4_ctx* c = m->ctx;
  const g4_model_config& k = m->cfg;
  if (c->world < 2 || !c->comm) {
    c->set_err("g4_batch_expert_parallel: needs g4_dist_init with two or more ranks");
    return G4_E_ARG;
  }
  if (k.n_expert <= 0 || k.n_expert % c->world) {
    c->set_err("g4_batch_expert_parallel: %d experts do not split over %d ranks", k.n_expert, c->world);
    return G4_E_ARG;
  }
  const int El = k.n_expert / c->world;
  b->ep_views.assign(2 * (size_t)k.n_layers, g4_tensor{});
  b->ep_moe.assign(k.n_layers, g4_moe_weights{});
  for (int l = 0; l < k.n_layers; ++l) {
    const LayerDev& L = m->L[l];
    g4_moe_weights w = L.moe;
    const g4_tensor* full[2] = {L.moe.gate_up_exps, L.moe.down_exps};
    for (int i = 0; i < 2; ++i) {
      const g4_tensor* t = full[i];
      const uint64_t per = t->n_elems / (uint64_t)k.n_expert;  // elements of one expert
      const int bs = block_size(t->type), ts = type_size(t->type);
      if (t->n_elems % (uint64_t)k.n_expert || bs <= 0 || per % (uint64_t)bs) {
        c->set_err("g4_batch_expert_parallel: layer %d: experts are not whole blocks", l);
        return G4_E_TYPE;
      }
      const uint64_t bytes = per / (uint64_t)bs * (uint64_t)ts;
      g4_tensor& v = b->ep_views[2 * (size_t)l + i];
      v.ctx = c;
      v.type = t->type;
      v.d = static_cast<uint8_t*>(t->d) + (size_t)c->rank * El * bytes;
      v.nbytes = (uint64_t)El * bytes;
      v.n_elems = (uint64_t)El * per;
    }
    w.gate_up_exps = &b->ep_views[2 * (size_t)l];
    w.down_exps = &b->ep_views[2 * (size_t)l + 1];
    b->ep_moe[l] = w;
  }
  b->ep = true;
  return 0;
}
