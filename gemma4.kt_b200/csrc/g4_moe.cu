// g4_moe.cu -- the expert half of gemma4.kt's MoE block (Llama.kt:247-346)
// for a batch of tokens, as a short chain of sm_100a kernels:
//
//   moe_prep        moeInput = rmsnorm(x, pre_ffw_norm_2)            Llama.kt:248-254
//                   router input x * rms/sqrt(dim) * gate_inp_scale   Llama.kt:257-268
//   moe_router      logits = gate_inp . router input (F32)            Llama.kt:269-270
//   moe_topk        softmax (double exp) + iterative top-k            Llama.kt:273-293
//   moe_permute     per-expert counts, offsets, slot permutation      (implicit ki loop :300)
//   moe_expert<GU>  grouped gate_up GEMV, epilogue gelu(gate)*up      Llama.kt:305-322
//   moe_expert<DN>  grouped down GEMV                                  Llama.kt:325-332
//   moe_combine     out = sum_k (prob_k*down_scale[e_k]) * down_k in k
//                   order, then rmsnorm(post_ffw_norm_2)              Llama.kt:334-346
//
// A "slot" is one (token, k) selection: slot = token * n_used + k.  The expert
// kernels stream each selected expert's weights once per token chunk with
// cp.async.bulk into a shared-memory ring (as the GEMV does) and read the
// chunk's activations through L1.  Every result is written to a fixed place,
// so the combine is deterministic and in the reference's order.
#include "g4.h"
#include "g4_ctx.h"
#include "g4_gemv.cuh"
#include "g4_gemv_rows.cuh"
#include "g4_moe_tc.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <map>
#include <mutex>
#include <vector>

namespace g4 {

constexpr int kMaxExperts = 256;
constexpr int kMaxUsed = 16;

// ---------------------------------------------------------------- helpers

// ---------------------------------------------------------------- prep

__global__ void __launch_bounds__(512) moe_prep_kernel(const float* __restrict__ x, const float* __restrict__ pre_norm,
                                                       const float* __restrict__ gate_scale, float* __restrict__ moe_in,
                                                       float* __restrict__ xr, float* __restrict__ moe_in_s16, int dim,
                                                       float eps) {
  __shared__ float red[33];
  const float4* xt = reinterpret_cast<const float4*>(x + (size_t)blockIdx.x * dim);
  const int n4 = dim >> 2;
  float ss = 0.f;
  for (int i = threadIdx.x; i < n4; i += blockDim.x) {
    float4 v = xt[i];
    ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
  }
  ss = block_sum(ss, red);
  // rmsnorm (Llama.kt:27-37): ss/size + eps, 1/sqrt in double
  float m = __fadd_rn(__fdiv_rn(ss, (float)dim), eps);
  float s_norm = (float)(1.0 / sqrt((double)m));
  // router scale (Llama.kt:258-261): (float)(1/sqrt(ss)) / (float)sqrt(dim)
  float s_router = __fdiv_rn(s_norm, (float)sqrt((double)dim));
  float4* mo = reinterpret_cast<float4*>(moe_in + (size_t)blockIdx.x * dim);
  float4* xo = reinterpret_cast<float4*>(xr + (size_t)blockIdx.x * dim);
  const float4* pn = reinterpret_cast<const float4*>(pre_norm);
  const float4* gs = reinterpret_cast<const float4*>(gate_scale);
  for (int i = threadIdx.x; i < n4; i += blockDim.x) {
    const float4 v = xt[i], w = pn[i], g = gs[i];
    mo[i] = make_float4(__fmul_rn(w.x, __fmul_rn(s_norm, v.x)), __fmul_rn(w.y, __fmul_rn(s_norm, v.y)),
                        __fmul_rn(w.z, __fmul_rn(s_norm, v.z)), __fmul_rn(w.w, __fmul_rn(s_norm, v.w)));
    xo[i] = make_float4(__fmul_rn(__fmul_rn(v.x, s_router), g.x), __fmul_rn(__fmul_rn(v.y, s_router), g.y),
                        __fmul_rn(__fmul_rn(v.z, s_router), g.z), __fmul_rn(__fmul_rn(v.w, s_router), g.w));
  }
  if (moe_in_s16 == nullptr) return;
  __syncthreads();
  const float* mi = moe_in + (size_t)blockIdx.x * dim;
  for (int k = threadIdx.x; k < dim / 16; k += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) t += mi[16 * k + i];
    moe_in_s16[(size_t)blockIdx.x * (dim / 16) + k] = t;
  }
}

// ---------------------------------------------------------------- router
// logits[t][e] = sum_k Wr[e][k] * xr[t][k]  (F32 matmul, Llama.kt:269-270).
// Few tokens: one CTA per (expert, 8 tokens); its 8 warps split K and the
// partial sums meet in shared memory in a fixed order.
__global__ void __launch_bounds__(256) moe_router_small_kernel(const float* __restrict__ wr,
                                                               const float* __restrict__ xr, float* __restrict__ logits,
                                                               int T, int dim, int n_expert) {
  __shared__ float part[8][8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x, t0 = blockIdx.y * 8;
  const int n4 = dim >> 2;
  const int k0 = (n4 * warp) / 8, k1 = (n4 * (warp + 1)) / 8;
  const float4* w4 = reinterpret_cast<const float4*>(wr + (size_t)e * dim);
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  for (int k = k0 + lane; k < k1; k += 32) {
    const float4 w = __ldg(w4 + k);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (t0 + j < T) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(xr + (size_t)(t0 + j) * dim) + k);
        acc[j] = fmaf(w.x, v.x, fmaf(w.y, v.y, fmaf(w.z, v.z, fmaf(w.w, v.w, acc[j]))));
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float v = warp_sum(acc[j]);
    if (lane == 0) part[warp][j] = v;
  }
  __syncthreads();
  if (threadIdx.x < 8 && t0 + threadIdx.x < T) {
    float v = 0.f;
    for (int w = 0; w < 8; ++w) v += part[w][threadIdx.x];
    logits[(size_t)(t0 + threadIdx.x) * n_expert + e] = v;
  }
}

// Many tokens: register-tiled fp32 GEMM.  A CTA (128 threads) computes 64
// tokens x 128 experts over one K range of a split-K partition; thread
// (ty, tx) = (tid / 16, tid % 16) holds tokens {4ty..4ty+3, 32+4ty..} x
// experts {4tx..4tx+3, 64+4tx..}, so every shared-memory read is a
// conflict-free 16-byte vector (64 FMAs per 4 reads).  K advances in tiles
// of 32 staged through registers (coalesced global loads, transposed into
// k-major shared rows).  Partial sums go to part[split][T][E]; the top-k
// kernel adds the splits in order.
constexpr int kRtM = 64, kRtN = 128, kRtK = 32, kRtMaxSplit = 32;
__global__ void __launch_bounds__(128) moe_router_gemm_kernel(const float* __restrict__ wr,
                                                              const float* __restrict__ xr, float* __restrict__ part,
                                                              int T, int dim, int E, int nsplit) {
  __shared__ __align__(16) float xs[kRtK][kRtM + 4];
  __shared__ __align__(16) float ws[kRtK][kRtN + 4];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int t0 = blockIdx.x * kRtM, e0 = blockIdx.z * kRtN, split = blockIdx.y;
  const int nk = (dim + kRtK - 1) / kRtK;
  const int kt0 = (int)((long long)nk * split / nsplit), kt1 = (int)((long long)nk * (split + 1) / nsplit);
  // loads: float4 number i = tid + 128j; row i / 8, columns 4*(i % 8) of the k tile
  float4 xv[4], wv[8];
  auto load = [&](int kt) {
    const int kb = kt * kRtK + 4 * (tid & 7);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = t0 + ((tid + 128 * j) >> 3);
      xv[j] = (r < T && kb < dim) ? __ldg(reinterpret_cast<const float4*>(xr + (size_t)r * dim + kb))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = e0 + ((tid + 128 * j) >> 3);
      wv[j] = (e < E && kb < dim) ? __ldg(reinterpret_cast<const float4*>(wr + (size_t)e * dim + kb))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto store = [&]() {
    const int k = 4 * (tid & 7);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = (tid + 128 * j) >> 3;
      xs[k][r] = xv[j].x;
      xs[k + 1][r] = xv[j].y;
      xs[k + 2][r] = xv[j].z;
      xs[k + 3][r] = xv[j].w;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = (tid + 128 * j) >> 3;
      ws[k][e] = wv[j].x;
      ws[k + 1][e] = wv[j].y;
      ws[k + 2][e] = wv[j].z;
      ws[k + 3][e] = wv[j].w;
    }
  };
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  if (kt0 < kt1) load(kt0);
  for (int kt = kt0; kt < kt1; ++kt) {
    __syncthreads();  // the previous tile's reads are done
    store();
    __syncthreads();
    if (kt + 1 < kt1) load(kt + 1);
#pragma unroll 4
    for (int k = 0; k < kRtK; ++k) {
      const float4 a0 = *reinterpret_cast<const float4*>(&xs[k][4 * ty]);
      const float4 a1 = *reinterpret_cast<const float4*>(&xs[k][32 + 4 * ty]);
      const float4 b0 = *reinterpret_cast<const float4*>(&ws[k][4 * tx]);
      const float4 b1 = *reinterpret_cast<const float4*>(&ws[k][64 + 4 * tx]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
  }
  float* out = part + (size_t)split * T * E;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int t = t0 + (i < 4 ? 4 * ty + i : 32 + 4 * ty + i - 4);
    if (t >= T) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = e0 + (j < 4 ? 4 * tx + j : 64 + 4 * tx + j - 4);
      if (e < E) out[(size_t)t * E + e] = acc[i][j];
    }
  }
}

// Router logits for T tokens.  Returns the number of K splits written to
// `part` ([nsplit][T][E]; the caller sums them in order), or 0 when the
// logits went straight to `logits`.  part needs nsplit*T*E floats, at most
// kRtMaxSplit*T*E.
static int launch_router(const float* wr, const float* xr, float* logits, float* part, int T, int dim, int E,
                         int sms, cudaStream_t st) {
  if (T < 32) {
    moe_router_small_kernel<<<dim3(E, (T + 7) / 8), 256, 0, st>>>(wr, xr, logits, T, dim, E);
    return 0;
  }
  const int tiles = ((T + kRtM - 1) / kRtM) * ((E + kRtN - 1) / kRtN);
  const int nk = (dim + kRtK - 1) / kRtK;
  int nsplit = (2 * sms + tiles - 1) / tiles;
  nsplit = nsplit < 1 ? 1 : nsplit > kRtMaxSplit ? kRtMaxSplit : nsplit;
  if (nsplit > nk) nsplit = nk;
  moe_router_gemm_kernel<<<dim3((T + kRtM - 1) / kRtM, nsplit, (E + kRtN - 1) / kRtN), 128, 0, st>>>(
      wr, xr, part, T, dim, E, nsplit);
  return nsplit;
}

// ---------------------------------------------------------------- softmax + top-k
// One warp per token.  softmaxInPlace (MutableFloatTensor.kt:54-59): max,
// exp((v-max) in double) -> float, sequential float sum, divide.  Top-k as
// Llama.kt:280-293: strict '>' over ascending index, so ties go to the lowest
// index; the selected entry is masked to -inf.
// `logits` holds nsplit >= 1 partial logit matrices [nsplit][T][E] (split-K
// router) that are added in split order first.
// Softmax and top-k of one token by one warp; p (E floats of shared memory)
// holds the token's logits on entry and the token's mx is their maximum.
__device__ __forceinline__ void topk_warp(float* p, float mx, int E, int K, int t, int32_t* __restrict__ idx_out,
                                          float* __restrict__ prob_out) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  for (int e = lane; e < E; e += 32) p[e] = (float)exp((double)__fsub_rn(p[e], mx));
  __syncwarp();
  float sum = 0.f;
  if (lane == 0)
    for (int e = 0; e < E; ++e) sum = __fadd_rn(sum, p[e]);
  sum = __shfl_sync(0xffffffffu, sum, 0);
  for (int e = lane; e < E; e += 32) p[e] = __fdiv_rn(p[e], sum);
  __syncwarp();
  for (int k = 0; k < K; ++k) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int e = lane; e < E; e += 32) {
      float v = p[e];
      if (v > bv) {  // ascending e within the lane: first maximum wins
        bv = v;
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (bi == 0x7fffffff) bi = 0;  // every entry -inf: the reference keeps bestIdx = 0
    if (lane == 0) {
      idx_out[(size_t)t * K + k] = bi;
      prob_out[(size_t)t * K + k] = bv;
      p[bi] = -INFINITY;
    }
    __syncwarp();
  }
}

__global__ void moe_topk_kernel(const float* __restrict__ logits, int nsplit, int T, int E, int K,
                                int32_t* __restrict__ idx_out, float* __restrict__ prob_out) {
  __shared__ float probs[8][kMaxExperts];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= T) return;
  float* p = probs[warp];
  float mx = -INFINITY;
  for (int e = lane; e < E; e += 32) {
    float v = logits[(size_t)t * E + e];
    for (int sp = 1; sp < nsplit; ++sp) v = __fadd_rn(v, logits[((size_t)sp * T + t) * E + e]);
    p[e] = v;
    mx = fmaxf(mx, v);
  }
  topk_warp(p, mx, E, K, t, idx_out, prob_out);
}

// ---------------------------------------------------------------- permutation
// Single CTA: counts per expert, exclusive offsets (offsets[E] = T*K), and
// perm[offsets[e] + j] = slot for the j-th slot routed to e.
// Block-wide body of the permutation (shared arrays passed in).
__device__ __forceinline__ void permute_block(const int32_t* __restrict__ idx, int n_slots, int E,
                                              int32_t* __restrict__ offsets, int32_t* __restrict__ perm, int* cnt,
                                              int* off, int* cur) {
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    cnt[e] = 0;
    cur[e] = 0;
  }
  __syncthreads();
  for (int s = threadIdx.x; s < n_slots; s += blockDim.x) atomicAdd(&cnt[idx[s]], 1);
  __syncthreads();
  if (threadIdx.x < 32) {  // exclusive scan of the counts, 32 experts at a time
    int carry = 0;
    for (int base = 0; base < E; base += 32) {
      const int e = base + (int)threadIdx.x;
      const int v = e < E ? cnt[e] : 0;
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if ((int)threadIdx.x >= o) incl += u;
      }
      if (e < E) off[e] = carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (threadIdx.x == 0) off[E] = carry;
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= E; e += blockDim.x) offsets[e] = off[e];
  for (int s = threadIdx.x; s < n_slots; s += blockDim.x) {
    int e = idx[s];
    int pos = off[e] + atomicAdd(&cur[e], 1);
    perm[pos] = s;
  }
}

__global__ void __launch_bounds__(1024) moe_permute_kernel(const int32_t* __restrict__ idx, int n_slots, int E,
                                                           int32_t* __restrict__ offsets, int32_t* __restrict__ perm) {
  __shared__ int cnt[kMaxExperts], off[kMaxExperts + 1], cur[kMaxExperts];
  permute_block(idx, n_slots, E, offsets, perm, cnt, off, cur);
}

// Small batches (T <= 8): prep, router, softmax/top-k and permutation in one
// launch.  CTA e computes expert e's logit for every token: each thread holds
// its share of router row e and of the gate scale in registers (float4 columns
// tid, tid + 256, ...), so the sums of squares and the logits need a single
// round trip to memory.  The CTA also writes moe_in and its per-16 sums for
// the 16-column groups jj = e (mod E).  The last CTA to finish (ticket
// counter) runs softmax/top-k per token and the permutation, and puts the
// ticket back to 0 for the next call.
constexpr int kFrontMaxF4 = 4;  // float4 columns per thread: dim <= 4096
__global__ void __launch_bounds__(256) moe_front_small_kernel(
    const float* __restrict__ x, const float* __restrict__ pre_norm, const float* __restrict__ gate_scale,
    const float* __restrict__ wr, float* __restrict__ moe_in, float* __restrict__ moe_in_s16,
    float* __restrict__ logits, int32_t* __restrict__ idx, float* __restrict__ prob, int32_t* __restrict__ offsets,
    int32_t* __restrict__ perm, unsigned* __restrict__ ticket, int T, int dim, int E, int K, float eps) {
  __shared__ float s_norm[8], s_router[8];
  __shared__ float part[8][8];
  __shared__ float probs[8][kMaxExperts];
  __shared__ int cnt[kMaxExperts], off[kMaxExperts + 1], cur[kMaxExperts];
  __shared__ int is_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, e = blockIdx.x;
  const int n4 = dim >> 2;
  const float4* w4 = reinterpret_cast<const float4*>(wr + (size_t)e * dim);
  const float4* g4 = reinterpret_cast<const float4*>(gate_scale);
  float4 wv[kFrontMaxF4], gv[kFrontMaxF4];
#pragma unroll
  for (int i = 0; i < kFrontMaxF4; ++i) {
    const int k = tid + 256 * i;
    if (k < n4) {
      wv[i] = __ldg(w4 + k);
      gv[i] = __ldg(g4 + k);
    }
  }
  grid_dep_launch();
  grid_dep_wait();  // x comes from the previous grid
  // per-token sums of squares (rmsnorm, Llama.kt:27-37)
  float acc[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) acc[t] = 0.f;
#pragma unroll
  for (int i = 0; i < kFrontMaxF4; ++i) {
    const int k = tid + 256 * i;
    if (k < n4) {
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        if (t < T) {
          const float4 v = __ldg(reinterpret_cast<const float4*>(x + (size_t)t * dim) + k);
          acc[t] = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, acc[t]))));
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const float v = warp_sum(acc[t]);
    if (lane == 0) part[warp][t] = v;
  }
  __syncthreads();
  if (tid < T) {
    float ss = 0.f;
    for (int w = 0; w < 8; ++w) ss += part[w][tid];
    const float m = __fadd_rn(__fdiv_rn(ss, (float)dim), eps);
    const float sn = (float)(1.0 / sqrt((double)m));
    s_norm[tid] = sn;
    s_router[tid] = __fdiv_rn(sn, (float)sqrt((double)dim));  // router scale, Llama.kt:258-261
  }
  __syncthreads();
  // router logit of expert e (F32 matmul, Llama.kt:269-270) on xr = (x * s) * gate_scale
#pragma unroll
  for (int t = 0; t < 8; ++t) acc[t] = 0.f;
#pragma unroll
  for (int i = 0; i < kFrontMaxF4; ++i) {
    const int k = tid + 256 * i;
    if (k < n4) {
      const float4 w = wv[i], g = gv[i];
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        if (t < T) {
          const float4 v = __ldg(reinterpret_cast<const float4*>(x + (size_t)t * dim) + k);
          const float sr = s_router[t];
          acc[t] = fmaf(w.x, __fmul_rn(__fmul_rn(v.x, sr), g.x),
                        fmaf(w.y, __fmul_rn(__fmul_rn(v.y, sr), g.y),
                             fmaf(w.z, __fmul_rn(__fmul_rn(v.z, sr), g.z),
                                  fmaf(w.w, __fmul_rn(__fmul_rn(v.w, sr), g.w), acc[t]))));
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const float v = warp_sum(acc[t]);
    if (lane == 0) part[warp][t] = v;  // every thread read part before the last barrier
  }
  // moe_in and its per-16 sums for this CTA's column groups
  for (int item = tid; item < T * (dim / 16); item += blockDim.x) {
    const int t = item / (dim / 16), jj = item % (dim / 16);
    if (jj % gridDim.x != (unsigned)e) continue;
    const float* xr_ = x + (size_t)t * dim + 16 * jj;
    float* mo = moe_in + (size_t)t * dim + 16 * jj;
    float s16 = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float v = __fmul_rn(pre_norm[16 * jj + i], __fmul_rn(s_norm[t], xr_[i]));
      mo[i] = v;
      s16 += v;
    }
    moe_in_s16[(size_t)t * (dim / 16) + jj] = s16;
  }
  __syncthreads();
  if (tid < T) {
    float v = 0.f;
    for (int w = 0; w < 8; ++w) v += part[w][tid];
    logits[(size_t)tid * E + e] = v;
  }
  // the last CTA to get here routes every token
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!is_last) return;
  if (tid == 0) *ticket = 0u;  // every CTA has counted
  __threadfence();
  if (warp < T) {
    float* p = probs[warp];
    float mx = -INFINITY;
    for (int ee = lane; ee < E; ee += 32) {
      const float v = __ldcg(logits + (size_t)warp * E + ee);
      p[ee] = v;
      mx = fmaxf(mx, v);
    }
    topk_warp(p, mx, E, K, warp, idx, prob);
  }
  __syncthreads();
  __threadfence_block();
  permute_block(idx, T * K, E, offsets, perm, cnt, off, cur);
}

// Wide batches: the same result from three kernels over chunks of slots.
// Within an expert the slots come in no fixed order; nothing downstream
// depends on it (every slot's products are independent of its neighbours).
constexpr int kPermChunk = 2048;
__global__ void __launch_bounds__(256) moe_perm_count_kernel(const int32_t* __restrict__ idx, int n_slots, int E,
                                                             int32_t* __restrict__ cnt) {
  __shared__ int h[kMaxExperts];
  for (int e = threadIdx.x; e < E; e += blockDim.x) h[e] = 0;
  __syncthreads();
  const int s0 = blockIdx.x * kPermChunk, s1 = min(n_slots, s0 + kPermChunk);
  for (int s = s0 + threadIdx.x; s < s1; s += blockDim.x) atomicAdd(&h[idx[s]], 1);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[(size_t)blockIdx.x * E + e] = h[e];
}
// One CTA of kMaxExperts threads: offsets[e] (offsets[E] = n_slots) and, in
// place of the chunk counts, each chunk's first position for each expert.
__global__ void __launch_bounds__(kMaxExperts) moe_perm_scan_kernel(int32_t* __restrict__ cnt, int nb, int E,
                                                                    int32_t* __restrict__ offsets) {
  __shared__ int tot[kMaxExperts + 1];
  const int e = threadIdx.x;
  int sum = 0;
  if (e < E)
    for (int b = 0; b < nb; ++b) sum += cnt[(size_t)b * E + e];
  tot[e] = sum;
  __syncthreads();
  if (e == 0) {
    int a = 0;
    for (int i = 0; i < E; ++i) {
      const int v = tot[i];
      tot[i] = a;
      a += v;
    }
    tot[E] = a;
    offsets[E] = a;
  }
  __syncthreads();
  if (e < E) {
    int run = tot[e];
    offsets[e] = run;
    for (int b = 0; b < nb; ++b) {
      const int c = cnt[(size_t)b * E + e];
      cnt[(size_t)b * E + e] = run;
      run += c;
    }
  }
}
__global__ void __launch_bounds__(256) moe_perm_place_kernel(const int32_t* __restrict__ idx, int n_slots, int E,
                                                             const int32_t* __restrict__ base,
                                                             int32_t* __restrict__ perm) {
  __shared__ int cur[kMaxExperts];
  for (int e = threadIdx.x; e < E; e += blockDim.x) cur[e] = base[(size_t)blockIdx.x * E + e];
  __syncthreads();
  const int s0 = blockIdx.x * kPermChunk, s1 = min(n_slots, s0 + kPermChunk);
  for (int s = s0 + threadIdx.x; s < s1; s += blockDim.x) perm[atomicAdd(&cur[idx[s]], 1)] = s;
}

// Threads for a one-row-per-CTA kernel over n4 float4 columns: about 512,
// with every thread doing the same number of columns.
static int row_threads(int n4) {
  const int iters = (n4 + 511) / 512;
  int t = (n4 + iters - 1) / iters;
  t = (t + 31) / 32 * 32;
  return t < 32 ? 32 : t;
}

// ---------------------------------------------------------------- grouped experts
// Work item = (expert e, row tile, token chunk of <= NB slots).  Items of
// expert e are tile-major with the chunk fastest, so CTAs working on the same
// tile at the same time share its weights through L2.
//
// GATEUP: tile = NCW gate rows r and their up rows ff+r (one pair per consumer
//         warp); epilogue g = gelu(gate) * up -> G[slot][r].
// DOWN:   tile = NCW virtual rows (pr real rows each) of the [dim, ff] expert
//         matrix; output D[slot][row].
struct ExpertArgs {
  const uint8_t* w;         // expert tensor block stream
  const float* act;         // GATEUP: moe_in [T, K_in]; DOWN: G [slots, ff]
  float* out;               // GATEUP: G [slots, ff]; DOWN: D [slots, dim]
  const int32_t* offsets;   // [E+1]
  const int32_t* perm;      // [slots]
  unsigned* status;
  int E, n_used;
  int rows_e;               // output rows per expert (GATEUP: 2*ff; DOWN: dim)
  int cols;                 // K (GATEUP: dim; DOWN: ff)
  int ff;                   // expert_ff
  int pr;                   // DOWN: rows per virtual row
  int vb;                   // bytes per (virtual) row
  int units;                // 16-weight units per (virtual) row
  int tiles_e;              // row tiles per expert
  int tile_rows;            // GATEUP: pairs per tile; DOWN: virtual rows per tile
  int stage_bytes, nstages;
  int region_bytes;         // GATEUP: offset of the up-row region in a stage
  long long expert_elems;   // elements per expert matrix
};

template <int FMT, bool GATEUP, int PR, int NB, int NCW>
__global__ void __launch_bounds__(32 * (NCW + 1)) moe_expert_kernel(const __grid_constant__ ExpertArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int BS = block_size(FMT), TS = type_size(FMT);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + 4;
  int* s_items = reinterpret_cast<int*>(smem + 64);            // [E+1] item prefix
  int* s_chunks = s_items + (kMaxExperts + 1);                 // [E] chunks per expert
  uint8_t* stages = smem + 64 + 4 * (2 * kMaxExperts + 8);
  stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(stages) + 127) & ~uintptr_t(127));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NS = a.nstages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NCW);
    }
    fence_barrier_init();
  }
  // per-expert chunk counts, then an exclusive scan of chunks * tiles (warp 0)
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) {
    const int n = a.offsets[e + 1] - a.offsets[e];
    s_chunks[e] = (n + NB - 1) / NB;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    int carry = 0;
    for (int base = 0; base < a.E; base += 32) {
      const int e = base + (int)threadIdx.x;
      const int v = e < a.E ? s_chunks[e] * a.tiles_e : 0;
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if ((int)threadIdx.x >= o) incl += u;
      }
      if (e < a.E) s_items[e] = carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (threadIdx.x == 0) s_items[a.E] = carry;
  }
  __syncthreads();
  const int n_items = s_items[a.E];

  auto locate = [&](int item, int& e, int& tile, int& chunk) {
    int lo = 0, hi = a.E - 1;  // last e with s_items[e] <= item
    while (lo < hi) {
      int mid = (lo + hi + 1) >> 1;
      if (s_items[mid] <= item) lo = mid;
      else hi = mid - 1;
    }
    e = lo;
    int local = item - s_items[e];
    tile = local / s_chunks[e];
    chunk = local - tile * s_chunks[e];
  };

  if (warp == 0) {
    if (lane != 0) return;
    int it = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++it) {
      int s = it % NS;
      if (it >= NS && !mbar_wait_bounded(&empty[s], ((it / NS) - 1) & 1)) {
        record_error(a.status, ERR_TIMEOUT_EMPTY);
        break;
      }
      int e, tile, chunk;
      locate(item, e, tile, chunk);
      uint8_t* dst = stages + (size_t)s * a.stage_bytes;
      long long eb = (long long)e * a.expert_elems;  // expert's first element (block aligned)
      if (GATEUP) {
        int r0 = tile * a.tile_rows;
        int nr = min(a.tile_rows, a.ff - r0);
        long long g0 = (eb + (long long)r0 * a.cols) / BS * TS;
        long long u0 = (eb + (long long)(a.ff + r0) * a.cols) / BS * TS;
        long long bytes = (long long)nr * a.vb;
        // copy the 16-byte aligned superset of each row range
        long long ga = g0 & ~15ll, gb = (g0 + bytes + 15) & ~15ll;
        long long ua = u0 & ~15ll, ub = (u0 + bytes + 15) & ~15ll;
        mbar_arrive_expect_tx(&full[s], (uint32_t)((gb - ga) + (ub - ua)));
        bulk_g2s(dst, a.w + ga, (uint32_t)(gb - ga), &full[s]);
        bulk_g2s(dst + a.region_bytes, a.w + ua, (uint32_t)(ub - ua), &full[s]);
      } else {
        int v0 = tile * a.tile_rows;
        int nv = min(a.tile_rows, a.rows_e / PR - v0);
        long long b0 = (eb + (long long)v0 * PR * a.cols) / BS * TS;
        long long ba = b0 & ~15ll, bb = (b0 + (long long)nv * a.vb + 15) & ~15ll;
        mbar_arrive_expect_tx(&full[s], (uint32_t)(bb - ba));
        bulk_g2s(dst, a.w + ba, (uint32_t)(bb - ba), &full[s]);
      }
    }
    for (int j = max(0, it - NS); j < it; ++j)
      if (!mbar_wait_bounded(&full[j % NS], (j / NS) & 1)) record_error(a.status, ERR_TIMEOUT_DRAIN);
    return;
  }

  const int cw = warp - 1;
  int it = 0;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++it) {
    int s = it % NS;
    if (!mbar_wait_bounded(&full[s], (it / NS) & 1)) {
      record_error(a.status, ERR_TIMEOUT_FULL);
      return;
    }
    int e, tile, chunk;
    locate(item, e, tile, chunk);
    const int p0 = a.offsets[e] + chunk * NB;
    const int nb = min(NB, a.offsets[e + 1] - p0);
    int slot[NB];
    const float* xrow[NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      slot[j] = j < nb ? a.perm[p0 + j] : 0;
      // GATEUP reads the token's moeInput row, DOWN the slot's gelu*up row
      xrow[j] = GATEUP ? a.act + (size_t)(slot[j] / a.n_used) * a.cols : a.act + (size_t)slot[j] * a.cols;
    }
    const uint8_t* st = stages + (size_t)s * a.stage_bytes;

    if (GATEUP) {
      const int r0 = tile * a.tile_rows;
      const int r = r0 + cw;  // gate row; up row = ff + r
      const bool valid = r < a.ff;
      const long long eb = (long long)e * a.expert_elems;
      const int gmis = (int)(((eb + (long long)r0 * a.cols) / BS * TS) & 15);
      const int umis = (int)(((eb + (long long)(a.ff + r0) * a.cols) / BS * TS) & 15);
      const uint8_t* vg = st + gmis + (size_t)cw * a.vb;
      const uint8_t* vu = st + a.region_bytes + umis + (size_t)cw * a.vb;
      float ag[NB], au[NB];
#pragma unroll
      for (int j = 0; j < NB; ++j) ag[j] = au[j] = 0.f;
      if (valid) {
        for (int u = lane; u < a.units; u += 32) {
          float wg[16], wu[16];
          deq16<FMT>(vg, u, wg);
          deq16<FMT>(vu, u, wu);
#pragma unroll
          for (int j = 0; j < NB; ++j) {
            if (j < nb) {
              const float4* xp = reinterpret_cast<const float4*>(xrow[j] + u * 16);
              float g0 = 0.f, g1 = 0.f, u0 = 0.f, u1 = 0.f;
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                float4 v = __ldg(xp + k);
                g0 = fmaf(wg[4 * k], v.x, g0);
                g1 = fmaf(wg[4 * k + 1], v.y, g1);
                g0 = fmaf(wg[4 * k + 2], v.z, g0);
                g1 = fmaf(wg[4 * k + 3], v.w, g1);
                u0 = fmaf(wu[4 * k], v.x, u0);
                u1 = fmaf(wu[4 * k + 1], v.y, u1);
                u0 = fmaf(wu[4 * k + 2], v.z, u0);
                u1 = fmaf(wu[4 * k + 3], v.w, u1);
              }
              ag[j] += g0 + g1;
              au[j] += u0 + u1;
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        float g = warp_sum(ag[j]);
        float up = warp_sum(au[j]);
        if (lane == 0 && valid && j < nb) a.out[(size_t)slot[j] * a.ff + r] = __fmul_rn(gelu_ref(g), up);
      }
    } else {
      const int v = tile * a.tile_rows + cw;
      const bool valid = v < a.rows_e / PR;
      const long long eb = (long long)e * a.expert_elems;
      const int mis = (int)(((eb + (long long)tile * a.tile_rows * PR * a.cols) / BS * TS) & 15);
      const uint8_t* vbp = st + mis + (size_t)cw * a.vb;
      float acc[PR][NB];
#pragma unroll
      for (int r = 0; r < PR; ++r)
#pragma unroll
        for (int j = 0; j < NB; ++j) acc[r][j] = 0.f;
      if (valid) {
        for (int u = lane; u < a.units; u += 32) {
          const int e0 = u * 16;
          const int col = PR == 1 ? e0 : e0 % a.cols;
          const int rip = PR == 1 ? 0 : e0 / a.cols;
          float w[16];
          deq16<FMT>(vbp, u, w);
#pragma unroll
          for (int j = 0; j < NB; ++j) {
            if (j < nb) {
              const float4* xp = reinterpret_cast<const float4*>(xrow[j] + col);
              float s0 = 0.f, s1 = 0.f;
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                float4 xv = __ldg(xp + k);
                s0 = fmaf(w[4 * k], xv.x, s0);
                s1 = fmaf(w[4 * k + 1], xv.y, s1);
                s0 = fmaf(w[4 * k + 2], xv.z, s0);
                s1 = fmaf(w[4 * k + 3], xv.w, s1);
              }
              float part = s0 + s1;
#pragma unroll
              for (int r = 0; r < PR; ++r) acc[r][j] += (rip == r) ? part : 0.f;
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
      for (int r = 0; r < PR; ++r)
#pragma unroll
        for (int j = 0; j < NB; ++j) {
          float sum = warp_sum(acc[r][j]);
          if (lane == 0 && valid && j < nb) a.out[(size_t)slot[j] * a.rows_e + (size_t)v * PR + r] = sum;
        }
    }
  }
}

// ---------------------------------------------------------------- grouped experts, lane-per-row
// The expert GEMVs in the GEMV kernel's style (csrc/g4_gemv.cu): each warp
// streams 16 (virtual) rows of one expert through its own bulk-copy ring, two
// lanes per row, and multiplies every decoded weight into the NB tokens routed
// to that expert (activations through L1, their per-16-column sums from a
// table).  Work item = (expert, token chunk of <= NB slots, row group).
//   GATEUP: lane (rs, half) copies gate row r = 16g+rs (half 0) or up row
//           ff+r (half 1); both lanes of a row decode alternate blocks of both
//           rows; epilogue g = gelu(gate) * up -> G[slot][r] and the sum of the
//           group's 16 G values -> Gs16[slot][g].
//   DOWN:   lane (rs, half) owns virtual row 16g+rs (pr real rows of the
//           [dim, ff] expert matrix); D[slot][row].
struct RowsArgs {
  const uint8_t* w;
  const float* act;      // GATEUP: moe_in [T][cols]; DOWN: G [slots][cols]
  const float* act_s16;  // per-16-column sums of the activation rows
  float* out;            // GATEUP: G [slots][ff]; DOWN: D [slots][dim]
  float* out_s16;        // GATEUP: Gs16 [slots][ff/16]
  const int32_t* offsets;
  const int32_t* perm;
  unsigned* status;
  int E, n_used, ff, dim;
  int cols;              // K of the product
  int nvrows;            // GATEUP: ff; DOWN: dim / pr
  int bpv;               // blocks per virtual row
  int cb, nchunks, pitch, ns;
  int ngroups;           // ceil(nvrows / 16)
  int split;             // 1: warps own items; >1: CTA owns an item, its warps split the chunks
  int xcols;             // activation floats staged per token per stage (GATEUP: the chunk; DOWN: the row)
  int xs16n;             // per-16 sums staged per token per stage
  int x_at, xs_at;       // byte offsets of those areas inside a stage
  int stage_bytes;
  long long expert_elems;
};

// xr[j] / xs16[j]: token j's activations / per-16-column sums staged in shared
// memory, holding columns from `xoff` on.
template <int FMT, int PR, int NB>
__device__ __forceinline__ void blk_nb(const uint8_t* blk, int e0, int cols, const float* const* xr,
                                       const float* const* xs16, int xoff, int nbv, float (&acc)[NB][PR]) {
  constexpr uint32_t C = 0x3F800000u;
  if constexpr (FMT == Q4_K) {
    const uint4 h = lds128(blk);
    const float d = f16_bits_to_f32((uint16_t)(h.x & 0xFFFFu));
    const float dmin = f16_bits_to_f32((uint16_t)(h.x >> 16));
    const uint32_t sc03 = h.y & 0x3F3F3F3Fu, mn03 = h.z & 0x3F3F3F3Fu;
    const uint32_t sc47 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    const uint32_t mn47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int eg = e0 + 64 * g;
      const int col = PR == 1 ? eg : eg % cols;
      const int rr = PR == 1 ? 0 : eg / cols;
      float2 alo[NB], ahi[NB];
      float xlo[NB], xhi[NB];
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        if (j < nbv) {
          const float* q = xs16[j] + (col - xoff) / 16;
          xlo[j] = q[0] + q[1];
          xhi[j] = q[2] + q[3];
        } else {
          xlo[j] = xhi[j] = 0.f;
        }
        alo[j] = f2(-xlo[j], 0.f);
        ahi[j] = f2(-xhi[j], 0.f);
      }
      const uint4 qa = lds128(blk + 16 + 32 * g), qb = lds128(blk + 32 + 32 * g);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t w = k == 0 ? qa.x : k == 1 ? qa.y : k == 2 ? qa.z : k == 3 ? qa.w
                         : k == 4 ? qb.x : k == 5 ? qb.y : k == 6 ? qb.z : qb.w;
        const uint32_t ml = (w & 0x0F0F0F0Fu) | 0x80808080u, mh = w & 0xF0F0F0F0u;
        const float2 l01 = f2(__uint_as_float(__byte_perm(ml, C, 0x7054u)), __uint_as_float(__byte_perm(ml, C, 0x7154u)));
        const float2 l23 = f2(__uint_as_float(__byte_perm(ml, C, 0x7254u)), __uint_as_float(__byte_perm(ml, C, 0x7354u)));
        const float2 h01 = f2(__uint_as_float(__byte_perm(mh, C, 0x7604u)), __uint_as_float(__byte_perm(mh, C, 0x7614u)));
        const float2 h23 = f2(__uint_as_float(__byte_perm(mh, C, 0x7624u)), __uint_as_float(__byte_perm(mh, C, 0x7634u)));
#pragma unroll
        for (int j = 0; j < NB; ++j) {
          if (j < nbv) {
            const float4 xl = lds_f4(xr[j] + (col - xoff) + 4 * k);
            const float4 xh = lds_f4(xr[j] + (col - xoff) + 32 + 4 * k);
            alo[j] = __ffma2_rn(l01, f2(xl.x, xl.y), alo[j]);
            alo[j] = __ffma2_rn(l23, f2(xl.z, xl.w), alo[j]);
            ahi[j] = __ffma2_rn(h01, f2(xh.x, xh.y), ahi[j]);
            ahi[j] = __ffma2_rn(h23, f2(xh.z, xh.w), ahi[j]);
          }
        }
      }
      const uint32_t scw = g < 2 ? sc03 : sc47, mnw = g < 2 ? mn03 : mn47;
      const int b0 = (2 * g) & 3;
      const float c_lo = 128.f * d * (float)((scw >> (8 * b0)) & 0xFFu);
      const float c_hi = 2048.f * d * (float)((scw >> (8 * b0 + 8)) & 0xFFu);
      const float m_lo = dmin * (float)((mnw >> (8 * b0)) & 0xFFu);
      const float m_hi = dmin * (float)((mnw >> (8 * b0 + 8)) & 0xFFu);
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        float v = c_lo * (alo[j].x + alo[j].y);
        v = fmaf(c_hi, ahi[j].x + ahi[j].y, v);
        v = fmaf(-m_lo, xlo[j], fmaf(-m_hi, xhi[j], v));
        add_row<PR>(acc[j], rr, v);
      }
    }
  } else if constexpr (FMT == Q8_0) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(blk);
    const uint8_t* b4 = reinterpret_cast<const uint8_t*>(a & ~uintptr_t(3));
    const uint32_t sh = (uint32_t)(a & 3u);
    uint32_t w[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) w[i] = lds32(b4 + 4 * i);
    const float d = f16_bits_to_f32((uint16_t)(sh ? (w[0] >> 16) : (w[0] & 0xFFFFu)));
    const int col = e0;  // Q8_0 rows are whole blocks here (pr == 1)
    float2 s[NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) s[j] = f2(0.f, 0.f);
    const float2 nb2 = f2(-8388736.0f, -8388736.0f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t m = __funnelshift_rc(w[k], w[k + 1], 16u + 8u * sh) ^ 0x80808080u;
      const float2 q01 = __fadd2_rn(f2(f_magic23(m, 0), f_magic23(m, 1)), nb2);
      const float2 q23 = __fadd2_rn(f2(f_magic23(m, 2), f_magic23(m, 3)), nb2);
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        if (j < nbv) {
          const float4 xv = lds_f4(xr[j] + (col - xoff) + 4 * k);
          s[j] = __ffma2_rn(q01, f2(xv.x, xv.y), s[j]);
          s[j] = __ffma2_rn(q23, f2(xv.z, xv.w), s[j]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < NB; ++j) acc[j][0] = fmaf(s[j].x + s[j].y, d, acc[j][0]);
  } else {  // Q6_K
    const uintptr_t a = reinterpret_cast<uintptr_t>(blk);
    const uint8_t* b4 = reinterpret_cast<const uint8_t*>(a & ~uintptr_t(3));
    const uint32_t sh = 8u * (uint32_t)(a & 3u);
    const float d = f16_bits_to_f32((uint16_t)(__funnelshift_r(lds32(b4 + 208), lds32(b4 + 212), sh) & 0xFFFFu));
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t qa[8], qb[8], qh[8], w[9];
#pragma unroll
      for (int i = 0; i < 9; ++i) w[i] = lds32(b4 + 64 * h + 4 * i);
#pragma unroll
      for (int i = 0; i < 8; ++i) qa[i] = __funnelshift_r(w[i], w[i + 1], sh);
#pragma unroll
      for (int i = 0; i < 9; ++i) w[i] = lds32(b4 + 64 * h + 32 + 4 * i);
#pragma unroll
      for (int i = 0; i < 8; ++i) qb[i] = __funnelshift_r(w[i], w[i + 1], sh);
#pragma unroll
      for (int i = 0; i < 9; ++i) w[i] = lds32(b4 + 128 + 32 * h + 4 * i);
#pragma unroll
      for (int i = 0; i < 8; ++i) qh[i] = __funnelshift_r(w[i], w[i + 1], sh);
      const uint32_t s0 = lds32(b4 + 192 + 8 * h), s1 = lds32(b4 + 196 + 8 * h), s2 = lds32(b4 + 200 + 8 * h);
      const uint32_t scw0 = __funnelshift_r(s0, s1, sh), scw1 = __funnelshift_r(s1, s2, sh);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int ebase = e0 + 128 * h + 16 * c;
#pragma unroll
        for (int sub = 0; sub < 4; ++sub) {
          const int e = ebase + 32 * sub;
          const int col = PR == 1 ? e : e % cols;
          const int rr = PR == 1 ? 0 : e / cols;
          float2 a4[NB];
          float xsum[NB];
#pragma unroll
          for (int j = 0; j < NB; ++j) {
            xsum[j] = j < nbv ? xs16[j][(col - xoff) / 16] : 0.f;
            a4[j] = f2(-xsum[j], 0.f);
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t la = qa[4 * c + k], lb = qb[4 * c + k], hh = qh[4 * c + k];
            uint32_t m;
            if (sub == 0) m = ((la & 0x0F0F0F0Fu) | 0x80808080u) | ((hh << 4) & 0x30303030u);
            else if (sub == 1) m = ((lb & 0x0F0F0F0Fu) | 0x80808080u) | ((hh << 2) & 0x30303030u);
            else if (sub == 2) m = (((la >> 4) & 0x0F0F0F0Fu) | 0x80808080u) | (hh & 0x30303030u);
            else m = (((lb >> 4) & 0x0F0F0F0Fu) | 0x80808080u) | ((hh >> 2) & 0x30303030u);
            const float2 f01 = f2(__uint_as_float(__byte_perm(m, C, 0x7054u)), __uint_as_float(__byte_perm(m, C, 0x7154u)));
            const float2 f23 = f2(__uint_as_float(__byte_perm(m, C, 0x7254u)), __uint_as_float(__byte_perm(m, C, 0x7354u)));
#pragma unroll
            for (int j = 0; j < NB; ++j) {
              if (j < nbv) {
                const float4 xv = lds_f4(xr[j] + (col - xoff) + 4 * k);
                a4[j] = __ffma2_rn(f01, f2(xv.x, xv.y), a4[j]);
                a4[j] = __ffma2_rn(f23, f2(xv.z, xv.w), a4[j]);
              }
            }
          }
          const int si = 2 * sub + c;
          const int8_t sc = (int8_t)((((si >> 2) ? scw1 : scw0) >> (8 * (si & 3))) & 0xFFu);
          const float ds = d * (float)sc;
#pragma unroll
          for (int j = 0; j < NB; ++j) add_row<PR>(acc[j], rr, ds * fmaf(128.f, a4[j].x + a4[j].y, -32.f * xsum[j]));
        }
      }
    }
  }
}

template <int FMT, bool GATEUP, int PR, int NB>
__global__ void __launch_bounds__(NB >= 4 ? 256 : 512) moe_rows_kernel(const __grid_constant__ RowsArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int BS = block_size(FMT), TS = type_size(FMT);
  constexpr int RPW = 16, LPR = 2;
  constexpr int SLOTS = GATEUP ? 2 * RPW : RPW;  // row slots per stage
  int* s_items = reinterpret_cast<int*>(smem);           // [E+1]
  int* s_chunks = s_items + (kMaxExperts + 1);           // [E]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 8 * (kMaxExperts + 8));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, W = blockDim.x >> 5;
  const int NS = a.ns;
  uint8_t* ring = smem + 8 * (kMaxExperts + 8) + 128 * ((W * NS * 8 + 127) / 128);
  const size_t stage_bytes = (size_t)a.stage_bytes;
  uint64_t* mybars = bars + warp * NS;
  uint8_t* myring = ring + (size_t)warp * NS * stage_bytes;
  const int rs = lane % RPW, half = lane / RPW;
  (void)SLOTS;

  if (threadIdx.x < W * NS) mbar_init(&bars[threadIdx.x], 1);
  if (threadIdx.x == 0) fence_barrier_init();
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) {
    const int n = a.offsets[e + 1] - a.offsets[e];
    s_chunks[e] = (n + NB - 1) / NB;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    int carry = 0;
    for (int base = 0; base < a.E; base += 32) {
      const int e = base + (int)threadIdx.x;
      const int v = e < a.E ? s_chunks[e] * a.ngroups : 0;
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if ((int)threadIdx.x >= o) incl += u;
      }
      if (e < a.E) s_items[e] = carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (threadIdx.x == 0) s_items[a.E] = carry;
  }
  __syncthreads();
  const int n_items = s_items[a.E];

  struct Item {
    int e, g, k;
  };
  auto locate = [&](int item) {
    int lo = 0, hi = a.E - 1;  // last e with s_items[e] <= item (never an empty expert)
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_items[mid] <= item) lo = mid;
      else hi = mid - 1;
    }
    const int local = item - s_items[lo];
    const int ch = s_chunks[lo];
    return Item{lo, local / ch, local % ch};
  };
  const long long vrow_bytes = (long long)a.bpv * TS;
  const long long chunk_bytes = (long long)a.cb * TS;
  const long long blk_row = (long long)(GATEUP ? 1 : PR) * a.cols / BS;  // blocks per virtual row
  // first byte of this lane's copied row in item `it` (GATEUP: gate or up row by half)
  auto row_start = [&](const Item& it, bool& ok) {
    const int v = it.g * RPW + rs;
    ok = v < a.nvrows;
    const long long eb = (long long)it.e * a.expert_elems / BS;  // expert's first block
    const long long row = GATEUP ? (long long)(half ? a.ff + v : v) : (long long)v;
    return (eb + row * blk_row) * TS;
  };
  // lane j < NB: slot of token j of the item at the issue pointer (-1: none)
  int islot = -1;
  auto item_slot = [&](const Item& it) {
    const int p0 = a.offsets[it.e] + it.k * NB;
    const int n = min(NB, a.offsets[it.e + 1] - p0);
    return lane < n ? a.perm[p0 + lane] : -1;
  };
  auto issue = [&](const Item& it, int c, int slot) {
    uint64_t* bar = &mybars[slot];
    uint32_t mine = 0;
    if (lane < NB && islot >= 0) {
      // this token's activations for the stage (and their per-16 sums)
      uint8_t* st = myring + (size_t)slot * stage_bytes;
      const int row = GATEUP ? islot / a.n_used : islot;
      const int col0 = GATEUP ? c * a.cb * BS : 0;
      const int ncols = GATEUP ? min(a.cb * BS, a.cols - col0) : a.cols;
      bulk_g2s(st + a.x_at + (size_t)lane * a.xcols * 4, a.act + (size_t)row * a.cols + col0, (uint32_t)ncols * 4u, bar);
      const uint32_t sb = (uint32_t)(((ncols / 16) * 4 + 15) & ~15);
      bulk_g2s(st + a.xs_at + (size_t)lane * a.xs16n * 4, a.act_s16 + (size_t)row * (a.cols / 16) + col0 / 16, sb, bar);
      mine += (uint32_t)ncols * 4u + sb;
    }
    if (GATEUP || half == 0) {
      bool ok;
      const long long rstart = row_start(it, ok);
      if (ok) {
        const long long start = rstart + c * chunk_bytes;
        const long long len = min(chunk_bytes, vrow_bytes - c * chunk_bytes);
        const long long a0 = start & ~15ll, a1 = (start + len + 15) & ~15ll;
        const int slot_row = GATEUP ? half * RPW + rs : rs;
        bulk_g2s(myring + (size_t)slot * stage_bytes + (size_t)slot_row * a.pitch, a.w + a0, (uint32_t)(a1 - a0), bar);
        mine += (uint32_t)(a1 - a0);
      }
    }
    const uint32_t total = __reduce_add_sync(0xffffffffu, mine);
    if (lane == 0) mbar_arrive_expect_tx(bar, total);
  };

  // split == 1: warp-owned items gw, gw+GW, ..., each with all its chunks.
  // split  > 1: item blockIdx.x; warp w takes chunks w, w+W, ...
  const bool split = a.split > 1;
  const int gw = split ? (int)blockIdx.x : (int)blockIdx.x * W + warp;
  const int GW = split ? n_items : (int)gridDim.x * W;  // split: a single item
  const int c0 = split ? warp : 0, cstep = split ? W : 1;
  bool okw = true;
  int issued = 0, consumed = 0;
  int ii = gw, ci = c0;  // issue pointer (item, chunk)
  if (ci >= a.nchunks) ii = n_items;  // split: more warps than chunks
  Item iti = ii < n_items ? locate(ii) : Item{0, 0, 0};
  if (ii < n_items) islot = item_slot(iti);
  for (; issued < NS && ii < n_items; ++issued) {
    issue(iti, ci, issued);
    ci += cstep;
    if (ci >= a.nchunks) {
      ci = c0;
      ii += GW;
      if (ii < n_items) {
        iti = locate(ii);
        islot = item_slot(iti);
      }
    }
  }

  float acc[NB][PR], acc2[NB];  // acc2: up-row sums (GATEUP)
  int item = (c0 < a.nchunks) ? gw : n_items, c = c0;
  Item it{};
  int slots[NB];
  int nbv = 0;
  if (split && gw < n_items) {  // a warp without chunks still joins the reduction
    it = locate(gw);
    const int p0 = a.offsets[it.e] + it.k * NB;
    nbv = min(NB, a.offsets[it.e + 1] - p0);
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      const int sj = j < nbv ? a.perm[p0 + j] : 0;
      slots[j] = sj;
#pragma unroll
      for (int r = 0; r < PR; ++r) acc[j][r] = 0.f;
      acc2[j] = 0.f;
    }
  }
  for (int i = 0; item < n_items; ++i) {
    if (c == c0 && !split) {
      it = locate(item);
      const int p0 = a.offsets[it.e] + it.k * NB;
      nbv = min(NB, a.offsets[it.e + 1] - p0);
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        const int sj = j < nbv ? a.perm[p0 + j] : 0;
        slots[j] = sj;
#pragma unroll
        for (int r = 0; r < PR; ++r) acc[j][r] = 0.f;
        acc2[j] = 0.f;
      }
    }
    const int slot = i % NS;
    if (!mbar_wait_bounded(&mybars[slot], (i / NS) & 1)) {
      record_error(a.status, ERR_TIMEOUT_FULL);
      okw = false;
      consumed = i;
      break;
    }
    {
      const Item& cur = it;
      const int v = cur.g * RPW + rs;
      if (v < a.nvrows) {
        const long long start_c = (long long)c * chunk_bytes;
        const int nb = (int)(min(chunk_bytes, vrow_bytes - start_c) / TS);
        const int e0 = c * a.cb * BS;
        const uint8_t* sbase = myring + (size_t)slot * stage_bytes;
        const float* xr[NB];
        const float* xs16[NB];
#pragma unroll
        for (int j = 0; j < NB; ++j) {
          xr[j] = reinterpret_cast<const float*>(sbase + a.x_at) + (size_t)j * a.xcols;
          xs16[j] = reinterpret_cast<const float*>(sbase + a.xs_at) + (size_t)j * a.xs16n;
        }
        const int xoff = GATEUP ? c * a.cb * BS : 0;
        if constexpr (GATEUP) {
          // both rows' segments: gate in slots [0,16), up in [16,32)
          const long long eb = (long long)cur.e * a.expert_elems / BS;
          const long long g_start = (eb + (long long)v * blk_row) * TS + start_c;
          const long long u_start = (eb + (long long)(a.ff + v) * blk_row) * TS + start_c;
          const uint8_t* gb = sbase + (size_t)rs * a.pitch + (g_start & 15);
          const uint8_t* ub = sbase + (size_t)(RPW + rs) * a.pitch + (u_start & 15);
          for (int b = half; b < nb; b += LPR) {
            float tmp[NB][1];
#pragma unroll
            for (int j = 0; j < NB; ++j) tmp[j][0] = 0.f;
            blk_nb<FMT, 1, NB>(gb + b * TS, e0 + b * BS, a.cols, xr, xs16, xoff, nbv, tmp);
#pragma unroll
            for (int j = 0; j < NB; ++j) acc[j][0] += tmp[j][0];
#pragma unroll
            for (int j = 0; j < NB; ++j) tmp[j][0] = 0.f;
            blk_nb<FMT, 1, NB>(ub + b * TS, e0 + b * BS, a.cols, xr, xs16, xoff, nbv, tmp);
#pragma unroll
            for (int j = 0; j < NB; ++j) acc2[j] += tmp[j][0];
          }
        } else {
          const long long eb = (long long)cur.e * a.expert_elems / BS;
          const long long r_start = (eb + (long long)v * blk_row) * TS + start_c;
          const uint8_t* rb = sbase + (size_t)rs * a.pitch + (r_start & 15);
          for (int b = half; b < nb; b += LPR) blk_nb<FMT, PR, NB>(rb + b * TS, e0 + b * BS, a.cols, xr, xs16, xoff, nbv, acc);
        }
      }
    }
    // refill this slot with the stage NS ahead
    __syncwarp();
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (ii < n_items) {
      issue(iti, ci, slot);
      ++issued;
      ci += cstep;
      if (ci >= a.nchunks) {
        ci = c0;
        ii += GW;
        if (ii < n_items) {
          iti = locate(ii);
          islot = item_slot(iti);
        }
      }
    }
    c += cstep;
    if (split) {
      if (c >= a.nchunks) break;  // this warp's share of the item is done
      continue;
    }
    if (c >= a.nchunks) {
      // item finished: combine the two lanes of each row, write the results
      const int v = it.g * RPW + rs;
      const bool ok = v < a.nvrows;
      if constexpr (GATEUP) {
#pragma unroll
        for (int j = 0; j < NB; ++j) {
          const float hg = acc[j][0] + __shfl_xor_sync(0xffffffffu, acc[j][0], 16);
          const float hu = acc2[j] + __shfl_xor_sync(0xffffffffu, acc2[j], 16);
          float gv = 0.f;
          if (ok && j < nbv) gv = __fmul_rn(gelu_ref(hg), hu);  // Llama.kt:316-322
          if (half == 0 && ok && j < nbv) a.out[(size_t)slots[j] * a.ff + v] = gv;
          // per-16-column sum of G for the down product (the group's 16 rows)
          float t = (half == 0) ? gv : 0.f;
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
          if (lane == 0 && j < nbv) a.out_s16[(size_t)slots[j] * (a.ff / 16) + it.g] = t;
        }
      } else {
#pragma unroll
        for (int j = 0; j < NB; ++j)
#pragma unroll
          for (int r = 0; r < PR; ++r) {
            const float t = acc[j][r] + __shfl_xor_sync(0xffffffffu, acc[j][r], 16);
            if (half == 0 && ok && j < nbv) a.out[(size_t)slots[j] * a.dim + (size_t)v * PR + r] = t;
          }
      }
      c = 0;
      item += GW;
    }
  }
  if (split && gw < n_items) {
    // CTA-owned item: warps hold partial sums over disjoint chunks; reduce them
    // in shared memory in warp order, then finish as the per-warp path does.
    float* red = reinterpret_cast<float*>(ring);  // the rings are idle now
    constexpr int PER = GATEUP ? 2 * NB : NB * PR;
    __syncthreads();  // every warp is done reading its ring
    {
      float* mine = red + ((size_t)warp * 32 + lane) * PER;
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        if constexpr (GATEUP) {
          mine[2 * j] = acc[j][0];
          mine[2 * j + 1] = acc2[j];
        } else {
#pragma unroll
          for (int r = 0; r < PR; ++r) mine[j * PR + r] = acc[j][r];
        }
      }
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        float t0[PR], t1 = 0.f;
#pragma unroll
        for (int r = 0; r < PR; ++r) t0[r] = 0.f;
        for (int w2 = 0; w2 < W; ++w2) {
          const float* src = red + ((size_t)w2 * 32 + lane) * PER;
          if constexpr (GATEUP) {
            t0[0] += src[2 * j];
            t1 += src[2 * j + 1];
          } else {
#pragma unroll
            for (int r = 0; r < PR; ++r) t0[r] += src[j * PR + r];
          }
        }
#pragma unroll
        for (int r = 0; r < PR; ++r) acc[j][r] = t0[r];
        acc2[j] = t1;
      }
      const int v = it.g * RPW + rs;
      const bool ok = v < a.nvrows;
      if constexpr (GATEUP) {
#pragma unroll
        for (int j = 0; j < NB; ++j) {
          const float hg = acc[j][0] + __shfl_xor_sync(0xffffffffu, acc[j][0], 16);
          const float hu = acc2[j] + __shfl_xor_sync(0xffffffffu, acc2[j], 16);
          float gv = 0.f;
          if (ok && j < nbv) gv = __fmul_rn(gelu_ref(hg), hu);
          if (half == 0 && ok && j < nbv) a.out[(size_t)slots[j] * a.ff + v] = gv;
          float t = (half == 0) ? gv : 0.f;
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
          if (lane == 0 && j < nbv) a.out_s16[(size_t)slots[j] * (a.ff / 16) + it.g] = t;
        }
      } else {
#pragma unroll
        for (int j = 0; j < NB; ++j)
#pragma unroll
          for (int r = 0; r < PR; ++r) {
            const float t = acc[j][r] + __shfl_xor_sync(0xffffffffu, acc[j][r], 16);
            if (half == 0 && ok && j < nbv) a.out[(size_t)slots[j] * a.dim + (size_t)v * PR + r] = t;
          }
      }
    }
  }
  if (!okw) {
    for (int q = consumed + 1; q < issued; ++q)
      if (!mbar_wait_bounded(&mybars[q % NS], (q / NS) & 1)) record_error(a.status, ERR_TIMEOUT_DRAIN);
  }
}

// ---------------------------------------------------------------- combine
// moeOutput = 0; for ki: moeOutput += (prob*downScale) * down  (saxpyInPlace,
// MutableFloatTensor.kt:61-66: product rounded, then added); then
// rmsnorm(post_ffw_norm_2) (Llama.kt:340-346) when a weight is given.
__global__ void __launch_bounds__(512) moe_combine_kernel(const float* __restrict__ D, const int32_t* __restrict__ idx,
                                                          const float* __restrict__ prob,
                                                          const float* __restrict__ down_scale,
                                                          const float* __restrict__ post_norm, float* __restrict__ out,
                                                          int dim, int K, float eps) {
  __shared__ float red[33];
  __shared__ float fw[kMaxUsed];
  const int t = blockIdx.x;
  grid_dep_wait();
  grid_dep_launch();
  if (threadIdx.x < K) {
    int e = idx[(size_t)t * K + threadIdx.x];
    fw[threadIdx.x] = __fmul_rn(prob[(size_t)t * K + threadIdx.x], down_scale[e]);
  }
  __syncthreads();
  float4* o = reinterpret_cast<float4*>(out + (size_t)t * dim);
  const int n4 = dim >> 2;
  float ss = 0.f;
  for (int i = threadIdx.x; i < n4; i += blockDim.x) {
    float4 d[kMaxUsed];
#pragma unroll
    for (int k = 0; k < kMaxUsed; ++k)
      if (k < K) d[k] = __ldg(reinterpret_cast<const float4*>(D + ((size_t)t * K + k) * dim) + i);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < kMaxUsed; ++k) {
      if (k < K) {
        acc.x = __fadd_rn(__fmul_rn(fw[k], d[k].x), acc.x);
        acc.y = __fadd_rn(__fmul_rn(fw[k], d[k].y), acc.y);
        acc.z = __fadd_rn(__fmul_rn(fw[k], d[k].z), acc.z);
        acc.w = __fadd_rn(__fmul_rn(fw[k], d[k].w), acc.w);
      }
    }
    o[i] = acc;
    ss = fmaf(acc.x, acc.x, fmaf(acc.y, acc.y, fmaf(acc.z, acc.z, fmaf(acc.w, acc.w, ss))));
  }
  if (post_norm == nullptr) return;
  ss = block_sum(ss, red);
  const float m = __fadd_rn(__fdiv_rn(ss, (float)dim), eps);
  const float sn = (float)(1.0 / sqrt((double)m));
  const float4* pn = reinterpret_cast<const float4*>(post_norm);
  for (int i = threadIdx.x; i < n4; i += blockDim.x) {
    float4 v = o[i];
    const float4 w = pn[i];
    v.x = __fmul_rn(w.x, __fmul_rn(sn, v.x));
    v.y = __fmul_rn(w.y, __fmul_rn(sn, v.y));
    v.z = __fmul_rn(w.z, __fmul_rn(sn, v.z));
    v.w = __fmul_rn(w.w, __fmul_rn(sn, v.w));
    o[i] = v;
  }
}

// Same arithmetic with the combined row held in registers between the sum and
// the post-norm (one write of the output instead of write + re-read +
// write): thread i owns float4 columns i, i + blockDim, ... (IT of them).
template <int IT>
__global__ void __launch_bounds__(512) moe_combine_reg_kernel(const float* __restrict__ D,
                                                              const int32_t* __restrict__ idx,
                                                              const float* __restrict__ prob,
                                                              const float* __restrict__ down_scale,
                                                              const float* __restrict__ post_norm,
                                                              float* __restrict__ out, int dim, int K, float eps) {
  __shared__ float red[33];
  __shared__ float fw[kMaxUsed];
  const int t = blockIdx.x;
  grid_dep_wait();
  grid_dep_launch();
  if (threadIdx.x < K) {
    const int e = idx[(size_t)t * K + threadIdx.x];
    fw[threadIdx.x] = __fmul_rn(prob[(size_t)t * K + threadIdx.x], down_scale[e]);
  }
  __syncthreads();
  const int n4 = dim >> 2;
  float4 acc[IT];
  float ss = 0.f;
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    const int i = threadIdx.x + it * blockDim.x;
    acc[it] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < n4) {
      for (int k0 = 0; k0 < K; k0 += 8) {  // eight rows in flight, summed in k order
        float4 d[8];
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (k0 + k < K) d[k] = __ldg(reinterpret_cast<const float4*>(D + ((size_t)t * K + k0 + k) * dim) + i);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if (k0 + k < K) {
            const float f = fw[k0 + k];
            acc[it].x = __fadd_rn(__fmul_rn(f, d[k].x), acc[it].x);
            acc[it].y = __fadd_rn(__fmul_rn(f, d[k].y), acc[it].y);
            acc[it].z = __fadd_rn(__fmul_rn(f, d[k].z), acc[it].z);
            acc[it].w = __fadd_rn(__fmul_rn(f, d[k].w), acc[it].w);
          }
        }
      }
      ss = fmaf(acc[it].x, acc[it].x, fmaf(acc[it].y, acc[it].y, fmaf(acc[it].z, acc[it].z,
                                                                      fmaf(acc[it].w, acc[it].w, ss))));
    }
  }
  float4* o = reinterpret_cast<float4*>(out + (size_t)t * dim);
  float sn = 1.f;
  if (post_norm != nullptr) {
    ss = block_sum(ss, red);
    const float m = __fadd_rn(__fdiv_rn(ss, (float)dim), eps);
    sn = (float)(1.0 / sqrt((double)m));
  }
  const float4* pn = reinterpret_cast<const float4*>(post_norm);
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    const int i = threadIdx.x + it * blockDim.x;
    if (i >= n4) continue;
    float4 v = acc[it];
    if (post_norm != nullptr) {
      const float4 w = pn[i];
      v.x = __fmul_rn(w.x, __fmul_rn(sn, v.x));
      v.y = __fmul_rn(w.y, __fmul_rn(sn, v.y));
      v.z = __fmul_rn(w.z, __fmul_rn(sn, v.z));
      v.w = __fmul_rn(w.w, __fmul_rn(sn, v.w));
    }
    o[i] = v;
  }
}

// ---------------------------------------------------------------- host side
// The CUDA error of the last failed expert-kernel launch on this thread (a
// launcher reads cudaGetLastError(), which clears it; callers report this).
static thread_local cudaError_t t_launch_err = cudaSuccess;
static int launch_status() {
  t_launch_err = cudaGetLastError();
  return t_launch_err == cudaSuccess ? 0 : -2;
}
static cudaError_t last_launch_err() {
  return t_launch_err != cudaSuccess ? t_launch_err : cudaErrorLaunchFailure;
}

struct MoeScratch {
  float *moe_in, *xr, *logits, *prob, *G, *D;
  float *moe_in_s16, *G_s16;  // per-16-column sums of moe_in rows and of G rows
  int32_t *idx, *offsets, *perm;
};

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

static size_t moe_scratch_bytes(int T, int dim, int E, int K, int ff) {
  size_t s = 0;
  s += align_up((size_t)T * dim * 4, 256) * 2;       // moe_in, xr
  s += align_up((size_t)T * E * 4, 256);             // logits
  s += align_up((size_t)T * K * 4, 256) * 3;         // prob, idx, perm
  s += align_up((size_t)(E + 1) * 4, 256);           // offsets
  s += align_up((size_t)T * K * ff * 4, 256);        // G
  s += align_up((size_t)T * K * dim * 4, 256);       // D
  s += align_up((size_t)T * (dim / 16) * 4, 256);    // moe_in_s16
  s += align_up((size_t)T * K * (ff / 16) * 4, 256); // G_s16
  return s;
}

static MoeScratch carve(uint8_t* base, int T, int dim, int E, int K, int ff) {
  MoeScratch m;
  size_t o = 0;
  auto take = [&](size_t b) {
    uint8_t* p = base + o;
    o += align_up(b, 256);
    return p;
  };
  m.moe_in = (float*)take((size_t)T * dim * 4);
  m.xr = (float*)take((size_t)T * dim * 4);
  m.logits = (float*)take((size_t)T * E * 4);
  m.prob = (float*)take((size_t)T * K * 4);
  m.idx = (int32_t*)take((size_t)T * K * 4);
  m.perm = (int32_t*)take((size_t)T * K * 4);
  m.offsets = (int32_t*)take((size_t)(E + 1) * 4);
  m.G = (float*)take((size_t)T * K * ff * 4);
  m.D = (float*)take((size_t)T * K * dim * 4);
  m.moe_in_s16 = (float*)take((size_t)T * (dim / 16) * 4);
  m.G_s16 = (float*)take((size_t)T * K * (ff / 16) * 4);
  return m;
}

// offsets[e] / perm for n_slots slots routed by idx[] to E buckets.  `work`
// holds ceil(n_slots / kPermChunk) * E ints (used when n_slots is large).
static void launch_permute(const int32_t* idx, int n_slots, int E, int32_t* offsets, int32_t* perm, int32_t* work,
                           cudaStream_t st) {
  if (n_slots <= 2 * kPermChunk) {
    moe_permute_kernel<<<1, 1024, 0, st>>>(idx, n_slots, E, offsets, perm);
  } else {
    const int nb = (n_slots + kPermChunk - 1) / kPermChunk;
    moe_perm_count_kernel<<<nb, 256, 0, st>>>(idx, n_slots, E, work);
    moe_perm_scan_kernel<<<1, kMaxExperts, 0, st>>>(work, nb, E, offsets);
    moe_perm_place_kernel<<<nb, 256, 0, st>>>(idx, n_slots, E, work, perm);
  }
}

// G4_PDL=0 launches the decode chain without programmatic dependent launch
static bool pdl_enabled() {
  const char* v = getenv("G4_PDL");
  return !(v && v[0] == '0');
}

// Launch with programmatic stream serialization: the grid may start while the
// previous grid in the stream is still running; the kernel's grid_dep_wait()
// orders it after that grid (kernels without the wait must not use this).
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), int grid, int block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((unsigned)block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Front of the layer, shared by every entry point: norms (prep), router
// logits, softmax + top-k, and the slot permutation.  The router's split-K
// partials and the permutation's chunk counts use the D buffer, which the
// expert products only write later.
static cudaError_t launch_front(g4_ctx* c, const g4_moe_weights* w, const float* x, const MoeScratch& m, int T,
                                bool want_s16, cudaStream_t st) {
  const int dim = w->dim, E = w->n_expert, K = w->n_used;
  if (T <= 8 && dim % 16 == 0 && dim <= 4 * 256 * kFrontMaxF4) {
    // one launch; its completion ticket is a context word that the last CTA resets
    return launch_pdl(moe_front_small_kernel, E, 256, 0, st, x, (const float*)w->pre_ffw_norm_2->d,
                      (const float*)w->gate_inp_scale->d, (const float*)w->gate_inp->d, m.moe_in, m.moe_in_s16,
                      m.logits, m.idx, m.prob, m.offsets, m.perm, c->ticket(), T, dim, E, K, w->eps);
  }
  moe_prep_kernel<<<T, row_threads(dim / 4), 0, st>>>(x, (const float*)w->pre_ffw_norm_2->d,
                                                      (const float*)w->gate_inp_scale->d, m.moe_in, m.xr,
                                                      want_s16 ? m.moe_in_s16 : nullptr, dim, w->eps);
  // D holds T*K*dim floats; the split-K router may use up to kRtMaxSplit*T*E of them
  int nsplit = 0;
  if ((long long)kRtMaxSplit * E <= (long long)K * dim)
    nsplit = launch_router((const float*)w->gate_inp->d, m.xr, m.logits, m.D, T, dim, E, c->dev.sms, st);
  else
    moe_router_small_kernel<<<dim3(E, (T + 7) / 8), 256, 0, st>>>((const float*)w->gate_inp->d, m.xr, m.logits, T,
                                                                  dim, E);
  moe_topk_kernel<<<(T + 7) / 8, 256, 0, st>>>(nsplit ? m.D : m.logits, nsplit ? nsplit : 1, T, E, K, m.idx,
                                               m.prob);
  launch_permute(m.idx, T * K, E, m.offsets, m.perm, reinterpret_cast<int32_t*>(m.D), st);
  return cudaGetLastError();
}

static cudaError_t launch_combine(const g4_moe_weights* w, const MoeScratch& m, float* out, int T, cudaStream_t st) {
  const int n4 = w->dim / 4, threads = row_threads(n4), iters = (n4 + threads - 1) / threads;
  const float* ds = (const float*)w->down_exps_scale->d;
  const float* pn = w->post_ffw_norm_2 ? (const float*)w->post_ffw_norm_2->d : nullptr;
  const float* D = m.D;
  const int32_t* idx = m.idx;
  const float* prob = m.prob;
  const int dim = w->dim, K = w->n_used;
  const float eps = w->eps;
  switch (iters) {
    case 1: return launch_pdl(moe_combine_reg_kernel<1>, T, threads, 0, st, D, idx, prob, ds, pn, out, dim, K, eps);
    case 2: return launch_pdl(moe_combine_reg_kernel<2>, T, threads, 0, st, D, idx, prob, ds, pn, out, dim, K, eps);
    case 3: return launch_pdl(moe_combine_reg_kernel<3>, T, threads, 0, st, D, idx, prob, ds, pn, out, dim, K, eps);
    case 4: return launch_pdl(moe_combine_reg_kernel<4>, T, threads, 0, st, D, idx, prob, ds, pn, out, dim, K, eps);
    default: return launch_pdl(moe_combine_kernel, T, threads, 0, st, D, idx, prob, ds, pn, out, dim, K, eps);
  }
}

using ExpertFn = void (*)(const ExpertArgs);

template <int FMT, bool GU, int PR>
static ExpertFn expert_fn(int nb) {
  if (nb >= 8) return moe_expert_kernel<FMT, GU, PR, 8, 8>;
  if (nb >= 4) return moe_expert_kernel<FMT, GU, PR, 4, 8>;
  if (nb >= 2) return moe_expert_kernel<FMT, GU, PR, 2, 8>;
  return moe_expert_kernel<FMT, GU, PR, 1, 8>;
}

template <bool GU, int PR>
static ExpertFn expert_fn_t(int type, int nb) {
  switch (type) {
    case Q8_0: return expert_fn<Q8_0, GU, PR>(nb);
    case Q4_K: return expert_fn<Q4_K, GU, PR>(nb);
    case Q6_K: return expert_fn<Q6_K, GU, PR>(nb);
    case BF16: return expert_fn<BF16, GU, PR>(nb);
    case F32: return expert_fn<F32, GU, PR>(nb);
  }
  return nullptr;
}

static ExpertFn select_expert(int type, bool gu, int pr, int nb) {
  if (gu) return expert_fn_t<true, 1>(type, nb);
  if (pr == 1) return expert_fn_t<false, 1>(type, nb);
  if (pr == 2) return expert_fn_t<false, 2>(type, nb);
  if (pr == 4) return expert_fn_t<false, 4>(type, nb);
  return nullptr;
}

static int gcd_i(int a, int b) {
  while (b) {
    int t = a % b;
    a = b;
    b = t;
  }
  return a;
}

static int launch_expert(g4_ctx* c, int type, bool gu, const uint8_t* w, const float* act, float* out,
                         const MoeScratch& m, int E, int K, int dim, int ff, int T, cudaStream_t st) {
  const int BS = block_size(type), TS = type_size(type);
  ExpertArgs a{};
  a.w = w;
  a.act = act;
  a.out = out;
  a.offsets = m.offsets;
  a.perm = m.perm;
  a.status = c->status;
  a.E = E;
  a.n_used = K;
  a.ff = ff;
  const int NCW = 8;
  if (gu) {
    a.rows_e = 2 * ff;
    a.cols = dim;
    a.pr = 1;
    if (dim % BS || dim % 16) return -1;
    a.vb = dim / BS * TS;
    if (a.vb % 2) return -1;
    a.units = dim / 16;
    a.tile_rows = NCW;
    a.tiles_e = (ff + NCW - 1) / NCW;
    a.region_bytes = (int)align_up((size_t)NCW * a.vb + 32, 128);
    a.stage_bytes = 2 * a.region_bytes;
    a.expert_elems = (long long)2 * ff * dim;
  } else {
    a.rows_e = dim;
    a.cols = ff;
    if (ff % 16) return -1;
    int pr = ff % BS == 0 ? 1 : BS / gcd_i(ff % BS, BS);
    if (pr != 1 && pr != 2 && pr != 4) return -1;
    if (dim % pr) return -1;
    a.pr = pr;
    a.vb = pr * ff / BS * TS;
    if (a.vb % 2) return -1;
    a.units = pr * ff / 16;
    a.tile_rows = NCW;
    a.tiles_e = (dim / pr + NCW - 1) / NCW;
    a.stage_bytes = (int)align_up((size_t)NCW * a.vb + 32, 128);
    a.expert_elems = (long long)dim * ff;
  }
  if (a.expert_elems % BS) return -1;
  // up to 4 stages, as many as fit in shared memory (wide BF16 / F32 rows take 2)
  const size_t fixed_smem = 64 + 4 * (2 * kMaxExperts + 8) + 128;
  a.nstages = 4;
  while (a.nstages > 2 && fixed_smem + (size_t)a.nstages * a.stage_bytes > c->dev.smem_optin) --a.nstages;
  if (fixed_smem + (size_t)a.nstages * a.stage_bytes > c->dev.smem_optin) return -1;
  // Token chunk: enough slots per expert on average -> wider chunks.
  int avg = (T * K + E - 1) / E;
  int nb = avg >= 8 ? 8 : avg >= 4 ? 4 : avg >= 2 ? 2 : 1;
  ExpertFn fn = select_expert(type, gu, a.pr, nb);
  if (!fn) return -1;
  size_t smem = fixed_smem + (size_t)a.nstages * a.stage_bytes;
  // kernel attributes and occupancy are queried once per (device, kernel, smem):
  // the shared-memory attribute is a per-device setting of the kernel
  static std::mutex occ_mu;
  static std::map<std::tuple<int, ExpertFn, size_t>, int> occ_cache;
  int occ = 1;
  {
    std::lock_guard<std::mutex> lk(occ_mu);
    auto key = std::make_tuple(c->dev.device, fn, smem);
    auto itc = occ_cache.find(key);
    if (itc == occ_cache.end()) {
      // per-kernel attribute: allow the device maximum, not just this launch's size
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c->dev.smem_optin);
      int o = 1;
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, fn, 32 * (NCW + 1), smem);
      cudaGetLastError();
      itc = occ_cache.emplace(key, o < 1 ? 1 : o).first;
    }
    occ = itc->second;
  }
  // Upper bound on items: every slot in its own chunk.
  long long max_items = (long long)std::min(T * K, E * ((T * K + nb - 1) / nb + 1)) * a.tiles_e;
  int grid = (int)std::min<long long>(max_items, (long long)c->dev.sms * occ);
  if (grid < 1) grid = 1;
  fn<<<grid, 32 * (NCW + 1), smem, st>>>(a);
  return launch_status();
}

// Q4_K for NB tokens on two-part int16 activations (quantize_x16 layout: xq[j]
// is token j's padded int16 row, xql[j] the remainders in units of 2^-16 of
// the scale, xsc[j] its per-32-column scales, xs16[j] its fp32 per-16-column
// sums), the dp2a form of blk_nb's Q4_K branch with fp32-level products.
template <int PR, int NB>
__device__ __forceinline__ void blk_q4k_nb_i16(const uint8_t* blk, int e0, int cols, const int16_t* const* xq,
                                               const int16_t* const* xql, const float* const* xsc,
                                               const float* const* xs16, int nbv, float (&acc)[NB][PR]) {
  const uint4 h = lds128(blk);
  const float d = f16_bits_to_f32((uint16_t)(h.x & 0xFFFFu));
  const float dmin = f16_bits_to_f32((uint16_t)(h.x >> 16));
  const uint32_t sc03 = h.y & 0x3F3F3F3Fu, mn03 = h.z & 0x3F3F3F3Fu;
  const uint32_t sc47 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
  const uint32_t mn47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int eg = e0 + 64 * g;
    const int col = PR == 1 ? eg : eg % cols;
    const int rr = PR == 1 ? 0 : eg / cols;
    const int xo = xq_at(col);
    const uint4 qa = lds128(blk + 16 + 32 * g), qb = lds128(blk + 32 + 32 * g);
    int alo[NB], ahi[NB], alo2[NB], ahi2[NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) alo[j] = ahi[j] = alo2[j] = ahi2[j] = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t w = k == 0 ? qa.x : k == 1 ? qa.y : k == 2 ? qa.z : k == 3 ? qa.w
                       : k == 4 ? qb.x : k == 5 ? qb.y : k == 6 ? qb.z : qb.w;
      const uint32_t lo = w & 0x0F0F0F0Fu, hi = w & 0xF0F0F0F0u;
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        if (j < nbv) {
          const uint2 xl = *reinterpret_cast<const uint2*>(xq[j] + xo + 4 * k);
          const uint2 xh = *reinterpret_cast<const uint2*>(xq[j] + xo + 32 + 4 * k);
          const uint2 yl = *reinterpret_cast<const uint2*>(xql[j] + xo + 4 * k);
          const uint2 yh = *reinterpret_cast<const uint2*>(xql[j] + xo + 32 + 4 * k);
          alo[j] = dp2a_lo_su(xl.x, lo, alo[j]);
          alo[j] = dp2a_hi_su(xl.y, lo, alo[j]);
          ahi[j] = dp2a_lo_su(xh.x, hi, ahi[j]);
          ahi[j] = dp2a_hi_su(xh.y, hi, ahi[j]);
          alo2[j] = dp2a_lo_su(yl.x, lo, alo2[j]);
          alo2[j] = dp2a_hi_su(yl.y, lo, alo2[j]);
          ahi2[j] = dp2a_lo_su(yh.x, hi, ahi2[j]);
          ahi2[j] = dp2a_hi_su(yh.y, hi, ahi2[j]);
        }
      }
    }
    const uint32_t scw = g < 2 ? sc03 : sc47, mnw = g < 2 ? mn03 : mn47;
    const int b0 = (2 * g) & 3;
    const float dsl = d * small_u2f((scw >> (8 * b0)) & 0xFFu), dsh = d * small_u2f((scw >> (8 * b0 + 8)) & 0xFFu);
    const float mn_lo = small_u2f((mnw >> (8 * b0)) & 0xFFu), mn_hi = small_u2f((mnw >> (8 * b0 + 8)) & 0xFFu);
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      if (j < nbv) {
        const float* q = xs16[j] + col / 16;
        const float xlo = q[0] + q[1], xhi = q[2] + q[3];
        const float s_lo = xsc[j][col / 32], s_hi = xsc[j][col / 32 + 1] * 0.0625f;
        const float flo = fmaf((float)alo2[j], kLoScale, (float)alo[j]);
        const float fhi = fmaf((float)ahi2[j], kLoScale, (float)ahi[j]);
        float v = dsl * (s_lo * flo);
        v = fmaf(dsh, s_hi * fhi, v);
        v = fmaf(-dmin, fmaf(mn_lo, xlo, mn_hi * xhi), v);
        add_row<PR>(acc[j], rr, v);
      }
    }
  }
}

// ---------------------------------------------------------------- decode batches
// T <= 2 tokens (at most 2K routed slots): the expert products as one wave of
// CTAs, one per SM.  The work is the list of units (expert e, token chunk of up
// to NB = T slots, row v) in expert-major order with v fastest, so a CTA's
// contiguous share of it is a few contiguous byte ranges of weights.  The CTA
// streams its share through a ring of NS stages (one bulk copy per physical
// row, issued as far ahead as the ring allows) and all its warps decode a
// stage together: task (block b, physical row r) in block-major order, so the
// lanes of a warp read the same activation columns (shared-memory broadcasts)
// and distinct rows' blocks.  Per-task partial sums go to shared memory; each
// unit then adds its blocks in block order (fixed order: deterministic).
//   GATEUP: physical rows of a unit = gate row v and up row ff+v of expert e;
//           G[slot][v] = gelu(gate) * up (Llama.kt:316-322).
//   DOWN:   one virtual row (PR real rows of the [dim, ff] matrix) per unit;
//           D[slot][v*PR + r].  The per-16-column sums of the staged G rows
//           are made here.
constexpr int kDecHeadInts = kMaxExperts + 4;  // s_units, s_off
constexpr int kDecMaxSlots = 2 * kMaxUsed;      // T <= 2
constexpr int kDecHeadBytes = 4 * (2 * kDecHeadInts + kDecMaxSlots);

struct DecArgs {
  const uint8_t* w;
  const float* act;      // GATEUP: moe_in [T][cols]; DOWN: G [T*K][cols]
  const float* act_s16;  // GATEUP: moe_in_s16 [T][cols/16]; DOWN: unused
  float* out;            // GATEUP: G [slots][ff]; DOWN: D [slots][dim]
  const int32_t* offsets;
  const int32_t* perm;
  unsigned* status;
  int E, n_used, ff, dim;
  int cols, nvrows, bpv;
  int act_rows;          // activation rows staged (GATEUP: T; DOWN: T*K)
  int rs, ns, pitch;     // units per stage, ring stages, bytes per physical row slot
  int stage_bytes;
  int tab_at, red_at, act_at, s16_at, ring_at;  // shared-memory layout (bytes)
  int xq_at_, xql_at, xsc_at, xq_stride;        // Q4_K: two-part int16 activations (padded rows), per-32 scales
  int red_stride;        // floats of one of the two partial-sum buffers
  int n_slots;           // T * n_used
  long long expert_elems;
  // GATEUP only: the down product's weights, prefetched into L2 for the down
  // kernel's CTA with the same index (nullptr: none)
  const uint8_t* pf_w;
  int pf_nvrows, pf_grid;
  long long pf_row_bytes, pf_expert_bytes;
};

struct DecUnit {
  int v, nbv;
  int arow[2];  // activation row of each token (GATEUP: its token; DOWN: its slot)
  int slot[2];  // output row (slot)
  int off[2];   // offset of each physical row's first byte in its ring row
};

template <int FMT, bool GATEUP, int PR, int NB>
__global__ void __launch_bounds__(512, 1) moe_dec_kernel(const __grid_constant__ DecArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int BS = block_size(FMT), TS = type_size(FMT);
  constexpr int PHYS = GATEUP ? 2 : 1;
  int* s_units = reinterpret_cast<int*>(smem);  // [E+1] first unit of each expert
  int* s_off = s_units + kDecHeadInts;           // [E+1] copy of offsets
  int* s_perm = s_off + kDecHeadInts;            // [n_slots] copy of perm
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kDecHeadBytes);  // [ns] stages, [1] activations
  DecUnit* tab = reinterpret_cast<DecUnit*>(smem + a.tab_at);          // [2 ns][rs]
  float* red = reinterpret_cast<float*>(smem + a.red_at);              // [2][red_stride]
  float* s_act = reinterpret_cast<float*>(smem + a.act_at);            // [act_rows][cols]
  float* s_s16 = reinterpret_cast<float*>(smem + a.s16_at);            // [act_rows][cols/16]
  int16_t* s_xq = reinterpret_cast<int16_t*>(smem + a.xq_at_);         // Q4_K: [act_rows][xq_stride]
  int16_t* s_xql = reinterpret_cast<int16_t*>(smem + a.xql_at);        // Q4_K: remainders, same layout
  float* s_xsc = reinterpret_cast<float*>(smem + a.xsc_at);            // Q4_K: [act_rows][cols/32]
  uint8_t* ring = smem + a.ring_at;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x;
  const int NS = a.ns, RS = a.rs, c16 = a.cols / 16;
  uint64_t* act_bar = bars + NS;

  if (tid <= NS) mbar_init(&bars[tid], 1);
  if (tid == 0) fence_barrier_init();
  // GATEUP waits for the front (offsets, perm, moe_in) and only then lets the
  // down grid launch, so the down grid may read offsets/perm and fetch its
  // weights before its own wait, which guards only G.
  if (GATEUP) {
    grid_dep_wait();
    grid_dep_launch();
  }
  // offsets and perm into shared memory (one round trip for all threads)
  for (int i = tid; i <= a.E; i += nthr) s_off[i] = a.offsets[i];
  for (int i = tid; i < a.n_slots; i += nthr) s_perm[i] = a.perm[i];
  __syncthreads();
  if (warp == 0) {  // units per expert: ceil(n_e / NB) token chunks x nvrows rows
    int carry = 0;
    for (int base = 0; base < a.E; base += 32) {
      const int e = base + lane;
      const int v = e < a.E ? (s_off[e + 1] - s_off[e] + NB - 1) / NB * a.nvrows : 0;
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
      }
      if (e < a.E) s_units[e] = carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) s_units[a.E] = carry;
  }
  __syncthreads();
  const int U = s_units[a.E];
  const int u0 = (int)((long long)U * blockIdx.x / gridDim.x);
  const int u1 = (int)((long long)U * (blockIdx.x + 1) / gridDim.x);
  const int nst = (u1 - u0 + RS - 1) / RS;
  if (nst == 0) {
    if (!GATEUP) {
      grid_dep_wait();
      grid_dep_launch();
    }
    return;
  }

  // stage s of this CTA: ring slot s % NS, unit table s % (2 NS) (the epilogue
  // of stage s still reads its table while stage s + NS is being issued)
  auto issue = [&](int s) {
    const int slot = s % NS;
    DecUnit* tb = tab + (size_t)(s % (2 * NS)) * RS;
    uint8_t* sbase = ring + (size_t)slot * a.stage_bytes;
    const int us = u0 + s * RS, nu = min(RS, u1 - us);
    uint32_t mine = 0;
    for (int i = lane; i < nu; i += 32) {
      const int u = us + i;
      int lo = 0, hi = a.E - 1;  // last expert whose first unit is <= u (never an empty one)
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_units[mid] <= u) lo = mid;
        else hi = mid - 1;
      }
      const int e = lo, local = u - s_units[e];
      const int k = local / a.nvrows, v = local - k * a.nvrows;
      const int p0 = s_off[e] + k * NB;
      DecUnit d;
      d.v = v;
      d.nbv = min(NB, s_off[e + 1] - p0);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int sl = (j < NB && j < d.nbv) ? s_perm[p0 + j] : s_perm[p0];
        d.slot[j] = sl;
        d.arow[j] = GATEUP ? sl / a.n_used : sl;
      }
      const long long eb = (long long)e * a.expert_elems / BS;  // expert's first block
#pragma unroll
      for (int ph = 0; ph < PHYS; ++ph) {
        const long long row = GATEUP ? (ph ? (long long)a.ff + v : (long long)v) : (long long)v;
        const long long start = (eb + row * a.bpv) * TS;
        const long long a0 = start & ~15ll, a1 = (start + (long long)a.bpv * TS + 15) & ~15ll;
        d.off[ph] = (int)(start & 15);
        bulk_g2s(sbase + (size_t)(ph * nu + i) * a.pitch, a.w + a0, (uint32_t)(a1 - a0), &bars[slot]);
        mine += (uint32_t)(a1 - a0);
      }
      if (PHYS == 1) d.off[1] = 0;
      tb[i] = d;
    }
    const uint32_t total = __reduce_add_sync(0xffffffffu, mine);
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      mbar_arrive_expect_tx(&bars[slot], total);
    }
  };

  if (warp == 0)
    for (int s = 0; s < NS && s < nst; ++s) issue(s);
  if (!GATEUP) {  // G is the previous grid's output
    grid_dep_wait();
    grid_dep_launch();
  }
  if (tid == 32) {  // activations, once (warp 1)
    const uint32_t ab = (uint32_t)a.act_rows * (uint32_t)a.cols * 4u;
    const uint32_t sb = GATEUP ? (uint32_t)a.act_rows * (uint32_t)c16 * 4u : 0u;
    mbar_arrive_expect_tx(act_bar, ab + sb);
    bulk_g2s(s_act, a.act, ab, act_bar);
    if (GATEUP) bulk_g2s(s_s16, a.act_s16, sb, act_bar);
  }
  if (GATEUP && a.pf_w && tid == 64 && (int)blockIdx.x < a.pf_grid) {
    // L2 prefetch of the down rows that down CTA blockIdx.x will read.  With
    // NB = T every routed expert has one token chunk, so down unit u is row
    // u % pf_nvrows of the (u / pf_nvrows)-th routed expert.
    const int Ud = U / a.nvrows * a.pf_nvrows;
    const int d0 = (int)((long long)Ud * blockIdx.x / a.pf_grid);
    const int d1 = (int)((long long)Ud * (blockIdx.x + 1) / a.pf_grid);
    for (int r = d0 / a.pf_nvrows; d0 < d1 && r <= (d1 - 1) / a.pf_nvrows; ++r) {
      int lo = 0, hi = a.E - 1;  // the expert whose units start at r * nvrows
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_units[mid] <= r * a.nvrows) lo = mid;
        else hi = mid - 1;
      }
      const int v0 = max(d0, r * a.pf_nvrows) - r * a.pf_nvrows;
      const int v1 = min(d1, (r + 1) * a.pf_nvrows) - r * a.pf_nvrows;
      const long long b0 = (long long)lo * a.pf_expert_bytes + v0 * a.pf_row_bytes;
      const long long b1 = (long long)lo * a.pf_expert_bytes + v1 * a.pf_row_bytes;
      const long long p0 = b0 & ~15ll, p1 = (b1 + 15) & ~15ll;
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.pf_w + p0), "r"((uint32_t)(p1 - p0))
                   : "memory");
    }
  }

  bool ok = mbar_wait_bounded(act_bar, 0);
  if (!GATEUP && ok) {
    for (int i = tid; i < a.act_rows * c16; i += nthr) {
      const float* q = s_act + (size_t)(i / c16) * a.cols + 16 * (i % c16);
      float t = 0.f;
#pragma unroll
      for (int k = 0; k < 16; ++k) t += q[k];
      s_s16[i] = t;
    }
  }
  int s = 0;
  if (FMT == Q4_K && ok) {
    // int16 activations per 32 columns (see quantize_x16), one warp per block
    const int c32 = a.cols / 32, W = nthr >> 5;
    for (int bk = warp; bk < a.act_rows * c32; bk += W) {
      const int r = bk / c32, b = bk - r * c32;
      const float v = s_act[(size_t)r * a.cols + 32 * b + lane];
      float m = fabsf(v);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const uint32_t t = __float_as_uint(m * (1.0f / 32760.0f));
      uint32_t e = t & 0x7F800000u;
      if (t & 0x007FFFFFu) e += 0x00800000u;
      const bool nz = m > 0.f && e != 0u;
      const float inv = nz ? __uint_as_float(0x7F000000u - e) : 1.0f;
      const float f = v * inv;  // exact (power of two)
      const float fq = rintf(f);
      const int lo = __float2int_rn(__fmul_rn(__fsub_rn(f, fq), 65536.0f));  // remainder, units of 2^-16
      const size_t xo = (size_t)r * a.xq_stride + xq_at(32 * b + lane);
      s_xq[xo] = (int16_t)__float2int_rn(fq);
      s_xql[xo] = (int16_t)max(-32767, min(32767, lo));
      if (lane == 0) s_xsc[(size_t)r * c32 + b] = nz ? __uint_as_float(e) : 1.0f;
    }
  }
  if (!__syncthreads_and(ok)) {
    if (tid == 0) record_error(a.status, ERR_TIMEOUT_FULL);
  } else {
    for (; s < nst; ++s) {
      const int slot = s % NS;
      const DecUnit* tb = tab + (size_t)(s % (2 * NS)) * RS;
      const int us = u0 + s * RS, nu = min(RS, u1 - us);
      const int prow = PHYS * nu, ntask = prow * a.bpv;
      float* rb = red + (size_t)(s & 1) * a.red_stride;
      const uint8_t* sbase = ring + (size_t)slot * a.stage_bytes;
      const bool okw = mbar_wait_bounded(&bars[slot], (s / NS) & 1);
      if (okw) {
        for (int t = tid; t < ntask; t += nthr) {
          const int b = t / prow, r = t - b * prow;
          const int ph = (PHYS == 2 && r >= nu) ? 1 : 0;
          const DecUnit& d = tb[r - ph * nu];
          const float* xr[NB];
          const float* xs16[NB];
#pragma unroll
          for (int j = 0; j < NB; ++j) {
            xr[j] = s_act + (size_t)d.arow[j] * a.cols;
            xs16[j] = s_s16 + (size_t)d.arow[j] * c16;
          }
          float acc[NB][PR];
#pragma unroll
          for (int j = 0; j < NB; ++j)
#pragma unroll
            for (int q = 0; q < PR; ++q) acc[j][q] = 0.f;
          const uint8_t* blk = sbase + (size_t)r * a.pitch + d.off[ph] + (size_t)b * TS;
          if constexpr (FMT == Q4_K) {
            const int16_t* xq[NB];
            const int16_t* xql[NB];
            const float* xsc[NB];
#pragma unroll
            for (int j = 0; j < NB; ++j) {
              xq[j] = s_xq + (size_t)d.arow[j] * a.xq_stride;
              xql[j] = s_xql + (size_t)d.arow[j] * a.xq_stride;
              xsc[j] = s_xsc + (size_t)d.arow[j] * (a.cols / 32);
            }
            blk_q4k_nb_i16<PR, NB>(blk, b * BS, a.cols, xq, xql, xsc, xs16, d.nbv, acc);
          } else {
            blk_nb<FMT, PR, NB>(blk, b * BS, a.cols, xr, xs16, 0, d.nbv, acc);
          }
          float* o = rb + (size_t)t * (NB * PR);
#pragma unroll
          for (int j = 0; j < NB; ++j)
#pragma unroll
            for (int q = 0; q < PR; ++q) o[j * PR + q] = acc[j][q];
        }
      }
      // the ring slot is read: order those reads before the bulk copies that refill it
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      if (__syncthreads_or(!okw)) {
        if (tid == 0) record_error(a.status, ERR_TIMEOUT_FULL);
        break;
      }
      if (warp == 0 && s + NS < nst) issue(s + NS);
      // unit results: blocks added in block order (the last threads, away from the issuing warp)
      for (int q = nthr - 1 - tid; q < nu * NB; q += nthr) {
        const int i = q / NB, j = q - (q / NB) * NB;
        const DecUnit& d = tb[i];
        if (j >= d.nbv) continue;
        if constexpr (GATEUP) {
          float g = 0.f, up = 0.f;
          for (int b = 0; b < a.bpv; ++b) {
            g += rb[((size_t)b * prow + i) * NB + j];
            up += rb[((size_t)b * prow + nu + i) * NB + j];
          }
          a.out[(size_t)d.slot[j] * a.ff + d.v] = __fmul_rn(gelu_ref(g), up);
        } else {
#pragma unroll
          for (int q2 = 0; q2 < PR; ++q2) {
            float sum = 0.f;
            for (int b = 0; b < a.bpv; ++b) sum += rb[((size_t)b * prow + i) * (NB * PR) + j * PR + q2];
            a.out[(size_t)d.slot[j] * a.dim + (size_t)d.v * PR + q2] = sum;
          }
        }
      }
    }
  }
  if (s < nst && warp == 0) {
    // stopped early: wait (bounded) for the copies still in flight before the CTA exits
    const int issued = min(nst, s + NS);
    for (int q = s; q < issued; ++q)
      if (!mbar_wait_bounded(&bars[q % NS], (q / NS) & 1)) record_error(a.status, ERR_TIMEOUT_DRAIN);
  }
}

using RowsFn = void (*)(const RowsArgs);

template <int FMT, bool GU, int PR>
static RowsFn rows_fn_nb(int nb) {
  if (nb >= 8) return moe_rows_kernel<FMT, GU, PR, 8>;
  if (nb >= 4) return moe_rows_kernel<FMT, GU, PR, 4>;
  if (nb >= 2) return moe_rows_kernel<FMT, GU, PR, 2>;
  return moe_rows_kernel<FMT, GU, PR, 1>;
}

static RowsFn rows_fn(int type, bool gu, int pr, int nb) {
  if (gu) {
    if (type == Q4_K) return rows_fn_nb<Q4_K, true, 1>(nb);
    if (type == Q6_K) return rows_fn_nb<Q6_K, true, 1>(nb);
    if (type == Q8_0) return rows_fn_nb<Q8_0, true, 1>(nb);
    return nullptr;
  }
  if (type == Q8_0) return pr == 1 ? rows_fn_nb<Q8_0, false, 1>(nb) : nullptr;
  if (type == Q4_K) {
    if (pr == 1) return rows_fn_nb<Q4_K, false, 1>(nb);
    if (pr == 2) return rows_fn_nb<Q4_K, false, 2>(nb);
    if (pr == 4) return rows_fn_nb<Q4_K, false, 4>(std::min(nb, 4));
  }
  if (type == Q6_K) {
    if (pr == 1) return rows_fn_nb<Q6_K, false, 1>(nb);
    if (pr == 2) return rows_fn_nb<Q6_K, false, 2>(nb);
    if (pr == 4) return rows_fn_nb<Q6_K, false, 4>(std::min(nb, 4));
  }
  return nullptr;
}

static int rows_pitch(int bytes) {
  int p = (bytes + 15) / 16;
  if ((p & 1) == 0) ++p;
  return 16 * p;
}

// Kernel set-up (smem attribute + occupancy) cached per kernel; the no-alloc
// path keeps its own fixed table so it never touches the heap.
static int rows_occ(RowsFn fn, size_t smem, int threads, int optin, bool noalloc_path);

// Returns 0, -1 when the layout needs the generic expert kernel, -2 on a launch error.
static int launch_expert_rows(g4_ctx* c, int type, bool gu, const uint8_t* w, const float* act, const float* act_s16,
                              float* out, float* out_s16, const MoeScratch& m, int E, int K, int dim, int ff, int T,
                              cudaStream_t st, bool noalloc_path) {
  if (type != Q4_K && type != Q6_K && type != Q8_0) return -1;
  const int BS = block_size(type), TS = type_size(type);
  RowsArgs a{};
  a.w = w;
  a.act = act;
  a.act_s16 = act_s16;
  a.out = out;
  a.out_s16 = out_s16;
  a.offsets = m.offsets;
  a.perm = m.perm;
  a.status = c->status;
  a.E = E;
  a.n_used = K;
  a.ff = ff;
  a.dim = dim;
  int pr = 1;
  if (gu) {
    if (dim % BS || dim % 64 || ff % 16) return -1;
    a.cols = dim;
    a.nvrows = ff;
    a.bpv = dim / BS;
    a.expert_elems = (long long)2 * ff * dim;
  } else {
    if (ff % 64) return -1;
    if (ff % BS) {
      if (type == Q8_0) return -1;
      int g = ff % BS, b = BS;
      while (b) {
        int t = g % b;
        g = b;
        b = t;
      }
      pr = BS / g;
      if (pr != 2 && pr != 4) return -1;
    }
    if (dim % pr) return -1;
    a.cols = ff;
    a.nvrows = dim / pr;
    a.bpv = pr * ff / BS;
    a.expert_elems = (long long)dim * ff;
  }
  if (a.expert_elems % BS) return -1;
  a.ngroups = (a.nvrows + 15) / 16;
  // about 288-560 bytes of a row per bulk copy, an even number of blocks (two lanes per row)
  int cb = type == Q4_K ? 2 : type == Q6_K ? 2 : 8;
  cb = std::min(cb, (a.bpv + 1) / 2 * 2);
  a.cb = std::max(2, cb);
  a.nchunks = (a.bpv + a.cb - 1) / a.cb;
  a.pitch = rows_pitch(a.cb * TS + 32);
  const int slots = gu ? 32 : 16;
  const int optin = (int)c->dev.smem_optin;
  const size_t head = 8 * (kMaxExperts + 8);
  const int avg = (T * K + E - 1) / E;
  // Wide token tiles belong to the tensor-core / generic kernels: this one
  // re-reads each token's activations per row, which only pays for <= 2.
  if (avg > 2) return -1;
  const int nb = avg >= 2 ? 2 : 1;
  // stage = weight row slots, then each token's activations for the stage and
  // their per-16-column sums
  a.xcols = gu ? a.cb * BS : a.cols;
  a.xs16n = ((a.xcols / 16) + 3) / 4 * 4;
  a.x_at = slots * a.pitch;
  a.xs_at = a.x_at + nb * a.xcols * 4;
  a.stage_bytes = (int)align_up((size_t)a.xs_at + (size_t)nb * a.xs16n * 4, 128);
  const size_t stage = (size_t)a.stage_bytes;
  // warps per CTA from the amount of work, so that every SM gets some
  // Upper bound on items: sum over experts of ceil(n_e / nb) token chunks is
  // at most (T*K + (nb - 1) * experts used) / nb, times the row groups.
  const long long tk = (long long)T * K;
  const long long max_items = ((tk + (long long)(nb - 1) * std::min(tk, (long long)E) + nb - 1) / nb) * a.ngroups;
  auto need = [&](int wv, int ns) { return head + 128 * ((wv * ns * 8 + 127) / 128) + (size_t)wv * ns * stage; };
  int warps;
  // Few items (small batches): one CTA per item, its warps split the chunks,
  // so that enough lanes stream weights at once.  Otherwise warps own items.
  const bool split = max_items < 8LL * c->dev.sms;
  if (split) {
    a.split = std::min(a.nchunks, 8);
    warps = a.split;
    // as many stages as a warp has chunks (up to 4): no idle ring slots, so
    // that more CTAs fit on an SM
    a.ns = 1;
    while (a.ns < 4 && a.ns * a.split < a.nchunks && need(warps, a.ns + 1) <= (size_t)optin) ++a.ns;
  } else {
    a.split = 1;
    warps = (int)std::min<long long>(16, std::max<long long>(1, (max_items + c->dev.sms - 1) / c->dev.sms));
    // deepest ring (up to 6 stages) that fits; fewer warps per SM leave room for more stages
    a.ns = 6;
    while (a.ns > 2 && need(warps, a.ns) > (size_t)optin) --a.ns;
    while (warps > 1 && need(warps, a.ns) > (size_t)optin) --warps;
  }
  if (need(warps, a.ns) > (size_t)optin) return -1;
  const size_t smem = need(warps, a.ns);
  RowsFn fn = rows_fn(type, gu, pr, nb);
  if (!fn) return -1;
  const int occ = rows_occ(fn, smem, 32 * warps, optin, noalloc_path);
  if (occ < 1) {
    t_launch_err = cudaErrorInvalidConfiguration;
    return -2;
  }
  const int grid = split ? (int)max_items
                         : (int)std::max<long long>(1, std::min<long long>((max_items + warps - 1) / warps,
                                                                           (long long)c->dev.sms * occ));
  fn<<<grid, 32 * warps, smem, st>>>(a);
  return launch_status();
}

// ---------------------------------------------------------------- decode launch
using DecFn = void (*)(const DecArgs);

template <int FMT, bool GU, int PR>
static DecFn dec_fn_nb(int nb) {
  return nb == 2 ? moe_dec_kernel<FMT, GU, PR, 2> : moe_dec_kernel<FMT, GU, PR, 1>;
}

static DecFn dec_fn(int type, bool gu, int pr, int nb) {
  if (type == Q4_K) {
    if (gu) return dec_fn_nb<Q4_K, true, 1>(nb);
    return pr == 1 ? dec_fn_nb<Q4_K, false, 1>(nb) : pr == 2 ? dec_fn_nb<Q4_K, false, 2>(nb)
                                                             : dec_fn_nb<Q4_K, false, 4>(nb);
  }
  if (type == Q6_K) {
    if (gu) return dec_fn_nb<Q6_K, true, 1>(nb);
    return pr == 1 ? dec_fn_nb<Q6_K, false, 1>(nb) : pr == 2 ? dec_fn_nb<Q6_K, false, 2>(nb)
                                                             : dec_fn_nb<Q6_K, false, 4>(nb);
  }
  if (type == Q8_0 && pr == 1) return gu ? dec_fn_nb<Q8_0, true, 1>(nb) : dec_fn_nb<Q8_0, false, 1>(nb);
  return nullptr;
}

// Geometry and shared-memory layout of one decode product; false when the
// decode kernels do not handle it (the caller then takes the other kernels).
static bool dec_plan(const g4_ctx* c, int type, bool gu, int E, int K, int dim, int ff, int T, int per_sm,
                     DecArgs& a, int& grid, int& threads, size_t& smem, int& pr) {
  if (type != Q4_K && type != Q6_K && type != Q8_0) return false;
  if (T < 1 || T > 2 || E > kMaxExperts || K > kMaxUsed) return false;
  const int BS = block_size(type), TS = type_size(type);
  a = DecArgs{};
  a.E = E;
  a.n_used = K;
  a.ff = ff;
  a.dim = dim;
  a.n_slots = T * K;
  pr = 1;
  if (gu) {
    if (dim % BS || dim % 64) return false;
    a.cols = dim;
    a.nvrows = ff;
    a.bpv = dim / BS;
    a.expert_elems = 2LL * ff * dim;
    a.act_rows = T;
  } else {
    if (ff % 64) return false;
    if (ff % BS) {
      if (type == Q8_0) return false;
      int g = ff % BS, b = BS;
      while (b) {
        const int t = g % b;
        g = b;
        b = t;
      }
      pr = BS / g;
      if (pr != 2 && pr != 4) return false;
    }
    if (dim % pr) return false;
    a.cols = ff;
    a.nvrows = dim / pr;
    a.bpv = pr * ff / BS;
    a.expert_elems = (long long)dim * ff;
    a.act_rows = T * K;
  }
  if (a.expert_elems % BS) return false;
  const int PHYS = gu ? 2 : 1, NB = T;
  a.pitch = rows_pitch(a.bpv * TS + 32);
  a.xq_stride = (a.cols + 8 * ((a.cols + 255) / 256) + 3) / 4 * 4;  // padded int16 row, 8-byte multiple
  // NB = T covers every expert's slots in one chunk (a token picks an expert once)
  const long long units_max = std::min((long long)T * K, (long long)E) * a.nvrows;
  // per_sm CTAs of 512 / per_sm threads on each SM: their stages interleave
  threads = 512 / per_sm;
  grid = (int)std::min<long long>((long long)c->dev.sms * per_sm, units_max);
  const long long share = (units_max + grid - 1) / grid;
  // about one block per thread per stage (four for 32-weight blocks), at most
  // 96 KB of rows per SM and stage
  int rs = std::max(1, (BS == 32 ? 4 : 1) * threads / (PHYS * a.bpv));
  rs = std::min(rs, std::max(1, 96 * 1024 / per_sm / (PHYS * a.pitch)));
  rs = (int)std::max<long long>(1, std::min<long long>(rs, share));
  int ns = (int)std::min<long long>(4, (share + rs - 1) / rs);
  auto layout = [&](int rs_, int ns_) {
    size_t o = kDecHeadBytes + 8 * (size_t)(ns_ + 1);
    o = align_up(o, 16);
    a.tab_at = (int)o;
    o += (size_t)2 * ns_ * rs_ * sizeof(DecUnit);
    o = align_up(o, 16);
    a.red_at = (int)o;
    a.red_stride = rs_ * PHYS * a.bpv * NB * pr;
    o += (size_t)2 * a.red_stride * 4;
    o = align_up(o, 128);
    a.act_at = (int)o;
    o += (size_t)a.act_rows * a.cols * 4;
    o = align_up(o, 16);
    a.s16_at = (int)o;
    o += (size_t)a.act_rows * (a.cols / 16) * 4;
    o = align_up(o, 16);
    a.xq_at_ = (int)o;
    o += type == Q4_K ? (size_t)a.act_rows * a.xq_stride * 2 : 0;
    o = align_up(o, 16);
    a.xql_at = (int)o;
    o += type == Q4_K ? (size_t)a.act_rows * a.xq_stride * 2 : 0;
    o = align_up(o, 16);
    a.xsc_at = (int)o;
    o += type == Q4_K ? (size_t)a.act_rows * (a.cols / 32) * 4 : 0;
    o = align_up(o, 128);
    a.ring_at = (int)o;
    a.stage_bytes = (int)align_up((size_t)rs_ * PHYS * a.pitch, 128);
    return o + (size_t)ns_ * a.stage_bytes;
  };
  // the SM's shared memory (the opt-in limit plus the 1 KB each CTA reserves) split over per_sm CTAs
  const size_t optin = std::min<size_t>(c->dev.smem_optin, (c->dev.smem_optin + 1024) / per_sm - 1024);
  smem = layout(rs, ns);
  while (smem > optin && ns > 2) smem = layout(rs, --ns);
  while (smem > optin && rs > 1) smem = layout(--rs, ns);
  if (smem > optin) return false;
  a.rs = rs;
  a.ns = ns;
  return true;
}

// CTAs per SM of the decode kernels (512 / this many threads each)
constexpr int kDecCtasPerSm = 1;

// Fixed table of (device, decode kernel) pairs whose shared-memory limit was
// raised (no heap use; the attribute is set per device).
static bool dec_prepare(DecFn fn, int optin, int device) {
  static std::mutex mu;
  struct Done {
    DecFn fn;
    int device;
  };
  static Done done[64];
  static int n = 0;
  std::lock_guard<std::mutex> lk(mu);
  for (int i = 0; i < n; ++i)
    if (done[i].fn == fn && done[i].device == device) return true;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, optin) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (n < 64) done[n++] = Done{fn, device};
  return true;
}

// Largest batch the decode kernels take: 1 by default (at T = 2 the rows
// kernels are faster on B200); G4_MOE_DEC=0 turns them off and G4_MOE_DEC=1
// uses them up to T = 2 (read at every call).
static int dec_max_tokens() {
  const char* v = getenv("G4_MOE_DEC");
  if (v && v[0] == '0') return 0;
  if (v && v[0] == '1') return 2;
  return 1;
}

// Both expert products of a decode batch (T <= dec_max_tokens()) on the decode kernels.
// Returns 0 when launched, -1 when they do not apply (nothing launched), -2 on
// a launch error.
static int launch_dec_pair(g4_ctx* c, const g4_moe_weights* w, const MoeScratch& m, int E, int K, int dim, int ff,
                           int T, cudaStream_t st) {
  if (T > dec_max_tokens()) return -1;
  DecArgs ga, da;
  int gg = 0, dg = 0, gt = 0, dt_ = 0, gpr = 1, dpr = 1;
  size_t gs = 0, ds = 0;
  const int per_sm = kDecCtasPerSm;
  if (!dec_plan(c, w->gate_up_exps->type, true, E, K, dim, ff, T, per_sm, ga, gg, gt, gs, gpr) ||
      !dec_plan(c, w->down_exps->type, false, E, K, dim, ff, T, per_sm, da, dg, dt_, ds, dpr))
    return -1;
  const DecFn gf = dec_fn(w->gate_up_exps->type, true, 1, T), df = dec_fn(w->down_exps->type, false, dpr, T);
  if (!gf || !df) return -1;
  const int optin = (int)c->dev.smem_optin;
  if (!dec_prepare(gf, optin, c->dev.device) || !dec_prepare(df, optin, c->dev.device)) return -1;
  ga.w = (const uint8_t*)w->gate_up_exps->d;
  ga.act = m.moe_in;
  ga.act_s16 = m.moe_in_s16;
  ga.out = m.G;
  da.w = (const uint8_t*)w->down_exps->d;
  da.act = m.G;
  da.act_s16 = nullptr;
  da.out = m.D;
  for (DecArgs* a : {&ga, &da}) {
    a->offsets = m.offsets;
    a->perm = m.perm;
    a->status = c->status;
  }
  const int dt = w->down_exps->type;
  ga.pf_w = da.w;
  ga.pf_nvrows = da.nvrows;
  ga.pf_grid = dg;
  ga.pf_row_bytes = (long long)da.bpv * type_size(dt);
  ga.pf_expert_bytes = da.expert_elems / block_size(dt) * type_size(dt);
  if (launch_pdl(gf, gg, gt, gs, st, ga) != cudaSuccess) return -2;
  if (launch_pdl(df, dg, dt_, ds, st, da) != cudaSuccess) return -2;
  return 0;
}

static int tensor_ok(const g4_tensor* t, int type, uint64_t n) {
  return t && (type < 0 || t->type == type) && t->n_elems == n;
}

static int rows_occ_fixed(RowsFn fn, size_t smem, int threads, int optin);

// Kernel set-up per (device, kernel, smem): the shared-memory attribute is a
// per-device setting, so a process using several devices sets it on each.
static int rows_occ(RowsFn fn, size_t smem, int threads, int optin, bool noalloc_path) {
  if (noalloc_path) return rows_occ_fixed(fn, smem, threads, optin);
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  static std::mutex mu;
  static std::map<std::tuple<int, RowsFn, size_t>, int> cache;
  std::lock_guard<std::mutex> lk(mu);
  auto key = std::make_tuple(device, fn, smem);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int o = 0;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, optin) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, fn, threads, smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  cache.emplace(key, o);
  return o;
}

// fixed table for the no-alloc path (no heap use), keyed by device as well
static int rows_occ_fixed(RowsFn fn, size_t smem, int threads, int optin) {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  static std::mutex mu;
  struct E {
    RowsFn fn;
    size_t smem;
    int device;
    int occ;
  };
  static E tab[128];
  static int n = 0;
  std::lock_guard<std::mutex> lk(mu);
  for (int i = 0; i < n; ++i)
    if (tab[i].fn == fn && tab[i].smem == smem && tab[i].device == device) return tab[i].occ;
  int o = 0;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, optin) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, fn, threads, smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (n < 128) tab[n++] = E{fn, smem, device, o};
  return o;
}

}  // namespace g4

using namespace g4;

extern "C" int g4_moe_topk(g4_ctx* c, const float* logits, int T, int E, int K, int32_t* idx, float* prob,
                           void* stream) {
  if (!c) return G4_E_ARG;
  if (!logits || !idx || !prob || T < 0 || E < 1 || E > kMaxExperts || K < 1 || K > E || K > kMaxUsed) {
    c->set_err("g4_moe_topk: bad argument");
    return G4_E_ARG;
  }
  if (T == 0) return 0;
  if (int r = c->bind()) return r;
  moe_topk_kernel<<<(T + 7) / 8, 256, 0, (cudaStream_t)stream>>>(logits, 1, T, E, K, idx, prob);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : c->cuda_fail(e, "g4_moe_topk");
}

extern "C" int g4_moe_layer(g4_ctx* c, const g4_moe_weights* w, const float* x, float* out, int T,
                            int32_t* topk_idx, float* topk_prob, void* stream) {
  if (!c) return G4_E_ARG;
  if (!w || !x || !out || T < 0) {
    c->set_err("g4_moe_layer: bad argument");
    return G4_E_ARG;
  }
  const int dim = w->dim, E = w->n_expert, K = w->n_used, ff = w->expert_ff;
  if (dim <= 0 || E < 1 || E > kMaxExperts || K < 1 || K > E || K > kMaxUsed || ff <= 0 || dim % 4) {
    c->set_err("g4_moe_layer: unsupported geometry dim=%d experts=%d used=%d ff=%d", dim, E, K, ff);
    return G4_E_ARG;
  }
  if (!tensor_ok(w->gate_inp, G4_TYPE_F32, (uint64_t)dim * E) ||
      !tensor_ok(w->gate_inp_scale, G4_TYPE_F32, dim) || !tensor_ok(w->down_exps_scale, G4_TYPE_F32, E) ||
      !tensor_ok(w->pre_ffw_norm_2, G4_TYPE_F32, dim) ||
      (w->post_ffw_norm_2 && !tensor_ok(w->post_ffw_norm_2, G4_TYPE_F32, dim)) ||
      !tensor_ok(w->gate_up_exps, -1, (uint64_t)dim * 2 * ff * E) ||
      !tensor_ok(w->down_exps, -1, (uint64_t)ff * dim * E)) {
    c->set_err("g4_moe_layer: a weight tensor is missing or has the wrong type/size");
    return G4_E_ARG;
  }
  if (T == 0) return 0;
  if ((long long)T * K > (1 << 24)) {
    c->set_err("g4_moe_layer: too many tokens (%d)", T);
    return G4_E_ARG;
  }
  if (int r = c->bind()) return r;
  cudaStream_t st = (cudaStream_t)stream;
  const size_t base_need = moe_scratch_bytes(T, dim, E, K, ff);
  // wide batches: grouped expert products on the tensor cores (g4_moe_tc.cu)
  const bool use_tc = moe_tc_supported(w->gate_up_exps->type, w->down_exps->type, dim, ff, E) &&
                      moe_tc_wanted(T, K, E);
  size_t need = base_need + (use_tc ? moe_tc_scratch_bytes(T, dim, E, K, ff) : 0);
  uint8_t* base = (uint8_t*)c->scratch(need);
  if (!base) {
    c->set_err("g4_moe_layer: cannot allocate %zu bytes of scratch", need);
    return G4_E_NOMEM;
  }
  MoeScratch m = carve(base, T, dim, E, K, ff);
  cudaError_t e = launch_front(c, w, x, m, T, !use_tc, st);
  if (e != cudaSuccess) return c->cuda_fail(e, "g4_moe_layer launch");
  bool done = false;
  if (use_tc) {
    e = launch_moe_tc(c, (const uint8_t*)w->gate_up_exps->d, (const uint8_t*)w->down_exps->d, m.moe_in, m.offsets,
                      m.perm, m.D, base + base_need, T, dim, E, K, ff, st);
    if (e != cudaSuccess) return c->cuda_fail(e, "g4_moe_layer tensor-core launch");
    done = true;
  }
  if (!done) {
    const int rd = launch_dec_pair(c, w, m, E, K, dim, ff, T, st);
    if (rd == -2) return c->cuda_fail(last_launch_err(), "g4_moe_layer decode launch");
    done = rd == 0;
  }
  if (!done) {
    int r = launch_expert_rows(c, w->gate_up_exps->type, true, (const uint8_t*)w->gate_up_exps->d, m.moe_in,
                               m.moe_in_s16, m.G, m.G_s16, m, E, K, dim, ff, T, st, false);
    const bool rows_gu = r == 0;
    if (r == -1)
      r = launch_expert(c, w->gate_up_exps->type, true, (const uint8_t*)w->gate_up_exps->d, m.moe_in, m.G, m, E, K,
                        dim, ff, T, st);
    if (r == 0) {
      // the down rows kernel needs G's per-16-column sums, written by the gate_up rows kernel
      r = rows_gu ? launch_expert_rows(c, w->down_exps->type, false, (const uint8_t*)w->down_exps->d, m.G, m.G_s16,
                                       m.D, nullptr, m, E, K, dim, ff, T, st, false)
                  : -1;
      if (r == -1)
        r = launch_expert(c, w->down_exps->type, false, (const uint8_t*)w->down_exps->d, m.G, m.D, m, E, K, dim, ff,
                          T, st);
    }
    if (r == -1) {
      c->set_err("g4_moe_layer: expert tensor layout not supported by the grouped kernels");
      return G4_E_ARG;
    }
    if (r) return c->cuda_fail(last_launch_err(), "g4_moe_layer expert launch");
  }
  if (cudaError_t ce = launch_combine(w, m, out, T, st)) return c->cuda_fail(ce, "g4_moe_layer combine launch");
  if (topk_idx) cudaMemcpyAsync(topk_idx, m.idx, (size_t)T * K * 4, cudaMemcpyDeviceToDevice, st);
  if (topk_prob) cudaMemcpyAsync(topk_prob, m.prob, (size_t)T * K * 4, cudaMemcpyDeviceToDevice, st);
  e = cudaGetLastError();
  return e == cudaSuccess ? 0 : c->cuda_fail(e, "g4_moe_layer");
}

extern "C" int g4_moe_layer_host(g4_ctx* c, const g4_moe_weights* w, const float* xh, float* outh, int T,
                                 int32_t* idx_h, float* prob_h) {
  if (!c) return G4_E_ARG;
  if (!w || !xh || !outh || T < 0) {
    c->set_err("g4_moe_layer_host: bad argument");
    return G4_E_ARG;
  }
  if (T == 0) return 0;
  if (int r = c->bind()) return r;
  const int dim = w->dim, K = w->n_used;
  size_t xb = align_up((size_t)T * dim * 4, 256), ib = align_up((size_t)T * K * 4, 256);
  // The io buffers live in their own arena: the layer's scratch arena may grow.
  size_t need = 2 * xb + 2 * ib;
  void* io = c->io(need);
  if (!io) {
    c->set_err("g4_moe_layer_host: cannot allocate %zu bytes", need);
    return G4_E_NOMEM;
  }
  uint8_t* b = (uint8_t*)io;
  float* xd = (float*)b;
  float* od = (float*)(b + xb);
  int32_t* id = (int32_t*)(b + 2 * xb);
  float* pd = (float*)(b + 2 * xb + ib);
  cudaStream_t st = 0;
  cudaError_t e = cudaMemcpyAsync(xd, xh, (size_t)T * dim * 4, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return c->cuda_fail(e, "g4_moe_layer_host H2D");
  int r = g4_moe_layer(c, w, xd, od, T, id, pd, st);
  if (r) return r;
  cudaMemcpyAsync(outh, od, (size_t)T * dim * 4, cudaMemcpyDeviceToHost, st);
  if (idx_h) cudaMemcpyAsync(idx_h, id, (size_t)T * K * 4, cudaMemcpyDeviceToHost, st);
  if (prob_h) cudaMemcpyAsync(prob_h, pd, (size_t)T * K * 4, cudaMemcpyDeviceToHost, st);
  return c->check_status(st);
}

// ============================================================================
// Expert-parallel MoE layer (one process per GPU, NCCL).
//
// Rank r holds experts [r*El, (r+1)*El) of the layer (El = n_expert / world)
// and the replicated router, scales and norms, and owns its own tokens.  A
// call routes the rank's tokens, sends every routed slot's moe_in row to the
// rank that owns its expert, runs the grouped expert products over what it
// received, sends the products back and combines them on the owner in the
// reference's selection order: the same arithmetic as g4_moe_layer.
// ============================================================================

// dest[s] = owning rank of slot s's expert
__global__ void moe_ep_dest_kernel(const int32_t* __restrict__ idx, int n, int e_local, int32_t* __restrict__ dest) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s < n) dest[s] = idx[s] / e_local;
}
// send order p (slots grouped by destination): row p = moe_in of the slot's
// token, eid[p] = the expert's index at the destination.  One warp per row.
__global__ void __launch_bounds__(256) moe_ep_pack_kernel(const float* __restrict__ moe_in,
                                                          const int32_t* __restrict__ idx,
                                                          const int32_t* __restrict__ perm, int n, int dim, int K,
                                                          int e_local, float* __restrict__ rows,
                                                          int32_t* __restrict__ eid) {
  const int p = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (p >= n) return;
  const int slot = perm[p];
  const float4* src = reinterpret_cast<const float4*>(moe_in + (size_t)(slot / K) * dim);
  float4* dst = reinterpret_cast<float4*>(rows + (size_t)p * dim);
  for (int i = lane; i < dim / 4; i += 32) dst[i] = __ldg(src + i);
  if (lane == 0) eid[p] = idx[slot] % e_local;
}
// D[slot of send position p] = back[p]
__global__ void __launch_bounds__(256) moe_ep_unpack_kernel(const float* __restrict__ back,
                                                            const int32_t* __restrict__ perm, int n, int dim,
                                                            float* __restrict__ D) {
  const int p = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (p >= n) return;
  const float4* src = reinterpret_cast<const float4*>(back + (size_t)p * dim);
  float4* dst = reinterpret_cast<float4*>(D + (size_t)perm[p] * dim);
  for (int i = lane; i < dim / 4; i += 32) dst[i] = src[i];
}

extern "C" int g4_moe_layer_ep(g4_ctx* c, const g4_moe_weights* w, const float* x, float* out, int T,
                               int32_t* topk_idx, float* topk_prob, void* stream) {
  if (!c) return G4_E_ARG;
  if (!w || (T > 0 && (!x || !out)) || T < 0) {
    c->set_err("g4_moe_layer_ep: bad argument");
    return G4_E_ARG;
  }
  const int world = c->world, rank = c->rank;
  const int dim = w->dim, E = w->n_expert, K = w->n_used, ff = w->expert_ff;
  if (dim <= 0 || E < 1 || E > kMaxExperts || K < 1 || K > E || K > kMaxUsed || ff <= 0 || dim % 4 ||
      E % world) {
    c->set_err("g4_moe_layer_ep: unsupported geometry dim=%d experts=%d used=%d ff=%d world=%d", dim, E, K, ff,
               world);
    return G4_E_ARG;
  }
  const int El = E / world;
  if (!tensor_ok(w->gate_inp, G4_TYPE_F32, (uint64_t)dim * E) ||
      !tensor_ok(w->gate_inp_scale, G4_TYPE_F32, dim) || !tensor_ok(w->down_exps_scale, G4_TYPE_F32, E) ||
      !tensor_ok(w->pre_ffw_norm_2, G4_TYPE_F32, dim) ||
      (w->post_ffw_norm_2 && !tensor_ok(w->post_ffw_norm_2, G4_TYPE_F32, dim)) ||
      !tensor_ok(w->gate_up_exps, -1, (uint64_t)dim * 2 * ff * El) ||
      !tensor_ok(w->down_exps, -1, (uint64_t)ff * dim * El)) {
    c->set_err("g4_moe_layer_ep: a weight tensor is missing or has the wrong type/size "
               "(expert tensors hold this rank's %d experts)", El);
    return G4_E_ARG;
  }
  if (!moe_tc_supported(w->gate_up_exps->type, w->down_exps->type, dim, ff, El)) {
    c->set_err("g4_moe_layer_ep: expert layout not supported (Q4_K experts, dim %% 256 == 0, ff %% 64 == 0)");
    return G4_E_TYPE;
  }
  if ((long long)T * K * world > (1 << 24)) {
    c->set_err("g4_moe_layer_ep: too many tokens (%d)", T);
    return G4_E_ARG;
  }
  if (world > 1 && !c->comm) {
    c->set_err("g4_moe_layer_ep: g4_dist_init not called");
    return G4_E_DIST;
  }
  if (int r = c->bind()) return r;
  cudaStream_t st = (cudaStream_t)stream;
  const int n_slots = T * K;

  // ---- send side: this rank's tokens (scratch arena)
  const size_t base_need = moe_scratch_bytes(T > 0 ? T : 1, dim, E, K, ff);
  const size_t ns_al = align_up((size_t)(n_slots > 0 ? n_slots : 1) * 4, 256);
  const size_t rows_al = align_up((size_t)(n_slots > 0 ? n_slots : 1) * dim * 4, 256);
  const size_t cnt_al = align_up((size_t)world * (world + 1) * 4, 256);
  const size_t need = base_need + 3 * ns_al + align_up((size_t)(world + 1) * 4, 256) + 2 * rows_al + cnt_al;
  uint8_t* base = (uint8_t*)c->scratch(need);
  if (!base) {
    c->set_err("g4_moe_layer_ep: cannot allocate %zu bytes of scratch", need);
    return G4_E_NOMEM;
  }
  MoeScratch m = carve(base, T > 0 ? T : 1, dim, E, K, ff);
  uint8_t* q = base + base_need;
  int32_t* dest = (int32_t*)q;                 q += ns_al;
  int32_t* perm_d = (int32_t*)q;               q += ns_al;
  int32_t* send_eid = (int32_t*)q;             q += ns_al;
  int32_t* off_d = (int32_t*)q;                q += align_up((size_t)(world + 1) * 4, 256);
  float* send_rows = (float*)q;                q += rows_al;
  float* back_rows = (float*)q;                q += rows_al;
  int32_t* off_all = (int32_t*)q;

  cudaError_t e = cudaSuccess;
  if (T > 0) {
    e = launch_front(c, w, x, m, T, false, st);
    if (e != cudaSuccess) return c->cuda_fail(e, "g4_moe_layer_ep launch");
    moe_ep_dest_kernel<<<(n_slots + 255) / 256, 256, 0, st>>>(m.idx, n_slots, El, dest);
    launch_permute(dest, n_slots, world, off_d, perm_d, reinterpret_cast<int32_t*>(m.G), st);
    moe_ep_pack_kernel<<<(n_slots + 7) / 8, 256, 0, st>>>(m.moe_in, m.idx, perm_d, n_slots, dim, K, El, send_rows,
                                                           send_eid);
  } else {
    e = cudaMemsetAsync(off_d, 0, (size_t)(world + 1) * 4, st);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return c->cuda_fail(e, "g4_moe_layer_ep dispatch");

  // ---- every rank's send offsets, so each rank knows what it receives from whom
  if (int r = g4_nccl_allgather_i32(c, off_d, off_all, (size_t)world + 1, st)) return r;
  int32_t* h_off = (int32_t*)c->pinned((size_t)world * (world + 1) * 4);
  if (!h_off) {
    c->set_err("g4_moe_layer_ep: cannot allocate pinned memory");
    return G4_E_NOMEM;
  }
  e = cudaMemcpyAsync(h_off, off_all, (size_t)world * (world + 1) * 4, cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) return c->cuda_fail(e, "g4_moe_layer_ep count exchange");
  // bounded wait: a peer that stopped answering ends in G4_E_DIST, not a hung host
  if (int r = g4_dist_stream_wait(c, st)) return r;
  std::vector<size_t> s_off(world), s_len(world), r_off(world), r_len(world);
  size_t R = 0;
  for (int p = 0; p < world; ++p) {
    const int32_t* mine = h_off + (size_t)rank * (world + 1);
    const int32_t* theirs = h_off + (size_t)p * (world + 1);
    s_off[p] = (size_t)mine[p];
    s_len[p] = (size_t)(mine[p + 1] - mine[p]);
    r_off[p] = R;
    r_len[p] = (size_t)(theirs[rank + 1] - theirs[rank]);
    R += r_len[p];
  }

  // ---- receive side (ep arena, sized now that the counts are known)
  const int Ri = (int)(R > 0 ? R : 1);
  const size_t rr_al = align_up((size_t)Ri * dim * 4, 256), ri_al = align_up((size_t)Ri * 4, 256);
  const size_t tc_need = moe_tc_scratch_bytes(Ri, dim, El, 1, ff);
  const size_t ep_need = 2 * rr_al + 2 * ri_al + align_up((size_t)(El + 1) * 4, 256) +
                         align_up((size_t)((Ri + kPermChunk - 1) / kPermChunk) * El * 4, 256) + tc_need;
  uint8_t* eb = (uint8_t*)c->ep(ep_need);
  if (!eb) {
    c->set_err("g4_moe_layer_ep: cannot allocate %zu bytes for received rows", ep_need);
    return G4_E_NOMEM;
  }
  float* recv_rows = (float*)eb;               eb += rr_al;
  float* recv_out = (float*)eb;                eb += rr_al;
  int32_t* recv_eid = (int32_t*)eb;            eb += ri_al;
  int32_t* perm_l = (int32_t*)eb;              eb += ri_al;
  int32_t* off_l = (int32_t*)eb;               eb += align_up((size_t)(El + 1) * 4, 256);
  int32_t* perm_work = (int32_t*)eb;           eb += align_up((size_t)((Ri + kPermChunk - 1) / kPermChunk) * El * 4, 256);
  void* tc_work = eb;

  // ---- dispatch: rows and their local expert ids
  {
    std::vector<size_t> so(world), sl(world), ro(world), rl(world);
    const size_t rb = (size_t)dim * 4;
    for (int p = 0; p < world; ++p) so[p] = s_off[p] * rb, sl[p] = s_len[p] * rb, ro[p] = r_off[p] * rb,
                                    rl[p] = r_len[p] * rb;
    if (int r = g4_nccl_alltoallv(c, send_rows, so.data(), sl.data(), recv_rows, ro.data(), rl.data(), st)) return r;
    for (int p = 0; p < world; ++p) so[p] = s_off[p] * 4, sl[p] = s_len[p] * 4, ro[p] = r_off[p] * 4, rl[p] = r_len[p] * 4;
    if (int r = g4_nccl_alltoallv(c, send_eid, so.data(), sl.data(), recv_eid, ro.data(), rl.data(), st)) return r;
  }

  // ---- this rank's experts over the received rows (each row one slot)
  if (R > 0) {
    launch_permute(recv_eid, (int)R, El, off_l, perm_l, perm_work, st);
    e = cudaGetLastError();
    if (e == cudaSuccess)
      e = launch_moe_tc(c, (const uint8_t*)w->gate_up_exps->d, (const uint8_t*)w->down_exps->d, recv_rows, off_l,
                        perm_l, recv_out, tc_work, (int)R, dim, El, 1, ff, st);
    if (e != cudaSuccess) return c->cuda_fail(e, "g4_moe_layer_ep expert launch");
  }

  // ---- products back to the ranks that own the tokens, in their send order
  {
    std::vector<size_t> so(world), sl(world), ro(world), rl(world);
    const size_t rb = (size_t)dim * 4;
    for (int p = 0; p < world; ++p) so[p] = r_off[p] * rb, sl[p] = r_len[p] * rb, ro[p] = s_off[p] * rb,
                                    rl[p] = s_len[p] * rb;
    if (int r = g4_nccl_alltoallv(c, recv_out, so.data(), sl.data(), back_rows, ro.data(), rl.data(), st)) return r;
  }
  if (T == 0) return 0;
  moe_ep_unpack_kernel<<<(n_slots + 7) / 8, 256, 0, st>>>(back_rows, perm_d, n_slots, dim, m.D);
  if (cudaError_t ce = launch_combine(w, m, out, T, st)) return c->cuda_fail(ce, "g4_moe_layer_ep combine launch");
  if (topk_idx) cudaMemcpyAsync(topk_idx, m.idx, (size_t)T * K * 4, cudaMemcpyDeviceToDevice, st);
  if (topk_prob) cudaMemcpyAsync(topk_prob, m.prob, (size_t)T * K * 4, cudaMemcpyDeviceToDevice, st);
  e = cudaGetLastError();
  return e == cudaSuccess ? 0 : c->cuda_fail(e, "g4_moe_layer_ep");
}

// ============================================================================
// Allocation-free MoE layer.
//
// Some hosts cannot let a library allocate device memory once they are
// running: a JVM host that reserves all free HBM for its own pool at start-up
// (a later cudaMalloc would fail), or a decode loop that must not pay for the
// device-wide synchronisation a cudaMalloc/cudaFree can cause mid-step.  For
// them g4_moe_layer_noalloc runs the same kernels as g4_moe_layer with its
// work buffers in one fixed array of device memory that belongs to the
// library image (every GPU that loads the library holds it until exit).
// ============================================================================
namespace g4 {

static __device__ __align__(256) uint8_t g_moe_noalloc_scratch[G4_MOE_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kNoallocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoallocMaxDevices];  // device address of the array, per device

struct FixedOcc {
  ExpertFn fn;
  size_t smem;
  int device;
  int occ;
};
FixedOcc g_noalloc_occ[128];  // kernel set-up done by the no-alloc path per device (fixed table, no heap)
int g_noalloc_occ_n = 0;

// Device address of the scratch array on the current device.  It is resolved
// (cudaGetSymbolAddress) once per device, normally by g4_init through
// noalloc_prepare_device; the symbol's host-side name is only a stand-in and
// must never be passed to a kernel.
int noalloc_scratch(g4_ctx* c, uint8_t** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  const int d = c->dev.device;
  if (d < 0 || d >= kNoallocMaxDevices) {
    c->set_err("g4_moe_layer_noalloc: device id %d out of range", d);
    return G4_E_ARG;
  }
  if (!g_noalloc_ptr[d]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_moe_noalloc_scratch);
    if (e != cudaSuccess || !p) return c->cuda_fail(e, "g4_moe_layer_noalloc: cudaGetSymbolAddress");
    g_noalloc_ptr[d] = p;
  }
  *out = static_cast<uint8_t*>(g_noalloc_ptr[d]);
  return 0;
}
}  // namespace

// Resolve the no-alloc array on `device` (current).  Under lazy module
// loading (CUDA's default) the array only comes into being when this
// translation unit's module is loaded on the device; resolving its address
// loads the module, so g4_init calls this before the host can hand the free
// HBM to a pool of its own.  Returns the cudaError_t of the lookup.
int noalloc_prepare_device(int device) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (device < 0 || device >= kNoallocMaxDevices) return (int)cudaErrorInvalidDevice;
  if (g_noalloc_ptr[device]) return 0;
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_moe_noalloc_scratch);
  if (e != cudaSuccess || !p) {
    cudaGetLastError();
    return (int)(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
  }
  g_noalloc_ptr[device] = p;
  return 0;
}

namespace {

int noalloc_occ(ExpertFn fn, size_t smem, int threads, int* occ) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  int dev = 0, optin = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  for (int i = 0; i < g_noalloc_occ_n; ++i)
    if (g_noalloc_occ[i].fn == fn && g_noalloc_occ[i].smem == smem && g_noalloc_occ[i].device == dev) {
      *occ = g_noalloc_occ[i].occ;
      return 0;
    }
  if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return -1;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, optin) != cudaSuccess) return -1;
  int o = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, fn, threads, smem) != cudaSuccess) return -1;
  if (o < 1) o = 1;
  if (g_noalloc_occ_n < 128) g_noalloc_occ[g_noalloc_occ_n++] = FixedOcc{fn, smem, dev, o};
  *occ = o;
  return 0;
}

// Same work decomposition as launch_expert, with the kernel set-up cached in a
// fixed table.
int launch_expert_noalloc(g4_ctx* c, int type, bool gu, const uint8_t* w, const float* act, float* out,
                          const MoeScratch& m, int E, int K, int dim, int ff, int T, cudaStream_t st) {
  const int BS = block_size(type), TS = type_size(type);
  const int NCW = 8;
  ExpertArgs a{};
  a.w = w;
  a.act = act;
  a.out = out;
  a.offsets = m.offsets;
  a.perm = m.perm;
  a.status = c->status;
  a.E = E;
  a.n_used = K;
  a.ff = ff;
  if (gu) {
    a.rows_e = 2 * ff;
    a.cols = dim;
    a.pr = 1;
    if (dim % BS || dim % 16) return -1;
    a.vb = dim / BS * TS;
    if (a.vb % 2) return -1;
    a.units = dim / 16;
    a.tile_rows = NCW;
    a.tiles_e = (ff + NCW - 1) / NCW;
    a.region_bytes = (int)align_up((size_t)NCW * a.vb + 32, 128);
    a.stage_bytes = 2 * a.region_bytes;
    a.expert_elems = (long long)2 * ff * dim;
  } else {
    a.rows_e = dim;
    a.cols = ff;
    if (ff % 16) return -1;
    int pr = ff % BS == 0 ? 1 : BS / gcd_i(ff % BS, BS);
    if (pr != 1 && pr != 2 && pr != 4) return -1;
    if (dim % pr) return -1;
    a.pr = pr;
    a.vb = pr * ff / BS * TS;
    if (a.vb % 2) return -1;
    a.units = pr * ff / 16;
    a.tile_rows = NCW;
    a.tiles_e = (dim / pr + NCW - 1) / NCW;
    a.stage_bytes = (int)align_up((size_t)NCW * a.vb + 32, 128);
    a.expert_elems = (long long)dim * ff;
  }
  if (a.expert_elems % BS) return -1;
  const size_t fixed_smem = 64 + 4 * (2 * kMaxExperts + 8) + 128;
  a.nstages = 4;
  while (a.nstages > 2 && fixed_smem + (size_t)a.nstages * a.stage_bytes > c->dev.smem_optin) --a.nstages;
  if (fixed_smem + (size_t)a.nstages * a.stage_bytes > c->dev.smem_optin) return -1;
  int avg = (T * K + E - 1) / E;
  int nb = avg >= 8 ? 8 : avg >= 4 ? 4 : avg >= 2 ? 2 : 1;
  ExpertFn fn = select_expert(type, gu, a.pr, nb);
  if (!fn) return -1;
  size_t smem = fixed_smem + (size_t)a.nstages * a.stage_bytes;
  int occ = 1;
  if (noalloc_occ(fn, smem, 32 * (NCW + 1), &occ)) {
    t_launch_err = cudaErrorInvalidConfiguration;
    return -2;
  }
  long long max_items = (long long)std::min(T * K, E * ((T * K + nb - 1) / nb + 1)) * a.tiles_e;
  int grid = (int)std::min<long long>(max_items, (long long)c->dev.sms * occ);
  if (grid < 1) grid = 1;
  fn<<<grid, 32 * (NCW + 1), smem, st>>>(a);
  return launch_status();
}
}  // namespace

}  // namespace g4

extern "C" int g4_moe_layer_noalloc(g4_ctx* c, const g4_moe_weights* w, const float* x, float* out, int T,
                                    int32_t* topk_idx, float* topk_prob, void* stream) {
  if (!c) return G4_E_ARG;
  if (!w || !x || !out || T < 0) {
    c->set_err("g4_moe_layer_noalloc: bad argument");
    return G4_E_ARG;
  }
  const int dim = w->dim, E = w->n_expert, K = w->n_used, ff = w->expert_ff;
  if (dim <= 0 || E < 1 || E > kMaxExperts || K < 1 || K > E || K > kMaxUsed || ff <= 0 || dim % 4) {
    c->set_err("g4_moe_layer_noalloc: unsupported geometry dim=%d experts=%d used=%d ff=%d", dim, E, K, ff);
    return G4_E_ARG;
  }
  if (!tensor_ok(w->gate_inp, G4_TYPE_F32, (uint64_t)dim * E) ||
      !tensor_ok(w->gate_inp_scale, G4_TYPE_F32, dim) || !tensor_ok(w->down_exps_scale, G4_TYPE_F32, E) ||
      !tensor_ok(w->pre_ffw_norm_2, G4_TYPE_F32, dim) ||
      (w->post_ffw_norm_2 && !tensor_ok(w->post_ffw_norm_2, G4_TYPE_F32, dim)) ||
      !tensor_ok(w->gate_up_exps, -1, (uint64_t)dim * 2 * ff * E) ||
      !tensor_ok(w->down_exps, -1, (uint64_t)ff * dim * E)) {
    c->set_err("g4_moe_layer_noalloc: a weight tensor is missing or has the wrong type/size");
    return G4_E_ARG;
  }
  if (T == 0) return 0;
  const size_t need = moe_scratch_bytes(T, dim, E, K, ff);
  if (need > (size_t)G4_MOE_NOALLOC_SCRATCH_BYTES) {
    c->set_err("g4_moe_layer_noalloc: %d tokens need %zu bytes of work memory, more than the fixed %u; "
               "split the batch or use g4_moe_layer",
               T, need, (unsigned)G4_MOE_NOALLOC_SCRATCH_BYTES);
    return G4_E_ARG;
  }
  if (int r = c->bind()) return r;
  uint8_t* base = nullptr;
  if (int r = noalloc_scratch(c, &base)) return r;
  cudaStream_t st = (cudaStream_t)stream;
  // Every work buffer is fully written before it is read, so nothing has to
  // be cleared between calls.
  MoeScratch m = carve(base, T, dim, E, K, ff);
  cudaError_t e = launch_front(c, w, x, m, T, true, st);
  if (e != cudaSuccess) return c->cuda_fail(e, "g4_moe_layer_noalloc launch");
  int r = launch_dec_pair(c, w, m, E, K, dim, ff, T, st);
  const bool dec = r == 0;
  if (r == -1)
    r = launch_expert_rows(c, w->gate_up_exps->type, true, (const uint8_t*)w->gate_up_exps->d, m.moe_in,
                           m.moe_in_s16, m.G, m.G_s16, m, E, K, dim, ff, T, st, true);
  const bool rows_gu = !dec && r == 0;
  if (r == -1)
    r = launch_expert_noalloc(c, w->gate_up_exps->type, true, (const uint8_t*)w->gate_up_exps->d, m.moe_in, m.G, m,
                              E, K, dim, ff, T, st);
  if (r == 0 && !dec) {
    r = rows_gu ? launch_expert_rows(c, w->down_exps->type, false, (const uint8_t*)w->down_exps->d, m.G, m.G_s16,
                                     m.D, nullptr, m, E, K, dim, ff, T, st, true)
                : -1;
    if (r == -1)
      r = launch_expert_noalloc(c, w->down_exps->type, false, (const uint8_t*)w->down_exps->d, m.G, m.D, m, E, K,
                                dim, ff, T, st);
  }
  if (r == -1) {
    c->set_err("g4_moe_layer_noalloc: expert tensor layout not supported by the grouped kernels");
    return G4_E_ARG;
  }
  if (r) return c->cuda_fail(last_launch_err(), "g4_moe_layer_noalloc expert launch");
  if (cudaError_t ce = launch_combine(w, m, out, T, st)) return c->cuda_fail(ce, "g4_moe_layer_noalloc combine launch");
  if (topk_idx) cudaMemcpyAsync(topk_idx, m.idx, (size_t)T * K * 4, cudaMemcpyDeviceToDevice, st);
  if (topk_prob) cudaMemcpyAsync(topk_prob, m.prob, (size_t)T * K * 4, cudaMemcpyDeviceToDevice, st);
  e = cudaGetLastError();
  return e == cudaSuccess ? 0 : c->cuda_fail(e, "g4_moe_layer_noalloc");
}
