// g4_fuse.cuh -- the fused prologues and epilogues of the decoder's GEMV
// launches (GemvFuse, g4_gemv.cuh): the activation vector computed from the
// kernel's inputs (norms, residual, embedding, MoE merge)
// and the row post-processing (GELU pairs, softcap + argmax).
#pragma once
#include "g4_gemv.cuh"

namespace g4 {

// ---------------------------------------------------------------- fused prologue
// The activation vector of a decoder GEMV, computed by every CTA into xs
// (shared memory, n floats) from the kernel's inputs; CTA 0 also stores the
// new residual stream xn to f.x_out.  The arithmetic follows the reference's
// rounding order per element (Llama.kt:27-37 rmsnorm: w * (s * x);
// MutableFloatTensor.addInPlace / mapInPlace); sums of squares use a fixed
// tree instead of the sequential float sum.
constexpr int kPrologueMaxE = 8;  // elements per thread held in registers by the one-round path

// The constant inputs of the one-round path (norm weights), loaded by each
// thread for its elements i = tid + k * blockDim.x.  They never change, so a
// kernel loads them before waiting for its predecessor.
struct PrologueConst {
  float wi[kPrologueMaxE], wr[kPrologueMaxE], wm[kPrologueMaxE];
  bool loaded;
};
// IN: the kernel's prologue mode when fixed at compile time (-1: f.in_mode).
template <int IN = -1>
static __device__ __forceinline__ void prologue_const(const GemvFuse& f, int n, PrologueConst& c) {
  const int mode = IN >= 0 ? IN : f.in_mode;
  c.loaded = mode != IN_PLAIN && n <= kPrologueMaxE * (int)blockDim.x;
  if (!c.loaded) return;
  const bool merge = mode == IN_MOE_MERGE, resid = mode == IN_RESID_NORM || merge;
#pragma unroll
  for (int k = 0; k < kPrologueMaxE; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    c.wi[k] = c.wr[k] = c.wm[k] = 0.f;
    if (i < n) {
      c.wi[k] = __ldg(f.w_in + i);
      if (resid && f.r) c.wr[k] = __ldg(f.w_r + i);
      if (merge) c.wm[k] = __ldg(f.w_m + i);
    }
  }
}

template <int IN = -1>
static __device__ void fused_prologue(const GemvFuse& f, const float* __restrict__ x, float* xs, float* red, int n,
                                      const PrologueConst* pc = nullptr) {
  const int mode = IN >= 0 ? IN : f.in_mode;
  const int tid = threadIdx.x, nt = blockDim.x;
  const bool store = f.x_out != nullptr && (f.store_all || blockIdx.x == 0);
  constexpr int kMaxE = kPrologueMaxE;
  if (n <= kMaxE * nt) {
    // every input this thread needs, loaded in one round, then the passes in registers
    const bool merge = mode == IN_MOE_MERGE, embed = mode == IN_EMBED_NORM;
    const bool resid = mode == IN_RESID_NORM || merge;
    float xv[kMaxE], rv[kMaxE], wr[kMaxE], mv[kMaxE], wm[kMaxE], wi[kMaxE];
    long long ebase = 0;
    if (embed) {
      const int s = *f.step;
      int tok = f.in_tok[s];
      if (tok < 0) tok = *f.next_tok;
      ebase = (long long)tok * n;
    }
#pragma unroll
    for (int k = 0; k < kMaxE; ++k) {
      const int i = tid + k * nt;
      const bool in = i < n;
      xv[k] = rv[k] = wr[k] = mv[k] = wm[k] = wi[k] = 0.f;
      if (pc && pc->loaded) {
        wi[k] = pc->wi[k];
        wr[k] = pc->wr[k];
        wm[k] = pc->wm[k];
      }
      if (in) {
        if (!(pc && pc->loaded)) {
          wi[k] = f.w_in[i];
          if (resid && f.r) wr[k] = f.w_r[i];
          if (merge) wm[k] = f.w_m[i];
        }
        if (embed) xv[k] = get_elem(f.emb_type, f.emb, ebase + i);
        else xv[k] = x[i];
        if (resid && f.r) rv[k] = f.r[i];
        if (merge) mv[k] = f.m[i];
      }
    }
    float s_r = 0.f;
    if (resid && f.r) {
      float sr = 0.f;
#pragma unroll
      for (int k = 0; k < kMaxE; ++k) sr = __fadd_rn(sr, __fmul_rn(rv[k], rv[k]));
      s_r = rms_scale(block_sum(sr, red), n, f.eps);
    }
    float ss = 0.f;
    if (merge) {
      // xb = rmsnorm(shared, post_ffw_norm_1) + moeOutput (Llama.kt:237-243, 349)
      float st = 0.f;
#pragma unroll
      for (int k = 0; k < kMaxE; ++k) {
        mv[k] = __fadd_rn(__fmul_rn(wr[k], __fmul_rn(s_r, rv[k])), mv[k]);
        st = __fadd_rn(st, __fmul_rn(mv[k], mv[k]));
      }
      const float s_m = rms_scale(block_sum(st, red), n, f.eps);
#pragma unroll
      for (int k = 0; k < kMaxE; ++k) xv[k] = __fadd_rn(xv[k], __fmul_rn(wm[k], __fmul_rn(s_m, mv[k])));
    } else if (resid && f.r) {
#pragma unroll
      for (int k = 0; k < kMaxE; ++k) xv[k] = __fadd_rn(xv[k], __fmul_rn(wr[k], __fmul_rn(s_r, rv[k])));
    } else if (embed) {
#pragma unroll
      for (int k = 0; k < kMaxE; ++k) xv[k] = __fmul_rn(xv[k], f.sqrt_dim);  // Llama.kt:113
    }
#pragma unroll
    for (int k = 0; k < kMaxE; ++k) {
      if (resid && f.scale != 1.f) xv[k] = __fmul_rn(xv[k], f.scale);  // Llama.kt:393-397
      ss = __fadd_rn(ss, __fmul_rn(xv[k], xv[k]));
    }
    const float sx = rms_scale(block_sum(ss, red), n, f.eps);
#pragma unroll
    for (int k = 0; k < kMaxE; ++k) {
      const int i = tid + k * nt;
      if (i < n) {
        if (store) f.x_out[i] = xv[k];
        xs[i] = __fmul_rn(wi[k], __fmul_rn(sx, xv[k]));
      }
    }
    __syncthreads();
    return;
  }
  float ss = 0.f;
  if (mode == IN_NORM) {
    for (int i = tid; i < n; i += nt) {
      const float v = x[i];
      xs[i] = v;
      ss = __fadd_rn(ss, __fmul_rn(v, v));
    }
  } else if (mode == IN_EMBED_NORM) {
    // Llama.kt:112-113: x = tokenEmbeddingTable.get(token * dim + i) * sqrt(dim)
    const int s = *f.step;
    int tok = f.in_tok[s];
    if (tok < 0) tok = *f.next_tok;
    const long long base = (long long)tok * n;
    for (int i = tid; i < n; i += nt) {
      const float v = __fmul_rn(get_elem(f.emb_type, f.emb, base + i), f.sqrt_dim);
      xs[i] = v;
      if (store) f.x_out[i] = v;
      ss = __fadd_rn(ss, __fmul_rn(v, v));
    }
  } else {
    // IN_RESID_NORM / IN_MOE_MERGE: xn = (x + branch) * scale
    float s_r = 0.f;
    if (f.r) {
      float sr = 0.f;
      for (int i = tid; i < n; i += nt) sr = __fadd_rn(sr, __fmul_rn(f.r[i], f.r[i]));
      s_r = rms_scale(block_sum(sr, red), n, f.eps);
    }
    float s_m = 0.f;
    if (mode == IN_MOE_MERGE) {
      // xb = rmsnorm(shared, post_ffw_norm_1) + moeOutput (Llama.kt:237-243, 349)
      float st = 0.f;
      for (int i = tid; i < n; i += nt) {
        const float t = __fadd_rn(__fmul_rn(f.w_r[i], __fmul_rn(s_r, f.r[i])), f.m[i]);
        xs[i] = t;
        st = __fadd_rn(st, __fmul_rn(t, t));
      }
      s_m = rms_scale(block_sum(st, red), n, f.eps);
    }
    for (int i = tid; i < n; i += nt) {
      float v = x[i];
      if (mode == IN_MOE_MERGE) v = __fadd_rn(v, __fmul_rn(f.w_m[i], __fmul_rn(s_m, xs[i])));
      else if (f.r) v = __fadd_rn(v, __fmul_rn(f.w_r[i], __fmul_rn(s_r, f.r[i])));
      if (f.scale != 1.f) v = __fmul_rn(v, f.scale);  // Llama.kt:393-397
      xs[i] = v;
      if (store) f.x_out[i] = v;
      ss = __fadd_rn(ss, __fmul_rn(v, v));
    }
  }
  const float sx = rms_scale(block_sum(ss, red), n, f.eps);
  for (int i = tid; i < n; i += nt) xs[i] = __fmul_rn(f.w_in[i], __fmul_rn(sx, xs[i]));
  __syncthreads();
}

// Order-preserving key of an output for the argmax: larger value first, and
// among equal values the lower row (FloatTensor.argmax keeps the first maximum).
static __device__ __forceinline__ unsigned long long argmax_key(float v, long long row) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)row);
}

static __device__ __forceinline__ float softcap_ref(float v, float cap) {
  // Llama.kt:403-406: cap * tanh((v / cap).toDouble()).toFloat()
  return cap > 0.f ? __fmul_rn(cap, (float)tanh((double)__fdiv_rn(v, cap))) : v;
}

}  // namespace g4
