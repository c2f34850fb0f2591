// g4_block.cu -- the whole FFN half of a MoE layer in one call
// (g4_ffn_moe_block: Llama.kt:226-353, and the layer output scale of
// Llama.kt:393-397): the shared MLP, the expert half (g4_moe_layer) and the
// merge, on the residual stream in place.
//
// Per token: h = rmsnorm(x, ffn_norm); gate / up GEMVs; hb = gelu(gate) * up;
// down GEMV; then one kernel per token finishes the block:
//   xb = rmsnorm(down, post_ffw_norm_1) + moeOutput      Llama.kt:237-243, 349
//   x += rmsnorm(xb, post_ffw_norm); x *= scale          Llama.kt:352-353, 393-397
// The GEMVs are g4_matmul (every format); the expert half is g4_moe_layer on
// the same residual stream (Llama.kt:247 reads state.x, not xb).
#include "g4.h"
#include "g4_common.cuh"
#include "g4_ctx.h"
#include "g4_internal.h"

namespace g4 {

// out[t] = w * (s * x[t]) per token (Llama.kt:27-37); one CTA per token
__global__ void __launch_bounds__(256) blk_rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                          float* __restrict__ out, int dim, float eps) {
  __shared__ float red[33];
  const float* xt = x + (size_t)blockIdx.x * dim;
  float* ot = out + (size_t)blockIdx.x * dim;
  float ss = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) ss = __fadd_rn(ss, __fmul_rn(xt[i], xt[i]));
  const float s = rms_scale(block_sum(ss, red), dim, eps);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) ot[i] = __fmul_rn(w[i], __fmul_rn(s, xt[i]));
}

// hb = gelu(gate) * up (Llama.kt:234-235)
__global__ void blk_gelu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ hb,
                                    long long n) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) hb[i] = __fmul_rn(gelu_ref(g[i]), u[i]);
}

// Llama.kt:237-243, 349-353, 393-397 for one token per CTA
__global__ void __launch_bounds__(256) blk_merge_kernel(float* __restrict__ x, const float* __restrict__ down,
                                                        const float* __restrict__ moe, const float* __restrict__ w1,
                                                        const float* __restrict__ wp, int dim, float eps, float scale) {
  __shared__ float red[33];
  float* xt = x + (size_t)blockIdx.x * dim;
  const float* dt = down + (size_t)blockIdx.x * dim;
  const float* mt = moe + (size_t)blockIdx.x * dim;
  float ss = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) ss = __fadd_rn(ss, __fmul_rn(dt[i], dt[i]));
  const float s1 = rms_scale(block_sum(ss, red), dim, eps);
  float st = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float v = __fadd_rn(__fmul_rn(w1[i], __fmul_rn(s1, dt[i])), mt[i]);
    st = __fadd_rn(st, __fmul_rn(v, v));
  }
  const float s2 = rms_scale(block_sum(st, red), dim, eps);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float v = __fadd_rn(__fmul_rn(w1[i], __fmul_rn(s1, dt[i])), mt[i]);
    float r = __fadd_rn(xt[i], __fmul_rn(wp[i], __fmul_rn(s2, v)));
    if (scale != 1.f) r = __fmul_rn(r, scale);
    xt[i] = r;
  }
}

}  // namespace g4

using namespace g4;

static bool f32_vec(const g4_tensor* t, int n) { return t && t->type == F32 && t->n_elems == (uint64_t)n; }

extern "C" int g4_ffn_moe_block(g4_ctx* c, const g4_ffn_moe_weights* w, float* x, int T, void* stream) {
  if (!c) return G4_E_ARG;
  if (!w || !w->moe || (!x && T > 0) || T < 0 || w->ff <= 0) {
    c->set_err("g4_ffn_moe_block: bad argument");
    return G4_E_ARG;
  }
  if (T == 0) return 0;
  const int dim = w->moe->dim, ff = w->ff;
  const float eps = w->moe->eps;
  if (!f32_vec(w->ffn_norm, dim) || !f32_vec(w->post_ffw_norm_1, dim) || !f32_vec(w->post_ffw_norm, dim) || !w->ffn_gate ||
      !w->ffn_up || !w->ffn_down || w->ffn_gate->n_elems != (uint64_t)dim * ff ||
      w->ffn_up->n_elems != (uint64_t)dim * ff || w->ffn_down->n_elems != (uint64_t)dim * ff) {
    c->set_err("g4_ffn_moe_block: the shared MLP needs F32 [%d] norms and [%d, %d] gate / up / down tensors", dim,
               dim, ff);
    return G4_E_ARG;
  }
  if (int r = c->bind()) return r;
  cudaStream_t st = (cudaStream_t)stream;
  auto al = [](size_t b) { return (b + 255) / 256 * 256; };
  const size_t bx = al((size_t)T * dim * 4), bf = al((size_t)T * ff * 4);
  uint8_t* b = (uint8_t*)c->blk(4 * bx + 3 * bf);
  if (!b) {
    c->set_err("g4_ffn_moe_block: cannot allocate %zu bytes of work memory", 4 * bx + 3 * bf);
    return G4_E_NOMEM;
  }
  float* h = (float*)b;
  float* dn = (float*)(b + bx);
  float* moe = (float*)(b + 2 * bx);
  float* g = (float*)(b + 4 * bx);
  float* u = (float*)(b + 4 * bx + bf);
  float* hb = (float*)(b + 4 * bx + 2 * bf);
  // shared MLP (Llama.kt:231-236)
  blk_rmsnorm_kernel<<<T, 256, 0, st>>>(x, (const float*)w->ffn_norm->d, h, dim, eps);
  if (cudaError_t e = cudaGetLastError()) return c->cuda_fail(e, "g4_ffn_moe_block: norm");
  for (int t = 0; t < T; ++t) {
    if (int r = g4_matmul(c, w->ffn_gate, 0, h + (size_t)t * dim, g + (size_t)t * ff, ff, dim, st)) return r;
    if (int r = g4_matmul(c, w->ffn_up, 0, h + (size_t)t * dim, u + (size_t)t * ff, ff, dim, st)) return r;
  }
  const long long n = (long long)T * ff;
  blk_gelu_mul_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(g, u, hb, n);
  if (cudaError_t e = cudaGetLastError()) return c->cuda_fail(e, "g4_ffn_moe_block: gelu");
  for (int t = 0; t < T; ++t)
    if (int r = g4_matmul(c, w->ffn_down, 0, hb + (size_t)t * ff, dn + (size_t)t * dim, dim, ff, st)) return r;
  // expert half on the same residual stream (Llama.kt:247-346)
  if (int r = g4_moe_layer(c, w->moe, x, moe, T, nullptr, nullptr, st)) return r;
  // merge and layer output scale (Llama.kt:237-243, 349-353, 393-397)
  blk_merge_kernel<<<T, 256, 0, st>>>(x, dn, moe, (const float*)w->post_ffw_norm_1->d,
                                      (const float*)w->post_ffw_norm->d, dim, eps, w->layer_output_scale);
  if (cudaError_t e = cudaGetLastError()) return c->cuda_fail(e, "g4_ffn_moe_block: merge");
  return 0;
}

extern "C" int g4_ffn_moe_block_host(g4_ctx* c, const g4_ffn_moe_weights* w, float* xh, int T) {
  if (!c) return G4_E_ARG;
  if (!w || !w->moe || (!xh && T > 0) || T < 0) {
    c->set_err("g4_ffn_moe_block_host: bad argument");
    return G4_E_ARG;
  }
  if (T == 0) return 0;
  if (int r = c->bind()) return r;
  const size_t nb = (size_t)T * w->moe->dim * 4;
  float* xd = (float*)c->io(nb);
  if (!xd) {
    c->set_err("g4_ffn_moe_block_host: cannot allocate %zu bytes", nb);
    return G4_E_NOMEM;
  }
  cudaStream_t st = 0;
  if (cudaError_t e = cudaMemcpyAsync(xd, xh, nb, cudaMemcpyHostToDevice, st))
    return c->cuda_fail(e, "g4_ffn_moe_block_host H2D");
  if (int r = g4_ffn_moe_block(c, w, xd, T, st)) return r;
  if (cudaError_t e = cudaMemcpyAsync(xh, xd, nb, cudaMemcpyDeviceToHost, st))
    return c->cuda_fail(e, "g4_ffn_moe_block_host D2H");
  return c->check_status(st);
}
