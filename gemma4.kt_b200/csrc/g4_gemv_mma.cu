// g4_gemv_mma.cu -- the decoder's Q8_0 matrix-vector products on the tensor
// cores (mma.sync m16n8k32, int8 x int8 -> int32), sm_100a.
//
// At model load every Q8_0 projection is repacked into tiles of 16 rows x one
// 32-column block: the 512 code bytes in the order of the mma A fragment (lane
// l holds rows l/4 and l/4 + 8, columns 4(l%4)..+3 and 16 + 4(l%4)..+3 as 16
// contiguous bytes, so a warp loads a tile with one coalesced 16-byte load per
// lane) and the 16 fp16 scales as 8 words (row g and g + 8 in word g).
//
// The activation of each 32-column block is held as three int8 limbs,
// x / s = h + m/254 + l/254^2 (s a power of two with max|x|/s <= 127; each
// limb in [-127, 127]): about 23 bits per value, fp32-level products.  The
// limbs are the B operand's columns 0, 1, 2 (the other five are zero), so one
// mma gives, for 16 rows, the exact int32 sums of the codes times each limb;
// the fp32 accumulation scales them by d_row * s_block per block and the
// limbs are combined once per row at the end.
//
// CTAs of 8 warps take tasks of 8/ks row tiles; the ks warps of a row tile
// split its blocks (K), loading four tiles ahead into registers, and meet in
// shared memory for the epilogue (plain, gelu(gate) * up on interleaved rows,
// or softcap + arg-max).  The first task's weights are requested before the
// kernel waits for its predecessor (programmatic dependent launch).
//
// The batched decoder's kernels follow: batch_prologue_kernel (a token's fused
// prologue and its limbs, one CTA per token) and gemm_mma_batch_kernel (the
// same tiles for up to 64 tokens, the tokens as the B operand's columns, the
// limbs staged in shared memory, split-K with a deterministic reduction).
#include "g4_fuse.cuh"
#include "g4_gemv.cuh"
#include "g4_internal.h"

#include <algorithm>

namespace g4 {

constexpr int kMmaWarps = 8;
constexpr int kMmaAhead = 4;  // tiles a warp has in flight

struct MmaGemvArgs {
  MmaGemvPlan p;
  const uint4* q;       // [nrt][nkb][32 lanes] 16-byte fragments
  const uint32_t* sc;   // [nrt][nkb][8] scale pairs
  const float* x;
  float* y;
  unsigned* status;
  GemvFuse f;
};

// D = A.B + C with C = 0x4B400000 in every element: each int32 sum s (|s| <
// 2^22; a block's code x limb sums stay below 32*127*127) comes out as the bit
// pattern of the float 1.5*2^23 + s, so one subtraction (mma_f32) turns it into
// an exact float instead of an integer-to-float conversion.
constexpr int kMmaMagic = 0x4B400000;
__device__ __forceinline__ void mma_s8(int (&d)[4], const uint4& a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1), "r"(kMmaMagic));
}
__device__ __forceinline__ float mma_f32(int d) { return __fsub_rn(__int_as_float(d), 12582912.0f); }

// x rounded to the nearest integer (ties to even), |x| < 2^22, as float and int
__device__ __forceinline__ float rint_small(float x, int& i) {
  constexpr float kMagic = 12582912.0f;
  const float t = __fadd_rn(x, kMagic);
  i = __float_as_int(t) - 0x4B400000;
  return __fsub_rn(t, kMagic);
}

// Repack a Q8_0 matrix [rows][cols] (GGUF rows of 34-byte blocks) into the
// fragment tiles; rows past the end are zero.  One thread per (tile, lane).
__global__ void repack_q8_0_mma_kernel(const uint8_t* __restrict__ raw, int rows, int cols, uint4* __restrict__ q,
                                       uint32_t* __restrict__ sc) {
  const int nkb = cols / 32, nrt = (rows + 15) / 16;
  const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= (long long)nrt * nkb * 32) return;
  const int lane = (int)(id & 31);
  const long long tile = id >> 5;
  const int rt = (int)(tile / nkb), kb = (int)(tile % nkb);
  const int g = lane >> 2, t = lane & 3;
  const size_t row_bytes = (size_t)nkb * 34;
  auto code4 = [&](int r, int c0) {
    uint32_t v = 0;
    if (r < rows) {
      const uint8_t* b = raw + (size_t)r * row_bytes + (size_t)kb * 34 + 2 + c0;
      v = (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24);
    }
    return v;
  };
  const int r0 = rt * 16 + g, r1 = r0 + 8;
  q[tile * 32 + lane] = make_uint4(code4(r0, 4 * t), code4(r1, 4 * t), code4(r0, 16 + 4 * t), code4(r1, 16 + 4 * t));
  if (t == 0) {
    auto scale = [&](int r) -> uint32_t {
      if (r >= rows) return 0u;
      const uint8_t* b = raw + (size_t)r * row_bytes + (size_t)kb * 34;
      return (uint32_t)b[0] | ((uint32_t)b[1] << 8);
    };
    sc[tile * 8 + g] = scale(r0) | (scale(r1) << 16);
  }
}

// The activation of one CTA as three int8 limbs per value (layout [nkb][96]:
// limb h at +0, m at +32, l at +64 of each 32-column block) and the block's
// power-of-two scale.  kGlobal: src is global memory written by an earlier
// grid (read through L2), else shared memory.
template <bool kGlobal>
__device__ __forceinline__ void limbs_cta(const float* src, int cols, int8_t* lim, float* xsc) {
  constexpr int kQ = 6;
  const int n4 = cols / 4;
  for (int i0 = 0; i0 < n4; i0 += kQ * (int)blockDim.x) {
    float4 vq[kQ];
#pragma unroll
    for (int qq = 0; qq < kQ; ++qq) {
      const int i = i0 + qq * (int)blockDim.x + (int)threadIdx.x;
      vq[qq] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < n4) {
        if constexpr (kGlobal) vq[qq] = __ldcg(reinterpret_cast<const float4*>(src) + i);
        else vq[qq] = reinterpret_cast<const float4*>(src)[i];
      }
    }
#pragma unroll
    for (int qq = 0; qq < kQ; ++qq) {
      if (i0 + qq * (int)blockDim.x >= n4) break;  // uniform over the CTA
      const int i = i0 + qq * (int)blockDim.x + (int)threadIdx.x;
      const float4 v = vq[qq];
      float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
      // smallest power of two sc with m / sc <= 127 (1 for an all-zero block)
      const uint32_t tt = __float_as_uint(m * (1.0f / 127.0f));
      uint32_t e = tt & 0x7F800000u;
      if (tt & 0x007FFFFFu) e += 0x00800000u;
      const bool nz = m > 0.f && e != 0u;
      const float inv = nz ? __uint_as_float(0x7F000000u - e) : 1.0f;
      if (i < n4) {
        const float f[4] = {v.x * inv, v.y * inv, v.z * inv, v.w * inv};  // exact (power of two)
        uint32_t wh = 0, wm = 0, wl = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          int h, mi, li;
          const float hr = rint_small(f[j], h);
          const float r1 = __fsub_rn(f[j], hr);  // exact, |r1| <= 1/2
          const float mr = rint_small(__fmul_rn(r1, 254.f), mi);
          const float r2 = fmaf(r1, 254.f, -mr);  // |r2| <= 1/2
          rint_small(__fmul_rn(r2, 254.f), li);
          wh |= (uint32_t)(uint8_t)h << (8 * j);
          wm |= (uint32_t)(uint8_t)mi << (8 * j);
          wl |= (uint32_t)(uint8_t)li << (8 * j);
        }
        const int c = 4 * i, kb = c >> 5, cc = c & 31;
        *reinterpret_cast<uint32_t*>(lim + kb * 96 + cc) = wh;
        *reinterpret_cast<uint32_t*>(lim + kb * 96 + 32 + cc) = wm;
        *reinterpret_cast<uint32_t*>(lim + kb * 96 + 64 + cc) = wl;
        if ((i & 7) == 0) xsc[kb] = nz ? __uint_as_float(e) : 1.0f;
      }
    }
  }
}

template <int IN>
__global__ void __launch_bounds__(kMmaWarps * 32, 3) gemv_mma_kernel(const __grid_constant__ MmaGemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const MmaGemvPlan& p = a.p;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int sub = warp / p.ks, kw = warp % p.ks;  // row tile of the task, K part
  const int kb0 = kw * p.kpw, kb1 = min(p.nkb, kb0 + p.kpw);
  float* xs = reinterpret_cast<float*>(smem + p.xs_off);
  int8_t* lim = reinterpret_cast<int8_t*>(smem + p.lim_off);  // [nkb][3 limbs][32]
  float* xsc = reinterpret_cast<float*>(smem + p.xsc_off);    // [nkb]
  float* misc = reinterpret_cast<float*>(smem + p.misc_off);
  float* red = reinterpret_cast<float*>(smem + p.red_off);    // [2][8 warps][16 rows]

  uint4 A[kMmaAhead];
  uint32_t S[kMmaAhead];
  auto load = [&](int task, int k) {
    const int rt = task * p.tiles + sub;
#pragma unroll
    for (int u = 0; u < kMmaAhead; ++u) {
      const int kb = k + u;
      if (rt < p.nrt && kb < kb1) {
        const size_t tile = (size_t)rt * p.nkb + kb;
        A[u] = __ldg(a.q + tile * 32 + lane);
        S[u] = __ldg(a.sc + tile * 8 + g);
      } else {
        A[u] = make_uint4(0u, 0u, 0u, 0u);
        S[u] = 0u;
      }
    }
  };
  PrologueConst pc;
  prologue_const<IN>(a.f, p.cols, pc);
  int task = blockIdx.x;
  load(task, kb0);  // weights only: before the dependency wait
  issue_l2_prefetch(a.f);
  grid_dep_wait();
  grid_dep_launch();

  // activation: fused prologue (or x), then three int8 limbs per value
  if constexpr (IN != IN_PLAIN) fused_prologue<IN>(a.f, a.x, xs, misc, p.cols, &pc);
  if constexpr (IN == IN_PLAIN) limbs_cta<true>(a.x, p.cols, lim, xsc);
  else limbs_cta<false>(xs, p.cols, lim, xsc);
  __syncthreads();

  const int out_mode = a.f.out_mode;
  const int erows = p.tiles * 16;  // output rows of a task
  unsigned long long best = 0ull;
  constexpr float kInv1 = 1.0f / 254.0f, kInv2 = 1.0f / 64516.0f;
  for (int it = 0; task < p.ntasks; task += gridDim.x, ++it) {
    const int rt = task * p.tiles + sub;
    float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
    for (int k = kb0; k < kb1; k += kMmaAhead) {
      uint4 Ac[kMmaAhead];
      uint32_t Sc[kMmaAhead];
#pragma unroll
      for (int u = 0; u < kMmaAhead; ++u) {
        Ac[u] = A[u];
        Sc[u] = S[u];
      }
      if (k + kMmaAhead < kb1) load(task, k + kMmaAhead);           // the row tile's next blocks
      else if (task + (int)gridDim.x < p.ntasks) load(task + gridDim.x, kb0);  // the next task's first
#pragma unroll
      for (int u = 0; u < kMmaAhead; ++u) {
        const int kb = k + u;
        if (kb < kb1 && rt < p.nrt) {
          uint32_t b0 = 0u, b1 = 0u;
          if (g < 3) {
            b0 = *reinterpret_cast<const uint32_t*>(lim + kb * 96 + g * 32 + 4 * t);
            b1 = *reinterpret_cast<const uint32_t*>(lim + kb * 96 + g * 32 + 16 + 4 * t);
          }
          int d[4];
          mma_s8(d, Ac[u], b0, b1);
          const float s = xsc[kb];
          const float dg = __fmul_rn(f16_bits_to_f32((uint16_t)(Sc[u] & 0xFFFFu)), s);
          const float dg8 = __fmul_rn(f16_bits_to_f32((uint16_t)(Sc[u] >> 16)), s);
          acc0 = fmaf(mma_f32(d[0]), dg, acc0);
          acc1 = fmaf(mma_f32(d[1]), dg, acc1);
          acc2 = fmaf(mma_f32(d[2]), dg8, acc2);
          acc3 = fmaf(mma_f32(d[3]), dg8, acc3);
        }
      }
    }
    // limbs: lane t = 0 holds columns 0 (h) and 1 (m), lane t = 1 column 2 (l)
    const float lo_g = __shfl_down_sync(0xffffffffu, acc0, 1);
    const float lo_g8 = __shfl_down_sync(0xffffffffu, acc2, 1);
    float* rb = red + (it & 1) * (kMmaWarps * 16);
    if (t == 0) {
      rb[warp * 16 + g] = fmaf(lo_g, kInv2, fmaf(acc1, kInv1, acc0));
      rb[warp * 16 + g + 8] = fmaf(lo_g8, kInv2, fmaf(acc3, kInv1, acc2));
    }
    __syncthreads();
    if ((int)threadIdx.x < erows) {
      const unsigned emask = erows >= 32 ? 0xffffffffu : 0x0000ffffu;  // erows: 16, 32, 64 or 128
      const int sr = threadIdx.x >> 4, rr = threadIdx.x & 15;
      float s = 0.f;
      for (int w = 0; w < p.ks; ++w) s += rb[(sr * p.ks + w) * 16 + rr];
      const int row = (task * p.tiles + sr) * 16 + rr;
      const bool ok = row < p.rows;
      if (out_mode == OUT_GELU_PAIR) {
        const float up = __shfl_xor_sync(emask, s, 1);
        if (ok && !(row & 1)) a.y[row >> 1] = __fmul_rn(gelu_ref(s), up);
      } else if (out_mode == OUT_SOFTCAP_ARGMAX) {
        if (ok) {
          const float c = softcap_ref(s, a.f.softcap);
          a.y[row] = c;
          const unsigned long long key = argmax_key(c, row);
          best = key > best ? key : best;
        }
      } else if (ok) {
        a.y[row] = s;
      }
    }
  }
  if (out_mode == OUT_SOFTCAP_ARGMAX && (int)threadIdx.x < erows) {
    const unsigned emask = erows >= 32 ? 0xffffffffu : 0x0000ffffu;
    for (int o = erows >= 32 ? 16 : 8; o > 0; o >>= 1) {
      const unsigned long long v = __shfl_xor_sync(emask, best, o);
      best = v > best ? v : best;
    }
    if (lane == 0 && best) atomicMax(a.f.argmax, best);
  }
}

using MmaFn = void (*)(const MmaGemvArgs);

static MmaFn mma_fn(int in_mode) {
  switch (in_mode) {
    case IN_PLAIN: return gemv_mma_kernel<IN_PLAIN>;
    case IN_NORM: return gemv_mma_kernel<IN_NORM>;
    case IN_RESID_NORM: return gemv_mma_kernel<IN_RESID_NORM>;
    case IN_EMBED_NORM: return gemv_mma_kernel<IN_EMBED_NORM>;
    case IN_MOE_MERGE: return gemv_mma_kernel<IN_MOE_MERGE>;
    default: return nullptr;
  }
}

size_t mma_packed_bytes(int rows, int cols) {
  const size_t tiles = (size_t)((rows + 15) / 16) * (size_t)(cols / 32);
  return tiles * 512 + tiles * 32;
}

int repack_q8_0_mma(const uint8_t* raw, int rows, int cols, uint8_t* packed, cudaStream_t st) {
  if (rows <= 0 || cols <= 0 || cols % 32) return (int)cudaErrorInvalidValue;
  const size_t tiles = (size_t)((rows + 15) / 16) * (size_t)(cols / 32);
  const long long threads = (long long)tiles * 32;
  repack_q8_0_mma_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
      raw, rows, cols, reinterpret_cast<uint4*>(packed), reinterpret_cast<uint32_t*>(packed + tiles * 512));
  return (int)cudaGetLastError();
}

MmaGemvPlan plan_gemv_mma(const DeviceInfo& dev, int rows, int cols, bool pair, bool fused) {
  MmaGemvPlan p{};
  p.rows = rows;
  p.cols = cols;
  p.pair = pair ? 1 : 0;
  if (rows <= 0 || cols <= 0 || cols % 32 || (pair && rows % 2)) return p;
  p.nrt = (rows + 15) / 16;
  p.nkb = cols / 32;
  p.tiles_total = (size_t)p.nrt * p.nkb;
  auto al = [](size_t v) { return (int)((v + 127) / 128 * 128); };
  p.fused = fused ? 1 : 0;
  p.xs_off = 0;
  p.lim_off = fused ? al((size_t)cols * 4) : 0;
  p.xsc_off = p.lim_off + al((size_t)p.nkb * 96);
  p.misc_off = p.xsc_off + al((size_t)p.nkb * 4);
  p.red_off = p.misc_off + 512;
  p.smem = (size_t)p.red_off + 2 * kMmaWarps * 16 * 4;
  if (p.smem > dev.smem_optin) return p;
  int occ = 3;
  for (int in = IN_PLAIN; in <= IN_MOE_MERGE; ++in) {
    MmaFn fn = mma_fn(in);
    int o = 0;
    if (!fn || cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dev.smem_optin) ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, fn, kMmaWarps * 32, p.smem) || o < 1) {
      cudaGetLastError();
      return p;
    }
    occ = std::min(occ, o);
  }
  // K split: the number of warps per row tile that gives the shortest
  // critical path, counted as task waves x blocks per warp (ties: more CTAs)
  const int resident = occ * dev.sms;
  long long best = -1;
  for (int ks = 1; ks <= kMmaWarps; ks *= 2) {
    const int tiles = kMmaWarps / ks;
    const int ntasks = (p.nrt + tiles - 1) / tiles;
    const int grid = std::min(ntasks, resident);
    const int waves = (ntasks + grid - 1) / grid;
    int kpw = (p.nkb + ks - 1) / ks;
    kpw = (kpw + kMmaAhead - 1) / kMmaAhead * kMmaAhead;  // whole load rounds
    const long long cost = (long long)waves * kpw;
    if (best < 0 || cost < best || (cost == best && grid > p.grid)) {
      best = cost;
      p.ks = ks;
      p.tiles = tiles;
      p.kpw = kpw;
      p.ntasks = ntasks;
      p.grid = grid;
    }
  }
  p.fast = 1;
  return p;
}

int launch_gemv_mma(const MmaGemvPlan& p, const uint8_t* packed, const float* x, float* y, const GemvFuse& f,
                    unsigned* status, cudaStream_t st, bool pdl) {
  cudaGetLastError();
  if (!p.fast || (f.out_mode == OUT_GELU_PAIR) != (p.pair != 0) || (f.in_mode != IN_PLAIN && !p.fused))
    return (int)cudaErrorInvalidValue;
  MmaFn fn = mma_fn(f.in_mode);
  if (!fn) return (int)cudaErrorInvalidValue;
  MmaGemvArgs a{p, reinterpret_cast<const uint4*>(packed),
                reinterpret_cast<const uint32_t*>(packed + p.tiles_total * 512), x, y, status, f};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(32 * kMmaWarps);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return (int)cudaLaunchKernelEx(&cfg, fn, a);
}

// ---------------------------------------------------------------- batched decode
// Many sequences at one step each (g4_batch_step): T <= kBatchMaxT tokens.

__device__ int g_batch_step0 = 0;  // step index 0: the batched embedding prologue reads in_tok[0]

struct BatchPrologueArgs {
  GemvFuse f;        // token 0's pointers; token s adds s * dim to x, f.r, f.m, f.x_out; f.in_tok = tokens[T]
  const float* x;    // [T][dim]: the residual stream (norm modes) or the activation (IN_PLAIN)
  int dim;
  int8_t* lim;       // [T][dim/32][96] int8 limbs
  float* lsc;        // [T][dim/32] block scales
};

// One CTA per token: the decoder's fused prologue of that token (norms,
// residual, embedding, MoE merge; the new residual stored by every CTA), then
// its activation as int8 limbs for gemm_mma_batch_kernel.
__global__ void __launch_bounds__(512) batch_prologue_kernel(const __grid_constant__ BatchPrologueArgs a) {
  extern __shared__ __align__(16) float bxs[];  // [dim] activation, then 64 floats of reduction space
  const int s = blockIdx.x, nkb = a.dim / 32;
  const size_t off = (size_t)s * a.dim;
  int8_t* lim = a.lim + (size_t)s * nkb * 96;
  float* lsc = a.lsc + (size_t)s * nkb;
  if (a.f.in_mode == IN_PLAIN) {
    limbs_cta<true>(a.x + off, a.dim, lim, lsc);
    return;
  }
  GemvFuse f = a.f;
  f.store_all = 1;
  if (f.r) f.r += off;
  if (f.m) f.m += off;
  if (f.x_out) f.x_out += off;
  if (f.in_mode == IN_EMBED_NORM) {
    f.in_tok = a.f.in_tok + s;
    f.step = &g_batch_step0;
  }
  fused_prologue<-1>(f, a.x ? a.x + off : nullptr, bxs, bxs + a.dim, a.dim, nullptr);
  limbs_cta<false>(bxs, a.dim, lim, lsc);
}

struct MmaBatchArgs {
  MmaBatchPlan p;
  const uint4* q;       // repacked weights (repack_q8_0_mma)
  const uint32_t* sc;
  const int8_t* lim;    // [T][nkb][96]
  const float* lsc;     // [T][nkb]
  float* y;             // [T][ldy]
  int T, ldy, out_mode;
  float softcap;
  unsigned long long* argmax;  // OUT_SOFTCAP_ARGMAX: [T] keys (atomicMax)
  float* part;          // [splits][T][nrb * rows per block] partial sums (splits > 1)
  unsigned* tickets;    // [nrb] splits finished per row block
};

constexpr int kBatchKc = 4;      // blocks (32 columns) per staged chunk of the activations
constexpr int kBatchRow = 112;   // bytes per token in a staged block: 96 limb bytes + 16 (bank spread)
// Warps per row tile: two (each with half of the token groups) from 16 tokens
// on, so a warp holds fewer accumulators and more warps fit an SM.
__host__ __device__ constexpr int batch_wt(int ng) { return ng >= 2 ? 2 : 1; }
__host__ __device__ constexpr int batch_rt(int ng) { return 8 / batch_wt(ng); }  // row tiles per row block

// One output of the batched GEMM: plain, gelu(gate) * up (value of the even
// row, `up` its odd neighbour), or softcap with the token's arg-max key.
__device__ __forceinline__ void batch_out(const MmaBatchArgs& a, int row, int tk, float v, float up,
                                          unsigned long long& best) {
  if (a.out_mode == OUT_GELU_PAIR) {
    if (!(row & 1)) a.y[(size_t)tk * a.ldy + (row >> 1)] = __fmul_rn(gelu_ref(v), up);
  } else if (a.out_mode == OUT_SOFTCAP_ARGMAX) {
    const float c = softcap_ref(v, a.softcap);
    a.y[(size_t)tk * a.ldy + row] = c;
    const unsigned long long key = argmax_key(c, row);
    best = key > best ? key : best;
  } else {
    a.y[(size_t)tk * a.ldy + row] = v;
  }
}

// Y[t][row] = W[row] . x_t for T tokens on the repacked tiles.  A CTA task is
// a row block (batch_rt row tiles; batch_wt warps per tile, each with its share
// of the token groups) x one of `splits` K ranges;
// per block of 32 columns a warp runs one mma per limb and group of 8 tokens
// (the group's tokens are the B operand's columns), its next weight tile in
// flight.  The tokens' limbs travel through shared memory in chunks of
// kBatchKc blocks (cp.async, two stages) that the CTA's warps share.  With
// one split the warps finish their outputs directly; otherwise each split
// stores its partial sums, and the row block's last split to finish (a ticket
// counter) adds them in split order and finishes the outputs.
template <int NG>
__global__ void __launch_bounds__(kMmaWarps * 32, 3) gemm_mma_batch_kernel(const __grid_constant__ MmaBatchArgs a) {
  // [2][kBatchKc][8 NG][kBatchRow] limbs, [2][kBatchKc][8 NG] scales, [8 NG] arg-max keys, the last-split flag
  extern __shared__ __align__(16) uint8_t bsm[];
  constexpr int TT = 8 * NG;
  constexpr int WT = batch_wt(NG), RT = batch_rt(NG), NGW = NG / WT, RB = RT * 16;
  constexpr int kStage = kBatchKc * TT * kBatchRow;
  float* ssc = reinterpret_cast<float*>(bsm + 2 * kStage);
  unsigned long long* sbest = reinterpret_cast<unsigned long long*>(ssc + 2 * kBatchKc * TT);
  int& s_last = *reinterpret_cast<int*>(sbest + TT);
  const MmaBatchPlan& p = a.p;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int T = a.T, nkb = p.nkb;
  constexpr float kInv1 = 1.0f / 254.0f, kInv2 = 1.0f / 64516.0f;
  const int sub = warp % RT, half = warp / RT;  // row tile of the block, share of the token groups
  unsigned long long best[NGW][2];
#pragma unroll
  for (int gg = 0; gg < NGW; ++gg) best[gg][0] = best[gg][1] = 0ull;
  if (a.out_mode == OUT_SOFTCAP_ARGMAX)
    for (int i = threadIdx.x; i < TT; i += blockDim.x) sbest[i] = 0ull;

  auto stage = [&](int kb0, int kb_end, int b) {
    uint8_t* dst = bsm + b * kStage;
    for (int i = threadIdx.x; i < kBatchKc * T * 6; i += blockDim.x) {
      const int piece = i % 6, r = i / 6, tok = r % T, kk = r / T, kb = kb0 + kk;
      if (kb < kb_end)
        cp16(dst + (kk * TT + tok) * kBatchRow + 16 * piece, a.lim + ((size_t)tok * nkb + kb) * 96 + 16 * piece);
    }
    for (int i = threadIdx.x; i < kBatchKc * T; i += blockDim.x) {
      const int tok = i % T, kk = i / T, kb = kb0 + kk;
      if (kb < kb_end) ssc[(b * kBatchKc + kk) * TT + tok] = __ldcg(a.lsc + (size_t)tok * nkb + kb);
    }
    cp_commit();
  };

  for (int task = blockIdx.x; task < p.ntasks; task += gridDim.x) {
    const int rb = task / p.splits, sp = task % p.splits;
    const int rt = rb * RT + sub;
    const bool ract = rt < p.nrt && half * NGW * 8 < T;
    const int kb_beg = sp * p.kps, kb_end = min(nkb, kb_beg + p.kps);
    const int nch = (kb_end - kb_beg + kBatchKc - 1) / kBatchKc;
    float acc[NGW][4];
#pragma unroll
    for (int gg = 0; gg < NGW; ++gg) acc[gg][0] = acc[gg][1] = acc[gg][2] = acc[gg][3] = 0.f;
    const uint4* qt = a.q + (size_t)rt * nkb * 32 + lane;
    const uint32_t* st = a.sc + (size_t)rt * nkb * 8 + g;
    uint4 An = make_uint4(0u, 0u, 0u, 0u);
    uint32_t Sn = 0u;
    if (ract && kb_beg < kb_end) {
      An = __ldg(qt + (size_t)kb_beg * 32);
      Sn = __ldg(st + (size_t)kb_beg * 8);
    }
    if (nch > 0) stage(kb_beg, kb_end, 0);
    for (int ch = 0; ch < nch; ++ch) {
      if (ch + 1 < nch) {
        stage(kb_beg + (ch + 1) * kBatchKc, kb_end, (ch + 1) & 1);
        cp_wait<1>();
      } else {
        cp_wait<0>();
      }
      __syncthreads();  // chunk ch is in shared memory for every warp
      const uint8_t* bsrc = bsm + (ch & 1) * kStage;
      const float* scs = ssc + (ch & 1) * kBatchKc * TT;
      const int kn = min(kBatchKc, kb_end - kb_beg - ch * kBatchKc);
      for (int kk = 0; kk < kn; ++kk) {
        const int kb = kb_beg + ch * kBatchKc + kk;
        const uint4 A = An;
        const uint32_t S = Sn;
        if (ract && kb + 1 < kb_end) {  // the next weight tile in flight
          An = __ldg(qt + (size_t)(kb + 1) * 32);
          Sn = __ldg(st + (size_t)(kb + 1) * 8);
        }
        if (ract) {
          const float d0 = f16_bits_to_f32((uint16_t)(S & 0xFFFFu)), d8 = f16_bits_to_f32((uint16_t)(S >> 16));
#pragma unroll
          for (int gg = 0; gg < NGW; ++gg) {
            const int G = half * NGW + gg;
            if (G * 8 < T) {  // uniform
              const uint32_t* bp =
                  reinterpret_cast<const uint32_t*>(bsrc + (kk * TT + G * 8 + g) * kBatchRow + 4 * t);
              int dh[4], dm[4], dl[4];
              mma_s8(dh, A, bp[0], bp[4]);
              mma_s8(dm, A, bp[8], bp[12]);
              mma_s8(dl, A, bp[16], bp[20]);
              const float s0 = scs[kk * TT + G * 8 + 2 * t], s1 = scs[kk * TT + G * 8 + 2 * t + 1];
              const float sc[4] = {d0 * s0, d0 * s1, d8 * s0, d8 * s1};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float v = fmaf(mma_f32(dl[i]), kInv2, fmaf(mma_f32(dm[i]), kInv1, mma_f32(dh[i])));
                acc[gg][i] = fmaf(v, sc[i], acc[gg][i]);
              }
            }
          }
        }
      }
      __syncthreads();  // buffer (ch & 1) is free for chunk ch + 2
    }
    // lane: rows r0 = rt*16 + g and r0 + 8; tokens G*8 + 2t and G*8 + 2t + 1
    const int r0 = rt * 16 + g;
    if (p.splits == 1) {
      if (ract) {
#pragma unroll
        for (int gg = 0; gg < NGW; ++gg) {
          const int G = half * NGW + gg;
          if (G * 8 < T) {
            float o[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) o[i] = __shfl_xor_sync(0xffffffffu, acc[gg][i], 4);  // row g ^ 1
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int row = r0 + 8 * (i >> 1), tk = G * 8 + 2 * t + (i & 1);
              if (row < p.rows && tk < T) batch_out(a, row, tk, acc[gg][i], o[i], best[gg][i & 1]);
            }
          }
        }
      }
      continue;
    }
    // split-K: partial sums of this split, then the row block's last split finishes
    float* pp = a.part + (size_t)sp * T * (p.nrb * RB);
    if (ract) {
#pragma unroll
      for (int gg = 0; gg < NGW; ++gg) {
        const int G = half * NGW + gg;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = r0 + 8 * (i >> 1), tk = G * 8 + 2 * t + (i & 1);
          if (tk < T) pp[(size_t)tk * (p.nrb * RB) + row] = acc[gg][i];
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      s_last = atomicAdd(a.tickets + rb, 1u) + 1 == (unsigned)p.splits;
    }
    __syncthreads();
    if (!s_last) continue;
    __threadfence();  // acquire: the other splits' partials are visible
    // thread -> (token, row pair) of the row block; sums in split order
    for (int e = threadIdx.x; e < T * (RB / 2); e += blockDim.x) {
      const int tk = e / (RB / 2), row = rb * RB + 2 * (e % (RB / 2));
      float v0 = 0.f, v1 = 0.f;
      for (int s2 = 0; s2 < p.splits; ++s2) {
        const float* q2 = a.part + ((size_t)s2 * T + tk) * (p.nrb * RB) + row;
        v0 += __ldcg(q2);
        v1 += __ldcg(q2 + 1);
      }
      unsigned long long bb = 0ull;
      if (row < p.rows) batch_out(a, row, tk, v0, v1, bb);
      if (row + 1 < p.rows && a.out_mode != OUT_GELU_PAIR) batch_out(a, row + 1, tk, v1, 0.f, bb);
      if (bb) atomicMax(&sbest[tk], bb);
    }
    if (threadIdx.x == 0) a.tickets[rb] = 0u;  // ready for the next launch
  }
  if (a.out_mode == OUT_SOFTCAP_ARGMAX) {
    // per token: the warps' bests (lanes g of one column t) and the split-K finishers' into shared memory
#pragma unroll
    for (int gg = 0; gg < NGW; ++gg)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int G = half * NGW + gg;
        unsigned long long b = best[gg][j];
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          const unsigned long long v = __shfl_xor_sync(0xffffffffu, b, o);
          b = v > b ? v : b;
        }
        const int tk = G * 8 + 2 * t + j;
        if (g == 0 && b && tk < T) atomicMax(&sbest[tk], b);
      }
    __syncthreads();
    for (int i = threadIdx.x; i < T; i += blockDim.x)
      if (sbest[i]) atomicMax(a.argmax + i, sbest[i]);
  }
}

using BatchFn = void (*)(const MmaBatchArgs);

static BatchFn batch_fn(int ng) {
  switch (ng) {
    case 1: return gemm_mma_batch_kernel<1>;
    case 2: return gemm_mma_batch_kernel<2>;
    case 4: return gemm_mma_batch_kernel<4>;
    case 8: return gemm_mma_batch_kernel<8>;
    default: return nullptr;
  }
}

MmaBatchPlan plan_gemm_mma_batch(const DeviceInfo& dev, int rows, int cols, int T) {
  MmaBatchPlan p{};
  p.rows = rows;
  p.cols = cols;
  if (rows <= 0 || cols <= 0 || cols % 32 || T <= 0 || T > kBatchMaxT) return p;
  p.ng = T <= 8 ? 1 : T <= 16 ? 2 : T <= 32 ? 4 : 8;
  p.nrt = (rows + 15) / 16;
  p.nkb = cols / 32;
  p.nrb = (p.nrt + batch_rt(p.ng) - 1) / batch_rt(p.ng);
  p.rb_rows = 16 * batch_rt(p.ng);
  p.smem = (size_t)2 * kBatchKc * 8 * p.ng * kBatchRow + (size_t)2 * kBatchKc * 8 * p.ng * 4 +
           (size_t)8 * p.ng * 8 + 16;
  BatchFn fn = batch_fn(p.ng);
  int occ = 0;
  if (!fn || cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dev.smem_optin) ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, kMmaWarps * 32, p.smem) || occ < 1) {
    cudaGetLastError();
    return p;
  }
  // K splits: enough tasks for every resident CTA, whole staged chunks per split
  const int resident = occ * dev.sms;
  int splits = std::max(1, std::min(16, (resident + p.nrb - 1) / p.nrb));
  p.kps = ((p.nkb + splits - 1) / splits + kBatchKc - 1) / kBatchKc * kBatchKc;
  p.splits = (p.nkb + p.kps - 1) / p.kps;
  p.ntasks = p.nrb * p.splits;
  p.grid = std::min(p.ntasks, resident);
  p.fast = 1;
  return p;
}

int launch_gemm_mma_batch(const MmaBatchPlan& p, const uint8_t* packed, const int8_t* lim, const float* lsc, int T,
                          float* y, int ldy, int out_mode, float softcap, unsigned long long* argmax,
                          float* partials, unsigned* tickets, cudaStream_t st) {
  cudaGetLastError();
  if (!p.fast || T <= 0 || T > 8 * p.ng || (out_mode == OUT_SOFTCAP_ARGMAX && !argmax) ||
      (out_mode == OUT_GELU_PAIR && p.rows % 2) || (p.splits > 1 && (!partials || !tickets)))
    return (int)cudaErrorInvalidValue;
  BatchFn fn = batch_fn(p.ng);
  const size_t tiles_total = (size_t)p.nrt * p.nkb;
  MmaBatchArgs a{p, reinterpret_cast<const uint4*>(packed),
                 reinterpret_cast<const uint32_t*>(packed + tiles_total * 512), lim, lsc, y, T, ldy, out_mode,
                 softcap, argmax, partials, tickets};
  fn<<<p.grid, kMmaWarps * 32, p.smem, st>>>(a);
  return (int)cudaGetLastError();
}

int launch_batch_prologue(const GemvFuse& f, const float* x, int dim, int T, int8_t* lim, float* lsc,
                          cudaStream_t st) {
  cudaGetLastError();
  // the activation row and the reduction space fit the default 48 KB of shared memory
  if (T <= 0 || dim <= 0 || dim % 32 || (size_t)(dim + 64) * 4 > 48 * 1024) return (int)cudaErrorInvalidValue;
  BatchPrologueArgs a{f, x, dim, lim, lsc};
  const size_t smem = (size_t)(dim + 64) * 4;
  batch_prologue_kernel<<<T, 512, smem, st>>>(a);
  return (int)cudaGetLastError();
}

}  // namespace g4
