// g4_gemv_dec.cu -- the decoder's matrix-vector products (Llama.forward's
// projections at batch 1: q|k|v, o, gate/up, down, the output projection),
// on sm_100a.
//
// A decode step runs dozens of small GEMVs (2-20 MB each) back to back, so
// what matters is the time to the first bytes and how many bytes are in
// flight per SM, not the streaming rate of a long kernel.  Design:
//  * CTAs of 8 warps take row groups of 8 rows in turn (persistent, 2-3 CTAs
//    per SM); the 8 warps split a group's blocks (K) into 8 segments;
//  * in a warp, 4 lanes share a row and the 8 rows of the group sit side by
//    side, so the 8 lanes at one column read the activations once (a
//    shared-memory broadcast) and each lane decodes whole units (a Q8_0
//    block, a 64-column group of a Q4_K block, half a Q6_K block);
//  * each warp copies its 8 row segments (16-byte aligned supersets) with
//    16-byte cp.async into its own slots, ns - 1 groups ahead of the one it
//    decodes; the first ns groups are requested before the kernel waits for
//    its predecessor (programmatic dependent launch: weights never change);
//  * the 8 warps' partial sums meet in shared memory (one barrier per group)
//    and warp 0 finishes the rows in a fixed order: plain, gelu(gate) * up on
//    interleaved rows, or the soft cap with the argmax key;
//  * the activation vector comes from the fused prologue (g4_fuse.cuh), once
//    per CTA, and is held as two-part int16 (fp32-level products).
#include "g4_fuse.cuh"
#include "g4_gemv.cuh"
#include "g4_gemv_rows.cuh"
#include "g4_internal.h"

#include <algorithm>

namespace g4 {

struct DecGemvArgs {
  DecGemvPlan p;
  const uint8_t* w;
  const float* x;
  float* y;
  unsigned* status;
  GemvFuse f;
};

// x rounded to the nearest integer (ties to even) for |x| < 2^22, as a float
// and as an int, on the FMA / ALU pipes (adding 1.5 * 2^23 leaves the integer
// in the low mantissa bits).
__device__ __forceinline__ float round_small(float x, int& i) {
  constexpr float kMagic = 12582912.0f;
  const float t = __fadd_rn(x, kMagic);
  i = __float_as_int(t) - 0x4B400000;
  return __fsub_rn(t, kMagic);
}


// Units a block is decoded in (one lane each).
template <int FMT>
struct DecUnits {
  static constexpr int kPerBlock = FMT == Q4_K ? 4 : FMT == Q6_K ? 2 : 1;
};

// Q4_K, 64-column group g of a block (Q4_KFloatTensor.kt:86-207): the same
// arithmetic as block_q4k_i16 for one group.
__device__ __forceinline__ float q4k_group_x2(const uint8_t* blk, int g, int e0, const int16_t* xq,
                                              const int16_t* xql, const float* xsc32, const float* xsum32) {
  const uint4 h = lds128(blk);
  const float d = f16_bits_to_f32((uint16_t)(h.x & 0xFFFFu));
  const float dmin = f16_bits_to_f32((uint16_t)(h.x >> 16));
  const uint32_t scw = g < 2 ? (h.y & 0x3F3F3F3Fu) : ((h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u));
  const uint32_t mnw = g < 2 ? (h.z & 0x3F3F3F3Fu) : (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u));
  const int col = e0 + 64 * g;
  const int16_t* xp = xq + xq_at(col);
  const int16_t* xpl = xql + xq_at(col);
  const uint4 qa = lds128(blk + 16 + 32 * g), qb = lds128(blk + 32 + 32 * g);
  int alo = 0, ahi = 0, alo2 = 0, ahi2 = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint2 xl = *reinterpret_cast<const uint2*>(xp + 4 * k);
    const uint2 xh = *reinterpret_cast<const uint2*>(xp + 32 + 4 * k);
    const uint2 yl = *reinterpret_cast<const uint2*>(xpl + 4 * k);
    const uint2 yh = *reinterpret_cast<const uint2*>(xpl + 32 + 4 * k);
    const uint32_t w = k == 0 ? qa.x : k == 1 ? qa.y : k == 2 ? qa.z : k == 3 ? qa.w
                     : k == 4 ? qb.x : k == 5 ? qb.y : k == 6 ? qb.z : qb.w;
    const uint32_t lo = w & 0x0F0F0F0Fu, hi = w & 0xF0F0F0F0u;
    alo = dp2a_lo_su(xl.x, lo, alo);
    alo = dp2a_hi_su(xl.y, lo, alo);
    ahi = dp2a_lo_su(xh.x, hi, ahi);
    ahi = dp2a_hi_su(xh.y, hi, ahi);
    alo2 = dp2a_lo_su(yl.x, lo, alo2);
    alo2 = dp2a_hi_su(yl.y, lo, alo2);
    ahi2 = dp2a_lo_su(yh.x, hi, ahi2);
    ahi2 = dp2a_hi_su(yh.y, hi, ahi2);
  }
  const float flo = fmaf((float)alo2, kLoScale, (float)alo);
  const float fhi = fmaf((float)ahi2, kLoScale, (float)ahi);
  const int b0 = (2 * g) & 3;
  const float sc_lo = small_u2f((scw >> (8 * b0)) & 0xFFu), sc_hi = small_u2f((scw >> (8 * b0 + 8)) & 0xFFu);
  const float mn_lo = small_u2f((mnw >> (8 * b0)) & 0xFFu), mn_hi = small_u2f((mnw >> (8 * b0 + 8)) & 0xFFu);
  const float s_lo = xsc32[col / 32], s_hi = xsc32[col / 32 + 1] * 0.0625f;
  const float xs_lo = xsum32[col / 32], xs_hi = xsum32[col / 32 + 1];
  float v = (d * sc_lo) * (s_lo * flo);
  v = fmaf(d * sc_hi, s_hi * fhi, v);
  return fmaf(-dmin, fmaf(mn_lo, xs_lo, mn_hi * xs_hi), v);
}

// Q6_K, 128-column half h of a block (Q6_KFloatTensor.kt:111-250): the same
// arithmetic as block_q6k_i16 for one half.
__device__ __forceinline__ float q6k_half_x2(const uint8_t* blk, int h, int e0, const int16_t* xq,
                                             const int16_t* xql, const float* xsc32, const float* xsum16) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(blk);
  const uint8_t* b4 = reinterpret_cast<const uint8_t*>(a & ~uintptr_t(3));
  const uint32_t sh = 8u * (uint32_t)(a & 3u);
  const float d = f16_bits_to_f32((uint16_t)(__funnelshift_r(lds32(b4 + 208), lds32(b4 + 212), sh) & 0xFFFFu));
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
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int ebase = e0 + 128 * h + 16 * c;
    int a4[4] = {0, 0, 0, 0}, b4s[4] = {0, 0, 0, 0};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t la = qa[4 * c + k], lb = qb[4 * c + k], hh = qh[4 * c + k];
      uint32_t m[4];
      m[0] = (la & 0x0F0F0F0Fu) | ((hh << 4) & 0x30303030u);
      m[1] = (lb & 0x0F0F0F0Fu) | ((hh << 2) & 0x30303030u);
      m[2] = ((la >> 4) & 0x0F0F0F0Fu) | (hh & 0x30303030u);
      m[3] = ((lb >> 4) & 0x0F0F0F0Fu) | ((hh >> 2) & 0x30303030u);
#pragma unroll
      for (int sub = 0; sub < 4; ++sub) {
        const int e = ebase + 32 * sub + 4 * k;
        const uint2 xv = *reinterpret_cast<const uint2*>(xq + xq_at(e));
        const uint2 yv = *reinterpret_cast<const uint2*>(xql + xq_at(e));
        a4[sub] = dp2a_lo_su(xv.x, m[sub], a4[sub]);
        a4[sub] = dp2a_hi_su(xv.y, m[sub], a4[sub]);
        b4s[sub] = dp2a_lo_su(yv.x, m[sub], b4s[sub]);
        b4s[sub] = dp2a_hi_su(yv.y, m[sub], b4s[sub]);
      }
    }
#pragma unroll
    for (int sub = 0; sub < 4; ++sub) {
      const int col = ebase + 32 * sub;
      const int si = 2 * sub + c;  // sc index 8h + 2*sub + c (Q6_KFloatTensor.kt:70)
      const uint32_t scb = ((((si >> 2) ? scw1 : scw0) >> (8 * (si & 3))) & 0xFFu) ^ 0x80u;
      const float scf = small_u2f(scb) - 128.f;
      const float qx = fmaf((float)b4s[sub], kLoScale, (float)a4[sub]);
      acc += (d * scf) * fmaf(xsc32[col / 32], qx, -32.f * xsum16[col / 16]);
    }
  }
  return acc;
}

template <int FMT>
__device__ __forceinline__ float dec_unit(const uint8_t* blk, int sub, int e0, const int16_t* xq, const int16_t* xql,
                                          const float* xsc32, const float* xsum16, const float* xsum32) {
  if constexpr (FMT == Q4_K) return q4k_group_x2(blk, sub, e0, xq, xql, xsc32, xsum32);
  else if constexpr (FMT == Q6_K) return q6k_half_x2(blk, sub, e0, xq, xql, xsc32, xsum16);
  else {
    float acc = 0.f;
    block_q8_0_i16<true>(blk, e0, xq, xsc32, acc, xql);
    return acc;
  }
}

// Waits until at most n of this thread's cp.async groups are pending (n < kDecGemvMaxSlots).
__device__ __forceinline__ void cp_wait_n(int n) {
  if (n <= 0) cp_wait<0>();
  else if (n == 1) cp_wait<1>();
  else cp_wait<2>();
}

// p.ns slots per warp: groups it + 1 .. it + ns - 1 stream in while group it
// is decoded.  IN: the prologue mode (each kernel holds only its own code).
template <int FMT, int IN>
__global__ void __launch_bounds__(kDecWarps * 32, 3) gemv_dec_kernel(const __grid_constant__ DecGemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const DecGemvPlan& p = a.p;
  constexpr int BS = block_size(FMT), TS = type_size(FMT), UPB = DecUnits<FMT>::kPerBlock;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rs = lane & 7, sl = lane >> 3;  // row of the group, lane of the row
  const int b0 = warp * p.bps, b1 = min(p.bpr, b0 + p.bps);  // this warp's blocks of each row
  const int seg_len = b1 > b0 ? (b1 - b0) * TS : 0;
  uint8_t* slots = smem + p.stage_off + (size_t)warp * p.stage_bytes;  // ns x 8 rows x seg_cap
  float* xs = reinterpret_cast<float*>(smem + p.xs_off);
  float* xsum16 = reinterpret_cast<float*>(smem + p.xsum_off);
  float* xsum32 = xsum16 + p.cols / 16;
  float* xsc32 = xsum32 + p.cols / 32;
  int16_t* xq = reinterpret_cast<int16_t*>(smem + p.xq_off);
  int16_t* xql = reinterpret_cast<int16_t*>(smem + p.xq2_off);
  float* misc = reinterpret_cast<float*>(smem + p.misc_off);
  float* red = reinterpret_cast<float*>(smem + p.red_off);  // [2][8 warps][8 rows]

  // lane (rs, sl) copies chunks sl, sl + 4, ... of row rs's segment of group g
  auto issue = [&](int g, int slot) {
    const int row = g * 8 + rs;
    if (g < p.ngroups && row < p.rows && seg_len > 0) {
      const long long start = (long long)row * p.row_bytes + (long long)b0 * TS;
      const long long a0 = start & ~15ll;
      const int nch = (int)((start + seg_len - a0 + 15) >> 4);
      const uint8_t* src = a.w + a0;
      uint8_t* dst = slots + ((size_t)slot * 8 + rs) * p.seg_cap;
      for (int c = sl; c < nch; c += 4) cp16(dst + (size_t)c * 16, src + (size_t)c * 16);
    }
    cp_commit();  // one commit group per group, empty or not
  };
  PrologueConst pc;
  prologue_const<IN>(a.f, p.cols, pc);  // constant inputs: before the dependency wait
  const int g0 = blockIdx.x, G = gridDim.x, ns = p.ns;
  for (int k = 0; k < ns; ++k) issue(g0 + k * G, k);  // weights only: before the dependency wait
  issue_l2_prefetch(a.f);
  grid_dep_wait();
  grid_dep_launch();

  // activation: fused prologue (or x itself), then two-part int16 per 32 columns
  if constexpr (IN != IN_PLAIN)
    fused_prologue<IN>(a.f, a.x, xs, misc, p.cols, &pc);
  {
    constexpr int kQ = 6;  // float4s per thread loaded in one round
    const int n4 = p.cols / 4;
    for (int i0 = 0; i0 < n4; i0 += kQ * (int)blockDim.x) {
      float4 vq[kQ];
#pragma unroll
      for (int q = 0; q < kQ; ++q) {
        const int i = i0 + q * (int)blockDim.x + (int)threadIdx.x;
        vq[q] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < n4) {
          if constexpr (IN == IN_PLAIN) vq[q] = __ldcg(reinterpret_cast<const float4*>(a.x) + i);
          else vq[q] = reinterpret_cast<const float4*>(xs)[i];
        }
      }
#pragma unroll
      for (int q = 0; q < kQ; ++q) {
      if (i0 + q * (int)blockDim.x >= n4) break;  // uniform over the CTA
      const int i = i0 + q * (int)blockDim.x + (int)threadIdx.x;
      const bool act = i < n4;
      const float4 v = vq[q];
      float s16 = (v.x + v.y) + (v.z + v.w);
      s16 += __shfl_xor_sync(0xffffffffu, s16, 1);
      s16 += __shfl_xor_sync(0xffffffffu, s16, 2);
      const float s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 4);
      float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
      // smallest power of two sc with m / sc <= 32760 (1 for an all-zero block)
      const uint32_t t = __float_as_uint(m * (1.0f / 32760.0f));
      uint32_t e = t & 0x7F800000u;
      if (t & 0x007FFFFFu) e += 0x00800000u;
      const bool nz = m > 0.f && e != 0u;
      const float inv = nz ? __uint_as_float(0x7F000000u - e) : 1.0f;
      if (act) {
        const float f0 = v.x * inv, f1 = v.y * inv, f2 = v.z * inv, f3 = v.w * inv;  // exact (power of two)
        int i0q, i1q, i2q, i3q;
        const float r0 = round_small(f0, i0q), r1 = round_small(f1, i1q);
        const float r2 = round_small(f2, i2q), r3 = round_small(f3, i3q);
        *reinterpret_cast<uint2*>(xq + xq_at(4 * i)) =
            make_uint2((uint32_t)(uint16_t)i0q | ((uint32_t)(uint16_t)i1q << 16),
                       (uint32_t)(uint16_t)i2q | ((uint32_t)(uint16_t)i3q << 16));
        auto lo16 = [](float sv, float rv) {  // the remainder in units of 2^-16
          int r;
          round_small(__fmul_rn(__fsub_rn(sv, rv), 65536.0f), r);
          return (uint32_t)(uint16_t)max(-32767, min(32767, r));
        };
        *reinterpret_cast<uint2*>(xql + xq_at(4 * i)) =
            make_uint2(lo16(f0, r0) | (lo16(f1, r1) << 16), lo16(f2, r2) | (lo16(f3, r3) << 16));
        if ((i & 3) == 0) xsum16[i >> 2] = s16;
        if ((i & 7) == 0) {
          xsum32[i >> 3] = s32;
          xsc32[i >> 3] = nz ? __uint_as_float(e) : 1.0f;
        }
      }
      }
    }
  }
  __syncthreads();

  const int out_mode = a.f.out_mode;
  const int nunits = (b1 - b0) * UPB;
  unsigned long long best = 0ull;
  int slot = 0;
  for (int g = g0, it = 0; g < p.ngroups; g += G, ++it) {
    cp_wait_n(ns - 1);  // this warp's copies of group it have landed
    __syncwarp();
    float acc = 0.f;
    const int row = g * 8 + rs;
    if (row < p.rows) {
      const long long start = (long long)row * p.row_bytes + (long long)b0 * TS;
      const uint8_t* seg = slots + ((size_t)slot * 8 + rs) * p.seg_cap + (start & 15);
      for (int u = sl; u < nunits; u += 4) {
        const int bl = u / UPB, sub = u % UPB;
        acc += dec_unit<FMT>(seg + (size_t)bl * TS, sub, (b0 + bl) * BS, xq, xql, xsc32, xsum16, xsum32);
      }
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 8);
    acc += __shfl_xor_sync(0xffffffffu, acc, 16);
    float* rb = red + (it & 1) * 64;
    if (lane < 8) rb[warp * 8 + lane] = acc;
    __syncwarp();
    issue(g + ns * G, slot);  // this warp is done with the slot
    slot = slot + 1 == ns ? 0 : slot + 1;
    __syncthreads();
    if (warp == 0) {
      float s = 0.f;
      if (lane < 8) {
#pragma unroll
        for (int w = 0; w < kDecWarps; ++w) s += rb[w * 8 + lane];
      }
      const int r = g * 8 + lane;
      const bool ok = lane < 8 && r < p.rows;
      if (out_mode == OUT_GELU_PAIR) {
        const float up = __shfl_xor_sync(0xffffffffu, s, 1);
        if (ok && !(lane & 1)) a.y[r >> 1] = __fmul_rn(gelu_ref(s), up);
      } else if (out_mode == OUT_SOFTCAP_ARGMAX) {
        if (ok) {
          const float c = softcap_ref(s, a.f.softcap);
          a.y[r] = c;
          const unsigned long long k = argmax_key(c, r);
          best = k > best ? k : best;
        }
      } else if (ok) {
        a.y[r] = s;
      }
    }
  }
  cp_wait<0>();
  if (out_mode == OUT_SOFTCAP_ARGMAX && warp == 0) {
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
      const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
      best = v > best ? v : best;
    }
    if (lane == 0 && best) atomicMax(a.f.argmax, best);
  }
}

using DecFnG = void (*)(const DecGemvArgs);

template <int FMT>
static DecFnG dec_fn_in(int in_mode) {
  switch (in_mode) {
    case IN_PLAIN: return gemv_dec_kernel<FMT, IN_PLAIN>;
    case IN_NORM: return gemv_dec_kernel<FMT, IN_NORM>;
    case IN_RESID_NORM: return gemv_dec_kernel<FMT, IN_RESID_NORM>;
    case IN_EMBED_NORM: return gemv_dec_kernel<FMT, IN_EMBED_NORM>;
    case IN_MOE_MERGE: return gemv_dec_kernel<FMT, IN_MOE_MERGE>;
    default: return nullptr;
  }
}

static DecFnG dec_gemv_fn(int type, int in_mode) {
  switch (type) {
    case Q8_0: return dec_fn_in<Q8_0>(in_mode);
    case Q4_K: return dec_fn_in<Q4_K>(in_mode);
    case Q6_K: return dec_fn_in<Q6_K>(in_mode);
    default: return nullptr;
  }
}

DecGemvPlan plan_gemv_dec(const DeviceInfo& dev, int type, int rows, int cols, bool pair, bool fused) {
  DecGemvPlan p{};
  p.type = type;
  p.rows = rows;
  p.cols = cols;
  p.pair = pair ? 1 : 0;
  if (type != Q8_0 && type != Q4_K && type != Q6_K) return p;
  const int BS = block_size(type), TS = type_size(type);
  if (rows <= 0 || cols <= 0 || cols % BS || cols % 32 || (pair && rows % 2)) return p;
  p.row_bytes = cols / BS * TS;
  p.bpr = cols / BS;
  p.bps = (p.bpr + kDecWarps - 1) / kDecWarps;
  // 16-byte chunks of the aligned superset, rounded to an odd count: the
  // 8 row slots then start in 8 different bank quads
  int nch = (15 + p.bps * TS + 15) / 16;
  if (!(nch & 1)) ++nch;
  p.seg_cap = nch * 16;
  p.ngroups = (rows + 7) / 8;
  auto al = [](size_t v) { return (int)((v + 127) / 128 * 128); };
  p.fused = fused ? 1 : 0;
  p.xs_off = 0;
  p.xsum_off = fused ? al((size_t)cols * 4) : 0;
  p.xq_off = p.xsum_off + al((size_t)(cols / 16 + 2 * (cols / 32)) * 4);
  const int xq1 = al((size_t)(cols + 8 * ((cols + 255) / 256)) * 2);
  p.xq2_off = p.xq_off + xq1;
  p.misc_off = p.xq2_off + xq1;
  p.red_off = p.misc_off + 512;
  p.stage_off = p.red_off + 512;
  // slots per warp: as many groups in flight as a CTA will take (at most 3),
  // fewer when that costs a CTA per SM
  const int slot_bytes = 8 * p.seg_cap;
  DecGemvPlan best{};
  long long best_score = -1;
  for (int ns = 1; ns <= 3; ++ns) {
    DecGemvPlan q = p;
    q.stage_bytes = ns * slot_bytes;
    q.smem = (size_t)q.stage_off + (size_t)kDecWarps * q.stage_bytes;
    if (q.smem > dev.smem_optin) break;
    // every prologue mode's kernel: the attribute is per kernel and device and
    // shared by every plan, so the device maximum; the occupancy is the least
    int occ = 3;
    bool ok = true;
    for (int in = IN_PLAIN; in <= IN_MOE_MERGE && ok; ++in) {
      DecFnG fn = dec_gemv_fn(type, in);
      int o = 0;
      ok = fn && cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dev.smem_optin) ==
                     cudaSuccess &&
           cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, fn, kDecWarps * 32, q.smem) == cudaSuccess && o >= 1;
      occ = std::min(occ, o);
    }
    if (!ok) {
      cudaGetLastError();
      break;
    }
    q.ns = ns;
    const int slots_total = occ * dev.sms;
    const int gpc = (q.ngroups + slots_total - 1) / slots_total;  // groups per CTA
    q.grid = (q.ngroups + gpc - 1) / gpc;
    q.fast = 1;
    // bytes in flight per SM while a CTA decodes, ties to fewer slots
    const long long score = (long long)occ * std::min(ns, gpc) * 1000 - ns;
    if (score > best_score) {
      best_score = score;
      best = q;
    }
    if (gpc <= ns) break;  // more slots than groups per CTA buy nothing
  }
  if (!best.fast) return p;
  return best;
}

int launch_gemv_dec(const DecGemvPlan& p, const uint8_t* w, const float* x, float* y, const GemvFuse& f,
                    unsigned* status, cudaStream_t st, bool pdl) {
  cudaGetLastError();
  if (!p.fast || (f.out_mode == OUT_GELU_PAIR) != (p.pair != 0) || (f.in_mode != IN_PLAIN && !p.fused))
    return (int)cudaErrorInvalidValue;
  DecGemvArgs a{p, w, x, y, status, f};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(32 * kDecWarps);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  DecFnG fn = dec_gemv_fn(p.type, f.in_mode);
  if (!fn) return (int)cudaErrorInvalidValue;
  return (int)cudaLaunchKernelEx(&cfg, fn, a);
}

}  // namespace g4
