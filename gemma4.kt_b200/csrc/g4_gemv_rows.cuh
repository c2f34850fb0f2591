// g4_gemv_rows.cuh -- per-block dot products for the lane-per-row GEMV and
// the MoE expert kernels.
//
// Each lane owns one row (or a share of its blocks when several lanes split a
// row) and walks its row segment in shared memory block by block; the
// activations are read as broadcasts.  The arithmetic restates the reference vectorDots
// (Q8_0FloatTensor.kt:39-142, Q4_KFloatTensor.kt:86-207,
// Q6_KFloatTensor.kt:111-250, BF16FloatTensor.kt:35-74,
// F32FloatTensor.kt:37-66) with a different summation order; results agree
// within rounding, not bitwise.
//
// The quantized formats multiply on the integer pipe (int16 activations, dp2a
// on the stored codes, below).  BF16 / F32 use packed fp32 fma.  f_magic23
// (int -> float without the quarter-rate I2F: byte b under exponent 150 is
// 2^23 + b) serves the MoE kernels' float decoders.
#pragma once
#include "g4_common.cuh"

namespace g4 {

__device__ __forceinline__ float f_magic23(uint32_t m, uint32_t byte) {
  // byte 0 <- m.byte[byte], byte 3 <- 0x4B: 2^23 + b
  return __uint_as_float(__byte_perm(m, 0x4B000000u, 0x7440u | byte));
}

__device__ __forceinline__ float4 lds_f4(const float* p) {
  uint4 v = lds128(p);
  return make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w));
}

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

template <int PR>
__device__ __forceinline__ void add_row(float (&acc)[PR], int r, float v) {
  if constexpr (PR == 1) {
    acc[0] += v;
  } else {
#pragma unroll
    for (int k = 0; k < PR; ++k) acc[k] += (k == r) ? v : 0.f;
  }
}

// ---------------------------------------------------------------- int16 activations
// The quantized formats' dot products also run on the integer pipe: the
// activation vector is held as int16 per 32-column block b, x ~= s_b * xq with
// s_b a power of two and |xq| <= 32760, and dp2a multiplies two int16
// activations by two weight bytes into an exact int32 sum (the 4- or 6-bit
// codes are used as bytes, no conversion to float).  The rounding of x is
// below 2^-15 of the block's largest entry, about 1e-5 relative error on a
// dot product.  The min / offset terms keep using the fp32 column sums.
// The int16 array has 8 entries of padding after every 256 columns, so the
// lanes that share a row (reading blocks 256 columns apart) hit different
// shared-memory banks: column c is entry xq_at(c).
__device__ __forceinline__ int xq_at(int c) { return c + 8 * (c >> 8); }
__device__ __forceinline__ int dp2a_lo_su(uint32_t a_s16x2, uint32_t b_u8x4, int c) {
  int d;
  asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_s16x2), "r"(b_u8x4), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2a_hi_su(uint32_t a_s16x2, uint32_t b_u8x4, int c) {
  int d;
  asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_s16x2), "r"(b_u8x4), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2a_lo_ss(uint32_t a_s16x2, uint32_t b_s8x4, int c) {
  int d;
  asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_s16x2), "r"(b_s8x4), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2a_hi_ss(uint32_t a_s16x2, uint32_t b_s8x4, int c) {
  int d;
  asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_s16x2), "r"(b_s8x4), "r"(c));
  return d;
}
// 0 <= v < 2^23 as float without the quarter-rate I2F
__device__ __forceinline__ float small_u2f(uint32_t v) { return __uint_as_float(0x4B000000u | v) - 8388608.0f; }

// One warp per 32-column block: xq = rint(x / s), s = the smallest power of
// two with max|x| / s <= 32760 (s = 1 for an all-zero block).
__device__ __forceinline__ void quantize_x16(const float* xs, int cols, int16_t* xq, float* xsc32) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, W = blockDim.x >> 5;
  for (int bk = warp; bk < cols / 32; bk += W) {
    const float v = xs[32 * bk + lane];
    float m = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const uint32_t t = __float_as_uint(m * (1.0f / 32760.0f));
    uint32_t e = t & 0x7F800000u;
    if (t & 0x007FFFFFu) e += 0x00800000u;
    const bool nz = m > 0.f && e != 0u;
    const float sc = nz ? __uint_as_float(e) : 1.0f;
    const float inv = nz ? __uint_as_float(0x7F000000u - e) : 1.0f;  // 1 / sc, exact
    xq[xq_at(32 * bk + lane)] = (int16_t)__float2int_rn(v * inv);
    if (lane == 0) xsc32[bk] = sc;
  }
}

// Two-part activations (X2): x = s_b * (xq + xql / 65536), the second int16
// holding the rounding remainder of the first, so the products carry about
// 31 bits of each activation (fp32-level dot products) at twice the dp2a
// work.  The whole-model decoder uses this form: its attention (scale 1.0 on
// RMS-normalised q and k) turns activation errors of a few 1e-5 into
// visibly different attention weights.
constexpr float kLoScale = 1.0f / 65536.0f;

// Q4_K on int16 activations.  Low nibbles are the bytes w & 0x0F, high nibbles
// stay in place as 16 * q (w & 0xF0): one mask per four codes each.
template <int PR, bool X2 = false>
__device__ __forceinline__ void block_q4k_i16(const uint8_t* blk, int e0, int cols, const int16_t* xq,
                                              const float* xsc32, const float* xsum32, float (&acc)[PR],
                                              const int16_t* xql = nullptr) {
  const uint4 h = lds128(blk);
  const float d = f16_bits_to_f32((uint16_t)(h.x & 0xFFFFu));
  const float dmin = f16_bits_to_f32((uint16_t)(h.x >> 16));
  // getScaleMinK4 (Q4_KFloatTensor.kt:70-84) for all 8 sub-blocks, byte-parallel
  const uint32_t sc03 = h.y & 0x3F3F3F3Fu, mn03 = h.z & 0x3F3F3F3Fu;
  const uint32_t sc47 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
  const uint32_t mn47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int eg = e0 + 64 * g;
    const int col = PR == 1 ? eg : eg % cols;
    const int rr = PR == 1 ? 0 : eg / cols;
    const int16_t* xp = xq + xq_at(col);  // the 64 columns of a group share one 256-column span
    const uint4 qa = lds128(blk + 16 + 32 * g), qb = lds128(blk + 32 + 32 * g);
    int alo = 0, ahi = 0, alo2 = 0, ahi2 = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint2 xl = *reinterpret_cast<const uint2*>(xp + 4 * k);
      const uint2 xh = *reinterpret_cast<const uint2*>(xp + 32 + 4 * k);
      const uint32_t w = k == 0 ? qa.x : k == 1 ? qa.y : k == 2 ? qa.z : k == 3 ? qa.w
                       : k == 4 ? qb.x : k == 5 ? qb.y : k == 6 ? qb.z : qb.w;
      const uint32_t lo = w & 0x0F0F0F0Fu, hi = w & 0xF0F0F0F0u;
      alo = dp2a_lo_su(xl.x, lo, alo);
      alo = dp2a_hi_su(xl.y, lo, alo);
      ahi = dp2a_lo_su(xh.x, hi, ahi);
      ahi = dp2a_hi_su(xh.y, hi, ahi);
      if constexpr (X2) {
        const int16_t* xpl = xql + xq_at(col);
        const uint2 yl = *reinterpret_cast<const uint2*>(xpl + 4 * k);
        const uint2 yh = *reinterpret_cast<const uint2*>(xpl + 32 + 4 * k);
        alo2 = dp2a_lo_su(yl.x, lo, alo2);
        alo2 = dp2a_hi_su(yl.y, lo, alo2);
        ahi2 = dp2a_lo_su(yh.x, hi, ahi2);
        ahi2 = dp2a_hi_su(yh.y, hi, ahi2);
      }
    }
    const float flo = X2 ? fmaf((float)alo2, kLoScale, (float)alo) : (float)alo;
    const float fhi = X2 ? fmaf((float)ahi2, kLoScale, (float)ahi) : (float)ahi;
    const uint32_t scw = g < 2 ? sc03 : sc47, mnw = g < 2 ? mn03 : mn47;
    const int b0 = (2 * g) & 3;
    const float sc_lo = small_u2f((scw >> (8 * b0)) & 0xFFu), sc_hi = small_u2f((scw >> (8 * b0 + 8)) & 0xFFu);
    const float mn_lo = small_u2f((mnw >> (8 * b0)) & 0xFFu), mn_hi = small_u2f((mnw >> (8 * b0 + 8)) & 0xFFu);
    const float s_lo = xsc32[col / 32], s_hi = xsc32[col / 32 + 1] * 0.0625f;
    const float xs_lo = xsum32[col / 32], xs_hi = xsum32[col / 32 + 1];
    // sum_i (d*sc*q_i - dmin*m) x_i over both sub-blocks of the group
    float v = (d * sc_lo) * (s_lo * flo);
    v = fmaf(d * sc_hi, s_hi * fhi, v);
    v = fmaf(-dmin, fmaf(mn_lo, xs_lo, mn_hi * xs_hi), v);
    add_row<PR>(acc, rr, v);
  }
}

// Q8_0 on int16 activations: the int8 codes are dp2a's signed bytes as stored.
template <bool X2 = false>
__device__ __forceinline__ void block_q8_0_i16(const uint8_t* blk, int col, const int16_t* xq, const float* xsc32,
                                               float& acc, const int16_t* xql = nullptr) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(blk);
  const uint8_t* b4 = reinterpret_cast<const uint8_t*>(a & ~uintptr_t(3));
  const uint32_t sh = (uint32_t)(a & 3u);  // 0 or 2
  uint32_t w[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) w[i] = lds32(b4 + 4 * i);
  const float d = f16_bits_to_f32((uint16_t)(sh ? (w[0] >> 16) : (w[0] & 0xFFFFu)));
  int s = 0, s2 = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    // quants start at byte 2 + sh of b4: a 16- or 32-bit clamped funnel shift
    const uint32_t m = __funnelshift_rc(w[k], w[k + 1], 16u + 8u * sh);
    const uint2 xv = *reinterpret_cast<const uint2*>(xq + xq_at(col) + 4 * k);
    s = dp2a_lo_ss(xv.x, m, s);
    s = dp2a_hi_ss(xv.y, m, s);
    if constexpr (X2) {
      const uint2 yv = *reinterpret_cast<const uint2*>(xql + xq_at(col) + 4 * k);
      s2 = dp2a_lo_ss(yv.x, m, s2);
      s2 = dp2a_hi_ss(yv.y, m, s2);
    }
  }
  const float fs = X2 ? fmaf((float)s2, kLoScale, (float)s) : (float)s;
  acc = fmaf(fs * xsc32[col / 32], d, acc);  // fma(sum, d, acc) as Q8_0FloatTensor.kt:77
}

// Q6_K on int16 activations: the 6-bit codes as bytes 0..63; sum (q - 32) x =
// s_b * sum(q xq) - 32 * sum x per 16-weight group.
template <int PR, bool X2 = false>
__device__ __forceinline__ void block_q6k_i16(const uint8_t* blk, int e0, int cols, const int16_t* xq,
                                              const float* xsc32, const float* xsum16, float (&acc)[PR],
                                              const int16_t* xql = nullptr) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(blk);
  const uint8_t* b4 = reinterpret_cast<const uint8_t*>(a & ~uintptr_t(3));
  const uint32_t sh = 8u * (uint32_t)(a & 3u);  // 0 or 16 bits
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
    const uint32_t scw0 = __funnelshift_r(s0, s1, sh);  // sc[8h + 0..3]
    const uint32_t scw1 = __funnelshift_r(s1, s2, sh);  // sc[8h + 4..7]
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int ebase = e0 + 128 * h + 16 * c;
      int a4[4] = {0, 0, 0, 0}, b4[4] = {0, 0, 0, 0};
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
          const uint2 xv = *reinterpret_cast<const uint2*>(xq + xq_at(PR == 1 ? e : e % cols));
          a4[sub] = dp2a_lo_su(xv.x, m[sub], a4[sub]);
          a4[sub] = dp2a_hi_su(xv.y, m[sub], a4[sub]);
          if constexpr (X2) {
            const uint2 yv = *reinterpret_cast<const uint2*>(xql + xq_at(PR == 1 ? e : e % cols));
            b4[sub] = dp2a_lo_su(yv.x, m[sub], b4[sub]);
            b4[sub] = dp2a_hi_su(yv.y, m[sub], b4[sub]);
          }
        }
      }
#pragma unroll
      for (int sub = 0; sub < 4; ++sub) {
        const int e = ebase + 32 * sub;
        const int col = PR == 1 ? e : e % cols;
        const int rr = PR == 1 ? 0 : e / cols;
        // sc index 8h + 2*sub + c (Q6_KFloatTensor.kt:70)
        const int si = 2 * sub + c;
        // int8 scale as float without I2F: (sc + 128) as an unsigned byte, minus 128
        const uint32_t scb = ((((si >> 2) ? scw1 : scw0) >> (8 * (si & 3))) & 0xFFu) ^ 0x80u;
        const float scf = small_u2f(scb) - 128.f;
        const float qx = X2 ? fmaf((float)b4[sub], kLoScale, (float)a4[sub]) : (float)a4[sub];
        const float v = (d * scf) * fmaf(xsc32[col / 32], qx, -32.f * xsum16[col / 16]);
        add_row<PR>(acc, rr, v);
      }
    }
  }
}

// ---------------------------------------------------------------- BF16 / F32
// 8 (BF16) or 4 (F32) weights per 16-byte load; segments are 16-byte aligned.
__device__ __forceinline__ void unit16_bf16(const uint8_t* p, int col, const float* xs, float2& s) {
  const float4 xa = lds_f4(xs + col), xb = lds_f4(xs + col + 4);
  const uint4 w = lds128(p);
  s = __ffma2_rn(f2(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xFFFF0000u)), f2(xa.x, xa.y), s);
  s = __ffma2_rn(f2(__uint_as_float(w.y << 16), __uint_as_float(w.y & 0xFFFF0000u)), f2(xa.z, xa.w), s);
  s = __ffma2_rn(f2(__uint_as_float(w.z << 16), __uint_as_float(w.z & 0xFFFF0000u)), f2(xb.x, xb.y), s);
  s = __ffma2_rn(f2(__uint_as_float(w.w << 16), __uint_as_float(w.w & 0xFFFF0000u)), f2(xb.z, xb.w), s);
}

__device__ __forceinline__ void unit16_f32(const uint8_t* p, int col, const float* xs, float2& s) {
  const float4 xa = lds_f4(xs + col);
  const uint4 w = lds128(p);
  s = __ffma2_rn(f2(__uint_as_float(w.x), __uint_as_float(w.y)), f2(xa.x, xa.y), s);
  s = __ffma2_rn(f2(__uint_as_float(w.z), __uint_as_float(w.w)), f2(xa.z, xa.w), s);
}

}  // namespace g4
