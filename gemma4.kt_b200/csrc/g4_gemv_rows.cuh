// g4_gemv_rows.cuh -- per-block dot products for the lane-per-row GEMV.
//
// Each lane owns one row (RL rows with activation reuse) and walks its row
// segment in shared memory block by block; the activations are read as
// warp-wide broadcasts.  The arithmetic restates the reference vectorDots
// (Q8_0FloatTensor.kt:39-142, Q4_KFloatTensor.kt:86-207,
// Q6_KFloatTensor.kt:111-250, BF16FloatTensor.kt:35-74,
// F32FloatTensor.kt:37-66) in fp32 with a different summation order; results
// agree within rounding, not bitwise.
//
// Integer -> float without the quarter-rate I2F pipe: a 4-bit or 6-bit code q
// placed in mantissa bits 16..21 under exponent 127 is the float 1 + q/128
// (one PRMT builds it from a byte that already holds 0x80|q).  Then
// sum_i q_i x_i = 128 * (sum_i f_i x_i - sum_i x_i), with sum_i x_i taken from a
// per-16-column table computed once per CTA.  The 1 stays within ~8x of the
// q/128 term, so the subtraction costs a few ulp, far inside the tolerance.
// Int8 codes use the exact 2^23 + b form plus one packed subtraction.
#pragma once
#include "g4_common.cuh"

namespace g4 {

__device__ __forceinline__ float f_one_plus(uint32_t m, uint32_t byte) {
  // byte 2 <- m.byte[byte] (0x80 | q), byte 3 <- 0x3F: 1 + q/128
  return __uint_as_float(__byte_perm(m, 0x3F000000u, 0x7044u | (byte << 8)));
}

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

// ---------------------------------------------------------------- Q4_K
// [fp16 d][fp16 dmin][scales 12][qs 128]; group g (64 weights) = low nibbles
// of qs[32g..32g+31] (sub-block 2g) then their high nibbles (sub-block 2g+1).
// Blocks are 144 = 9*16 bytes, so every block start is 16-byte aligned.
template <int RL, int PR>
__device__ __forceinline__ void block_q4k(const uint8_t* const* blk, int e0, int cols, const float* xs,
                                          const float* xsum16, float (&acc)[RL][PR]) {
  float d[RL], dm[RL];
  uint32_t sc03[RL], mn03[RL], sc47[RL], mn47[RL];
#pragma unroll
  for (int j = 0; j < RL; ++j) {
    uint4 h = lds128(blk[j]);
    d[j] = f16_bits_to_f32((uint16_t)(h.x & 0xFFFFu));
    dm[j] = f16_bits_to_f32((uint16_t)(h.x >> 16));
    // getScaleMinK4 (Q4_KFloatTensor.kt:70-84) for all 8 sub-blocks, byte-parallel
    sc03[j] = h.y & 0x3F3F3F3Fu;
    mn03[j] = h.z & 0x3F3F3F3Fu;
    sc47[j] = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    mn47[j] = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
  }
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int eg = e0 + 64 * g;
    const int col = PR == 1 ? eg : eg % cols;
    const int rr = PR == 1 ? 0 : eg / cols;
    const float* xp = xs + col;
    const float xs_lo = xsum16[col / 16] + xsum16[col / 16 + 1];
    const float xs_hi = xsum16[col / 16 + 2] + xsum16[col / 16 + 3];
    float2 alo[RL], ahi[RL];
    uint4 qa[RL], qb[RL];
#pragma unroll
    for (int j = 0; j < RL; ++j) {
      alo[j] = f2(0.f, 0.f);
      ahi[j] = f2(0.f, 0.f);
      qa[j] = lds128(blk[j] + 16 + 32 * g);
      qb[j] = lds128(blk[j] + 32 + 32 * g);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float4 xl = lds_f4(xp + 4 * k);
      const float4 xh = lds_f4(xp + 32 + 4 * k);
#pragma unroll
      for (int j = 0; j < RL; ++j) {
        const uint32_t w = k == 0 ? qa[j].x : k == 1 ? qa[j].y : k == 2 ? qa[j].z : k == 3 ? qa[j].w
                         : k == 4 ? qb[j].x : k == 5 ? qb[j].y : k == 6 ? qb[j].z : qb[j].w;
        const uint32_t ml = (w & 0x0F0F0F0Fu) | 0x80808080u;
        const uint32_t mh = ((w >> 4) & 0x0F0F0F0Fu) | 0x80808080u;
        alo[j] = __ffma2_rn(f2(f_one_plus(ml, 0), f_one_plus(ml, 1)), f2(xl.x, xl.y), alo[j]);
        alo[j] = __ffma2_rn(f2(f_one_plus(ml, 2), f_one_plus(ml, 3)), f2(xl.z, xl.w), alo[j]);
        ahi[j] = __ffma2_rn(f2(f_one_plus(mh, 0), f_one_plus(mh, 1)), f2(xh.x, xh.y), ahi[j]);
        ahi[j] = __ffma2_rn(f2(f_one_plus(mh, 2), f_one_plus(mh, 3)), f2(xh.z, xh.w), ahi[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < RL; ++j) {
      const uint32_t scw = g < 2 ? sc03[j] : sc47[j], mnw = g < 2 ? mn03[j] : mn47[j];
      const int b0 = (2 * g) & 3;
      const float d1 = d[j] * (float)((scw >> (8 * b0)) & 0xFFu);
      const float m1 = dm[j] * (float)((mnw >> (8 * b0)) & 0xFFu);
      const float d2 = d[j] * (float)((scw >> (8 * b0 + 8)) & 0xFFu);
      const float m2 = dm[j] * (float)((mnw >> (8 * b0 + 8)) & 0xFFu);
      // sum_i (d1*q_i - m1) x_i  with  sum_i q_i x_i = 128 * (s - sum_i x_i)
      const float slo = (alo[j].x + alo[j].y) - xs_lo;
      const float shi = (ahi[j].x + ahi[j].y) - xs_hi;
      float v = fmaf(128.f * d1, slo, -m1 * xs_lo);
      v += fmaf(128.f * d2, shi, -m2 * xs_hi);
      add_row<PR>(acc[j], rr, v);
    }
  }
}

// ---------------------------------------------------------------- Q8_0
// [fp16 d][int8 q x32]: 34 bytes, so a block starts on a 2-byte boundary.
template <int RL>
__device__ __forceinline__ void block_q8_0(const uint8_t* const* blk, int col, const float* xs,
                                           float (&acc)[RL][1]) {
  uint32_t q[RL][8];
  float d[RL];
#pragma unroll
  for (int j = 0; j < RL; ++j) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(blk[j]);
    const uint8_t* b4 = reinterpret_cast<const uint8_t*>(a & ~uintptr_t(3));
    const uint32_t sh = (uint32_t)(a & 3u);  // 0 or 2
    uint32_t w[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) w[i] = lds32(b4 + 4 * i);
    d[j] = f16_bits_to_f32((uint16_t)(sh ? (w[0] >> 16) : (w[0] & 0xFFFFu)));
    // quants start at byte 2 + sh of b4: shift by 16 or 32 bits (clamped funnel)
#pragma unroll
    for (int k = 0; k < 8; ++k) q[j][k] = __funnelshift_rc(w[k], w[k + 1], 16u + 8u * sh) ^ 0x80808080u;
  }
  float2 s[RL];
#pragma unroll
  for (int j = 0; j < RL; ++j) s[j] = f2(0.f, 0.f);
  const float2 bias = f2(8388736.0f, 8388736.0f);  // 2^23 + 128
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float4 xv = lds_f4(xs + col + 4 * k);
#pragma unroll
    for (int j = 0; j < RL; ++j) {
      const uint32_t m = q[j][k];
      const float2 q01 = __fadd2_rn(f2(f_magic23(m, 0), f_magic23(m, 1)), f2(-bias.x, -bias.y));
      const float2 q23 = __fadd2_rn(f2(f_magic23(m, 2), f_magic23(m, 3)), f2(-bias.x, -bias.y));
      s[j] = __ffma2_rn(q01, f2(xv.x, xv.y), s[j]);
      s[j] = __ffma2_rn(q23, f2(xv.z, xv.w), s[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < RL; ++j) acc[j][0] = fmaf(s[j].x + s[j].y, d[j], acc[j][0]);
}

// ---------------------------------------------------------------- Q6_K
// [ql 128][qh 64][int8 sc 16][fp16 d]: 210 bytes, 2-byte aligned starts.
// Half h (128 weights): for 16-byte column c and word k, qlA = ql[64h+16c+4k..],
// qlB = ql[64h+32+16c+4k..], qh = qh[32h+16c+4k..] give the codes of weights
// 128h + 32*sub + 16c + 4k + (0..3), sub = 0..3 (Q6_KFloatTensor.kt:163-178).
template <int RL, int PR>
__device__ __forceinline__ void block_q6k(const uint8_t* const* blk, int e0, int cols, const float* xs,
                                          const float* xsum16, float (&acc)[RL][PR]) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t qa[RL][8], qb[RL][8], qh[RL][8];
    float d[RL];
    uint32_t scw[RL][2];
#pragma unroll
    for (int j = 0; j < RL; ++j) {
      const uintptr_t a = reinterpret_cast<uintptr_t>(blk[j]);
      const uint8_t* b4 = reinterpret_cast<const uint8_t*>(a & ~uintptr_t(3));
      const uint32_t sh = 8u * (uint32_t)(a & 3u);  // 0 or 16 bits
      uint32_t w[9];
#pragma unroll
      for (int i = 0; i < 9; ++i) w[i] = lds32(b4 + 64 * h + 4 * i);
#pragma unroll
      for (int i = 0; i < 8; ++i) qa[j][i] = __funnelshift_r(w[i], w[i + 1], sh);
#pragma unroll
      for (int i = 0; i < 9; ++i) w[i] = lds32(b4 + 64 * h + 32 + 4 * i);
#pragma unroll
      for (int i = 0; i < 8; ++i) qb[j][i] = __funnelshift_r(w[i], w[i + 1], sh);
#pragma unroll
      for (int i = 0; i < 9; ++i) w[i] = lds32(b4 + 128 + 32 * h + 4 * i);
#pragma unroll
      for (int i = 0; i < 8; ++i) qh[j][i] = __funnelshift_r(w[i], w[i + 1], sh);
      uint32_t s0 = lds32(b4 + 192 + 8 * h), s1 = lds32(b4 + 196 + 8 * h), s2 = lds32(b4 + 200 + 8 * h);
      scw[j][0] = __funnelshift_r(s0, s1, sh);  // sc[8h + 0..3]
      scw[j][1] = __funnelshift_r(s1, s2, sh);  // sc[8h + 4..7]
      uint32_t dw = lds32(b4 + 208);
      uint32_t dw2 = lds32(b4 + 212);
      d[j] = f16_bits_to_f32((uint16_t)(__funnelshift_r(dw, dw2, sh) & 0xFFFFu));
    }
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float2 a4[RL][4];
#pragma unroll
      for (int j = 0; j < RL; ++j)
#pragma unroll
        for (int sub = 0; sub < 4; ++sub) a4[j][sub] = f2(0.f, 0.f);
      const int ebase = e0 + 128 * h + 16 * c;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float4 xv[4];
#pragma unroll
        for (int sub = 0; sub < 4; ++sub) {
          const int e = ebase + 32 * sub + 4 * k;
          xv[sub] = lds_f4(xs + (PR == 1 ? e : e % cols));
        }
#pragma unroll
        for (int j = 0; j < RL; ++j) {
          const uint32_t la = qa[j][4 * c + k], lb = qb[j][4 * c + k], hh = qh[j][4 * c + k];
          uint32_t m[4];
          m[0] = ((la & 0x0F0F0F0Fu) | 0x80808080u) | ((hh << 4) & 0x30303030u);
          m[1] = ((lb & 0x0F0F0F0Fu) | 0x80808080u) | ((hh << 2) & 0x30303030u);
          m[2] = (((la >> 4) & 0x0F0F0F0Fu) | 0x80808080u) | (hh & 0x30303030u);
          m[3] = (((lb >> 4) & 0x0F0F0F0Fu) | 0x80808080u) | ((hh >> 2) & 0x30303030u);
#pragma unroll
          for (int sub = 0; sub < 4; ++sub) {
            a4[j][sub] = __ffma2_rn(f2(f_one_plus(m[sub], 0), f_one_plus(m[sub], 1)), f2(xv[sub].x, xv[sub].y),
                                    a4[j][sub]);
            a4[j][sub] = __ffma2_rn(f2(f_one_plus(m[sub], 2), f_one_plus(m[sub], 3)), f2(xv[sub].z, xv[sub].w),
                                    a4[j][sub]);
          }
        }
      }
#pragma unroll
      for (int sub = 0; sub < 4; ++sub) {
        const int e = ebase + 32 * sub;
        const int col = PR == 1 ? e : e % cols;
        const int rr = PR == 1 ? 0 : e / cols;
        const float xsum = xsum16[col / 16];
#pragma unroll
        for (int j = 0; j < RL; ++j) {
          // sc index 8h + 2*sub + c (Q6_KFloatTensor.kt:70)
          const int si = 2 * sub + c;
          const int8_t sc = (int8_t)((scw[j][si >> 2] >> (8 * (si & 3))) & 0xFFu);
          // sum (q6 - 32) x = 128 * (s - xsum) - 32 * xsum
          const float s = (a4[j][sub].x + a4[j][sub].y) - xsum;
          const float v = (d[j] * (float)sc) * fmaf(128.f, s, -32.f * xsum);
          add_row<PR>(acc[j], rr, v);
        }
      }
    }
  }
}

// ---------------------------------------------------------------- BF16 / F32
// 8 (BF16) or 4 (F32) weights per 16-byte load; segments are 16-byte aligned.
template <int RL>
__device__ __forceinline__ void chunk16_bf16(const uint8_t* const* p, int col, const float* xs,
                                             float2 (&s)[RL]) {
  const float4 xa = lds_f4(xs + col), xb = lds_f4(xs + col + 4);
#pragma unroll
  for (int j = 0; j < RL; ++j) {
    const uint4 w = lds128(p[j]);
    s[j] = __ffma2_rn(f2(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xFFFF0000u)), f2(xa.x, xa.y), s[j]);
    s[j] = __ffma2_rn(f2(__uint_as_float(w.y << 16), __uint_as_float(w.y & 0xFFFF0000u)), f2(xa.z, xa.w), s[j]);
    s[j] = __ffma2_rn(f2(__uint_as_float(w.z << 16), __uint_as_float(w.z & 0xFFFF0000u)), f2(xb.x, xb.y), s[j]);
    s[j] = __ffma2_rn(f2(__uint_as_float(w.w << 16), __uint_as_float(w.w & 0xFFFF0000u)), f2(xb.z, xb.w), s[j]);
  }
}

template <int RL>
__device__ __forceinline__ void chunk16_f32(const uint8_t* const* p, int col, const float* xs, float2 (&s)[RL]) {
  const float4 xa = lds_f4(xs + col);
#pragma unroll
  for (int j = 0; j < RL; ++j) {
    const uint4 w = lds128(p[j]);
    s[j] = __ffma2_rn(f2(__uint_as_float(w.x), __uint_as_float(w.y)), f2(xa.x, xa.y), s[j]);
    s[j] = __ffma2_rn(f2(__uint_as_float(w.z), __uint_as_float(w.w)), f2(xa.z, xa.w), s[j]);
  }
}

}  // namespace g4
