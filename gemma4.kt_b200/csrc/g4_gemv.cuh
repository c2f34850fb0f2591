// g4_gemv.cuh -- launch plan of the streaming GEMV, the reference-exact
// element decoder (get) and the 16-weight unit dequantizer shared with the
// MoE expert kernels.
#pragma once
#include "g4_common.cuh"

namespace g4 {

struct GemvPlan {
  int type;
  int rows, cols;
  long long off;     // element offset into the tensor (thisOffset), block aligned
  int pr;            // rows per virtual row: after pr rows the block pattern repeats
  int nvrows;        // rows / pr
  int bpv;           // blocks per virtual row
  int cb;            // blocks per chunk (one bulk copy per row and chunk)
  int nchunks;       // chunks per virtual row
  int pitch;         // bytes per row slot in a stage (16 * odd: conflict-free)
  int lpr;           // lanes sharing one row (1, 2 or 4)
  int ns;            // stages per warp
  int warps;         // warps per CTA
  int split;         // 1: persistent, each warp owns whole row groups; >1: CTA per group
  int ngroups;       // row groups of 32/lpr virtual rows
  int grid;
  int xs_off, xsum_off, xq_off, xq2_off, bar_off, misc_off, ring_off, red_off;  // shared-memory carve-up
  size_t smem;
  int fast;          // 1: streaming kernel; 0: generic fallback
  int fused;         // planned for a fused prologue (fp32 activation staged in shared memory)
  int x2;            // two-part int16 activations (fp32-level products) for the quantized formats
};

// Plan of the decoder's GEMV (gemv_dec_kernel): CTAs of kDecWarps warps, each
// CTA taking row groups of 8 rows in turn, its warps splitting a group's
// blocks (K) between them; a warp's 8 rows are decoded by 4 lanes each, so
// the 8 lanes at one column read the activations once (shared-memory
// broadcast).  Row segments are copied with 16-byte cp.async into per-warp
// slots, the next group's in flight while this one is decoded.  Q8_0 / Q4_K /
// Q6_K rows of whole blocks, two-part activations.
constexpr int kDecWarps = 8;
constexpr int kDecGemvMaxSlots = 3;
struct DecGemvPlan {
  int type, rows, cols;
  int pair;          // 1: rows (2i, 2i + 1) -> one output each (gelu(gate) * up)
  int row_bytes;     // bytes of one row (whole blocks)
  int bpr, bps;      // blocks per row, per warp (K split)
  int seg_cap;       // bytes of a row-segment slot (16-byte multiple)
  int ngroups;       // row groups of 8
  int grid;
  int fused;         // room for a fused prologue (fp32 activation in shared memory at xs_off)
  int xs_off, xsum_off, xq_off, xq2_off, misc_off, red_off, stage_off;
  int ns;            // slots per warp (groups in flight), 1..kDecGemvMaxSlots
  int stage_bytes;   // per warp: ns slots x 8 rows x seg_cap
  size_t smem;
  int fast;
};

// Plan of the decoder's Q8_0 GEMV on the tensor cores (gemv_mma_kernel,
// g4_gemv_mma.cu): weights repacked into 16-row x 32-column mma tiles.
struct MmaGemvPlan {
  int rows, cols, pair, fused;
  int nrt, nkb;        // row tiles of 16, column blocks of 32
  size_t tiles_total;  // nrt * nkb (the scale words follow the tiles' code bytes)
  int ks;              // warps sharing one row tile (K split)
  int tiles;           // row tiles per CTA task (8 / ks)
  int kpw;             // blocks per warp
  int ntasks, grid;
  int xs_off, lim_off, xsc_off, misc_off, red_off;
  size_t smem;
  int fast;
};

// Plan of the batched decode GEMM (gemm_mma_batch_kernel, g4_gemv_mma.cu):
// T <= kBatchMaxT tokens on the repacked Q8_0 tiles, groups of 8 tokens.
constexpr int kBatchMaxT = 64;
struct MmaBatchPlan {
  int rows, cols, nrt, nkb;
  int ng;              // token groups of 8 the kernel is compiled for (1, 2, 4, 8)
  int nrb, rb_rows;    // row blocks (of 8 row tiles, or 4 from 16 tokens on) and their rows
  int splits, kps;     // K splits over CTAs and blocks per split (a multiple of the staged chunk)
  int ntasks, grid;
  size_t smem;
  int fast;
};
// Partial sums (floats) and tickets (row blocks) the batched GEMM needs for T tokens.
inline size_t mma_batch_partials(const MmaBatchPlan& p, int T) {
  return p.splits > 1 ? (size_t)p.splits * (size_t)T * (size_t)p.nrb * (size_t)p.rb_rows : 0;
}

// Options of plan_gemv.
struct GemvOpts {
  bool fused = false;     // room for a fused prologue (fp32 activation in shared memory)
  size_t max_smem = 0;    // cap on the plan's shared memory (0: the device maximum)
  bool exact_x = false;   // two-part int16 activations (Q8_0 / Q4_K / Q6_K, rows of whole blocks)
  bool latency = false;   // decode-size matrix: persistent CTAs with a warp (or half) per row
  bool pair_rows = false; // the epilogue pairs rows 2i, 2i + 1 (needs two rows per warp)
};

// Fused prologue / epilogue of the decoder's GEMV launches (GemvFuse.in_mode /
// out_mode).  The prologue turns the kernel's inputs into the activation
// vector before it is quantized; the epilogue post-processes each output row.
enum FuseIn : int {
  IN_PLAIN = 0,       // act = x
  IN_NORM = 1,        // act = rmsnorm(x, w_in)                                   Llama.kt:27-37
  IN_RESID_NORM = 2,  // xn = (x + rmsnorm(r, w_r)) * scale [r optional]; act = rmsnorm(xn, w_in)
  IN_EMBED_NORM = 3,  // xn = emb.get(tok * dim + i) * sqrt(dim); act = rmsnorm(xn, w_in)  Llama.kt:112-113
  IN_MOE_MERGE = 4,   // xn = (x + rmsnorm(rmsnorm(r, w_r) + m, w_m)) * scale; act = rmsnorm(xn, w_in)  Llama.kt:349-353
};
enum FuseOut : int {
  OUT_PLAIN = 0,           // y[row] = dot
  OUT_GELU_PAIR = 1,       // rows (2i, 2i+1) = (gate_i, up_i): y[i] = gelu(gate_i) * up_i   Llama.kt:357-360
  OUT_SOFTCAP_ARGMAX = 2,  // y[row] = cap * tanh(dot / cap) (cap > 0); argmax key (first maximum)  Llama.kt:403-406
};

struct GemvFuse {
  int in_mode = IN_PLAIN, out_mode = OUT_PLAIN;
  float eps = 1e-6f;
  float scale = 1.f;          // layer output scale (IN_RESID_NORM / IN_MOE_MERGE)
  float sqrt_dim = 1.f;       // IN_EMBED_NORM
  float softcap = 0.f;        // OUT_SOFTCAP_ARGMAX
  const float* w_in = nullptr;
  const float* r = nullptr;   // residual-branch output to normalise and add
  const float* w_r = nullptr;
  const float* m = nullptr;   // IN_MOE_MERGE: the expert half's output
  const float* w_m = nullptr;
  float* x_out = nullptr;     // CTA 0 stores xn (the new residual stream) here; must not alias x
  int store_all = 0;          // every CTA stores (batched prologues: one CTA per token, pointers offset)
  const uint8_t* emb = nullptr;  // IN_EMBED_NORM: embedding table (GGUF blocks)
  int emb_type = 0;
  const int* step = nullptr;     // IN_EMBED_NORM: token = in_tok[*step] >= 0 ? in_tok[*step] : *next_tok
  const int* in_tok = nullptr;
  const int* next_tok = nullptr;
  unsigned long long* argmax = nullptr;  // OUT_SOFTCAP_ARGMAX: atomicMax of (ordered value << 32 | ~row)
  // Weights of later kernels to pull into L2 while this one runs (16-byte
  // aligned ranges, sizes rounded up to 16 inside the tensors' padding); the
  // CTAs split each range and request it before they wait for their inputs.
  static constexpr int kPrefetch = 4;
  const uint8_t* pf[kPrefetch] = {nullptr, nullptr, nullptr, nullptr};
  long long pf_bytes[kPrefetch] = {0, 0, 0, 0};
};

// Bulk prefetch of global memory into L2 (no shared-memory destination).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// This CTA's share of the GemvFuse prefetch ranges, issued by one thread.
__device__ __forceinline__ void issue_l2_prefetch(const GemvFuse& f) {
  if (threadIdx.x != 0) return;
#pragma unroll
  for (int k = 0; k < GemvFuse::kPrefetch; ++k) {
    if (!f.pf[k] || f.pf_bytes[k] <= 0) continue;
    const long long n = (f.pf_bytes[k] + 15) & ~15ll;
    const long long share = ((n + gridDim.x - 1) / gridDim.x + 15) & ~15ll;
    const long long b0 = share * blockIdx.x, b1 = b0 + share < n ? b0 + share : n;
    for (long long o = b0; o < b1; o += 65536) {
      const long long len = b1 - o < 65536 ? b1 - o : 65536;
      prefetch_l2(f.pf[k] + o, (uint32_t)len);
    }
  }
}

// Magic-number int->float: 2^23 + b as float bits, then subtract 2^23 (+bias).
// Exact for 0 <= b < 2^23 and avoids the quarter-rate I2F path.
__device__ __forceinline__ float byte_as_float(uint32_t word, uint32_t sel_byte) {
  return __int_as_float((int)__byte_perm(word, 0x4B000000u, 0x7440u | sel_byte));
}

// Element get() with the reference's rounding order, no contraction
// (Q8_0FloatTensor.kt:21-28, Q4_KFloatTensor.kt:23-55, Q6_KFloatTensor.kt:26-73,
// BF16FloatTensor.kt:20-24, F32FloatTensor.kt:18-20).  Used by the dequant
// kernel (bit-exact check) and the generic GEMV fallback.
__device__ __forceinline__ float get_elem(int type, const uint8_t* base, long long idx) {
  switch (type) {
    case F32: return __ldg(reinterpret_cast<const float*>(base) + idx);
    case F16: {
      const uint8_t* p = base + idx * 2;
      return f16_bits_to_f32((uint16_t)(p[0] | (p[1] << 8)));
    }
    case BF16: {
      const uint8_t* p = base + idx * 2;
      return __uint_as_float((uint32_t)(p[0] | (p[1] << 8)) << 16);
    }
    case Q8_0: {
      const uint8_t* blk = base + (idx >> 5) * 34;
      float d = f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
      return __fmul_rn((float)(int8_t)blk[2 + (idx & 31)], d);
    }
    case Q4_K: {
      const uint8_t* blk = base + (idx >> 8) * 144;
      int w = (int)(idx & 255);
      float d = f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
      float dmin = f16_bits_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
      const uint8_t* s = blk + 4;
      int group = w >> 6, ig = w & 63;
      int sub = group * 2 + (ig >= 32), nib = ig & 31;
      int sc, m;
      if (sub < 4) {
        sc = s[sub] & 63;
        m = s[sub + 4] & 63;
      } else {
        sc = (s[sub + 4] & 0xF) | (((s[sub - 4] >> 6) & 3) << 4);
        m = (s[sub + 4] >> 4) | (((s[sub] >> 6) & 3) << 4);
      }
      uint8_t b = blk[16 + group * 32 + nib];
      int q = ig >= 32 ? (b >> 4) : (b & 0xF);
      float t = __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
      return __fsub_rn(t, __fmul_rn(dmin, (float)m));
    }
    case Q6_K: {
      const uint8_t* blk = base + (idx >> 8) * 210;
      int w = (int)(idx & 255);
      int half = w >> 7, rem = w & 127, sub32 = rem >> 5, l = rem & 31;
      const uint8_t* ql = blk + half * 64 + (sub32 & 1) * 32;
      int nib = (sub32 >> 1) ? (ql[l] >> 4) : (ql[l] & 0xF);
      int hb = (blk[128 + half * 32 + l] >> (2 * sub32)) & 3;
      int q6 = (nib | (hb << 4)) - 32;
      int sc = (int8_t)blk[192 + half * 8 + sub32 * 2 + l / 16];
      float d = f16_bits_to_f32((uint16_t)(blk[208] | (blk[209] << 8)));
      return __fmul_rn(__fmul_rn(d, (float)sc), (float)q6);
    }
    case Q4_0: {  // Q4_0FloatTensor.kt:20-38: (q - 8) * scale
      const uint8_t* blk = base + (idx >> 5) * 18;
      const int w = (int)(idx & 31);
      const int q = w < 16 ? (blk[2 + w] & 0xF) : (blk[2 + w - 16] >> 4);
      return __fmul_rn((float)(q - 8), f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8))));
    }
    case Q4_1: {  // Q4_1FloatTensor.kt:22-41: delta * quant + min (two roundings)
      const uint8_t* blk = base + (idx >> 5) * 20;
      const int w = (int)(idx & 31);
      const int q = w < 16 ? (blk[4 + w] & 0xF) : (blk[4 + w - 16] >> 4);
      const float d = f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
      const float m = f16_bits_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
      return __fadd_rn(__fmul_rn(d, (float)q), m);
    }
    case Q5_1: {  // Q5_1FloatTensor.kt:20-51: q * d + m, fifth bit from the 32-bit qh
      const uint8_t* blk = base + (idx >> 5) * 24;
      const int w = (int)(idx & 31);
      const uint32_t qh = (uint32_t)blk[4] | ((uint32_t)blk[5] << 8) | ((uint32_t)blk[6] << 16) |
                          ((uint32_t)blk[7] << 24);
      const int nib = w < 16 ? (blk[8 + w] & 0xF) : (blk[8 + w - 16] >> 4);
      const int xh = w < 16 ? (int)((qh >> w) << 4) & 0x10 : (int)(qh >> (w - 16 + 12)) & 0x10;
      const float d = f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
      const float m = f16_bits_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
      return __fadd_rn(__fmul_rn((float)(nib | xh), d), m);
    }
    case Q5_K: {  // Q5_KFloatTensor.kt:23-50: d * sc * quant - dmin * m
      const uint8_t* blk = base + (idx >> 8) * 176;
      const int w = (int)(idx & 255);
      const float d = f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
      const float dmin = f16_bits_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
      const uint8_t* s = blk + 4;
      const int group = w >> 6, ig = w & 63, hi = ig >= 32, l = ig & 31;
      const int sub = group * 2 + hi;
      int sc, m;
      if (sub < 4) {
        sc = s[sub] & 63;
        m = s[sub + 4] & 63;
      } else {
        sc = (s[sub + 4] & 0xF) | (((s[sub - 4] >> 6) & 3) << 4);
        m = (s[sub + 4] >> 4) | (((s[sub] >> 6) & 3) << 4);
      }
      const uint8_t b = blk[48 + group * 32 + l];
      const int nib = hi ? (b >> 4) : (b & 0xF);
      const int hbit = (blk[16 + l] >> (2 * group + hi)) & 1;
      const float t = __fmul_rn(__fmul_rn(d, (float)sc), (float)(nib | (hbit << 4)));
      return __fsub_rn(t, __fmul_rn(dmin, (float)m));
    }
    case MXFP4: {  // MXFP4FloatTensor.kt:22-36,49,209-216: E2M1 value * 2^(e8m0 - 128)
      const uint8_t* blk = base + (idx >> 5) * 17;
      const int w = (int)(idx & 31);
      const int e = blk[0];
      const float dd = __uint_as_float(e < 2 ? (0x00200000u << e) : ((uint32_t)(e - 1) << 23));
      const int packed = blk[1 + (w & 15)];
      const int nib = w < 16 ? (packed & 0xF) : (packed >> 4);
      const int mag = (nib & 7) < 4 ? (nib & 7) : (nib & 7) == 4 ? 4 : (nib & 7) == 5 ? 6 : (nib & 7) == 6 ? 8 : 12;
      return __fmul_rn((float)((nib & 8) ? -mag : mag), dd);
    }
    default: return __int_as_float(0x7fc00000);
  }
}

}  // namespace g4

namespace g4 {

// Dequantize one 16-weight unit into registers (for multi-token products).
// Q4_K uses the vectorDot form w = fma(q, d*sc, -(dmin*m)) (Q4_KFloatTensor.kt:145);
// Q6_K w = q6 * (d*sc) (Q6_KFloatTensor.kt:201); Q8_0 w = q * d.
template <int FMT>
__device__ __forceinline__ void deq16(const uint8_t* vb, int u, float* w) {
  if constexpr (FMT == Q8_0) {
    const uint8_t* blk = vb + (u >> 1) * 34;
    float d = f16_bits_to_f32(lds16(blk));
    uint32_t q[4];
    lds16B_unaligned(blk + 2 + (u & 1) * 16, q);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t wk = q[k] ^ 0x80808080u;
#pragma unroll
      for (int b = 0; b < 4; ++b) w[4 * k + b] = (byte_as_float(wk, b) - 8388736.0f) * d;
    }
  } else if constexpr (FMT == Q4_K) {
    const uint8_t* blk = vb + (u >> 4) * 144;
    int i0 = (u & 15) * 16;
    int g = i0 >> 6, hi = (i0 >> 5) & 1, c = (i0 >> 4) & 1;
    uint4 h = lds128(blk);
    float d = f16_bits_to_f32((uint16_t)(h.x & 0xFFFFu));
    float dmin = f16_bits_to_f32((uint16_t)(h.x >> 16));
    int j = 2 * g + hi;
    uint32_t sc, mn;
    if (j < 4) {
      sc = (h.y >> (8 * j)) & 63u;
      mn = (h.z >> (8 * j)) & 63u;
    } else {
      int jj = j - 4;
      uint32_t lo = (h.w >> (8 * jj)) & 0xFFu;
      sc = (lo & 0xFu) | (((h.y >> (8 * jj + 6)) & 3u) << 4);
      mn = (lo >> 4) | (((h.z >> (8 * jj + 6)) & 3u) << 4);
    }
    float d1 = d * (float)sc, negm = -(dmin * (float)mn);
    uint4 q = lds128(blk + 16 + g * 32 + c * 16);
    uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t nib = (hi ? (qw[k] >> 4) : qw[k]) & 0x0F0F0F0Fu;
#pragma unroll
      for (int b = 0; b < 4; ++b) w[4 * k + b] = fmaf(byte_as_float(nib, b) - 8388608.0f, d1, negm);
    }
  } else if constexpr (FMT == Q6_K) {
    const uint8_t* blk = vb + (u >> 4) * 210;
    int i0 = (u & 15) * 16;
    int half = i0 >> 7, rem = i0 & 127, sub32 = rem >> 5, l0 = rem & 31;
    uint32_t ql[4], qh[4];
    lds16B_unaligned(blk + half * 64 + (sub32 & 1) * 32 + l0, ql);
    lds16B_unaligned(blk + 128 + half * 32 + l0, qh);
    int8_t scv = (int8_t)(lds16(blk + 192 + ((u & 15) & ~1)) >> (8 * (u & 1)));
    float ds = f16_bits_to_f32(lds16(blk + 208)) * (float)scv;
    uint32_t nsh = (sub32 >> 1) * 4u, hsh = 2u * (uint32_t)sub32;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t q6 = ((ql[k] >> nsh) & 0x0F0F0F0Fu) | (((qh[k] >> hsh) & 0x03030303u) << 4);
#pragma unroll
      for (int b = 0; b < 4; ++b) w[4 * k + b] = (byte_as_float(q6, b) - 8388640.0f) * ds;
    }
  } else if constexpr (FMT == BF16) {
    const uint8_t* p = vb + u * 32;
    uint4 a = lds128(p), b = lds128(p + 16);
    uint32_t v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      w[2 * k] = __uint_as_float(v[k] << 16);
      w[2 * k + 1] = __uint_as_float(v[k] & 0xFFFF0000u);
    }
  } else {
    const uint8_t* p = vb + u * 64;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint4 a = lds128(p + 16 * k);
      w[4 * k] = __uint_as_float(a.x);
      w[4 * k + 1] = __uint_as_float(a.y);
      w[4 * k + 2] = __uint_as_float(a.z);
      w[4 * k + 3] = __uint_as_float(a.w);
    }
  }
}

}  // namespace g4
