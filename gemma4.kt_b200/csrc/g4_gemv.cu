// g4_gemv.cu -- quantized matrix-vector product y = W[off : off+rows*cols] . x
// for GGUF Q8_0 / Q4_K / Q6_K / BF16 / F32 block streams, on sm_100a.
//
// Replaces FloatTensor.matmul(that, out, dim0, dim1[, thisOffset])
// (FloatTensor.kt:18-29) and the per-type vectorDot it fans out to.
//
// Design (HBM-bound, CUDA cores):
//  * Persistent CTAs, sized so that every SM gets one.  Each warp owns row
//    groups of 32/LPR virtual rows (LPR lanes share a row) and streams their
//    segments through its own ring of shared-memory stages: one cp.async.bulk
//    (into this CTA only) per row segment, one mbarrier per stage.  The weights keep
//    their on-disk layout; unaligned block strides (34 B, 210 B) are handled by
//    copying the 16-byte-aligned superset of each segment and decoding at a
//    byte offset.  Few row groups: one CTA per group, its warps split the row.
//  * Quantized formats: the CTA's prologue turns x, in one pass, into int16 per
//    32-column block (power-of-two scales) plus fp32 column sums, and the block
//    decoders multiply the stored codes as bytes with dp2a (g4_gemv_rows.cuh).
//    BF16 / F32 read fp32 x with packed fma.
//  * Rows whose length is not a multiple of the block size (e.g. 704-wide Q4_K
//    expert down rows) are grouped into virtual rows of `pr` real rows, after
//    which the block pattern repeats; accumulators are kept per real row.
//  * Each warp reduces its rows with shuffles and writes y directly: no atomics,
//    deterministic.
#include "g4_gemv.cuh"
#include "g4_gemv_rows.cuh"
#include "g4_fuse.cuh"
#include "g4_internal.h"

#include <algorithm>
#include <cstdio>
#include <cstdlib>

namespace g4 {

struct GemvArgs {
  GemvPlan p;
  const uint8_t* w;  // tensor base (block stream), 256B aligned, padded by >=256 B
  const float* x;    // cols floats, 16B aligned
  float* y;          // rows floats
  unsigned* status;  // device error word
  GemvFuse f;        // fused prologue / epilogue (IN_PLAIN / OUT_PLAIN: none)
};

// LPR lanes share a row: a warp covers 32/LPR rows; lane l owns row slot
// l % (32/LPR) and, within each chunk, the blocks b with b % LPR == l / (32/LPR).
// FUSED: the decoder's variant with the fused prologue / epilogue and L2
// prefetch compiled in; the plain variant (g4_matmul) keeps them out, so its
// register count (and CTAs per SM) is that of the bare product.
template <int FMT, int PR, int LPR, bool X2, bool FUSED>
__global__ void __launch_bounds__(512) gemv_rows_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const GemvPlan& p = a.p;
  constexpr int BS = block_size(FMT), TS = type_size(FMT);
  constexpr int RPW = 32 / LPR;  // rows per warp
  float* xs = reinterpret_cast<float*>(smem + p.xs_off);
  float* xsum = reinterpret_cast<float*>(smem + p.xsum_off);  // per 16 columns, then per 32 columns
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  uint8_t* ring = smem + p.ring_off;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, W = blockDim.x >> 5;
  const int rs = lane % RPW, sl = lane / RPW;
  const int NS = p.ns;
  const size_t stage_bytes = (size_t)RPW * p.pitch;
  uint64_t* mybars = bars + warp * NS;
  uint8_t* myring = ring + (size_t)warp * NS * stage_bytes;
  const int n16 = p.cols / 16;
  float* xsum16 = xsum;
  float* xsum32 = xsum + n16;

  if (threadIdx.x < W * NS) mbar_init(&bars[threadIdx.x], 1);
  if (threadIdx.x == 0) fence_barrier_init();
  __syncthreads();

  const long long blk0 = p.off / BS;  // first block of the matrix
  const int bpv = p.bpv, cb = p.cb, nchunks = p.nchunks;
  const long long vrow_bytes = (long long)bpv * TS;
  const long long chunk_bytes = (long long)cb * TS;
  // Stage sequence of this warp, advanced incrementally: (group, chunk).
  // split == 1: groups gw, gw + GW, ... each with chunks 0..nchunks-1;
  // split  > 1: the CTA's one group, chunks warp, warp + W, ...
  const int gstep = gridDim.x * W;
  const int g_first = p.split == 1 ? (int)blockIdx.x * W + warp : (int)blockIdx.x;
  const int c_first = p.split == 1 ? 0 : warp;
  const int c_step = p.split == 1 ? 1 : W;
  auto advance = [&](int& g, int& c) {
    c += c_step;
    if (p.split == 1 && c == nchunks) {
      c = 0;
      g += gstep;
    }
  };
  auto valid = [&](int g, int c) { return g < p.ngroups && c < nchunks; };
  // byte offset of this lane's row in group g (only lanes with a row use it)
  auto row_start = [&](int g) { return (blk0 * TS) + ((long long)g * RPW + rs) * vrow_bytes; };
  auto row_ok = [&](int g) { return (long long)g * RPW + rs < p.nvrows; };

  // Lanes of sub-slot 0 copy their rows' segments of stage (g, c) into `slot`.
  auto issue = [&](int g, int c, long long rstart, int slot) {
    uint64_t* bar = &mybars[slot];
    uint32_t mine = 0;
    if (sl == 0 && row_ok(g)) {
      const long long start = rstart + c * chunk_bytes;
      const long long len = min(chunk_bytes, vrow_bytes - c * chunk_bytes);
      const long long a0 = start & ~15ll, a1 = (start + len + 15) & ~15ll;
      bulk_g2s(myring + (size_t)slot * stage_bytes + (size_t)rs * p.pitch, a.w + a0, (uint32_t)(a1 - a0), bar);
      mine = (uint32_t)(a1 - a0);
    }
    const uint32_t total = __reduce_add_sync(0xffffffffu, mine);
    if (lane == 0) mbar_arrive_expect_tx(bar, total);
  };

  bool ok = true;
  int issued = 0, consumed = 0;
  int gi = g_first, ci = c_first;  // issue pointer
  long long rs_i = row_start(gi);
  for (; issued < NS && valid(gi, ci); ++issued) {
    issue(gi, ci, rs_i, issued);
    const int g0 = gi;
    advance(gi, ci);
    if (gi != g0) rs_i = row_start(gi);
  }
  // Weights are never written by preceding kernels: the first stages are in
  // flight before this waits for them (programmatic dependent launch; both
  // are no-ops for a plain launch).  Dependents launch only after the wait,
  // so everything two kernels back has completed when they start.
  if constexpr (FUSED) issue_l2_prefetch(a.f);
  grid_dep_wait();
  grid_dep_launch();
  float* misc = reinterpret_cast<float*>(smem + p.misc_off);
  const float* src = a.x;
  if constexpr (FUSED) {
    if (a.f.in_mode != IN_PLAIN) {
      fused_prologue(a.f, a.x, xs, misc, p.cols);
      src = xs;
    }
  }

  // x -> shared memory while the first weight stages are in flight, in one
  // pass: thread t takes float4 columns t, t + blockDim, ...; for the quantized
  // formats 4 lanes form a 16-column sum, 8 lanes (one 32-column block) the
  // 32-column sum and the block's int16 values (quantize_x16's rule)
  int16_t* xq = reinterpret_cast<int16_t*>(smem + p.xq_off);
  int16_t* xql = X2 ? reinterpret_cast<int16_t*>(smem + p.xq2_off) : nullptr;  // remainders (two-part form)
  float* xsc32 = xsum32 + n16 / 2;
  {
    const int n4 = p.cols / 4;  // a multiple of 8 (cols % 32 == 0)
    for (int i0 = 0; i0 < n4; i0 += blockDim.x) {
      const int i = i0 + (int)threadIdx.x;
      const bool act = i < n4;
      const float4 v = !act ? make_float4(0.f, 0.f, 0.f, 0.f)
                       : src == a.x ? __ldg(reinterpret_cast<const float4*>(a.x) + i)
                                    : reinterpret_cast<const float4*>(src)[i];
      if constexpr (FMT == Q4_K || FMT == Q6_K || FMT == Q8_0) {
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
          const float s0 = v.x * inv, s1 = v.y * inv, s2 = v.z * inv, s3 = v.w * inv;  // exact (power of two)
          const int i0 = __float2int_rn(s0), i1 = __float2int_rn(s1), i2 = __float2int_rn(s2), i3 = __float2int_rn(s3);
          const uint32_t q01 = (uint32_t)(uint16_t)i0 | ((uint32_t)(uint16_t)i1 << 16);
          const uint32_t q23 = (uint32_t)(uint16_t)i2 | ((uint32_t)(uint16_t)i3 << 16);
          *reinterpret_cast<uint2*>(xq + xq_at(4 * i)) = make_uint2(q01, q23);
          if constexpr (X2) {
            // remainder s - rint(s) in [-0.5, 0.5] (exact), in units of 1/65536
            auto lo16 = [](float sv, int iv) {
              const int r = __float2int_rn((sv - (float)iv) * 65536.0f);
              return (uint32_t)(uint16_t)max(-32767, min(32767, r));
            };
            *reinterpret_cast<uint2*>(xql + xq_at(4 * i)) =
                make_uint2(lo16(s0, i0) | (lo16(s1, i1) << 16), lo16(s2, i2) | (lo16(s3, i3) << 16));
          }
          if ((i & 3) == 0) xsum16[i >> 2] = s16;
          if ((i & 7) == 0) {
            xsum32[i >> 3] = s32;
            xsc32[i >> 3] = nz ? __uint_as_float(e) : 1.0f;
          }
        }
      } else {
        if (act && src != xs) *reinterpret_cast<float4*>(xs + 4 * i) = v;
      }
    }
  }
  __syncthreads();

  float acc[PR];
#pragma unroll
  for (int r = 0; r < PR; ++r) acc[r] = 0.f;
  const int out_mode = FUSED ? a.f.out_mode : (int)OUT_PLAIN;
  unsigned long long best = 0ull;  // OUT_SOFTCAP_ARGMAX: this lane's best key

  int g = g_first, c = c_first;  // consume pointer
  long long rs_c = row_start(g);
  bool have_row = row_ok(g);
  int slot = 0;
  uint32_t phase = 0;  // slot = i % NS and phase = (i / NS) & 1, kept incrementally
  for (int i = 0; valid(g, c); ++i) {
    if (i > 0 && ++slot == NS) {
      slot = 0;
      phase ^= 1u;
    }
    if (!mbar_wait_bounded(&mybars[slot], phase)) {
      record_error(a.status, ERR_TIMEOUT_FULL);
      ok = false;
      consumed = i;
      break;
    }
    // ---- compute on this lane's share of its row segment
    if (have_row) {
      const long long start = rs_c + c * chunk_bytes;
      const int nb = min(cb, bpv - c * cb);  // blocks (elements for BF16 / F32) in this chunk
      const uint8_t* base = myring + (size_t)slot * stage_bytes + (size_t)rs * p.pitch + (start & 15);
      const int e0 = c * cb * BS;  // first element of the chunk within the virtual row
      if constexpr (FMT == Q4_K || FMT == Q6_K || FMT == Q8_0) {
        for (int b = sl; b < nb; b += LPR) {
          const uint8_t* blk = base + b * TS;
          if constexpr (FMT == Q4_K) block_q4k_i16<PR, X2>(blk, e0 + b * BS, p.cols, xq, xsc32, xsum32, acc, xql);
          else if constexpr (FMT == Q6_K) block_q6k_i16<PR, X2>(blk, e0 + b * BS, p.cols, xq, xsc32, xsum16, acc, xql);
          else block_q8_0_i16<X2>(blk, e0 + b * BS, xq, xsc32, acc[0], xql);
        }
      } else {
        // BF16 / F32: `blocks` are elements; 16-byte loads of 8 or 4 of them
        constexpr int EPL = 16 / TS;
        float2 s2 = f2(0.f, 0.f);
        for (int e = sl * EPL; e < nb; e += LPR * EPL) {
          if constexpr (FMT == BF16) unit16_bf16(base + e * TS, e0 + e, xs, s2);
          else unit16_f32(base + e * TS, e0 + e, xs, s2);
        }
        acc[0] += s2.x + s2.y;
      }
    }
    // ---- refill this slot with the stage NS ahead (same warp: no other reader)
    __syncwarp();
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (valid(gi, ci)) {
      issue(gi, ci, rs_i, slot);
      ++issued;
      const int g0 = gi;
      advance(gi, ci);
      if (gi != g0) rs_i = row_start(gi);
    }
    // ---- row group finished: combine the lanes of each row and write
    const int gprev = g;
    advance(g, c);
    if (p.split == 1 && g != gprev) {
      const long long v = (long long)gprev * RPW + rs;
#pragma unroll
      for (int r = 0; r < PR; ++r) {
        float t = acc[r];
#pragma unroll
        for (int o = RPW; o < 32; o <<= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (out_mode == OUT_PLAIN) {
          if (sl == 0 && have_row) a.y[v * PR + r] = t;
        } else if (out_mode == OUT_GELU_PAIR) {
          // rows 2i (gate) and 2i + 1 (up) sit in lanes rs, rs ^ 1 (PR == 1)
          const float u = __shfl_xor_sync(0xffffffffu, t, 1);
          if (sl == 0 && have_row && (v & 1) == 0) a.y[v >> 1] = __fmul_rn(gelu_ref(t), u);
        } else {
          const float capped = softcap_ref(t, a.f.softcap);
          if (sl == 0 && have_row) {
            a.y[v] = capped;
            const unsigned long long k = argmax_key(capped, v);
            best = k > best ? k : best;
          }
        }
        acc[r] = 0.f;
      }
      rs_c = row_start(g);
      have_row = row_ok(g);
    }
  }

  if (p.split > 1) {
    // CTA = one row group; warps hold partial sums over disjoint chunks.
    float* red = reinterpret_cast<float*>(smem + p.red_off);
#pragma unroll
    for (int r = 0; r < PR; ++r) {
      float t = acc[r];
#pragma unroll
      for (int o = RPW; o < 32; o <<= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
      if (sl == 0) red[((size_t)warp * RPW + rs) * PR + r] = t;
    }
    __syncthreads();
    if (out_mode == OUT_PLAIN) {
      for (int t = threadIdx.x; t < RPW * PR; t += blockDim.x) {
        const long long v = (long long)blockIdx.x * RPW + t / PR;
        float sum = 0.f;
        for (int w = 0; w < W; ++w) sum += red[(size_t)w * RPW * PR + t];
        if (v < p.nvrows) a.y[v * PR + (t % PR)] = sum;
      }
    } else if (warp == 0) {
      // fused epilogues (PR == 1): row t of the group in lane t
      const int t = lane;
      const long long v = (long long)blockIdx.x * RPW + t;
      float sum = 0.f;
      if (t < RPW)
        for (int w = 0; w < W; ++w) sum += red[(size_t)w * RPW + t];
      if (out_mode == OUT_GELU_PAIR) {
        const float u = __shfl_xor_sync(0xffffffffu, sum, 1);
        if (t < RPW && v < p.nvrows && (v & 1) == 0) a.y[v >> 1] = __fmul_rn(gelu_ref(sum), u);
      } else if (t < RPW && v < p.nvrows) {
        const float capped = softcap_ref(sum, a.f.softcap);
        a.y[v] = capped;
        best = argmax_key(capped, v);
      }
    }
  }
  if (out_mode == OUT_SOFTCAP_ARGMAX) {
    // CTA maximum, one atomic per CTA
    unsigned long long* kb = reinterpret_cast<unsigned long long*>(misc + 64);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
      best = k > best ? k : best;
    }
    __syncthreads();
    if (lane == 0) kb[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long b = 0ull;
      for (int w = 0; w < W; ++w) b = kb[w] > b ? kb[w] : b;
      atomicMax(a.f.argmax, b);
    }
  }
  // Never leave the CTA with bulk copies still landing in its shared memory
  // (only possible after a bounded wait expired).
  if (!ok) {
    for (int q = consumed + 1; q < issued; ++q)
      if (!mbar_wait_bounded(&mybars[q % NS], (q / NS) & 1)) record_error(a.status, ERR_TIMEOUT_DRAIN);
  }
}

// Generic path: any offset / width.  One warp per row, element-wise decode
// straight from global memory (FloatTensor.dot semantics, slow but total).
__global__ void gemv_generic_kernel(int type, const uint8_t* __restrict__ w, long long off, int rows,
                                    int cols, const float* __restrict__ x, float* __restrict__ y) {
  int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (row >= rows) return;
  long long base = off + (long long)row * cols;
  float s = 0.f;
  for (int c = lane; c < cols; c += 32) s = fmaf(get_elem(type, w, base + c), x[c], s);
  s = warp_sum(s);
  if (lane == 0) y[row] = s;
}

__global__ void dequant_kernel(int type, const uint8_t* __restrict__ w, long long off, long long n,
                               float* __restrict__ out) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long stride = (long long)gridDim.x * blockDim.x;
  for (; i < n; i += stride) out[i] = get_elem(type, w, off + i);
}

// ---------------------------------------------------------------- host side

static int gcd_i(int a, int b) {
  while (b) {
    int t = a % b;
    a = b;
    b = t;
  }
  return a;
}

using KernelFn = void (*)(const GemvArgs);

template <int FMT, bool X2, bool F>
static KernelFn pick_pr1(int lpr) {
  return lpr == 32 ? gemv_rows_kernel<FMT, 1, 32, X2, F> : lpr == 16 ? gemv_rows_kernel<FMT, 1, 16, X2, F>
       : lpr == 4  ? gemv_rows_kernel<FMT, 1, 4, X2, F>  : lpr == 2  ? gemv_rows_kernel<FMT, 1, 2, X2, F>
                                                                     : gemv_rows_kernel<FMT, 1, 1, X2, F>;
}

template <int FMT>
static KernelFn pick_kernel(int pr, int lpr, bool x2, bool fused) {
  if (x2) {
    // two-part activations: the decoder's row-aligned projections only
    if constexpr (FMT == Q8_0 || FMT == Q4_K || FMT == Q6_K)
      if (pr == 1) return fused ? pick_pr1<FMT, true, true>(lpr) : pick_pr1<FMT, true, false>(lpr);
    return nullptr;
  }
  if (pr == 1) return fused ? pick_pr1<FMT, false, true>(lpr) : pick_pr1<FMT, false, false>(lpr);
  if constexpr (FMT == Q4_K || FMT == Q6_K) {
    if (fused) return nullptr;  // fused prologues / epilogues take one row per lane group
    if (pr == 2) return lpr == 2 ? gemv_rows_kernel<FMT, 2, 2, false, false> : gemv_rows_kernel<FMT, 2, 1, false, false>;
    if (pr == 4) return lpr == 2 ? gemv_rows_kernel<FMT, 4, 2, false, false> : gemv_rows_kernel<FMT, 4, 1, false, false>;
  }
  return nullptr;
}

static KernelFn kernel_for(int type, int pr, int lpr, bool x2, bool fused) {
  switch (type) {
    case Q8_0: return pick_kernel<Q8_0>(pr, lpr, x2, fused);
    case Q4_K: return pick_kernel<Q4_K>(pr, lpr, x2, fused);
    case Q6_K: return pick_kernel<Q6_K>(pr, lpr, x2, fused);
    case BF16: return pick_kernel<BF16>(pr, lpr, false, fused);
    case F32: return pick_kernel<F32>(pr, lpr, false, fused);
    default: return nullptr;
  }
}

// Overridable for tuning sweeps: G4_GEMV_CHUNK_BYTES, G4_GEMV_WARPS, G4_GEMV_STAGES, G4_GEMV_LPR.
static int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return v && *v ? atoi(v) : dflt;
}

static int pitch_for(int bytes) {
  int p = (bytes + 15) / 16;
  if ((p & 1) == 0) ++p;  // 16 * odd: 8 lanes' 16-byte loads hit distinct bank groups
  return 16 * p;
}

GemvPlan plan_gemv(const DeviceInfo& dev, int type, long long off, int rows, int cols) {
  return plan_gemv(dev, type, off, rows, cols, GemvOpts{});
}

GemvPlan plan_gemv(const DeviceInfo& dev, int type, long long off, int rows, int cols, const GemvOpts& o) {
  const bool fused = o.fused, exact_x = o.exact_x, latency = o.latency;
  const size_t max_smem = o.max_smem;
  GemvPlan p{};
  p.type = type;
  p.rows = rows;
  p.cols = cols;
  p.off = off;
  p.fast = 0;
  p.fused = fused ? 1 : 0;
  p.x2 = exact_x && (type == Q8_0 || type == Q4_K || type == Q6_K) ? 1 : 0;
  const int BS = block_size(type), TS = type_size(type);
  // the lane-per-row kernel decodes F32, BF16, Q8_0, Q4_K and Q6_K; the other formats take the
  // generic kernel (one warp per row, element decoder)
  const bool fast_type = type == F32 || type == BF16 || type == Q8_0 || type == Q4_K || type == Q6_K;
  if (TS == 0 || !fast_type || rows <= 0 || cols <= 0) return p;
  if (cols % 32 != 0 || off % BS != 0) return p;
  if ((type == BF16 || type == F32) && ((off * TS) % 16) != 0) return p;
  int pr = 1;
  if (cols % BS != 0) {
    if (type == Q8_0 || cols % 64 != 0) return p;  // K-quant groups must not straddle rows
    pr = BS / gcd_i(cols % BS, BS);
    if (pr != 2 && pr != 4) return p;
  }
  if (rows % pr != 0) return p;
  // fp32 x in shared memory only for BF16 / F32; the quantized formats read the int16 form
  const bool quantized = type == Q8_0 || type == Q4_K || type == Q6_K;
  // a fused prologue stages the fp32 activation in shared memory for every format
  const int xbytes = quantized && !fused ? 0 : ((cols * 4 + 127) / 128) * 128;
  constexpr int kMiscBytes = 512;  // block reductions and the argmax epilogue
  // per-16 and per-32 column sums, per-32 int16 scales; int16 activations
  const int xsbytes = (((cols / 16 + 2 * (cols / 32)) * 4 + 127) / 128) * 128;
  const int xq1 = (((cols + 8 * ((cols + 255) / 256)) * 2 + 127) / 128) * 128;
  const int xqbytes = xq1 * (p.x2 ? 2 : 1);  // two-part form: the remainders follow the first part
  if (xbytes > 96 * 1024) return p;
  p.pr = pr;
  p.nvrows = rows / pr;
  p.bpv = (int)((long long)pr * cols / BS);
  // defaults from a sweep of 262144 x 1536 on B200 (lanes per row, bytes per copy)
  const int lpr_default = (type == Q4_K || type == Q6_K) ? 2 : 4;
  p.lpr = env_int("G4_GEMV_LPR", lpr_default);
  if (p.lpr != 1 && p.lpr != 2 && p.lpr != 4) p.lpr = 1;
  if (pr > 1 && p.lpr > 2) p.lpr = 2;
  // decode-size matrices: a warp per row (half a warp when rows are paired),
  // so that a row's blocks are decoded side by side, not one after another
  if (latency && pr == 1) p.lpr = o.pair_rows ? 16 : 32;
  int rows_per_group = 32 / p.lpr;
  p.ngroups = (p.nvrows + rows_per_group - 1) / rows_per_group;

  // chunk: about `target` bytes of one row per bulk copy (copies below ~256 B
  // cap the copy engine well under HBM speed), at least one block per lane
  const int target = env_int("G4_GEMV_CHUNK_BYTES", type == Q4_K ? 288 : type == Q6_K ? 420 : 576);
  const int unit = (type == BF16 ? 8 : type == F32 ? 4 : 1) * p.lpr;  // elements (blocks) per lane step
  int cb = std::max(unit, std::min(p.bpv, target / TS) / unit * unit);
  const bool small = latency ? p.ngroups < dev.sms : p.ngroups < 2 * dev.sms;
  if (small) {
    // few row groups: split each row over up to 8 warps of one CTA
    int want = std::max(unit, (p.bpv + 7) / 8);
    want = (want + unit - 1) / unit * unit;
    cb = std::min(cb, want);
  }
  p.cb = cb;
  p.nchunks = (p.bpv + cb - 1) / cb;
  p.pitch = pitch_for(cb * TS + 32);
  size_t stage = (size_t)rows_per_group * p.pitch;
  const size_t optin = dev.smem_optin > 0 ? dev.smem_optin : 227 * 1024;
  const size_t budget = max_smem > 0 ? std::min(max_smem, optin) : optin;
  const size_t fixed = (size_t)xbytes + xsbytes + xqbytes + kMiscBytes + 256;
  if (small) {
    p.split = std::min(p.nchunks, 8);
    p.warps = p.split;
    p.ns = 2;
  } else {
    p.split = 1;
    // enough CTAs to cover every SM: a warp streams one row group at a time, so
    // fewer than 16 groups per SM means fewer warps per CTA, not fewer CTAs
    p.warps = env_int("G4_GEMV_WARPS", std::max(1, std::min(16, latency ? (p.ngroups + dev.sms - 1) / dev.sms
                                                                           : p.ngroups / dev.sms)));
    p.ns = env_int("G4_GEMV_STAGES", p.warps >= 16 ? 2 : 4);  // deeper rings when few warps share the SM
  }
  for (;;) {
    size_t red = p.split > 1 ? (size_t)p.warps * rows_per_group * pr * 4 : 0;
    size_t need = fixed + red + (size_t)p.warps * p.ns * stage;
    if (need <= budget) break;
    if (p.ns > 2) --p.ns;
    else if (p.split == 1 && p.warps > 2) --p.warps;
    else if (p.split > 1 && p.cb > unit && type != BF16 && type != F32) {
      // narrower chunks, more of them: keeps the CTA's rings within shared memory
      p.cb = std::max(unit, p.cb / 2 / unit * unit);
      p.nchunks = (p.bpv + p.cb - 1) / p.cb;
      p.pitch = pitch_for(p.cb * TS + 32);
      stage = (size_t)rows_per_group * p.pitch;
    } else if (p.split > 1 && p.warps > 1) {
      p.warps /= 2;
      p.split = p.warps;
    } else {
      return p;  // rows too wide for the fast path
    }
  }
  p.xs_off = 0;
  p.xsum_off = xbytes;
  p.xq_off = xbytes + xsbytes;
  p.xq2_off = p.xq_off + xq1;
  p.misc_off = p.xq_off + xqbytes;
  p.bar_off = p.misc_off + kMiscBytes;
  p.ring_off = p.bar_off + 128 * ((p.warps * p.ns * 8 + 127) / 128);
  p.red_off = (int)(p.ring_off + (size_t)p.warps * p.ns * stage);
  p.smem = (size_t)p.red_off + (p.split > 1 ? (size_t)p.warps * rows_per_group * pr * 4 : 0);
  KernelFn k = kernel_for(type, pr, p.lpr, p.x2 != 0, p.fused != 0);
  if (!k) return p;
  int occ = 0;
  // The attribute belongs to the kernel, not to this plan: always allow the
  // device maximum so plans of other shapes stay launchable.
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)optin) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, 32 * p.warps, p.smem) != cudaSuccess || occ < 1) {
    cudaGetLastError();
    return p;
  }
  if (p.split > 1) p.grid = p.ngroups;
  else p.grid = (int)std::min<long long>((p.ngroups + p.warps - 1) / p.warps, (long long)dev.sms * occ);
  p.fast = 1;
  if (env_int("G4_DEBUG_PLAN", 0))
    fprintf(stderr, "g4 gemv plan: type %d %dx%d pr %d lpr %d cb %d pitch %d warps %d ns %d split %d grid %d smem %zu occ %d\n",
            type, rows, cols, pr, p.lpr, p.cb, p.pitch, p.warps, p.ns, p.split, p.grid, p.smem, occ);
  return p;
}

int launch_gemv_fused(const GemvPlan& p, const uint8_t* w, const float* x, float* y, const GemvFuse& f,
                      unsigned* status, cudaStream_t st, bool pdl) {
  cudaGetLastError();
  if (!p.fast || ((f.in_mode != IN_PLAIN || f.out_mode != OUT_PLAIN || f.pf[0]) && !p.fused) ||
      (f.out_mode != OUT_PLAIN && p.pr != 1))
    return (int)cudaErrorInvalidValue;
  GemvArgs a{p, w, x, y, status, f};
  KernelFn k = kernel_for(p.type, p.pr, p.lpr, p.x2 != 0, p.fused != 0);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(32 * p.warps);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return (int)cudaLaunchKernelEx(&cfg, k, a);
}

int launch_gemv(const GemvPlan& p, const uint8_t* w, const float* x, float* y, unsigned* status,
                cudaStream_t st) {
  cudaGetLastError();  // launch errors below must not be confused with stale ones
  if (p.fast) {
    GemvArgs a{p, w, x, y, status, GemvFuse{}};
    KernelFn k = kernel_for(p.type, p.pr, p.lpr, p.x2 != 0, p.fused != 0);
    k<<<p.grid, 32 * p.warps, p.smem, st>>>(a);
  } else {
    int wpb = 8;
    gemv_generic_kernel<<<(p.rows + wpb - 1) / wpb, 32 * wpb, 0, st>>>(p.type, w, p.off, p.rows, p.cols, x, y);
  }
  return (int)cudaGetLastError();
}

int launch_dequant(int type, const uint8_t* w, long long off, long long n, float* out, cudaStream_t st) {
  if (n <= 0) return 0;
  long long blocks = std::min<long long>((n + 255) / 256, 148 * 32);
  dequant_kernel<<<(int)blocks, 256, 0, st>>>(type, w, off, n, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace g4
