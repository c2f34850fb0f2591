// g4_gemv_dec.cu -- the decoder's matrix-vector products (Llama.forward's
// projections at batch 1: q|k|v, o, gate/up, down), on sm_100a.
//
// A decode step runs dozens of small GEMVs (2-20 MB each) back to back, so
// what matters is the time to first byte and how many rows progress at once,
// not the streaming rate of a long kernel.  Design:
//  * one CTA of 16 warps per SM; a warp owns a row (or the pair gate_i, up_i)
//    at a time and its 32 lanes decode the row's blocks side by side;
//  * a row (the 16-byte-aligned superset of its bytes) is copied by the
//    warp's lanes with 16-byte cp.async into the warp's slot in shared
//    memory and decoded there by the block decoders of g4_gemv_rows.cuh;
//    the warp's next row streams into a second slot while this one is
//    decoded, and the first row is requested before the kernel waits for
//    its predecessor (programmatic dependent launch: weights never change);
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

// 16-byte global -> shared copy (cp.async, L2 only); completion by commit groups.
__device__ __forceinline__ void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// NSLOT shared-memory slots per warp (2: the next unit streams in while this
// one is decoded; 1 for long rows, which come one per warp).
template <int FMT, int NSLOT, bool PAIR>
__global__ void __launch_bounds__(512, 1) gemv_dec_kernel(const __grid_constant__ DecGemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const DecGemvPlan& p = a.p;
  constexpr int BS = block_size(FMT), TS = type_size(FMT);
  constexpr int RPU = PAIR ? 2 : 1;  // rows per unit
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, W = blockDim.x >> 5;
  const int GW = gridDim.x * W;
  const int nunits = p.rows / RPU, nblk = p.cols / BS;
  const int row_cap = p.nchunk16 * 16;  // bytes of a row slot
  uint8_t* slots = smem + p.stage_off + (size_t)warp * p.stage_bytes;  // NSLOT x RPU rows
  float* xs = reinterpret_cast<float*>(smem + p.xs_off);
  float* xsum16 = reinterpret_cast<float*>(smem + p.xsum_off);
  float* xsum32 = xsum16 + p.cols / 16;
  float* xsc32 = xsum32 + p.cols / 32;
  int16_t* xq = reinterpret_cast<int16_t*>(smem + p.xq_off);
  int16_t* xql = reinterpret_cast<int16_t*>(smem + p.xq2_off);
  float* misc = reinterpret_cast<float*>(smem + p.misc_off);

  // the aligned superset of unit u's rows -> slot `slot` (one commit group)
  auto issue = [&](int u, int slot) {
#pragma unroll
    for (int r = 0; r < RPU; ++r) {
      const long long start = (long long)(u * RPU + r) * p.row_bytes;
      const uint8_t* src = a.w + (start & ~15ll);
      uint8_t* dst = slots + ((size_t)slot * RPU + r) * row_cap;
      for (int c = lane; c < p.nchunk16; c += 32) cp16(dst + (size_t)c * 16, src + (size_t)c * 16);
    }
    cp_commit();
  };
  int u = blockIdx.x * W + warp;
  if (u < nunits) issue(u, 0);  // weights only: before the dependency wait
  grid_dep_wait();
  grid_dep_launch();

  // activation: fused prologue (or x itself), then two-part int16 per 32 columns
  const float* src = a.x;
  if (a.f.in_mode != IN_PLAIN) {
    fused_prologue(a.f, a.x, xs, misc, p.cols, reinterpret_cast<float*>(smem + p.extra_off));
    src = xs;
  }
  {
    const int n4 = p.cols / 4;
    for (int i0 = 0; i0 < n4; i0 += blockDim.x) {
      const int i = i0 + (int)threadIdx.x;
      const bool act = i < n4;
      const float4 v = !act ? make_float4(0.f, 0.f, 0.f, 0.f)
                       : src == a.x ? __ldg(reinterpret_cast<const float4*>(a.x) + i)
                                    : reinterpret_cast<const float4*>(src)[i];
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
        const int i0q = __float2int_rn(f0), i1q = __float2int_rn(f1), i2q = __float2int_rn(f2), i3q = __float2int_rn(f3);
        *reinterpret_cast<uint2*>(xq + xq_at(4 * i)) =
            make_uint2((uint32_t)(uint16_t)i0q | ((uint32_t)(uint16_t)i1q << 16),
                       (uint32_t)(uint16_t)i2q | ((uint32_t)(uint16_t)i3q << 16));
        auto lo16 = [](float sv, int iv) {
          const int r = __float2int_rn((sv - (float)iv) * 65536.0f);
          return (uint32_t)(uint16_t)max(-32767, min(32767, r));
        };
        *reinterpret_cast<uint2*>(xql + xq_at(4 * i)) =
            make_uint2(lo16(f0, i0q) | (lo16(f1, i1q) << 16), lo16(f2, i2q) | (lo16(f3, i3q) << 16));
        if ((i & 3) == 0) xsum16[i >> 2] = s16;
        if ((i & 7) == 0) {
          xsum32[i >> 3] = s32;
          xsc32[i >> 3] = nz ? __uint_as_float(e) : 1.0f;
        }
      }
    }
  }
  __syncthreads();

  const int out_mode = a.f.out_mode;
  unsigned long long best = 0ull;
  for (int it = 0; u < nunits; u += GW, ++it) {
    const int cur = NSLOT == 2 ? (it & 1) : 0;
    if (NSLOT == 2 && u + GW < nunits) {
      issue(u + GW, cur ^ 1);  // the next unit streams in during this decode
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncwarp();
    float s[RPU];
#pragma unroll
    for (int r = 0; r < RPU; ++r) {
      const long long start = (long long)(u * RPU + r) * p.row_bytes;
      const uint8_t* rowp = slots + ((size_t)cur * RPU + r) * row_cap + (start & 15);
      float acc[1] = {0.f};
      for (int b = lane; b < nblk; b += 32) {
        const uint8_t* blk = rowp + (size_t)b * TS;
        if constexpr (FMT == Q4_K) block_q4k_i16<1, true>(blk, b * BS, p.cols, xq, xsc32, xsum32, acc, xql);
        else if constexpr (FMT == Q6_K) block_q6k_i16<1, true>(blk, b * BS, p.cols, xq, xsc32, xsum16, acc, xql);
        else block_q8_0_i16<true>(blk, b * BS, xq, xsc32, acc[0], xql);
      }
      s[r] = warp_sum(acc[0]);
    }
    if (lane == 0) {
      if (out_mode == OUT_GELU_PAIR) {
        a.y[u] = __fmul_rn(gelu_ref(s[0]), s[RPU - 1]);
      } else if (out_mode == OUT_SOFTCAP_ARGMAX) {
        const float c = softcap_ref(s[0], a.f.softcap);
        a.y[u] = c;
        const unsigned long long k = argmax_key(c, u);
        best = k > best ? k : best;
      } else {
        a.y[u] = s[0];
      }
    }
    __syncwarp();  // the slot is rewritten by a later unit
    if (NSLOT == 1 && u + GW < nunits) issue(u + GW, 0);
  }
  if (out_mode == OUT_SOFTCAP_ARGMAX) {
    unsigned long long* kb = reinterpret_cast<unsigned long long*>(misc + 64);
    __syncthreads();
    if (lane == 0) kb[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long b = 0ull;
      for (int w = 0; w < W; ++w) b = kb[w] > b ? kb[w] : b;
      atomicMax(a.f.argmax, b);
    }
  }
}

using DecFnG = void (*)(const DecGemvArgs);

template <int FMT>
static DecFnG dec_fn_slots(int nslot, bool pair) {
  if (pair) return nslot == 2 ? gemv_dec_kernel<FMT, 2, true> : gemv_dec_kernel<FMT, 1, true>;
  return nslot == 2 ? gemv_dec_kernel<FMT, 2, false> : gemv_dec_kernel<FMT, 1, false>;
}

static DecFnG dec_gemv_fn(int type, int nslot, bool pair) {
  switch (type) {
    case Q8_0: return dec_fn_slots<Q8_0>(nslot, pair);
    case Q4_K: return dec_fn_slots<Q4_K>(nslot, pair);
    case Q6_K: return dec_fn_slots<Q6_K>(nslot, pair);
    default: return nullptr;
  }
}

DecGemvPlan plan_gemv_dec(const DeviceInfo& dev, int type, int rows, int cols, bool pair, int fused_extra) {
  DecGemvPlan p{};
  p.type = type;
  p.rows = rows;
  p.cols = cols;
  p.pair = pair ? 1 : 0;
  if (type != Q8_0 && type != Q4_K && type != Q6_K) return p;
  const int BS = block_size(type), TS = type_size(type);
  if (rows <= 0 || cols <= 0 || cols % BS || cols % 32 || (pair && rows % 2)) return p;
  p.row_bytes = cols / BS * TS;
  p.nchunk16 = (p.row_bytes + 15) / 16 + 1;
  p.warps = 16;
  const int unit_bytes = (pair ? 2 : 1) * p.nchunk16 * 16;
  p.nslot = unit_bytes <= 4608 ? 2 : 1;  // double-buffer units of up to 4.5 KB
  p.stage_bytes = p.nslot * unit_bytes;
  auto al = [](size_t v) { return (int)((v + 127) / 128 * 128); };
  p.xs_off = 0;
  p.extra_off = al((size_t)cols * 4);
  p.xsum_off = p.extra_off + al((size_t)std::max(fused_extra, 0));
  p.xq_off = p.xsum_off + al((size_t)(cols / 16 + 2 * (cols / 32)) * 4);
  const int xq1 = al((size_t)(cols + 8 * ((cols + 255) / 256)) * 2);
  p.xq2_off = p.xq_off + xq1;
  p.misc_off = p.xq2_off + xq1;
  p.stage_off = p.misc_off + 512;
  p.smem = (size_t)p.stage_off + (size_t)p.warps * p.stage_bytes;
  if (p.smem > dev.smem_optin) return p;
  DecFnG fn = dec_gemv_fn(type, p.nslot, pair);
  if (!fn || cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dev.smem_optin)) {
    cudaGetLastError();
    return p;
  }
  const int units = rows / (pair ? 2 : 1);
  p.grid = std::min(dev.sms, (units + p.warps - 1) / p.warps);
  p.fast = 1;
  return p;
}

int launch_gemv_dec(const DecGemvPlan& p, const uint8_t* w, const float* x, float* y, const GemvFuse& f,
                    unsigned* status, cudaStream_t st, bool pdl) {
  cudaGetLastError();
  if (!p.fast || (f.out_mode == OUT_GELU_PAIR) != (p.pair != 0)) return (int)cudaErrorInvalidValue;
  DecGemvArgs a{p, w, x, y, status, f};
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
  return (int)cudaLaunchKernelEx(&cfg, dec_gemv_fn(p.type, p.nslot, p.pair != 0), a);
}

}  // namespace g4
