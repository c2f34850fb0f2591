// g4_moe_tc.cu -- the grouped expert products of the MoE block on the
// 5th-generation tensor cores (tcgen05), for token batches wide enough that
// the experts' weight tiles are reused across many tokens.
//
// The arithmetic is the expert block of Llama.forward (Llama.kt:297-337):
//   gate_up = W_gu[e] · moeInput   (rows 0..ff-1 gate, ff..2ff-1 up; Llama.kt:305-313)
//   g       = gelu(gate) * up      (Llama.kt:316-322)
//   down    = W_d[e] · g           (Llama.kt:325-332)
// for every routed slot, grouped by expert.  The weights stay in their GGUF
// Q4_K blocks in HBM and are dequantized inside the kernel to fp16
// (w = q*d*sc - dmin*m, Q4_KFloatTensor.kt:23-55, in packed fp16 arithmetic
// with the scale and min split into fp16 high and low parts, so the result is
// within about one fp16 rounding of the exact weight).  Activations enter the
// tensor cores as two fp16 parts, x = hi + lo (lo = fp16(x - hi), about 22
// bits between them): every K step issues one MMA on the high parts and one
// on the low parts into the same fp32 accumulator in tensor memory, so the
// result differs from the fp32 reference by the weights' fp16 rounding only.
//
// K order inside every aligned group of four columns is (0, 2, 1, 3) in the
// fp16 operands on both sides (weights as dequantized, activations as the
// gather and gate_up epilogue write them): the products are unchanged and
// the dequantizer needs no re-packing.
//
// One persistent CTA per SM, warp-specialised:
//   warp 0        allocates tensor memory; lane 0 issues tcgen05.mma
//                 (M = 128 weight rows, N = tokens, K = 16) into one of two
//                 accumulators, so the epilogue of one tile overlaps the
//                 main loop of the next;
//   warp 1        lane 0 loads token tiles [N x 64] fp16 with TMA (128-byte
//                 swizzle) from the expert-sorted activation matrix;
//   warps 2..9    dequantize the 128 x 64 weight tile of each stage into
//                 shared memory in the same swizzled K-major layout;
//   warps 10..13  read the accumulator (tcgen05.ld) and write the outputs:
//                 gelu(gate)*up as fp16 rows of G (gate_up), or fp32 rows of
//                 D by slot (down).
// Every wait is bounded (kWaitLimitNs) and reports through the status word.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "g4_common.cuh"
#include "g4_moe_tc.h"

namespace g4 {
namespace {

constexpr int kTileM = 128;                                 // weight rows per tile (MMA M)
constexpr int kKB = 64;                                     // K per pipeline stage: one 128-byte fp16 row
constexpr int kMmaK = 16;                                   // K of one kind::f16 MMA
constexpr int kEpiWarps = 4;                                // epilogue warps (one per TMEM lane quarter)
// NG producer groups of four dequantizing warps each
__host__ __device__ constexpr int tc_threads(int ng) { return 32 * (2 + 4 * ng + kEpiWarps); }
constexpr int kMaxStages = 8;
constexpr int kNumBoxes = 5;                                // token-tile heights 16, 32, 64, 128, 256
constexpr int kATile = kTileM * kKB * 2;                    // 16 KB of fp16
constexpr int kBarBytes = 512;
constexpr int kRawDepth = 4;                                // 64-column blocks of raw weights in flight per group
constexpr int kRawRow = 48;                                 // header 16 + codes 32 per row and 64 columns
__host__ __device__ constexpr int tc_raw_bytes(int ng) { return ng * kRawDepth * kTileM * kRawRow; }  // 24 KB a group
constexpr int kMaxExpertsTc = 256;

struct TcArgs {
  const uint8_t* w;        // expert weights, Q4_K block stream
  long long expert_elems;  // elements of one expert's matrix
  int cols;                // K of the product
  int ff;                  // gate_up: rows of each half
  int out_ld;              // row length of the output (ff for G, dim for D)
  int n_row_tiles;         // tiles of 128 rows per expert (pairs of 64 gate/up rows for gate_up)
  int nkb;                 // cols / 64
  int stages;
  int b_stage_bytes;       // token-tile cap * 128
  int acc_cols;            // tensor-memory columns per accumulator (= token-tile cap)
  uint32_t tmem_cols;      // allocated columns
  uint32_t tmem_a_col;     // first column of the weight stages when A lives in tensor memory
  int pipe_bytes;          // shared memory of one pipeline (1024-byte multiple)
  const int4* tiles;       // {expert, first sorted position, tokens, box index}
  const int32_t* n_tiles;
  const int32_t* perm;     // sorted position -> slot
  __half* g16;             // gate_up output [2][sorted position][ff]: high parts, then low parts
  float* D;                // down output [slot][dim]
  int lo_row;              // row of a position's low part in the token matrices (= positions)
  unsigned* status;
};

// ---------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Arrive on bar once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Same with the A operand (128 rows x 16 K, two fp16 per 32-bit column, row m
// in lane m) read from tensor memory.
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 32 consecutive tensor-memory columns of this warp's 32 lanes (one row per lane).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (start >> 4 | LBO 16 B | SBO 1024 B | version 1 | SWIZZLE_128B).
__device__ __forceinline__ uint64_t sw128_desc(const void* p) {
  const uint64_t a = (smem_u32(p) >> 4) & 0x3FFFu;
  return a | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor of kind::f16: fp32 accumulate, fp16 A and B, both K-major, M = 128.
__device__ __forceinline__ uint32_t idesc_f16(uint32_t n) {
  return (1u << 4) | ((n >> 3) << 17) | ((uint32_t)(kTileM >> 4) << 24);
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// 16-byte global -> shared copy through L2 only (cp.async, completion per thread by commit groups).
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// 32 consecutive accumulator columns of this warp's 32 lanes (one row per
// lane), waited for inside the same statement.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// try_wait that lets the hardware suspend the thread until the phase
// completes (or at most kSuspendNs), instead of spinning.
constexpr uint32_t kSuspendNs = 100000;
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return ok != 0;
}

// Bounded wait that also gives up as soon as another role of the CTA has
// given up (abort flag in shared memory).  On its own timeout it raises the
// flag and records `bit` in the status word.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, unsigned* status,
                                        unsigned bit) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait_suspend(bar, parity)) return true;
    if ((it & 7u) == 7u) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        *abort_flag = 1;
        record_error(status, bit);
        return false;
      }
    }
  }
}
// Short bounded wait used only while draining after an abort.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - t0 > 50000000ull) break;
}

__device__ __forceinline__ float gelu_f(float x) {
  // Llama.kt:23-25: 0.5x(1 + tanh(u)), u = sqrt(2/pi)(x + 0.044715x^3), written
  // as x * sigmoid(2u) = x / (1 + e^(-2u)); evaluated in float with the fast
  // exponential and division (relative error ~1e-6): the result is rounded to fp16 next.
  const float u = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
  return __fdividef(x, 1.f + __expf(-2.f * u));
}

// Byte k (0..11) of the 12 scale bytes held in three words.
__device__ __forceinline__ uint32_t scale_byte(uint32_t s0, uint32_t s1, uint32_t s2, int k) {
  const uint32_t w = k < 4 ? s0 : k < 8 ? s1 : s2;
  return (w >> (8 * (k & 3))) & 0xFFu;
}

// Position of logical K column k in the fp16 operands (bits 0 and 1 swapped).
__device__ __forceinline__ int kperm(int k) { return (k & ~3) | ((k & 1) << 1) | ((k >> 1) & 1); }

// Constants of one 32-weight sub-block for the fp16 dequantizer.  A code c
// arrives as v = 1024 + c*step (an fp16 bit pattern: step 1 for low nibbles,
// 16 for high ones) and w = c*s - m (s already divided by step) becomes
//   t = v*s_hi - c_hi,  u = v*s_lo - c_lo,  w = t + u
// with s_hi = fp16(s), s_lo = fp16(s - s_hi), c_hi = fp16(1024*s_hi + m) and
// c_lo = fp16(1024*s_lo + r), r the rounding residual of c_hi: t and u carry
// the whole of q*s - m between them, and each fp16 operation rounds once.
struct SubConst {
  __half2 s_hi, c_hi, s_lo, c_lo;  // c_* negated
};
__device__ __forceinline__ SubConst sub_const(float s, float m) {
  const __half shi = __float2half_rn(s);
  const float fshi = __half2float(shi);
  const __half slo = __float2half_rn(s - fshi);
  const float big = fmaf(1024.f, fshi, m);
  const __half chi = __float2half_rn(big);
  const float r = big - __half2float(chi);
  const __half clo = __float2half_rn(fmaf(1024.f, __half2float(slo), r));
  SubConst k;
  k.s_hi = __halves2half2(shi, shi);
  k.s_lo = __halves2half2(slo, slo);
  k.c_hi = __halves2half2(__hneg(chi), __hneg(chi));
  k.c_lo = __halves2half2(__hneg(clo), __hneg(clo));
  return k;
}
__device__ __forceinline__ uint32_t deq2(uint32_t v, const SubConst& k) {
  const __half2 hv = *reinterpret_cast<const __half2*>(&v);
  const __half2 t = __hfma2(hv, k.s_hi, k.c_hi);
  const __half2 u = __hfma2(hv, k.s_lo, k.c_lo);
  const __half2 w = __hadd2(t, u);
  return *reinterpret_cast<const uint32_t*>(&w);
}
// Four fp16 weights from one word of Q4_K codes (bytes b0..b3 = K 0..3 of a
// group of four): the low (mask 0x000F000F) or high (mask 0x00F000F0)
// nibbles as 1024 + code*step, in stored K order (0, 2, 1, 3).
__device__ __forceinline__ uint2 q4_word_to_f16(uint32_t x, uint32_t mask, const SubConst& k) {
  const uint32_t a02 = (x & mask) | 0x64006400u;         // bytes 0 and 2
  const uint32_t a13 = ((x >> 8) & mask) | 0x64006400u;  // bytes 1 and 3
  return make_uint2(deq2(a02, k), deq2(a13, k));
}

// ---------------------------------------------------------------- kernels
// Token tiles per expert: at most `cap` tokens each, balanced, heights rounded
// up to 16 (the MMA's N granule).  One CTA of 256 threads (E <= 256).
__global__ void __launch_bounds__(256) moe_tc_tiles_kernel(const int32_t* __restrict__ offsets, int E, int cap,
                                                           int4* __restrict__ tiles, int32_t* __restrict__ n_tiles) {
  __shared__ int cnt[kMaxExpertsTc];
  const int e = threadIdx.x;
  int ne = 0, nt = 0, tn = 0;
  if (e < E) {
    ne = offsets[e + 1] - offsets[e];
    if (ne > 0) {
      const int nt0 = (ne + cap - 1) / cap;
      tn = (((ne + nt0 - 1) / nt0) + 15) & ~15;
      nt = (ne + tn - 1) / tn;
    }
  }
  cnt[e] = nt;
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int i = 0; i < (int)blockDim.x; ++i) {
      const int v = cnt[i];
      cnt[i] = acc;
      acc += v;
    }
    *n_tiles = acc;
  }
  __syncthreads();
  const int base = cnt[e];
  for (int i = 0; i < nt; ++i) {
    const int start = i * tn, n = min(tn, ne - start), N = (n + 15) & ~15;
    const int box = N <= 16 ? 0 : N <= 32 ? 1 : N <= 64 ? 2 : N <= 128 ? 3 : 4;
    tiles[base + i] = make_int4(e, offsets[e] + start, n, box);
  }
}

// x16[p][:] = fp16(moe_in[token of slot perm[p]][:]) in stored K order and
// x16[n_pos + p][:] the remainders fp16(x - hi), one warp per sorted position.
__global__ void __launch_bounds__(256) moe_tc_gather_kernel(const float* __restrict__ moe_in,
                                                            const int32_t* __restrict__ perm,
                                                            __half* __restrict__ x16, int n_pos, int dim, int K) {
  const int p = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (p >= n_pos) return;
  const int tok = perm[p] / K;
  const float4* src = reinterpret_cast<const float4*>(moe_in + (size_t)tok * dim);
  uint2* dst = reinterpret_cast<uint2*>(x16 + (size_t)p * dim);
  for (int i = lane; i < dim / 4; i += 32) {
    const float4 v = __ldg(src + i);  // K 4i..4i+3 stored in the order (0, 2, 1, 3)
    const __half2 a = __floats2half2_rn(v.x, v.z), b = __floats2half2_rn(v.y, v.w);
    dst[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
    const float2 fa = __half22float2(a), fb = __half22float2(b);
    const __half2 al = __floats2half2_rn(v.x - fa.x, v.z - fa.y), bl = __floats2half2_rn(v.y - fb.x, v.w - fb.y);
    dst[(size_t)n_pos * dim / 4 + i] =
        make_uint2(*reinterpret_cast<const uint32_t*>(&al), *reinterpret_cast<const uint32_t*>(&bl));
  }
}

// One pipeline stage covers KSUB sub-tiles of 64 K columns (the last stage of
// an item may hold fewer): per sub-tile a 128-row x 64 weight tile and a
// token tile of up to cap rows x 64, each in the 128-byte-swizzled K-major
// layout.  Larger stages mean fewer barrier handshakes per K, which paces
// the pipeline when token tiles are narrow.
// TMEM_A: the dequantized weight tile of each stage goes to tensor memory
// (tcgen05.st, 32 columns per 64-column sub-tile) and the MMA reads it from
// there; shared memory then carries only the token tiles.  Chosen for token
// tiles of at most 128 rows, where fetching A from shared memory (4 KB per
// MMA) would cost more than the MMA itself.
// P independent pipelines share the CTA (each with its own issuing thread,
// token-tile loader, producers, epilogue warps, stage ring, barriers and
// 512/P tensor-memory columns) and split its items: a single thread issues
// one tcgen05.mma per ~120 cycles whatever the tile width, so narrow token
// tiles need several issuers to keep the tensor core fed.
template <bool GATEUP, int KSUB, bool TMEM_A, int NG, int P>
__global__ void __launch_bounds__(P * tc_threads(NG), 1)
    moe_tc_kernel(const __grid_constant__ TcArgs a, const __grid_constant__ CUtensorMap m0,
                  const __grid_constant__ CUtensorMap m1, const __grid_constant__ CUtensorMap m2,
                  const __grid_constant__ CUtensorMap m3, const __grid_constant__ CUtensorMap m4) {
  constexpr int kDepth = kRawDepth / KSUB;           // raw stages in flight per producer group
  constexpr int kRowRaw = KSUB * kRawRow;            // raw bytes per row and stage
  constexpr int kSlot = kTileM * kRowRaw;            // one raw stage of one group
  constexpr int kWpp = 2 + 4 * NG + kEpiWarps;       // warps per pipeline
  extern __shared__ uint8_t smem_raw[];
  const int gwarp = threadIdx.x >> 5;                // CTA warp (its % 4 is its tensor-memory lane quarter)
  const int pp = gwarp / kWpp;                       // this thread's pipeline
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023)) +
                (size_t)pp * a.pipe_bytes;
  const int S = a.stages, bsub = a.b_stage_bytes;
  uint8_t* a_st = sm;                                   // [S][KSUB] x [128 rows x 128 B] (unless TMEM_A)
  uint8_t* b_st = sm + (TMEM_A ? 0 : (size_t)S * KSUB * kATile);  // [S][KSUB][hi, lo] x [cap rows x 128 B]
  uint8_t* raw = b_st + (size_t)S * KSUB * 2 * bsub;    // [NG groups][kDepth] x [128 rows x kRowRaw]
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw + tc_raw_bytes(NG));
  uint64_t* full = bars;                                // producers (4 warps) + TMA bytes -> MMA
  uint64_t* empty = bars + kMaxStages;                  // MMA -> producers and TMA (tcgen05.commit)
  uint64_t* tfull = bars + 2 * kMaxStages;              // MMA -> epilogue   [2]
  uint64_t* tempty = tfull + 2;                         // epilogue -> MMA   [2] (count 4)
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = gwarp - pp * kWpp, lane = threadIdx.x & 31;  // warp within the pipeline
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 4 + 1);  // the four warps of the group that fills it + the TMA thread
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  // pipeline 0's first warp allocates all 512 columns; pipeline p uses columns [p*512/P, (p+1)*512/P)
  uint32_t* tmem_slot0 = reinterpret_cast<uint32_t*>(
      reinterpret_cast<uint8_t*>(tmem_slot) - (size_t)pp * a.pipe_bytes);
  if (gwarp == 0) {
    __syncwarp();
    tmem_alloc(tmem_slot0, a.tmem_cols);
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot0 + (uint32_t)pp * (512u / P);
  const int R = a.n_row_tiles, nkb = a.nkb;          // nkb: 64-column blocks per item
  const int nst = (nkb + KSUB - 1) / KSUB;           // stages per item
  const int n_items = *a.n_tiles * R;
  auto nsub_of = [&](int st) { return min(KSUB, nkb - st * KSUB); };

  if (warp == 0) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0, acc = 0, aph = 0;
      bool issued = false, ok = true;
      for (int item = blockIdx.x + pp * gridDim.x; ok && item < n_items; item += P * gridDim.x) {
        const int4 tl = a.tiles[item / R];
        const uint32_t idesc = idesc_f16((uint32_t)((tl.z + 15) & ~15));
        if (!tc_wait(&tempty[acc], aph ^ 1u, abort_flag, a.status, ERR_TIMEOUT_EMPTY)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * (uint32_t)a.acc_cols;
        for (int st = 0; st < nst; ++st) {
          if (!tc_wait(&full[s], ph, abort_flag, a.status, ERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int nsub = nsub_of(st);
#pragma unroll
          for (int sub = 0; sub < KSUB; ++sub) {
            if (sub < nsub) {
              // token tile: high parts, then low parts (bsub bytes each)
              const uint64_t bd = sw128_desc(b_st + (size_t)(s * KSUB + sub) * 2 * bsub);
              const uint64_t bl = sw128_desc(b_st + ((size_t)(s * KSUB + sub) * 2 + 1) * bsub);
              if (TMEM_A) {
                const uint32_t at = tmem_base + a.tmem_a_col + (uint32_t)(s * KSUB + sub) * 32u;
#pragma unroll
                for (int kk = 0; kk < kKB / kMmaK; ++kk) {  // 16 K = 8 columns of A, 32 bytes of B
                  tc_mma_f16_ts(d_tmem, at + 8u * kk, bd + 2 * kk, idesc, (st | sub | kk) != 0);
                  tc_mma_f16_ts(d_tmem, at + 8u * kk, bl + 2 * kk, idesc, 1u);
                }
              } else {
                const uint64_t ad = sw128_desc(a_st + (size_t)(s * KSUB + sub) * kATile);
#pragma unroll
                for (int kk = 0; kk < kKB / kMmaK; ++kk) {  // +32 bytes of K per step, inside the swizzle row
                  tc_mma_f16(d_tmem, ad + 2 * kk, bd + 2 * kk, idesc, (st | sub | kk) != 0);
                  tc_mma_f16(d_tmem, ad + 2 * kk, bl + 2 * kk, idesc, 1u);
                }
              }
            }
          }
          issued = true;
          tc_commit(&empty[s]);
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&tfull[acc]);
        acc ^= 1u;
        if (acc == 0) aph ^= 1u;
      }
      if (!ok && issued) {  // let every issued MMA finish before tensor memory is released
        tc_commit(drain);
        drain_wait(drain, 0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ TMA producer (token tiles)
    if (lane == 0) {
      int s = 0, n_issued = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int item = blockIdx.x + pp * gridDim.x; ok && item < n_items; item += P * gridDim.x) {
        const int4 tl = a.tiles[item / R];
        const CUtensorMap* map = tl.w == 0 ? &m0 : tl.w == 1 ? &m1 : tl.w == 2 ? &m2 : tl.w == 3 ? &m3 : &m4;
        const uint32_t box_bytes = (16u << tl.w) * 128u;
        for (int st = 0; st < nst; ++st) {
          if (!tc_wait(&empty[s], ph ^ 1u, abort_flag, a.status, ERR_TIMEOUT_EMPTY)) {
            ok = false;
            break;
          }
          const int nsub = nsub_of(st);
          mbar_arrive_expect_tx(&full[s], (uint32_t)nsub * 2u * box_bytes);
          for (int sub = 0; sub < nsub; ++sub) {
            uint8_t* dst = b_st + (size_t)(s * KSUB + sub) * 2 * bsub;
            tma_load_2d(dst, map, (st * KSUB + sub) * kKB, tl.y, &full[s]);
            tma_load_2d(dst + bsub, map, (st * KSUB + sub) * kKB, a.lo_row + tl.y, &full[s]);
          }
          ++n_issued;
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {  // let this thread's copies still in flight (the last S stages at most) land
        int ss = s;
        uint32_t pp = ph;
        for (int i = 0; i < S && i < n_issued; ++i) {
          if (--ss < 0) {
            ss = S - 1;
            pp ^= 1u;
          }
          drain_wait(&full[ss], pp);
        }
      }
    }
  } else if (warp < 2 + 4 * NG) {
    // ------------------------------------------------ dequantizing producers
    // NG groups of four warps take every NG-th stage of the CTA's sequence
    // (item, stage), so NG stages are dequantized at once.  In a group,
    // thread t owns A-tile row t: per 64-column sub-tile, the low nibbles of
    // its 32 code bytes (K 0..31, chunks 0..3) and the high nibbles (K 32..63,
    // chunks 4..7).  Chunk c of row t sits at (t/8)*1024 + (t%8)*128 +
    // ((c ^ t%8) * 16): the 128-byte swizzle the MMA descriptors name.  Raw
    // bytes travel kDepth group steps ahead through the thread's own slots of
    // a cp.async ring: per sub-tile 48 bytes = super-block header (d, dmin,
    // scales) + 32 code bytes.
    const int grp = (warp - 2) / 4;
    // with A in tensor memory a warp may only write its own lane quarter (warp % 4)
    const int t = TMEM_A ? 32 * (gwarp & 3) + lane : 32 * (warp - 2 - 4 * grp) + lane;
    const uint32_t row_off = (uint32_t)(t >> 3) * 1024u + (uint32_t)(t & 7) * 128u;
    uint8_t* my_raw = raw + (size_t)grp * kDepth * kSlot + (size_t)t * kRowRaw;
    auto row_e0 = [&](int item) {
      const int4 tl = a.tiles[item / R];
      const int rt = item % R;
      const long long wr = GATEUP ? (long long)((t & 1) ? a.ff : 0) + 64ll * rt + (t >> 1)
                                  : (long long)kTileM * rt + t;
      return (long long)tl.x * a.expert_elems + wr * a.cols;
    };
    // A cursor at the start of stage st of item `item`: its first 64-column
    // block is group g of the super-block at blk.
    struct Cursor {
      int item, st, g;
      const uint8_t* blk;
    };
    auto start = [&](Cursor& c, int item) {
      c.item = item;
      c.st = 0;
      c.g = 0;
      c.blk = a.w;
      if (item < n_items) {
        const long long e0 = row_e0(item);
        c.blk = a.w + (size_t)(e0 >> 8) * 144;
        c.g = (int)((e0 >> 6) & 3);
      }
    };
    auto step = [&](Cursor& c) {  // on to the next stage of the sequence
      const int n = nsub_of(c.st);
      c.g += n;
      c.blk += 144 * (c.g >> 2);
      c.g &= 3;
      if (++c.st == nst) start(c, c.item + P * gridDim.x);
    };
    Cursor fc, cc;  // fetch and compute cursors, both at this group's first stage
    start(fc, blockIdx.x + pp * gridDim.x);
    for (int i = 0; i < grp && fc.item < n_items; ++i) step(fc);
    cc = fc;
    int f_slot = 0;
    auto fetch = [&]() {  // copies for the fetch cursor (if any are left); always one commit group
      if (fc.item < n_items) {
        const int n = nsub_of(fc.st);
        const uint8_t* blk = fc.blk;
        int g = fc.g;
        uint8_t* dst = my_raw + (size_t)f_slot * kSlot;
#pragma unroll
        for (int sub = 0; sub < KSUB; ++sub) {
          if (sub < n) {
            cp_async16(dst + sub * kRawRow, blk);
            cp_async16(dst + sub * kRawRow + 16, blk + 16 + 32 * g);
            cp_async16(dst + sub * kRawRow + 32, blk + 32 + 32 * g);
            if (++g == 4) {
              g = 0;
              blk += 144;
            }
          }
        }
        for (int i = 0; i < NG && fc.item < n_items; ++i) step(fc);
      }
      cp_async_commit();
      if (++f_slot == kDepth) f_slot = 0;
    };
#pragma unroll 1
    for (int i = 0; i < kDepth - 1; ++i) fetch();
    int s = grp, c_slot = 0;  // ring stage of this group's first stage, then every NG-th one
    uint32_t ph = 0;
    while (cc.item < n_items) {
      fetch();
      cp_async_wait<kDepth - 1>();  // this thread's bytes for the compute cursor have landed
      const int n = nsub_of(cc.st);
      // every lane waits; the verdict is made warp-uniform so the warp never splits
      if (!__all_sync(0xffffffffu, tc_wait(&empty[s], ph ^ 1u, abort_flag, a.status, ERR_TIMEOUT_EMPTY))) break;
      int g = cc.g;
#pragma unroll
      for (int sub = 0; sub < KSUB; ++sub) {
        if (sub < n) {
          const uint8_t* src = my_raw + (size_t)c_slot * kSlot + sub * kRawRow;
          const uint4 hd = *reinterpret_cast<const uint4*>(src);
          const uint4 q0 = *reinterpret_cast<const uint4*>(src + 16);
          const uint4 q1 = *reinterpret_cast<const uint4*>(src + 32);
          // getScaleMinK4 (Q4_KFloatTensor.kt:70-84) for sub-blocks 2g (low nibbles) and 2g+1 (high)
          SubConst kc[2];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int j = 2 * g + hh;
            uint32_t sc, mn;
            if (j < 4) {
              sc = scale_byte(hd.y, hd.z, hd.w, j) & 63u;
              mn = scale_byte(hd.y, hd.z, hd.w, j + 4) & 63u;
            } else {
              const uint32_t bj4 = scale_byte(hd.y, hd.z, hd.w, j + 4);
              sc = (bj4 & 0xFu) | ((scale_byte(hd.y, hd.z, hd.w, j - 4) >> 6) << 4);
              mn = (bj4 >> 4) | ((scale_byte(hd.y, hd.z, hd.w, j) >> 6) << 4);
            }
            const float d = f16_bits_to_f32((uint16_t)(hd.x & 0xFFFFu));
            const float dmin = f16_bits_to_f32((uint16_t)(hd.x >> 16));
            const float sf = d * (float)sc;     // exact: 11-bit by 6-bit product
            const float mf = dmin * (float)mn;  // exact
            kc[hh] = sub_const(hh ? sf * 0.0625f : sf, mf);
          }
          const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
          if (TMEM_A) {
            // word i of the row (stored K positions 2i, 2i+1) goes to column i of the sub-tile
            uint32_t r[32];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint2 la = q4_word_to_f16(qw[2 * i], 0x000F000Fu, kc[0]);
              const uint2 lb = q4_word_to_f16(qw[2 * i + 1], 0x000F000Fu, kc[0]);
              const uint2 ha = q4_word_to_f16(qw[2 * i], 0x00F000F0u, kc[1]);
              const uint2 hb = q4_word_to_f16(qw[2 * i + 1], 0x00F000F0u, kc[1]);
              r[4 * i] = la.x, r[4 * i + 1] = la.y, r[4 * i + 2] = lb.x, r[4 * i + 3] = lb.y;
              r[16 + 4 * i] = ha.x, r[16 + 4 * i + 1] = ha.y, r[16 + 4 * i + 2] = hb.x, r[16 + 4 * i + 3] = hb.y;
            }
            tmem_st32(tmem_base + ((uint32_t)(32 * (gwarp & 3)) << 16) + a.tmem_a_col + (uint32_t)(s * KSUB + sub) * 32u,
                      r);
          } else {
            uint8_t* dst = a_st + (size_t)(s * KSUB + sub) * kATile + row_off;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint2 la = q4_word_to_f16(qw[2 * i], 0x000F000Fu, kc[0]);
              const uint2 lb = q4_word_to_f16(qw[2 * i + 1], 0x000F000Fu, kc[0]);
              const uint2 ha = q4_word_to_f16(qw[2 * i], 0x00F000F0u, kc[1]);
              const uint2 hb = q4_word_to_f16(qw[2 * i + 1], 0x00F000F0u, kc[1]);
              *reinterpret_cast<uint4*>(dst + (((uint32_t)i ^ (uint32_t)(t & 7)) << 4)) =
                  make_uint4(la.x, la.y, lb.x, lb.y);
              *reinterpret_cast<uint4*>(dst + (((uint32_t)(4 + i) ^ (uint32_t)(t & 7)) << 4)) =
                  make_uint4(ha.x, ha.y, hb.x, hb.y);
            }
          }
          g = (g + 1) & 3;
        }
      }
      if (++c_slot == kDepth) c_slot = 0;
      if (TMEM_A) {
        tmem_st_wait();  // the rows are in tensor memory before the MMA thread hears of them
        tc_fence_before();
      } else {
        fence_async_smem();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[s]);
      s += NG;  // this group's next stage is NG on (S >= NG)
      if (s >= S) {
        s -= S;
        ph ^= 1u;
      }
      for (int i = 0; i < NG && cc.item < n_items; ++i) step(cc);
    }
    cp_async_wait<0>();  // no copy of this thread outlives the role (after an abort too)
  } else {
    // ------------------------------------------------ epilogue
    const int q = gwarp & 3;  // tensor-memory lane quarter this warp may access
    uint32_t acc = 0, aph = 0;
    for (int item = blockIdx.x + pp * gridDim.x; item < n_items; item += P * gridDim.x) {
      const int4 tl = a.tiles[item / R];
      const int rt = item % R, n = tl.z, p0 = tl.y;
      if (!__all_sync(0xffffffffu, tc_wait(&tfull[acc], aph, abort_flag, a.status, ERR_TIMEOUT_FULL))) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + ((uint32_t)(32 * q) << 16) + acc * (uint32_t)a.acc_cols;
      for (int c0 = 0; c0 < n; c0 += 32) {
        float v[32];
        tmem_ld32(tb + (uint32_t)c0, v);
        if (GATEUP) {
          // Lanes 2i / 2i+1 hold the gate / up row of pair 16q + i.  Per two
          // token columns the even lane finishes column jj, the odd lane
          // column jj + 1, each after one exchange.
          const int col = kperm(64 * rt + 16 * q + (lane >> 1));  // stored K order of the down product
          const bool odd = lane & 1;
#pragma unroll
          for (int jj = 0; jj < 32; jj += 2) {
            const float recv = __shfl_xor_sync(0xffffffffu, odd ? v[jj] : v[jj + 1], 1);
            const float gate = odd ? recv : v[jj];
            const float up = odd ? v[jj + 1] : recv;
            const int tok = c0 + jj + (odd ? 1 : 0);
            if (tok < n) {
              const float gv = gelu_f(gate) * up;
              const __half hi = __float2half_rn(gv);
              a.g16[(size_t)(p0 + tok) * a.out_ld + col] = hi;
              a.g16[(size_t)(a.lo_row + p0 + tok) * a.out_ld + col] = __float2half_rn(gv - __half2float(hi));
            }
          }
        } else {
          const int my_slot = (c0 + lane < n) ? a.perm[p0 + c0 + lane] : 0;
          const int row = kTileM * rt + 32 * q + lane;
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            const int sl = __shfl_sync(0xffffffffu, my_slot, jj);
            if (c0 + jj < n) a.D[(size_t)sl * a.out_ld + row] = v[jj];
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1u;
      if (acc == 0) aph ^= 1u;
    }
  }

  __syncthreads();
  if (gwarp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(*tmem_slot0, a.tmem_cols);
  }
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    cudaGetLastError();
  });
  return fn;
}

// [rows][cols] fp16, row-major; box = 64 columns x box_rows rows, 128-byte swizzle.
bool make_map(PFN_cuTensorMapEncodeTiled_v12000 enc, CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols,
              uint32_t box_rows) {
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kKB, box_rows};
  const cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t al256(size_t v) { return (v + 255) / 256 * 256; }

struct TcWork {
  __half *x16, *g16;
  int4* tiles;
  int32_t* n_tiles;
};

TcWork carve_tc(void* base, int T, int dim, int E, int K, int ff) {
  TcWork w;
  uint8_t* p = static_cast<uint8_t*>(base);
  const size_t n_pos = (size_t)T * K;
  w.x16 = reinterpret_cast<__half*>(p);  // high parts, then low parts
  p += al256(2 * n_pos * dim * 2);
  w.g16 = reinterpret_cast<__half*>(p);
  p += al256(2 * n_pos * ff * 2);
  w.tiles = reinterpret_cast<int4*>(p);
  p += al256((n_pos / 16 + E + 1) * sizeof(int4));
  w.n_tiles = reinterpret_cast<int32_t*>(p);
  return w;
}

int token_cap(int T, int K, int E) {
  const long long avg = (long long)T * K / E;
  return avg >= 128 ? 256 : avg >= 48 ? 128 : avg >= 12 ? 64 : 32;
}

}  // namespace

size_t moe_tc_scratch_bytes(int T, int dim, int E, int K, int ff) {
  const size_t n_pos = (size_t)T * K;
  return al256(2 * n_pos * dim * 2) + al256(2 * n_pos * ff * 2) + al256((n_pos / 16 + E + 1) * sizeof(int4)) + 256;
}

bool moe_tc_supported(int gate_up_type, int down_type, int dim, int ff, int E) {
  return gate_up_type == Q4_K && down_type == Q4_K && dim % kTileM == 0 && ff % kKB == 0 && dim % 256 == 0 &&
         E <= kMaxExpertsTc && encode_fn() != nullptr;
}

bool moe_tc_wanted(int T, int K, int E) {
  const char* env = std::getenv("G4_MOE_TC");
  if (env && env[0] == '0') return false;
  if (env && env[0] == '1') return true;
  return 4ll * T * K >= (long long)E;  // a quarter of a token per expert on average, or more
}

cudaError_t launch_moe_tc(g4_ctx* c, const uint8_t* gate_up_w, const uint8_t* down_w, const float* moe_in,
                          const int32_t* offsets, const int32_t* perm, float* D, void* work, int T, int dim, int E,
                          int K, int ff, cudaStream_t st) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  const int n_pos = T * K;
  TcWork w = carve_tc(work, T, dim, E, K, ff);
  const int cap = token_cap(T, K, E);

  moe_tc_tiles_kernel<<<1, kMaxExpertsTc, 0, st>>>(offsets, E, cap, w.tiles, w.n_tiles);
  moe_tc_gather_kernel<<<(n_pos + 7) / 8, 256, 0, st>>>(moe_in, perm, w.x16, n_pos, dim, K);

  CUtensorMap mx[kNumBoxes], mg[kNumBoxes];
  for (int b = 0; b < kNumBoxes; ++b) {
    if (!make_map(enc, &mx[b], w.x16, 2ull * n_pos, (uint64_t)dim, 16u << b) ||
        !make_map(enc, &mg[b], w.g16, 2ull * n_pos, (uint64_t)ff, 16u << b))
      return cudaErrorInvalidValue;
  }
  const int bsub = cap * 128;  // one 64-column token sub-tile
  // Narrow token tiles: two pipelines (two MMA issuers), one producer group
  // each, weights in tensor memory.  128-token tiles: one pipeline, weights in
  // tensor memory next to the 256 accumulator columns.  256-token tiles: the
  // accumulators fill tensor memory, weights go through shared memory.
  const int P = cap <= 64 ? 2 : 1;
  const int ng = cap <= 64 ? 1 : 2;
  const int ksub = 1;
  const bool tmem_a = cap <= 128;
  const size_t optin = c->dev.smem_optin;
  const size_t a_bytes = tmem_a ? 0 : (size_t)kATile;
  const size_t raw_bytes = (size_t)tc_raw_bytes(ng);
  const size_t stage_bytes = (size_t)ksub * (a_bytes + 2 * bsub);  // token tiles: high and low parts
  const size_t pipe_budget = (optin - 1024) / P;
  if (pipe_budget < raw_bytes + kBarBytes + 2 * stage_bytes) return cudaErrorInvalidConfiguration;
  int stages = (int)((pipe_budget - raw_bytes - kBarBytes) / stage_bytes);
  if (tmem_a) stages = std::min(stages, (512 / P - 2 * cap) / (32 * ksub));
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages < ng || stages < 2) return cudaErrorInvalidConfiguration;  // every group needs a stage of its own
  const size_t pipe_bytes = (stages * stage_bytes + raw_bytes + kBarBytes + 1023) / 1024 * 1024;
  // at least 120 KB, so that one CTA per SM holds all 512 tensor-memory columns
  const size_t smem = std::max<size_t>(1024 + P * pipe_bytes, 120 * 1024);
  if (smem > optin) return cudaErrorInvalidConfiguration;

  TcArgs ga{};
  ga.w = gate_up_w;
  ga.expert_elems = 2ll * ff * dim;
  ga.cols = dim;
  ga.ff = ff;
  ga.out_ld = ff;
  ga.n_row_tiles = ff / 64;
  ga.nkb = dim / kKB;
  ga.stages = stages;
  ga.b_stage_bytes = bsub;
  ga.acc_cols = cap;
  ga.tmem_cols = 512;
  ga.tmem_a_col = 2u * (uint32_t)cap;
  ga.pipe_bytes = (int)pipe_bytes;
  ga.tiles = w.tiles;
  ga.n_tiles = w.n_tiles;
  ga.perm = perm;
  ga.g16 = w.g16;
  ga.D = nullptr;
  ga.lo_row = n_pos;
  ga.status = c->status;

  TcArgs da = ga;
  da.w = down_w;
  da.expert_elems = (long long)dim * ff;
  da.cols = ff;
  da.out_ld = dim;
  da.n_row_tiles = dim / kTileM;
  da.nkb = ff / kKB;
  da.g16 = nullptr;
  da.D = D;

  using Kern = void (*)(TcArgs, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap);
  const Kern kg = P == 2 ? moe_tc_kernel<true, 1, true, 1, 2> : tmem_a ? moe_tc_kernel<true, 1, true, 2, 1>
                                                                       : moe_tc_kernel<true, 1, false, 2, 1>;
  const Kern kd = P == 2 ? moe_tc_kernel<false, 1, true, 1, 2> : tmem_a ? moe_tc_kernel<false, 1, true, 2, 1>
                                                                        : moe_tc_kernel<false, 1, false, 2, 1>;
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(kg, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess ||
      (e = cudaFuncSetAttribute(kd, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess)
    return e;
  const int grid = c->dev.sms;
  const int threads = P * tc_threads(ng);
  kg<<<grid, threads, smem, st>>>(ga, mx[0], mx[1], mx[2], mx[3], mx[4]);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  kd<<<grid, threads, smem, st>>>(da, mg[0], mg[1], mg[2], mg[3], mg[4]);
  return cudaGetLastError();
}

}  // namespace g4
