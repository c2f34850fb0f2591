// g4_gemv.cu -- quantized matrix-vector product y = W[off : off+rows*cols] . x
// for GGUF Q8_0 / Q4_K / Q6_K / BF16 / F32 block streams, on sm_100a.
//
// Replaces FloatTensor.matmul(that, out, dim0, dim1[, thisOffset])
// (FloatTensor.kt:18-29) and the per-type vectorDot it fans out to.
//
// Design (HBM-bound, CUDA cores):
//  * Persistent CTAs (grid = #SMs x resident CTAs).  Warp 0 is a producer: one
//    lane streams contiguous row tiles of the raw block stream into a ring of
//    shared-memory stages with cp.async.bulk (TMA bulk copies, no multicast),
//    signalling an mbarrier per stage.  The weights keep their on-disk layout;
//    unaligned block strides (34 B, 210 B) are handled by copying the
//    16-byte-aligned superset of each tile and decoding at a byte offset.
//  * The other warps are consumers.  Each owns `rw` virtual rows of a tile and
//    walks 16-weight units across them; the 16 activations of a unit are loaded
//    once from shared memory and reused for every row (cuts smem traffic).
//  * Rows whose length is not a multiple of the block size (e.g. 704-wide Q4_K
//    expert down rows) are grouped into virtual rows of `pr` real rows, after
//    which the block pattern repeats; accumulators are kept per real row.
//  * Each warp reduces its rows with shuffles and writes y directly: no atomics,
//    deterministic.
#include "g4_gemv.cuh"
#include "g4_gemv_rows.cuh"
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
};

// Which (row group, chunk) the i-th stage of this warp holds.
struct Seq {
  int g, c;
};

__device__ __forceinline__ Seq seq_at(const GemvPlan& p, int i, int warp, int W) {
  if (p.split == 1) {
    const int gw = blockIdx.x * W + warp, GW = gridDim.x * W;
    return Seq{gw + (i / p.nchunks) * GW, i % p.nchunks};
  }
  return Seq{(int)blockIdx.x, warp + i * W};
}

__device__ __forceinline__ bool seq_valid(const GemvPlan& p, Seq s) { return s.g < p.ngroups && s.c < p.nchunks; }

template <int FMT, int PR, int RL>
__global__ void __launch_bounds__(512) gemv_rows_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const GemvPlan& p = a.p;
  constexpr int BS = block_size(FMT), TS = type_size(FMT);
  constexpr int ROWS = 32 * RL;
  float* xs = reinterpret_cast<float*>(smem + p.xs_off);
  float* xsum16 = reinterpret_cast<float*>(smem + p.xsum_off);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  uint8_t* ring = smem + p.ring_off;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, W = blockDim.x >> 5;
  const int NS = p.ns;
  const size_t stage_bytes = (size_t)ROWS * p.pitch;
  uint64_t* mybars = bars + warp * NS;
  uint8_t* myring = ring + (size_t)warp * NS * stage_bytes;

  if (threadIdx.x < W * NS) mbar_init(&bars[threadIdx.x], 1);
  if (threadIdx.x == 0) fence_barrier_init();
  // x -> shared memory, plus the sum of every 16 consecutive columns
  for (int i = threadIdx.x * 4; i < p.cols; i += blockDim.x * 4)
    *reinterpret_cast<float4*>(xs + i) = __ldg(reinterpret_cast<const float4*>(a.x + i));
  __syncthreads();
  for (int k = threadIdx.x; k < p.cols / 16; k += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) t += xs[16 * k + i];
    xsum16[k] = t;
  }
  __syncthreads();

  const long long blk0 = p.off / BS;  // first block of the matrix
  const int bpv = p.bpv;

  // Start of virtual row v, chunk c (bytes from the tensor base) and its length.
  auto seg = [&](long long v, int c, long long& start, int& len) {
    const int b = c * p.cb;
    const int nb = min(p.cb, bpv - b);
    start = (blk0 + v * bpv + b) * TS;
    len = nb * TS;
  };
  // All lanes copy their own rows' segments of stage (g, c) into slot `slot`.
  auto issue = [&](Seq sq, int slot) {
    uint64_t* bar = &mybars[slot];
    uint8_t* dst = myring + (size_t)slot * stage_bytes;
    uint32_t mine = 0;
#pragma unroll
    for (int j = 0; j < RL; ++j) {
      const long long v = (long long)sq.g * ROWS + j * 32 + lane;
      if (v < p.nvrows) {
        long long start;
        int len;
        seg(v, sq.c, start, len);
        const long long a0 = start & ~15ll, a1 = (start + len + 15) & ~15ll;
        bulk_g2s(dst + (size_t)(j * 32 + lane) * p.pitch, a.w + a0, (uint32_t)(a1 - a0), bar);
        mine += (uint32_t)(a1 - a0);
      }
    }
    const uint32_t total = __reduce_add_sync(0xffffffffu, mine);
    if (lane == 0) mbar_arrive_expect_tx(bar, total);
  };

  bool ok = true;
  int issued = 0, consumed = 0;
  for (; issued < NS; ++issued) {
    Seq sq = seq_at(p, issued, warp, W);
    if (!seq_valid(p, sq)) break;
    issue(sq, issued);
  }

  float acc[RL][PR];
#pragma unroll
  for (int j = 0; j < RL; ++j)
#pragma unroll
    for (int r = 0; r < PR; ++r) acc[j][r] = 0.f;

  int cur_g = -1;
  for (int i = 0;; ++i) {
    Seq sq = seq_at(p, i, warp, W);
    if (!seq_valid(p, sq)) break;
    const int slot = i % NS;
    if (!mbar_wait_bounded(&mybars[slot], (i / NS) & 1)) {
      record_error(a.status, ERR_TIMEOUT_FULL);
      ok = false;
      consumed = i;
      break;
    }
    if (p.split == 1 && sq.g != cur_g) {
      cur_g = sq.g;
#pragma unroll
      for (int j = 0; j < RL; ++j)
#pragma unroll
        for (int r = 0; r < PR; ++r) acc[j][r] = 0.f;
    }
    // ---- compute on this lane's row segments
    const uint8_t* base[RL];
#pragma unroll
    for (int j = 0; j < RL; ++j) {
      const long long v = (long long)sq.g * ROWS + j * 32 + lane;
      long long start = 0;
      int len = 0;
      if (v < p.nvrows) seg(v, sq.c, start, len);
      base[j] = myring + (size_t)slot * stage_bytes + (size_t)(j * 32 + lane) * p.pitch + (start & 15);
    }
    const int b0 = sq.c * p.cb;
    const int nb = min(p.cb, bpv - b0);
    if constexpr (FMT == Q4_K || FMT == Q6_K) {
      for (int b = 0; b < nb; ++b) {
        const uint8_t* blk[RL];
#pragma unroll
        for (int j = 0; j < RL; ++j) blk[j] = base[j] + b * TS;
        if constexpr (FMT == Q4_K) block_q4k<RL, PR>(blk, (b0 + b) * BS, p.cols, xs, xsum16, acc);
        else block_q6k<RL, PR>(blk, (b0 + b) * BS, p.cols, xs, xsum16, acc);
      }
    } else if constexpr (FMT == Q8_0) {
      for (int b = 0; b < nb; ++b) {
        const uint8_t* blk[RL];
#pragma unroll
        for (int j = 0; j < RL; ++j) blk[j] = base[j] + b * TS;
        float (&acc1)[RL][1] = *reinterpret_cast<float(*)[RL][1]>(&acc);
        block_q8_0<RL>(blk, (b0 + b) * BS, xs, acc1);
      }
    } else {
      // BF16 / F32: "blocks" are single elements; 16-byte loads
      constexpr int EPL = 16 / TS;  // elements per 16-byte load
      float2 s2[RL];
#pragma unroll
      for (int j = 0; j < RL; ++j) s2[j] = f2(0.f, 0.f);
      for (int e = 0; e < nb; e += EPL) {
        const uint8_t* pp[RL];
#pragma unroll
        for (int j = 0; j < RL; ++j) pp[j] = base[j] + e * TS;
        if constexpr (FMT == BF16) chunk16_bf16<RL>(pp, b0 + e, xs, s2);
        else chunk16_f32<RL>(pp, b0 + e, xs, s2);
      }
#pragma unroll
      for (int j = 0; j < RL; ++j) acc[j][0] += s2[j].x + s2[j].y;
    }
    // ---- refill this slot with stage i + NS (same warp: no other reader)
    __syncwarp();
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    {
      Seq nx = seq_at(p, i + NS, warp, W);
      if (seq_valid(p, nx)) {
        issue(nx, slot);
        ++issued;
      }
    }
    // ---- row group finished: write results
    if (p.split == 1) {
      if (sq.c == p.nchunks - 1) {
#pragma unroll
        for (int j = 0; j < RL; ++j) {
          const long long v = (long long)sq.g * ROWS + j * 32 + lane;
          if (v < p.nvrows)
#pragma unroll
            for (int r = 0; r < PR; ++r) a.y[v * PR + r] = acc[j][r];
        }
      }
    }
  }

  if (p.split > 1) {
    // CTA = one row group; warps hold partial sums over disjoint chunks.
    float* red = reinterpret_cast<float*>(smem + p.red_off);
#pragma unroll
    for (int j = 0; j < RL; ++j)
#pragma unroll
      for (int r = 0; r < PR; ++r) red[((size_t)warp * ROWS + j * 32 + lane) * PR + r] = acc[j][r];
    __syncthreads();
    for (int t = threadIdx.x; t < ROWS * PR; t += blockDim.x) {
      const long long v = (long long)blockIdx.x * ROWS + t / PR;
      float sum = 0.f;
      for (int w = 0; w < W; ++w) sum += red[(size_t)w * ROWS * PR + t];
      if (v < p.nvrows) a.y[v * PR + (t % PR)] = sum;
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

template <int FMT>
static KernelFn pick_kernel(int pr, int rl) {
  if (pr == 1) return rl == 2 ? gemv_rows_kernel<FMT, 1, 2> : gemv_rows_kernel<FMT, 1, 1>;
  if constexpr (FMT == Q4_K || FMT == Q6_K) {
    if (pr == 2 && rl == 1) return gemv_rows_kernel<FMT, 2, 1>;
    if (pr == 4 && rl == 1) return gemv_rows_kernel<FMT, 4, 1>;
  }
  return nullptr;
}

static KernelFn kernel_for(int type, int pr, int rl) {
  switch (type) {
    case Q8_0: return pick_kernel<Q8_0>(pr, rl);
    case Q4_K: return pick_kernel<Q4_K>(pr, rl);
    case Q6_K: return pick_kernel<Q6_K>(pr, rl);
    case BF16: return pick_kernel<BF16>(pr, rl);
    case F32: return pick_kernel<F32>(pr, rl);
    default: return nullptr;
  }
}

// Overridable for tuning sweeps: G4_GEMV_CHUNK_BYTES, G4_GEMV_WARPS, G4_GEMV_STAGES, G4_GEMV_RL.
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
  GemvPlan p{};
  p.type = type;
  p.rows = rows;
  p.cols = cols;
  p.off = off;
  p.fast = 0;
  const int BS = block_size(type), TS = type_size(type);
  if (TS == 0 || type == F16 || rows <= 0 || cols <= 0) return p;
  if (cols % 16 != 0 || off % BS != 0) return p;
  if ((type == BF16 || type == F32) && ((off * TS) % 16) != 0) return p;
  int pr = 1;
  if (cols % BS != 0) {
    if (type == Q8_0 || cols % 64 != 0) return p;  // K-quant groups must not straddle rows
    pr = BS / gcd_i(cols % BS, BS);
    if (pr != 2 && pr != 4) return p;
  }
  if (rows % pr != 0) return p;
  const int xbytes = ((cols * 4 + 127) / 128) * 128;
  const int xsbytes = ((cols / 16 * 4 + 127) / 128) * 128;
  if (xbytes > 96 * 1024) return p;
  p.pr = pr;
  p.nvrows = rows / pr;
  p.bpv = (int)((long long)pr * cols / BS);
  p.rl = env_int("G4_GEMV_RL", 1) == 2 && pr == 1 ? 2 : 1;
  const int rows_per_group = 32 * p.rl;
  p.ngroups = (p.nvrows + rows_per_group - 1) / rows_per_group;

  // chunk: about `target` bytes of one row per bulk copy, divisor of bpv if possible
  const int target = env_int("G4_GEMV_CHUNK_BYTES", 288);
  int cb = std::max(1, std::min(p.bpv, target / TS));
  if (type == BF16) cb = std::max(8, cb / 8 * 8);
  if (type == F32) cb = std::max(4, cb / 4 * 4);
  const bool small = p.ngroups < 2 * dev.sms;
  if (small) {
    // few row groups: split each row over up to 8 warps of one CTA
    int want = std::max(1, (p.bpv + 7) / 8);
    if (type == BF16) want = std::max(8, (want + 7) / 8 * 8);
    if (type == F32) want = std::max(4, (want + 3) / 4 * 4);
    cb = std::min(cb, want);
  }
  p.cb = cb;
  p.nchunks = (p.bpv + cb - 1) / cb;
  p.pitch = pitch_for(cb * TS + 32);
  size_t stage = (size_t)rows_per_group * p.pitch;
  const size_t budget = dev.smem_optin > 0 ? dev.smem_optin : 227 * 1024;
  const size_t fixed = (size_t)xbytes + xsbytes + 256;
  if (small) {
    p.split = std::min(p.nchunks, 8);
    p.warps = p.split;
    p.ns = 2;
  } else {
    p.split = 1;
    p.warps = env_int("G4_GEMV_WARPS", 8);
    p.ns = env_int("G4_GEMV_STAGES", 3);
  }
  for (;;) {
    size_t red = p.split > 1 ? (size_t)p.warps * rows_per_group * pr * 4 : 0;
    size_t need = fixed + red + (size_t)p.warps * p.ns * stage;
    if (need <= budget) break;
    if (p.ns > 2) --p.ns;
    else if (p.split == 1 && p.warps > 2) p.warps /= 2;
    else if (p.split > 1 && p.cb > 1 && type != BF16 && type != F32) {
      // narrower chunks, more of them: keeps the CTA's rings within shared memory
      p.cb = std::max(1, p.cb / 2);
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
  p.bar_off = xbytes + xsbytes;
  p.ring_off = p.bar_off + 128 * ((p.warps * p.ns * 8 + 127) / 128);
  p.red_off = (int)(p.ring_off + (size_t)p.warps * p.ns * stage);
  p.smem = (size_t)p.red_off + (p.split > 1 ? (size_t)p.warps * rows_per_group * pr * 4 : 0);
  KernelFn k = kernel_for(type, pr, p.rl);
  if (!k) return p;
  int occ = 0;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, 32 * p.warps, p.smem) != cudaSuccess || occ < 1) {
    cudaGetLastError();
    return p;
  }
  if (p.split > 1) p.grid = p.ngroups;
  else p.grid = (int)std::min<long long>((p.ngroups + p.warps - 1) / p.warps, (long long)dev.sms * occ);
  p.fast = 1;
  return p;
}

int launch_gemv(const GemvPlan& p, const uint8_t* w, const float* x, float* y, unsigned* status,
                cudaStream_t st) {
  if (p.fast) {
    GemvArgs a{p, w, x, y, status};
    KernelFn k = kernel_for(p.type, p.pr, p.rl);
    k<<<p.grid, 32 * p.warps, p.smem, st>>>(a);
  } else {
    int wpb = 8;
    gemv_generic_kernel<<<(p.rows + wpb - 1) / wpb, 32 * wpb, 0, st>>>(p.type, w, p.off, p.rows, p.cols, x, y);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_dequant(int type, const uint8_t* w, long long off, long long n, float* out, cudaStream_t st) {
  if (n <= 0) return 0;
  long long blocks = std::min<long long>((n + 255) / 256, 148 * 32);
  dequant_kernel<<<(int)blocks, 256, 0, st>>>(type, w, off, n, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace g4
