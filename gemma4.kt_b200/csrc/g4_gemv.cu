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
#include "g4_internal.h"

#include <algorithm>
#include <cstdio>

namespace g4 {

struct GemvArgs {
  GemvPlan p;
  const uint8_t* w;  // tensor base (block stream), 256B aligned, padded by >=32 B
  const float* x;    // cols floats, 16B aligned
  float* y;          // rows floats
  unsigned* status;  // device error word
};

template <int FMT, int PR, int RW>
__global__ void __launch_bounds__(288) gemv_stream_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const GemvPlan& p = a.p;
  constexpr int BS = block_size(FMT), TS = type_size(FMT);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + 4;
  uint64_t* xbar = full + 8;
  float* xs = reinterpret_cast<float*>(smem + 128);
  uint8_t* stages = smem + 128 + p.xbytes;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NS = p.nstages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], p.ncw);
    }
    mbar_init(xbar, 1);
    fence_barrier_init();
  }
  __syncthreads();

  const long long blk_base = p.off / BS;  // off is block aligned on this path
  const long long vrow_blocks = (long long)p.pr * p.cols / BS;

  if (warp == 0) {
    if (lane != 0) return;
    const uint32_t xb = (uint32_t)p.cols * 4u;
    mbar_arrive_expect_tx(xbar, xb);
    bulk_g2s(xs, a.x, xb, xbar);
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x, ++it) {
      int s = it % NS;
      if (it >= NS && !mbar_wait_bounded(&empty[s], ((it / NS) - 1) & 1)) {
        record_error(a.status, ERR_TIMEOUT_EMPTY);
        ok = false;
        break;
      }
      long long v0 = (long long)tile * p.tile_vrows;
      long long nv = min((long long)p.tile_vrows, (long long)p.nvrows - v0);
      long long byte0 = (blk_base + v0 * vrow_blocks) * TS;
      long long byte1 = (blk_base + (v0 + nv) * vrow_blocks) * TS;
      long long a0 = byte0 & ~15ll, a1 = (byte1 + 15) & ~15ll;
      uint32_t bytes = (uint32_t)(a1 - a0);
      mbar_arrive_expect_tx(&full[s], bytes);
      bulk_g2s(stages + (size_t)s * p.stage_bytes, a.w + a0, bytes, &full[s]);
    }
    // Never leave the CTA with bulk copies still landing in its shared memory.
    for (int j = max(0, it - NS); j < it; ++j)
      if (!mbar_wait_bounded(&full[j % NS], (j / NS) & 1)) record_error(a.status, ERR_TIMEOUT_DRAIN);
    if (!mbar_wait_bounded(xbar, 0)) record_error(a.status, ERR_TIMEOUT_DRAIN);
    (void)ok;
    return;
  }

  // ---------------- consumers ----------------
  const int cw = warp - 1;
  if (!mbar_wait_bounded(xbar, 0)) {
    record_error(a.status, ERR_TIMEOUT_FULL);
    return;
  }
  int it = 0;
  for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x, ++it) {
    int s = it % NS;
    if (!mbar_wait_bounded(&full[s], (it / NS) & 1)) {
      record_error(a.status, ERR_TIMEOUT_FULL);
      return;
    }
    const long long v0 = (long long)tile * p.tile_vrows;
    const long long byte0 = (blk_base + v0 * vrow_blocks) * TS;
    const uint8_t* st = stages + (size_t)s * p.stage_bytes + (byte0 & 15);
    const long long myv = v0 + (long long)cw * RW;

    float acc[RW][PR];
#pragma unroll
    for (int i = 0; i < RW; ++i)
#pragma unroll
      for (int r = 0; r < PR; ++r) acc[i][r] = 0.f;

    for (int u = lane; u < p.units; u += 32) {
      const int e0 = u * 16;
      const int col = (PR == 1) ? e0 : (e0 % p.cols);
      const int rip = (PR == 1) ? 0 : (e0 / p.cols);
      float xv[16];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint4 t = lds128(xs + col + 4 * k);
        xv[4 * k + 0] = __uint_as_float(t.x);
        xv[4 * k + 1] = __uint_as_float(t.y);
        xv[4 * k + 2] = __uint_as_float(t.z);
        xv[4 * k + 3] = __uint_as_float(t.w);
      }
      float sx = 0.f;
      if constexpr (FMT == Q4_K) {
#pragma unroll
        for (int k = 0; k < 16; ++k) sx += xv[k];
      }
#pragma unroll
      for (int i = 0; i < RW; ++i) {
        if (myv + i < p.nvrows) {
          const uint8_t* vbp = st + (size_t)(cw * RW + i) * p.vb;
          float part = dot16<FMT>(vbp, u, xv, sx);
#pragma unroll
          for (int r = 0; r < PR; ++r) acc[i][r] += (rip == r) ? part : 0.f;
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
    for (int i = 0; i < RW; ++i) {
#pragma unroll
      for (int r = 0; r < PR; ++r) {
        float v = warp_sum(acc[i][r]);
        if (lane == 0 && myv + i < p.nvrows) a.y[(myv + i) * PR + r] = v;
      }
    }
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
static KernelFn pick_kernel(int pr, int rw) {
#define G4_K(PR, RW) \
  if (pr == PR && rw == RW) return gemv_stream_kernel<FMT, PR, RW>;
  G4_K(1, 1) G4_K(1, 2) G4_K(1, 4) G4_K(2, 1) G4_K(2, 2) G4_K(4, 1) G4_K(4, 2)
#undef G4_K
  return nullptr;
}

static KernelFn kernel_for(int type, int pr, int rw) {
  switch (type) {
    case Q8_0: return pick_kernel<Q8_0>(pr, rw);
    case Q4_K: return pick_kernel<Q4_K>(pr, rw);
    case Q6_K: return pick_kernel<Q6_K>(pr, rw);
    case BF16: return pick_kernel<BF16>(pr, rw);
    case F32: return pick_kernel<F32>(pr, rw);
    default: return nullptr;
  }
}

static constexpr int kMaxStage = 32 * 1024;
static constexpr int kStages = 3;

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
  // 16-byte shared loads of BF16/F32 units need 16-byte aligned tile starts.
  if ((type == BF16 || type == F32) && ((off * TS) % 16) != 0) return p;
  int pr = BS / gcd_i(cols % BS == 0 ? BS : cols % BS, BS);
  if (cols % BS == 0) pr = 1;
  if (pr != 1 && pr != 2 && pr != 4) return p;
  if (rows % pr != 0) return p;
  p.pr = pr;
  p.nvrows = rows / pr;
  p.vb = (int)((long long)pr * cols / BS * TS);
  p.units = pr * cols / 16;
  p.xbytes = ((cols * 4 + 127) / 128) * 128;
  if (p.xbytes > 64 * 1024) return p;

  // Choose (ncw, rw): stage <= kMaxStage, prefer enough tiles to fill the GPU,
  // then activation reuse (rw), then wide CTAs.
  const int target_tiles = dev.sms * 2;
  int best_ncw = 0, best_rw = 0;
  long long best_score = -1;
  const int rw_opts[3] = {4, 2, 1};
  const int ncw_opts[4] = {8, 4, 2, 1};
  for (int a = 0; a < 4; ++a)
    for (int b = 0; b < 3; ++b) {
      int ncw = ncw_opts[a], rw = rw_opts[b];
      if (pr == 4 && rw > 2) continue;
      if (pr == 2 && rw > 2) continue;
      long long stage = (long long)ncw * rw * p.vb + 32;
      if (stage > kMaxStage) continue;
      long long tiles = (p.nvrows + (long long)ncw * rw - 1) / ((long long)ncw * rw);
      long long score = (tiles >= target_tiles ? 1000000 : tiles * 100) + rw * 10 + ncw;
      if (score > best_score) {
        best_score = score;
        best_ncw = ncw;
        best_rw = rw;
      }
    }
  if (best_ncw == 0) return p;
  p.ncw = best_ncw;
  p.rw = best_rw;
  p.tile_vrows = p.ncw * p.rw;
  p.ntiles = (p.nvrows + p.tile_vrows - 1) / p.tile_vrows;
  p.stage_bytes = (int)((((long long)p.tile_vrows * p.vb + 32) + 127) / 128 * 128);
  p.nstages = kStages;
  p.smem = 128 + (size_t)p.xbytes + (size_t)p.nstages * p.stage_bytes;
  KernelFn k = kernel_for(type, pr, p.rw);
  if (!k) return p;
  int threads = 32 * (p.ncw + 1);
  int occ = 0;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, threads, p.smem) != cudaSuccess || occ < 1) {
    cudaGetLastError();
    return p;
  }
  p.grid = (int)std::min<long long>(p.ntiles, (long long)dev.sms * occ);
  p.fast = 1;
  return p;
}

int launch_gemv(const DeviceInfo& dev, int type, const uint8_t* w, long long off, int rows, int cols,
                const float* x, float* y, unsigned* status, cudaStream_t st, GemvPlan* plan_out) {
  GemvPlan p = plan_gemv(dev, type, off, rows, cols);
  if (p.fast && ((uintptr_t)x & 15u) != 0) p.fast = 0;
  if (plan_out) *plan_out = p;
  if (p.fast) {
    GemvArgs a{p, w, x, y, status};
    KernelFn k = kernel_for(type, p.pr, p.rw);
    k<<<p.grid, 32 * (p.ncw + 1), p.smem, st>>>(a);
  } else {
    int wpb = 8;
    gemv_generic_kernel<<<(rows + wpb - 1) / wpb, 32 * wpb, 0, st>>>(type, w, off, rows, cols, x, y);
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
