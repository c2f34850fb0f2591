// g4_internal.h -- declarations shared by the translation units of libg4b200.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace g4 {

struct DeviceInfo {
  int device;
  int sms;
  size_t smem_optin;
};

struct GemvPlan;
struct GemvFuse;

struct GemvOpts;
// Launch plan of y = W . x (options: GemvOpts in g4_gemv.cuh; exact_x gives
// products at fp32 precision instead of ~3e-5, latency favours a warp per row).
GemvPlan plan_gemv(const DeviceInfo& dev, int type, long long off, int rows, int cols);
GemvPlan plan_gemv(const DeviceInfo& dev, int type, long long off, int rows, int cols, const GemvOpts& o);
// Launch with a plan from plan_gemv (the caller caches plans: planning queries
// occupancy and sets kernel attributes, which costs microseconds of host time).
// Returns the cudaError_t of the launch.
int launch_gemv(const GemvPlan& p, const uint8_t* w, const float* x, float* y, unsigned* status,
                cudaStream_t st);
struct MmaGemvPlan;
// The decoder's Q8_0 GEMV on the tensor cores (g4_gemv_mma.cu): the repacked
// layout's size, the repack of a GGUF Q8_0 matrix into it, plan and launch.
size_t mma_packed_bytes(int rows, int cols);
int repack_q8_0_mma(const uint8_t* raw, int rows, int cols, uint8_t* packed, cudaStream_t st);
MmaGemvPlan plan_gemv_mma(const DeviceInfo& dev, int rows, int cols, bool pair, bool fused);
int launch_gemv_mma(const MmaGemvPlan& p, const uint8_t* packed, const float* x, float* y, const GemvFuse& f,
                    unsigned* status, cudaStream_t st, bool pdl);
struct MmaBatchPlan;
// Batched decode (g4_gemv_mma.cu): the per-token prologue into int8 limbs and
// the T-token GEMM on the repacked Q8_0 tiles.
MmaBatchPlan plan_gemm_mma_batch(const DeviceInfo& dev, int rows, int cols, int T);
// partials: mma_batch_partials(p, T) floats; tickets: p.nrb words, zero between launches
int launch_gemm_mma_batch(const MmaBatchPlan& p, const uint8_t* packed, const int8_t* lim, const float* lsc, int T,
                          float* y, int ldy, int out_mode, float softcap, unsigned long long* argmax,
                          float* partials, unsigned* tickets, cudaStream_t st);
int launch_batch_prologue(const GemvFuse& f, const float* x, int dim, int T, int8_t* lim, float* lsc,
                          cudaStream_t st);
struct DecGemvPlan;
// The decoder's GEMV (g4_gemv_dec.cu): Q8_0 / Q4_K / Q6_K rows of whole blocks;
// fast == 0 when it does not apply.  fused: room for a fused prologue.
DecGemvPlan plan_gemv_dec(const DeviceInfo& dev, int type, int rows, int cols, bool pair, bool fused);
int launch_gemv_dec(const DecGemvPlan& p, const uint8_t* w, const float* x, float* y, const GemvFuse& f,
                    unsigned* status, cudaStream_t st, bool pdl);
// Same with a fused prologue / epilogue; pdl launches with programmatic
// stream serialization (weights stream in before the previous kernel ends).
// Needs a plan made with fused = true for a fused prologue, and the fast kernel.
int launch_gemv_fused(const GemvPlan& p, const uint8_t* w, const float* x, float* y, const GemvFuse& f,
                      unsigned* status, cudaStream_t st, bool pdl);
int launch_dequant(int type, const uint8_t* w, long long off, long long n, float* out, cudaStream_t st);
// Resolve the fixed work array of g4_moe_layer_noalloc on `device` (which must
// be current); returns a cudaError_t (0 on success).
int noalloc_prepare_device(int device);

}  // namespace g4
