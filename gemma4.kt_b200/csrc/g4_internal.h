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

// fused: reserve shared memory for a fused prologue (launch_gemv_fused).
// max_smem > 0 caps the plan's shared memory (room for a second CTA per SM).
// exact_x: two-part int16 activations for Q8_0 / Q4_K / Q6_K (rows of whole
// blocks only), products at fp32 precision instead of ~3e-5.
// latency: favour many warps per row (the split form) for decode-size matrices.
GemvPlan plan_gemv(const DeviceInfo& dev, int type, long long off, int rows, int cols, bool fused = false,
                   size_t max_smem = 0, bool exact_x = false, bool latency = false);
// Launch with a plan from plan_gemv (the caller caches plans: planning queries
// occupancy and sets kernel attributes, which costs microseconds of host time).
// Returns the cudaError_t of the launch.
int launch_gemv(const GemvPlan& p, const uint8_t* w, const float* x, float* y, unsigned* status,
                cudaStream_t st);
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
