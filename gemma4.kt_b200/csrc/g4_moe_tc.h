// g4_moe_tc.h -- tensor-core (tcgen05) grouped expert products for wide
// token batches, used by g4_moe_layer when experts see many tokens each.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "g4_ctx.h"

namespace g4 {

// Device buffers the tensor-core path needs on top of the layer's own work
// buffers (sizes in bytes, each 256-byte aligned).
size_t moe_tc_scratch_bytes(int T, int dim, int E, int K, int ff);

// True when the weight types and the geometry are ones the tensor-core path
// handles (Q4_K experts, dim % 256 == 0, ff % 64 == 0, at most 256 experts)
// and the driver can encode TMA tensor maps.
bool moe_tc_supported(int gate_up_type, int down_type, int dim, int ff, int E);

// True when g4_moe_layer should take the tensor-core path for T tokens
// (G4_MOE_TC=0 disables it, G4_MOE_TC=1 forces it when supported).
bool moe_tc_wanted(int T, int K, int E);

// gate_up and down products of every routed slot on the tensor cores:
//   moe_in [T][dim] fp32, offsets [E+1] / perm [T*K] from the permutation step,
//   D [T*K][dim] fp32 indexed by slot = token*K + k (what the combine reads).
// work points at moe_tc_scratch_bytes(...) bytes.  Returns a cudaError_t
// (cudaSuccess on success).  Call only when moe_tc_supported(...) is true.
cudaError_t launch_moe_tc(g4_ctx* c, const uint8_t* gate_up_w, const uint8_t* down_w, const float* moe_in,
                          const int32_t* offsets, const int32_t* perm, float* D, void* work, int T, int dim, int E,
                          int K, int ff, cudaStream_t st);

}  // namespace g4
