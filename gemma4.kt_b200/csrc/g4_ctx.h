// g4_ctx.h -- the opaque handles behind include/g4.h.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "g4_internal.h"
#include "g4_gemv.cuh"

#include <map>
#include <tuple>

constexpr int kStatusWords = 16;  // device words behind g4_ctx::status

struct g4_ctx {
  g4::DeviceInfo dev{};
  // device words: [0] error flags written by kernels (bounded waits), [1] the
  // MoE front kernel's completion ticket (its last CTA resets it to 0)
  unsigned* status = nullptr;
  unsigned* ticket() const { return status + 1; }
  unsigned* status_host = nullptr;  // pinned copy target of status[0] (one synchronisation per check)
  void* scratch_ptr = nullptr; // growable device arena (host-buffer staging, MoE work buffers)
  size_t scratch_bytes = 0;
  void* pinned_ptr = nullptr;  // growable pinned host staging
  size_t pinned_bytes = 0;
  void* io_ptr = nullptr;      // device staging for the *_host entry points
  size_t io_bytes = 0;
  void* ep_ptr = nullptr;      // receive-side buffers of the expert-parallel MoE layer
  size_t ep_bytes = 0;
  void* blk_ptr = nullptr;     // work buffers of the MoE FFN block (beside the MoE layer's own)
  size_t blk_bytes = 0;
  void* comm = nullptr;        // ncclComm_t when g4_dist_init has run
  int rank = 0;
  int world = 1;
  int dist_timeout_ms = 120000;  // bound on waits for peer ranks (g4_dist_init_timeout)
  char err[512] = {0};
  // launch plans, keyed by (type, offset, rows, cols, x 16B-aligned)
  std::map<std::tuple<int, long long, int, int, int>, g4::GemvPlan> gemv_plans;

  void set_err(const char* fmt, ...);
  int cuda_fail(cudaError_t e, const char* what);
  int bind();
  void* scratch(size_t bytes);
  void* pinned(size_t bytes);
  void* io(size_t bytes);
  void* ep(size_t bytes);
  void* blk(size_t bytes);
  int check_status(cudaStream_t st);
};

struct g4_tensor {
  g4_ctx* ctx = nullptr;
  void* d = nullptr;
  int type = 0;
  uint64_t nbytes = 0;
  uint64_t n_elems = 0;
};

void g4_dist_teardown(g4_ctx* c);

// Collectives of the expert-parallel MoE layer, over the context's NCCL
// communicator (g4_dist_init).  Return 0 or a G4_E_* code with the message set.
//   allgather: recv[r*count + i] = send_of_rank_r[i]
//   alltoallv: to every peer p, send[soff[p], soff[p]+slen[p]) bytes; from every
//              peer p, receive rlen[p] bytes at recv + roff[p] (one NCCL group)
int g4_nccl_allgather_i32(g4_ctx* c, const int32_t* send, int32_t* recv, size_t count, cudaStream_t st);
int g4_nccl_alltoallv(g4_ctx* c, const void* send, const size_t* soff, const size_t* slen, void* recv,
                      const size_t* roff, const size_t* rlen, cudaStream_t st);
// Wait for the stream's work within the context's distributed timeout (polls
// the stream and the communicator's error state; aborts it on expiry).
int g4_dist_stream_wait(g4_ctx* c, cudaStream_t st);
