// g4_ctx.h -- the opaque handles behind include/g4.h.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "g4_internal.h"
#include "g4_gemv.cuh"

#include <map>
#include <tuple>

struct g4_ctx {
  g4::DeviceInfo dev{};
  unsigned* status = nullptr;  // device error word written by kernels (bounded waits)
  void* scratch_ptr = nullptr; // growable device arena (host-buffer staging, MoE work buffers)
  size_t scratch_bytes = 0;
  void* pinned_ptr = nullptr;  // growable pinned host staging
  size_t pinned_bytes = 0;
  void* io_ptr = nullptr;      // device staging for the *_host entry points
  size_t io_bytes = 0;
  void* comm = nullptr;        // ncclComm_t when g4_dist_init has run
  int rank = 0;
  int world = 1;
  char err[512] = {0};
  // launch plans, keyed by (type, offset, rows, cols, x 16B-aligned)
  std::map<std::tuple<int, long long, int, int, int>, g4::GemvPlan> gemv_plans;

  void set_err(const char* fmt, ...);
  int cuda_fail(cudaError_t e, const char* what);
  int bind();
  void* scratch(size_t bytes);
  void* pinned(size_t bytes);
  void* io(size_t bytes);
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
