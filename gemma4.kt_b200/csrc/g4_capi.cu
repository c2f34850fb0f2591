// g4_capi.cu -- the C ABI (include/g4.h): contexts, tensor upload, matmul,
// dequant, status checks and the NCCL plumbing for row-sharded matmul.
#include "g4.h"
#include "g4_ctx.h"
#include "g4_gemv.cuh"

#include <dlfcn.h>
#include <nccl.h>

#include <time.h>
#include <sched.h>
#include <unistd.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>

using namespace g4;

static thread_local char g_init_err[512];

void g4_ctx::set_err(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(err, sizeof err, fmt, ap);
  va_end(ap);
}

int g4_ctx::cuda_fail(cudaError_t e, const char* what) {
  set_err("%s: %s", what, cudaGetErrorString(e));
  return G4_E_CUDA;
}

int g4_ctx::bind() {
  cudaError_t e = cudaSetDevice(dev.device);
  return e == cudaSuccess ? 0 : cuda_fail(e, "cudaSetDevice");
}

// A growable device arena: reallocated (after the queued work that may still
// read the old one) when a call needs more; slack: room for growth.
static void* grow_arena(void** p, size_t* have, size_t bytes, bool slack) {
  if (bytes <= *have) return *p;
  if (*p) {
    cudaDeviceSynchronize();  // the old arena may still be read by queued work
    cudaFree(*p);
  }
  *p = nullptr;
  *have = 0;
  const size_t want = slack ? bytes + bytes / 4 + (1u << 20) : bytes;
  if (cudaMalloc(p, want) != cudaSuccess) {
    cudaGetLastError();
    *p = nullptr;
    return nullptr;
  }
  *have = want;
  return *p;
}

void* g4_ctx::scratch(size_t bytes) { return grow_arena(&scratch_ptr, &scratch_bytes, bytes, true); }
void* g4_ctx::io(size_t bytes) { return grow_arena(&io_ptr, &io_bytes, bytes, false); }
void* g4_ctx::ep(size_t bytes) { return grow_arena(&ep_ptr, &ep_bytes, bytes, true); }
void* g4_ctx::blk(size_t bytes) { return grow_arena(&blk_ptr, &blk_bytes, bytes, true); }

void* g4_ctx::pinned(size_t bytes) {
  if (bytes <= pinned_bytes) return pinned_ptr;
  if (pinned_ptr) cudaFreeHost(pinned_ptr);
  pinned_ptr = nullptr;
  pinned_bytes = 0;
  if (cudaMallocHost(&pinned_ptr, bytes) != cudaSuccess) {
    cudaGetLastError();
    pinned_ptr = nullptr;
    return nullptr;
  }
  pinned_bytes = bytes;
  return pinned_ptr;
}

int g4_ctx::check_status(cudaStream_t st) {
  unsigned h = 0;
  if (status_host) {
    // the status word rides the stream into pinned memory: one synchronisation
    cudaError_t e = cudaMemcpyAsync(status_host, status, sizeof h, cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) return cuda_fail(e, "status read");
    e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "kernel execution");
    h = *status_host;
  } else {
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "kernel execution");
    e = cudaMemcpy(&h, status, sizeof h, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "status read");
  }
  if (h) {
    cudaMemset(status, 0, sizeof(unsigned));
    set_err("device status 0x%x (a bounded wait expired inside a kernel)", h);
    return G4_E_DEVICE;
  }
  return 0;
}

static bool supported_type(int t) {
  return t == G4_TYPE_F32 || t == G4_TYPE_F16 || t == G4_TYPE_Q4_0 || t == G4_TYPE_Q4_1 || t == G4_TYPE_Q5_1 ||
         t == G4_TYPE_Q8_0 || t == G4_TYPE_Q4_K || t == G4_TYPE_Q5_K || t == G4_TYPE_Q6_K || t == G4_TYPE_BF16 ||
         t == G4_TYPE_MXFP4;
}

extern "C" {

int g4_init(int device, g4_ctx** out) {
  if (!out) {
    snprintf(g_init_err, sizeof g_init_err, "g4_init: out is NULL");
    return G4_E_ARG;
  }
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || device < 0 || device >= n) {
    snprintf(g_init_err, sizeof g_init_err, "g4_init: device %d unavailable (%d devices, %s)", device, n,
             cudaGetErrorString(e));
    cudaGetLastError();
    return e != cudaSuccess ? G4_E_CUDA : G4_E_ARG;
  }
  cudaDeviceProp prop;
  if ((e = cudaSetDevice(device)) != cudaSuccess || (e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) {
    snprintf(g_init_err, sizeof g_init_err, "g4_init: %s", cudaGetErrorString(e));
    return G4_E_CUDA;
  }
  if (prop.major != 10) {
    snprintf(g_init_err, sizeof g_init_err, "g4_init: device %d is sm_%d%d; this library is built for sm_100a",
             device, prop.major, prop.minor);
    return G4_E_CUDA;
  }
  g4_ctx* c = new (std::nothrow) g4_ctx();
  if (!c) return G4_E_NOMEM;
  c->dev.device = device;
  c->dev.sms = prop.multiProcessorCount;
  c->dev.smem_optin = prop.sharedMemPerBlockOptin;
  if ((e = cudaMalloc(&c->status, kStatusWords * sizeof(unsigned))) != cudaSuccess) {
    snprintf(g_init_err, sizeof g_init_err, "g4_init: %s", cudaGetErrorString(e));
    delete c;
    return G4_E_NOMEM;
  }
  cudaMemset(c->status, 0, kStatusWords * sizeof(unsigned));
  if (cudaMallocHost(&c->status_host, sizeof(unsigned)) != cudaSuccess) {
    cudaGetLastError();
    c->status_host = nullptr;  // check_status falls back to a blocking copy
  }
  // Bring the allocation-free MoE entry point's fixed array into being now,
  // while the device still has room: under lazy module loading it would
  // otherwise appear at its first use, after a host may have reserved the
  // remaining HBM.  A failure here is reported by that entry point later.
  noalloc_prepare_device(device);
  *out = c;
  return 0;
}

int g4_destroy(g4_ctx* c) {
  if (!c) return G4_E_ARG;
  cudaSetDevice(c->dev.device);
  cudaDeviceSynchronize();
  g4_dist_teardown(c);
  if (c->scratch_ptr) cudaFree(c->scratch_ptr);
  if (c->pinned_ptr) cudaFreeHost(c->pinned_ptr);
  if (c->io_ptr) cudaFree(c->io_ptr);
  if (c->ep_ptr) cudaFree(c->ep_ptr);
  if (c->blk_ptr) cudaFree(c->blk_ptr);
  if (c->status) cudaFree(c->status);
  if (c->status_host) cudaFreeHost(c->status_host);
  delete c;
  return 0;
}

const char* g4_last_error(const g4_ctx* c) { return c ? c->err : g_init_err; }

static int upload_common(g4_ctx* c, int type, const void* host, uint64_t nbytes, uint64_t n_elems,
                         g4_tensor** out) {
  if (!c || !out || (!host && nbytes)) {
    if (c) c->set_err("g4_tensor_upload: NULL argument");
    return G4_E_ARG;
  }
  *out = nullptr;
  if (!supported_type(type)) {
    c->set_err("Quantization format %d is not supported", type);
    return G4_E_TYPE;
  }
  const int BS = block_size(type), TS = type_size(type);
  if (n_elems % BS != 0 || n_elems / BS * TS != nbytes) {
    c->set_err("g4_tensor_upload: %llu elements of type %d need %llu bytes, got %llu",
               (unsigned long long)n_elems, type, (unsigned long long)(n_elems / BS * TS),
               (unsigned long long)nbytes);
    return G4_E_ARG;
  }
  if (int r = c->bind()) return r;
  g4_tensor* t = new (std::nothrow) g4_tensor();
  if (!t) return G4_E_NOMEM;
  // Pad so 16-byte-rounded bulk copies of the last tile stay in bounds.
  size_t alloc = ((nbytes + 255) / 256) * 256 + 256;
  cudaError_t e = cudaMalloc(&t->d, alloc);
  if (e != cudaSuccess) {
    delete t;
    cudaGetLastError();
    c->set_err("g4_tensor_upload: cudaMalloc(%zu): %s", alloc, cudaGetErrorString(e));
    return G4_E_NOMEM;
  }
  cudaMemset(t->d, 0, alloc);
  if (nbytes && (e = cudaMemcpy(t->d, host, nbytes, cudaMemcpyHostToDevice)) != cudaSuccess) {
    cudaFree(t->d);
    delete t;
    return c->cuda_fail(e, "g4_tensor_upload: copy");
  }
  t->ctx = c;
  t->type = type;
  t->nbytes = nbytes;
  t->n_elems = n_elems;
  *out = t;
  return 0;
}

int g4_tensor_upload(g4_ctx* c, int type, const void* host, uint64_t nbytes, uint64_t n_elems, g4_tensor** out) {
  return upload_common(c, type, host, nbytes, n_elems, out);
}

int g4_tensor_upload_rows(g4_ctx* c, int type, const void* host, uint64_t cols, uint64_t row_begin,
                          uint64_t row_count, g4_tensor** out) {
  if (!c || !host || !out) {
    if (c) c->set_err("g4_tensor_upload_rows: NULL argument");
    return G4_E_ARG;
  }
  if (!supported_type(type)) {
    c->set_err("Quantization format %d is not supported", type);
    return G4_E_TYPE;
  }
  const uint64_t BS = block_size(type), TS = type_size(type);
  uint64_t e0 = row_begin * cols, n = row_count * cols;
  if (e0 % BS || n % BS) {
    c->set_err("g4_tensor_upload_rows: shard rows must start and end on %llu-element block boundaries",
               (unsigned long long)BS);
    return G4_E_ARG;
  }
  return upload_common(c, type, (const uint8_t*)host + e0 / BS * TS, n / BS * TS, n, out);
}

int g4_tensor_free(g4_tensor* t) {
  if (!t) return G4_E_ARG;
  if (t->ctx) cudaSetDevice(t->ctx->dev.device);
  cudaFree(t->d);
  delete t;
  return 0;
}

const void* g4_tensor_device_ptr(const g4_tensor* t) { return t ? t->d : nullptr; }
uint64_t g4_tensor_nbytes(const g4_tensor* t) { return t ? t->nbytes : 0; }
uint64_t g4_tensor_n_elems(const g4_tensor* t) { return t ? t->n_elems : 0; }
int g4_tensor_type(const g4_tensor* t) { return t ? t->type : -1; }

int g4_matmul(g4_ctx* c, const g4_tensor* w, int64_t off, const float* x, float* y, int dim0, int dim1,
              void* stream) {
  if (!c) return G4_E_ARG;
  if (!w || !x || !y || dim0 < 0 || dim1 < 0 || off < 0) {
    c->set_err("g4_matmul: bad argument");
    return G4_E_ARG;
  }
  if ((uint64_t)off + (uint64_t)dim0 * (uint64_t)dim1 > w->n_elems) {
    c->set_err("g4_matmul: rows %d x cols %d at offset %lld exceed the tensor's %llu elements", dim0, dim1,
               (long long)off, (unsigned long long)w->n_elems);
    return G4_E_ARG;
  }
  if (dim0 == 0) return 0;
  if (int r = c->bind()) return r;
  cudaStream_t st = (cudaStream_t)stream;
  if (dim1 == 0) {
    cudaError_t e = cudaMemsetAsync(y, 0, sizeof(float) * dim0, st);
    return e == cudaSuccess ? 0 : c->cuda_fail(e, "g4_matmul");
  }
  const int xal = ((uintptr_t)x & 15u) == 0;
  auto key = std::make_tuple(w->type, (long long)off, dim0, dim1, xal);
  auto itp = c->gemv_plans.find(key);
  if (itp == c->gemv_plans.end()) {
    GemvPlan p = plan_gemv(c->dev, w->type, off, dim0, dim1);
    if (!xal) p.fast = 0;
    itp = c->gemv_plans.emplace(key, p).first;
  }
  if (int e = launch_gemv(itp->second, (const uint8_t*)w->d, x, y, c->status, st)) {
    const GemvPlan& p = itp->second;
    c->set_err("g4_matmul launch (type %d, %dx%d, warps %d, smem %zu, grid %d): %s", p.type, dim0, dim1, p.warps,
               p.smem, p.grid, cudaGetErrorString((cudaError_t)e));
    return G4_E_CUDA;
  }
  return 0;
}

int g4_matmul_host(g4_ctx* c, const g4_tensor* w, int64_t off, const float* xh, float* yh, int dim0, int dim1) {
  if (!c) return G4_E_ARG;
  if (!xh || !yh) {
    c->set_err("g4_matmul_host: NULL buffer");
    return G4_E_ARG;
  }
  if (int r = c->bind()) return r;
  size_t xb = ((size_t)dim1 * 4 + 255) / 256 * 256, yb = (size_t)dim0 * 4;
  uint8_t* buf = (uint8_t*)c->io(xb + yb + 256);
  if (!buf) {
    c->set_err("g4_matmul_host: scratch allocation failed");
    return G4_E_NOMEM;
  }
  cudaStream_t st = 0;
  cudaError_t e = cudaMemcpyAsync(buf, xh, (size_t)dim1 * 4, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return c->cuda_fail(e, "g4_matmul_host: H2D");
  int r = g4_matmul(c, w, off, (const float*)buf, (float*)(buf + xb), dim0, dim1, st);
  if (r) return r;
  e = cudaMemcpyAsync(yh, buf + xb, yb, cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) return c->cuda_fail(e, "g4_matmul_host: D2H");
  return c->check_status(st);
}

int g4_dequant(g4_ctx* c, const g4_tensor* w, int64_t off, int64_t n, float* out, void* stream) {
  if (!c) return G4_E_ARG;
  if (!w || !out || off < 0 || n < 0 || (uint64_t)(off + n) > w->n_elems) {
    c->set_err("g4_dequant: bad argument");
    return G4_E_ARG;
  }
  if (int r = c->bind()) return r;
  if (launch_dequant(w->type, (const uint8_t*)w->d, off, n, out, (cudaStream_t)stream))
    return c->cuda_fail(cudaGetLastError(), "g4_dequant launch");
  return 0;
}

int g4_sync(g4_ctx* c, void* stream) {
  if (!c) return G4_E_ARG;
  if (int r = c->bind()) return r;
  return c->check_status((cudaStream_t)stream);
}

// ---------------------------------------------------------------- NCCL plumbing
// NCCL is resolved at run time (dlopen of libnccl.so.2) so that the library
// shares whichever NCCL the host process already loaded.
struct NcclApi {
  bool loaded = false;
  ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*commInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*commGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*commAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*allGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*groupStart)() = nullptr;
  ncclResult_t (*groupEnd)() = nullptr;
  const char* (*errStr)(ncclResult_t) = nullptr;
};

static NcclApi g_nccl;

static bool load_nccl(char* err, size_t n) {
  if (g_nccl.loaded) return true;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!h) {
    snprintf(err, n, "cannot load NCCL: %s", dlerror());
    return false;
  }
#define G4_SYM(f, name)                                       \
  *(void**)(&g_nccl.f) = dlsym(h, name);                      \
  if (!g_nccl.f) {                                            \
    snprintf(err, n, "NCCL symbol %s missing", name);         \
    return false;                                             \
  }
  G4_SYM(getUniqueId, "ncclGetUniqueId")
  G4_SYM(commInitRankConfig, "ncclCommInitRankConfig")
  G4_SYM(commGetAsyncError, "ncclCommGetAsyncError")
  G4_SYM(commAbort, "ncclCommAbort")
  G4_SYM(commDestroy, "ncclCommDestroy")
  G4_SYM(allGather, "ncclAllGather")
  G4_SYM(send, "ncclSend")
  G4_SYM(recv, "ncclRecv")
  G4_SYM(groupStart, "ncclGroupStart")
  G4_SYM(groupEnd, "ncclGroupEnd")
  G4_SYM(errStr, "ncclGetErrorString")
#undef G4_SYM
  g_nccl.loaded = true;
  return true;
}

int g4_dist_unique_id(void* id_out) {
  if (!id_out) return G4_E_ARG;
  if (!load_nccl(g_init_err, sizeof g_init_err)) return G4_E_DIST;
  ncclUniqueId id;
  ncclResult_t r = g_nccl.getUniqueId(&id);
  if (r != ncclSuccess) {
    snprintf(g_init_err, sizeof g_init_err, "ncclGetUniqueId: %s", g_nccl.errStr(r));
    return G4_E_DIST;
  }
  static_assert(sizeof(ncclUniqueId) == G4_NCCL_ID_BYTES, "nccl id size");
  memcpy(id_out, &id, sizeof id);
  return 0;
}

static long long now_ms() {
  struct timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (long long)ts.tv_sec * 1000 + ts.tv_nsec / 1000000;
}

// Default bound on g4_dist_init: G4_DIST_TIMEOUT_MS, else 120 s.
static int default_dist_timeout_ms() {
  const char* v = getenv("G4_DIST_TIMEOUT_MS");
  const int t = v && *v ? atoi(v) : 0;
  return t > 0 ? t : 120000;
}

// The communicator is non-blocking: a call may return ncclInProgress while
// NCCL finishes it in the background.  Poll its state until it settles or the
// deadline passes; on expiry (or any error) abort the communicator so no rank
// is left waiting on it, and report G4_E_DIST.
// Pause between polls of an operation in progress: the first polls only yield
// the CPU (a collective that is being enqueued finishes within microseconds;
// a sleep would add its whole length to every call), later ones sleep.
static void poll_pause(int& it) {
  if (++it < 4000) sched_yield();
  else usleep(it < 8000 ? 20 : 200);
}

static int nccl_settle(g4_ctx* c, ncclComm_t comm, ncclResult_t r, long long deadline_ms, const char* what) {
  int it = 0;
  while (r == ncclInProgress) {
    if (now_ms() > deadline_ms) {
      g_nccl.commAbort(comm);
      if (c->comm == (void*)comm) {
        c->comm = nullptr;
        c->rank = 0;
        c->world = 1;
      }
      c->set_err("%s: timed out (a peer rank did not answer); communicator aborted", what);
      return G4_E_DIST;
    }
    poll_pause(it);
    if (g_nccl.commGetAsyncError(comm, &r) != ncclSuccess) r = ncclSystemError;
  }
  if (r != ncclSuccess) {
    g_nccl.commAbort(comm);
    if (c->comm == (void*)comm) {
      c->comm = nullptr;
      c->rank = 0;
      c->world = 1;
    }
    c->set_err("%s: %s; communicator aborted", what, g_nccl.errStr(r));
    return G4_E_DIST;
  }
  return 0;
}

int g4_dist_init_timeout(g4_ctx* c, int rank, int world, const void* id, int timeout_ms) {
  if (!c) return G4_E_ARG;
  if (!id || world < 1 || rank < 0 || rank >= world || timeout_ms <= 0) {
    c->set_err("g4_dist_init: bad rank %d / world %d / timeout %d ms", rank, world, timeout_ms);
    return G4_E_ARG;
  }
  if (!load_nccl(c->err, sizeof c->err)) return G4_E_DIST;
  if (int r = c->bind()) return r;
  g4_dist_teardown(c);
  c->dist_timeout_ms = timeout_ms;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof uid);
  ncclComm_t comm = nullptr;
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  const long long deadline = now_ms() + timeout_ms;
  ncclResult_t r = g_nccl.commInitRankConfig(&comm, world, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    if (comm) g_nccl.commAbort(comm);
    c->set_err("ncclCommInitRankConfig: %s", g_nccl.errStr(r));
    return G4_E_DIST;
  }
  if (int e = nccl_settle(c, comm, r, deadline, "ncclCommInitRankConfig")) return e;
  c->comm = comm;
  c->rank = rank;
  c->world = world;
  return 0;
}

int g4_dist_init(g4_ctx* c, int rank, int world, const void* id) {
  return g4_dist_init_timeout(c, rank, world, id, default_dist_timeout_ms());
}

int g4_dist_abort(g4_ctx* c) {
  if (!c) return G4_E_ARG;
  if (c->comm && g_nccl.loaded) g_nccl.commAbort((ncclComm_t)c->comm);
  c->comm = nullptr;
  c->rank = 0;
  c->world = 1;
  return 0;
}

int g4_dist_rank(const g4_ctx* c) { return c ? c->rank : -1; }
int g4_dist_world(const g4_ctx* c) { return c ? c->world : -1; }

int g4_matmul_sharded(g4_ctx* c, const g4_tensor* w, const float* x, float* y, int rows, int cols, void* stream) {
  if (!c) return G4_E_ARG;
  if (!c->comm && c->world > 1) {
    c->set_err("g4_matmul_sharded: g4_dist_init not called");
    return G4_E_DIST;
  }
  int world = c->world, rank = c->rank;
  if (rows % world != 0) {
    c->set_err("g4_matmul_sharded: rows %d not divisible by world %d", rows, world);
    return G4_E_ARG;
  }
  int local = rows / world;
  float* my = y + (size_t)rank * local;
  int r = g4_matmul(c, w, 0, x, my, local, cols, stream);
  if (r || world == 1) return r;
  ncclResult_t nr = g_nccl.allGather(my, y, (size_t)local, ncclFloat32, (ncclComm_t)c->comm, (cudaStream_t)stream);
  return nccl_settle(c, (ncclComm_t)c->comm, nr, now_ms() + c->dist_timeout_ms, "ncclAllGather");
}

}  // extern "C"

void g4_dist_teardown(g4_ctx* c) {
  if (c->comm && g_nccl.loaded) g_nccl.commDestroy((ncclComm_t)c->comm);
  c->comm = nullptr;
  c->rank = 0;
  c->world = 1;
}

bool g4_nccl_send_recv_available() { return g_nccl.loaded; }

int g4_nccl_allgather_i32(g4_ctx* c, const int32_t* send, int32_t* recv, size_t count, cudaStream_t st) {
  if (!c->comm) {
    c->set_err("expert-parallel layer: g4_dist_init not called");
    return G4_E_DIST;
  }
  const ncclResult_t r = g_nccl.allGather(send, recv, count, ncclInt32, (ncclComm_t)c->comm, st);
  return nccl_settle(c, (ncclComm_t)c->comm, r, now_ms() + c->dist_timeout_ms, "ncclAllGather");
}

int g4_nccl_alltoallv(g4_ctx* c, const void* send, const size_t* soff, const size_t* slen, void* recv,
                      const size_t* roff, const size_t* rlen, cudaStream_t st) {
  if (!c->comm) {
    c->set_err("expert-parallel layer: g4_dist_init not called");
    return G4_E_DIST;
  }
  ncclComm_t comm = (ncclComm_t)c->comm;
  ncclResult_t r = g_nccl.groupStart();
  for (int p = 0; r == ncclSuccess && p < c->world; ++p) {
    if (slen[p]) r = g_nccl.send((const uint8_t*)send + soff[p], slen[p], ncclUint8, p, comm, st);
    if (r == ncclSuccess && rlen[p]) r = g_nccl.recv((uint8_t*)recv + roff[p], rlen[p], ncclUint8, p, comm, st);
  }
  const ncclResult_t r2 = g_nccl.groupEnd();
  if (r != ncclSuccess && r != ncclInProgress) {
    c->set_err("NCCL send/recv group: %s", g_nccl.errStr(r));
    return G4_E_DIST;
  }
  return nccl_settle(c, comm, r2, now_ms() + c->dist_timeout_ms, "NCCL send/recv group");
}

// Wait for the work queued on `st` (collectives included) with the context's
// distributed timeout: polls the stream and the communicator's asynchronous
// error instead of blocking in cudaStreamSynchronize, so a peer that stopped
// answering ends in G4_E_DIST (communicator aborted) rather than a hung host.
int g4_dist_stream_wait(g4_ctx* c, cudaStream_t st) {
  const long long deadline = now_ms() + c->dist_timeout_ms;
  int it = 0;
  for (;;) {
    const cudaError_t q = cudaStreamQuery(st);
    if (q == cudaSuccess) return 0;
    if (q != cudaErrorNotReady) return c->cuda_fail(q, "stream wait");
    if (c->comm) {
      ncclResult_t ar = ncclSuccess;
      if (g_nccl.commGetAsyncError((ncclComm_t)c->comm, &ar) != ncclSuccess) ar = ncclSystemError;
      if (ar != ncclSuccess && ar != ncclInProgress)
        return nccl_settle(c, (ncclComm_t)c->comm, ar, deadline, "collective");
    }
    if (now_ms() > deadline) {
      if (c->comm) g_nccl.commAbort((ncclComm_t)c->comm);
      c->comm = nullptr;
      c->rank = 0;
      c->world = 1;
      c->set_err("collective did not complete within %d ms (a peer rank stopped answering); communicator aborted",
                 c->dist_timeout_ms);
      return G4_E_DIST;
    }
    poll_pause(it);
  }
}
