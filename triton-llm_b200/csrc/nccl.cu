// NCCL all-reduce for the tensor-parallel decode, bound inside libtllm.so.
//
// The row-parallel projections of a KV-head-sharded model (o_proj, down_proj)
// leave partial sums that every rank needs in full; the sum runs over NVLink
// with NCCL, ordered on the library stream like the kernels around it, so it
// can sit inside the decode step's CUDA graph. NCCL is loaded with dlopen
// (libnccl.so.2, or the path in TLLM_NCCL_LIB) the first time one of these
// functions is called, so the library itself loads without it.
//
// Communicators are created non-blocking: every call that can wait for a
// peer (init, an enqueue that reports ncclInProgress, finalize) is polled
// with ncclCommGetAsyncError under a host-side time limit; when the limit
// runs out the communicator is aborted and TLLM_ERR_TIMEOUT returned, so a
// rank that never joins or has died ends the wait with an error instead of a
// hang. The unique id and the ranks' meeting point are the caller's (the
// Python side exchanges the id over its own TCP rendezvous).
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <mutex>
#include <thread>

#include "common.cuh"

namespace tllm {
namespace {

struct NcclApi {
  void *handle = nullptr;
  bool tried = false;
  char why[512] = {0};
  decltype(&ncclGetVersion) getVersion = nullptr;
  decltype(&ncclGetUniqueId) getUniqueId = nullptr;
  decltype(&ncclCommInitRankConfig) initRankConfig = nullptr;
  decltype(&ncclCommGetAsyncError) asyncError = nullptr;
  decltype(&ncclAllReduce) allReduce = nullptr;
  decltype(&ncclCommFinalize) finalize = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclCommAbort) abort = nullptr;
  decltype(&ncclGetErrorString) errorString = nullptr;
  decltype(&ncclGetLastError) lastError = nullptr;
};

NcclApi g_nccl;
std::mutex g_nccl_mu;

template <typename F>
bool bind(F &fn, const char *name) {
  fn = reinterpret_cast<F>(dlsym(g_nccl.handle, name));
  if (!fn) snprintf(g_nccl.why, sizeof(g_nccl.why), "symbol %s missing", name);
  return fn != nullptr;
}

int load_nccl() {
  std::lock_guard<std::mutex> lk(g_nccl_mu);
  if (!g_nccl.tried) {
    g_nccl.tried = true;
    const char *path = getenv("TLLM_NCCL_LIB");
    if (!path || !*path) path = "libnccl.so.2";
    g_nccl.handle = dlopen(path, RTLD_NOW | RTLD_LOCAL);
    if (!g_nccl.handle) {
      snprintf(g_nccl.why, sizeof(g_nccl.why), "dlopen(%s): %s", path, dlerror());
    } else if (!(bind(g_nccl.getVersion, "ncclGetVersion") &&
                 bind(g_nccl.getUniqueId, "ncclGetUniqueId") &&
                 bind(g_nccl.initRankConfig, "ncclCommInitRankConfig") &&
                 bind(g_nccl.asyncError, "ncclCommGetAsyncError") &&
                 bind(g_nccl.allReduce, "ncclAllReduce") &&
                 bind(g_nccl.finalize, "ncclCommFinalize") &&
                 bind(g_nccl.destroy, "ncclCommDestroy") &&
                 bind(g_nccl.abort, "ncclCommAbort") &&
                 bind(g_nccl.errorString, "ncclGetErrorString") &&
                 bind(g_nccl.lastError, "ncclGetLastError"))) {
      dlclose(g_nccl.handle);
      g_nccl.handle = nullptr;
    }
  }
  if (!g_nccl.handle) {
    set_error("NCCL library unavailable: %s", g_nccl.why);
    return TLLM_ERR_NCCL;
  }
  return TLLM_OK;
}

struct Comm {
  ncclComm_t comm = nullptr;
  int rank = 0, size = 0, device = 0;
  bool broken = false;   // aborted after a timeout or an error
};

int nccl_fail(Comm *c, ncclResult_t r, const char *what) {
  const char *last = (c && c->comm) ? g_nccl.lastError(c->comm) : nullptr;
  set_error("%s failed: %s%s%s", what, g_nccl.errorString(r),
            last && *last ? ": " : "", last ? last : "");
  return TLLM_ERR_NCCL;
}

// Polls the communicator's asynchronous state until it leaves
// ncclInProgress, for at most timeout_ms (<= 0: 120 s). On a timeout or an
// error the communicator is aborted (peers waiting on it fail too).
int wait_ready(Comm *c, int timeout_ms, const char *what) {
  if (timeout_ms <= 0) timeout_ms = 120000;
  const auto t0 = std::chrono::steady_clock::now();
  ncclResult_t st = ncclInProgress;
  for (int i = 0;; ++i) {
    ncclResult_t r = g_nccl.asyncError(c->comm, &st);
    if (r != ncclSuccess) st = r;
    if (st != ncclInProgress) break;
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                        std::chrono::steady_clock::now() - t0).count();
    if (ms > timeout_ms) {
      g_nccl.abort(c->comm);
      c->comm = nullptr;
      c->broken = true;
      set_error("%s: no completion after %d ms (a peer rank did not take part); "
                "communicator aborted", what, timeout_ms);
      return TLLM_ERR_TIMEOUT;
    }
    if (i > 64) std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
  if (st != ncclSuccess) {
    int rc = nccl_fail(c, st, what);
    g_nccl.abort(c->comm);
    c->comm = nullptr;
    c->broken = true;
    return rc;
  }
  return TLLM_OK;
}

Comm *as_comm(void *p) { return static_cast<Comm *>(p); }

}  // namespace
}  // namespace tllm

using namespace tllm;

extern "C" {

int tllm_nccl_version(int *version) {
  TLLM_CHECK_ARG(version, "version is NULL");
  int rc = load_nccl();
  if (rc) return rc;
  ncclResult_t r = g_nccl.getVersion(version);
  if (r != ncclSuccess) return nccl_fail(nullptr, r, "ncclGetVersion");
  return TLLM_OK;
}

int tllm_nccl_unique_id_bytes(void) { return (int)sizeof(ncclUniqueId); }

int tllm_nccl_unique_id(void *id) {
  TLLM_CHECK_ARG(id, "id is NULL");
  TLLM_INJECT("nccl");
  int rc = load_nccl();
  if (rc) return rc;
  ncclUniqueId u;
  ncclResult_t r = g_nccl.getUniqueId(&u);
  if (r != ncclSuccess) return nccl_fail(nullptr, r, "ncclGetUniqueId");
  memcpy(id, &u, sizeof(u));
  return TLLM_OK;
}

int tllm_nccl_init(void **comm, int size, int rank, const void *id,
                   int timeout_ms) {
  TLLM_CHECK_ARG(comm && id, "NULL argument");
  TLLM_CHECK_ARG(size >= 1 && rank >= 0 && rank < size,
                 "rank %d of %d is invalid", rank, size);
  *comm = nullptr;
  TLLM_INJECT("nccl");
  int rc = load_nccl();
  if (rc) return rc;
  Comm *c = new Comm();
  c->rank = rank;
  c->size = size;
  cudaError_t ce = cudaGetDevice(&c->device);
  if (ce != cudaSuccess) {
    delete c;
    set_error("cudaGetDevice failed: %s (%d)", cudaGetErrorString(ce), (int)ce);
    return TLLM_ERR_CUDA;
  }
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = g_nccl.initRankConfig(&c->comm, size, u, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    rc = nccl_fail(c, r, "ncclCommInitRankConfig");
    if (c->comm) g_nccl.abort(c->comm);
    delete c;
    return rc;
  }
  rc = wait_ready(c, timeout_ms, "ncclCommInitRankConfig");
  if (rc) {
    delete c;
    return rc;
  }
  *comm = c;
  return TLLM_OK;
}

int tllm_nccl_all_reduce(void *comm, void *buf, size_t count, int dtype,
                         tllm_stream_t stream, int timeout_ms) {
  Comm *c = as_comm(comm);
  TLLM_CHECK_ARG(c, "comm is NULL");
  TLLM_CHECK_ARG(!c->broken && c->comm, "communicator was aborted");
  TLLM_CHECK_ARG(dtype == TLLM_F32 || dtype == TLLM_BF16, "dtype F32 or BF16");
  if (count == 0) return TLLM_OK;
  TLLM_CHECK_ARG(buf, "buf is NULL");
  TLLM_INJECT("nccl");
  ncclResult_t r = g_nccl.allReduce(buf, buf, count,
                                    dtype == TLLM_F32 ? ncclFloat32 : ncclBfloat16,
                                    ncclSum, c->comm, resolve(stream));
  if (r == ncclInProgress) return wait_ready(c, timeout_ms, "ncclAllReduce");
  if (r != ncclSuccess) return nccl_fail(c, r, "ncclAllReduce");
  return TLLM_OK;
}

int tllm_nccl_check(void *comm, int *state) {
  Comm *c = as_comm(comm);
  TLLM_CHECK_ARG(c && state, "NULL argument");
  if (c->broken || !c->comm) {
    *state = (int)ncclInternalError;
    return TLLM_OK;
  }
  ncclResult_t st = ncclSuccess;
  ncclResult_t r = g_nccl.asyncError(c->comm, &st);
  *state = (int)(r != ncclSuccess ? r : st);
  return TLLM_OK;
}

int tllm_nccl_destroy(void *comm, int timeout_ms) {
  Comm *c = as_comm(comm);
  if (!c) return TLLM_OK;
  int rc = TLLM_OK;
  if (c->comm && !c->broken) {
    ncclResult_t r = g_nccl.finalize(c->comm);
    if (r == ncclSuccess || r == ncclInProgress) {
      rc = wait_ready(c, timeout_ms, "ncclCommFinalize");
    } else {
      rc = nccl_fail(c, r, "ncclCommFinalize");
      g_nccl.abort(c->comm);
      c->comm = nullptr;
    }
    if (c->comm) g_nccl.destroy(c->comm);
  }
  delete c;
  return rc;
}

int tllm_nccl_abort(void *comm) {
  Comm *c = as_comm(comm);
  if (!c) return TLLM_OK;
  if (c->comm) g_nccl.abort(c->comm);
  delete c;
  return TLLM_OK;
}

}  // extern "C"
