// Device runtime of libtllm.so: per-device library streams, a stream-ordered
// pool allocator, host<->device copies, events and error reporting.
//
// This is the native counterpart of triton_llm/gpu.py:114-263 in the
// reference, which binds cudaMalloc/cudaFree/cudaMemcpy/cudaDeviceSynchronize
// through ctypes. Here every allocation comes from the device's default
// memory pool on the library stream (cudaMallocAsync), so freeing a tensor in
// a decode loop never synchronises the device, and every copy is ordered on
// the same stream as the kernels.
#include <atomic>
#include <cstdlib>
#include <mutex>

#include "common.cuh"

namespace tllm {

static thread_local std::string g_err;

void set_error(const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
}
void clear_error() { g_err.clear(); }

// ---- fault injection -------------------------------------------------------
static std::atomic<long> g_site_count[3];
static long g_fault_at[3] = {-1, -1, -1};
static std::once_flag g_fault_once;

static void parse_fault_env() {
  const char *e = getenv("TLLM_FAULT_INJECT");
  if (!e) return;
  // comma separated "site:N" entries
  std::string s(e);
  size_t pos = 0;
  while (pos < s.size()) {
    size_t comma = s.find(',', pos);
    std::string item = s.substr(pos, comma == std::string::npos ? std::string::npos
                                                                : comma - pos);
    size_t colon = item.find(':');
    if (colon != std::string::npos) {
      std::string site = item.substr(0, colon);
      long n = atol(item.c_str() + colon + 1);
      if (site == "malloc") g_fault_at[0] = n;
      if (site == "launch") g_fault_at[1] = n;
      if (site == "nccl") g_fault_at[2] = n;
    }
    if (comma == std::string::npos) break;
    pos = comma + 1;
  }
}

bool inject_fault(const char *site) {
  std::call_once(g_fault_once, parse_fault_env);
  int idx = (site[0] == 'm') ? 0 : (site[0] == 'n' ? 2 : 1);
  if (g_fault_at[idx] < 0) return false;
  long n = ++g_site_count[idx];
  return n == g_fault_at[idx];
}

// ---- per-device state --------------------------------------------------------
static const int kMaxDevices = 64;
static cudaStream_t g_streams[kMaxDevices];
static int g_sms[kMaxDevices];
static std::mutex g_mu;

static int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

cudaStream_t lib_stream() {
  int d = current_device();
  if (d < 0 || d >= kMaxDevices) return nullptr;
  if (g_streams[d]) return g_streams[d];
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_streams[d]) {
    cudaStream_t s = nullptr;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) == cudaSuccess) {
      // Keep freed pool memory cached instead of returning it to the driver
      // at every synchronisation point.
      cudaMemPool_t pool;
      if (cudaDeviceGetDefaultMemPool(&pool, d) == cudaSuccess) {
        uint64_t thresh = ~0ull;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thresh);
      }
      g_streams[d] = s;
    }
  }
  return g_streams[d];
}

int sm_count() {
  int d = current_device();
  if (d < 0 || d >= kMaxDevices) return 148;
  if (!g_sms[d]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
    g_sms[d] = n > 0 ? n : 148;
  }
  return g_sms[d];
}

bool pdl_enabled() {
  static const bool on = [] {
    const char *v = getenv("TLLM_NO_PDL");
    return !(v && v[0] && v[0] != '0');
  }();
  return on;
}

static int *g_err_word[kMaxDevices];

int *device_error_ptr() {
  int d = current_device();
  if (d < 0 || d >= kMaxDevices) return nullptr;
  if (g_err_word[d]) return g_err_word[d];
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err_word[d]) {
    int *p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) == cudaSuccess) {
      cudaMemset(p, 0, sizeof(int));
      cudaDeviceSynchronize();
      g_err_word[d] = p;
    }
  }
  return g_err_word[d];
}

}  // namespace tllm

using namespace tllm;

extern "C" {

const char *tllm_last_error_string(void) { return g_err.c_str(); }
int tllm_version(void) { return 100; }

int tllm_device_count(int *count) {
  TLLM_CHECK_ARG(count, "count is NULL");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    cudaGetLastError();
    *count = 0;
    set_error("no CUDA device visible: %s", cudaGetErrorString(e));
    return TLLM_ERR_NO_DEVICE;
  }
  *count = n;
  return TLLM_OK;
}

int tllm_set_device(int device) {
  TLLM_CUDA(cudaSetDevice(device));
  return TLLM_OK;
}

int tllm_get_device(int *device) {
  TLLM_CHECK_ARG(device, "device is NULL");
  TLLM_CUDA(cudaGetDevice(device));
  return TLLM_OK;
}

int tllm_get_stream(tllm_stream_t *stream) {
  TLLM_CHECK_ARG(stream, "stream is NULL");
  cudaStream_t s = lib_stream();
  if (!s) {
    set_error("could not create the library stream");
    return TLLM_ERR_CUDA;
  }
  *stream = s;
  return TLLM_OK;
}

int tllm_malloc(void **ptr, size_t nbytes) {
  TLLM_CHECK_ARG(ptr, "ptr is NULL");
  TLLM_INJECT("malloc");
  *ptr = nullptr;
  if (nbytes == 0) return TLLM_OK;
  TLLM_CUDA(cudaMallocAsync(ptr, nbytes, lib_stream()));
  return TLLM_OK;
}

int tllm_free(void *ptr) {
  if (!ptr) return TLLM_OK;
  TLLM_CUDA(cudaFreeAsync(ptr, lib_stream()));
  return TLLM_OK;
}

int tllm_malloc_static(void **ptr, size_t nbytes) {
  TLLM_CHECK_ARG(ptr, "ptr is NULL");
  TLLM_INJECT("malloc");
  *ptr = nullptr;
  if (nbytes == 0) return TLLM_OK;
  TLLM_CUDA(cudaMalloc(ptr, nbytes));
  return TLLM_OK;
}

int tllm_free_static(void *ptr) {
  if (!ptr) return TLLM_OK;
  TLLM_CUDA(cudaFree(ptr));
  return TLLM_OK;
}

int tllm_host_alloc(void **ptr, size_t nbytes) {
  TLLM_CHECK_ARG(ptr, "ptr is NULL");
  *ptr = nullptr;
  if (nbytes == 0) return TLLM_OK;
  TLLM_CUDA(cudaMallocHost(ptr, nbytes));
  return TLLM_OK;
}

int tllm_host_free(void *ptr) {
  if (!ptr) return TLLM_OK;
  TLLM_CUDA(cudaFreeHost(ptr));
  return TLLM_OK;
}

static int copy_sync(void *dst, const void *src, size_t n, cudaMemcpyKind k) {
  if (n == 0) return TLLM_OK;
  TLLM_CHECK_ARG(dst && src, "NULL pointer in copy of %zu bytes", n);
  cudaStream_t s = lib_stream();
  TLLM_CUDA(cudaMemcpyAsync(dst, src, n, k, s));
  TLLM_CUDA(cudaStreamSynchronize(s));
  return TLLM_OK;
}

int tllm_memcpy_h2d(void *dst, const void *src, size_t nbytes) {
  return copy_sync(dst, src, nbytes, cudaMemcpyHostToDevice);
}
int tllm_memcpy_d2h(void *dst, const void *src, size_t nbytes) {
  return copy_sync(dst, src, nbytes, cudaMemcpyDeviceToHost);
}
int tllm_memcpy_d2d(void *dst, const void *src, size_t nbytes) {
  if (nbytes == 0) return TLLM_OK;
  TLLM_CHECK_ARG(dst && src, "NULL pointer in copy of %zu bytes", nbytes);
  TLLM_CUDA(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyDeviceToDevice,
                            lib_stream()));
  return TLLM_OK;
}
int tllm_memcpy_h2d_async(void *dst, const void *src, size_t nbytes,
                          tllm_stream_t stream) {
  if (nbytes == 0) return TLLM_OK;
  TLLM_CHECK_ARG(dst && src, "NULL pointer in copy of %zu bytes", nbytes);
  TLLM_CUDA(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyHostToDevice,
                            resolve(stream)));
  return TLLM_OK;
}
int tllm_memcpy_d2h_async(void *dst, const void *src, size_t nbytes,
                          tllm_stream_t stream) {
  if (nbytes == 0) return TLLM_OK;
  TLLM_CHECK_ARG(dst && src, "NULL pointer in copy of %zu bytes", nbytes);
  TLLM_CUDA(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyDeviceToHost,
                            resolve(stream)));
  return TLLM_OK;
}
int tllm_memset(void *ptr, int value, size_t nbytes, tllm_stream_t stream) {
  if (nbytes == 0) return TLLM_OK;
  TLLM_CHECK_ARG(ptr, "NULL pointer in memset");
  TLLM_CUDA(cudaMemsetAsync(ptr, value, nbytes, resolve(stream)));
  return TLLM_OK;
}

int tllm_synchronize(void) {
  TLLM_CUDA(cudaStreamSynchronize(lib_stream()));
  return TLLM_OK;
}
int tllm_stream_synchronize(tllm_stream_t stream) {
  TLLM_CUDA(cudaStreamSynchronize(resolve(stream)));
  return TLLM_OK;
}
int tllm_device_synchronize(void) {
  TLLM_CUDA(cudaDeviceSynchronize());
  return TLLM_OK;
}

int tllm_stream_create(tllm_stream_t *stream) {
  TLLM_CHECK_ARG(stream, "stream is NULL");
  cudaStream_t s;
  TLLM_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  *stream = s;
  return TLLM_OK;
}
int tllm_stream_destroy(tllm_stream_t stream) {
  if (!stream) return TLLM_OK;
  TLLM_CUDA(cudaStreamDestroy(static_cast<cudaStream_t>(stream)));
  return TLLM_OK;
}
int tllm_event_create(void **event) {
  TLLM_CHECK_ARG(event, "event is NULL");
  cudaEvent_t e;
  TLLM_CUDA(cudaEventCreate(&e));
  *event = e;
  return TLLM_OK;
}
int tllm_event_destroy(void *event) {
  if (!event) return TLLM_OK;
  TLLM_CUDA(cudaEventDestroy(static_cast<cudaEvent_t>(event)));
  return TLLM_OK;
}
int tllm_event_record(void *event, tllm_stream_t stream) {
  TLLM_CHECK_ARG(event, "event is NULL");
  TLLM_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(event), resolve(stream)));
  return TLLM_OK;
}
int tllm_event_elapsed_ms(void *start, void *end, float *ms) {
  TLLM_CHECK_ARG(start && end && ms, "NULL argument");
  TLLM_CUDA(cudaEventSynchronize(static_cast<cudaEvent_t>(end)));
  TLLM_CUDA(cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start),
                                 static_cast<cudaEvent_t>(end)));
  return TLLM_OK;
}
int tllm_stream_wait_event(tllm_stream_t stream, void *event) {
  TLLM_CHECK_ARG(event, "event is NULL");
  TLLM_CUDA(cudaStreamWaitEvent(resolve(stream),
                                static_cast<cudaEvent_t>(event), 0));
  return TLLM_OK;
}

int tllm_device_error(int *code, int reset) {
  TLLM_CHECK_ARG(code, "code is NULL");
  int *w = device_error_ptr();
  if (!w) {
    set_error("could not allocate the device error word");
    return TLLM_ERR_CUDA;
  }
  cudaStream_t s = lib_stream();
  TLLM_CUDA(cudaStreamSynchronize(s));
  TLLM_CUDA(cudaMemcpy(code, w, sizeof(int), cudaMemcpyDeviceToHost));
  if (reset) TLLM_CUDA(cudaMemset(w, 0, sizeof(int)));
  return TLLM_OK;
}

int tllm_graph_capture_begin(tllm_stream_t stream) {
  // Per-device state that kernels reach lazily (the device error word, the
  // library stream) is created now: allocation is not allowed during capture.
  TLLM_CHECK_ARG(device_error_ptr(), "device error word unavailable");
  TLLM_CUDA(cudaStreamBeginCapture(resolve(stream),
                                   cudaStreamCaptureModeThreadLocal));
  return TLLM_OK;
}

int tllm_graph_capture_end(tllm_stream_t stream, void **graph_exec) {
  TLLM_CHECK_ARG(graph_exec, "graph_exec is NULL");
  cudaGraph_t g = nullptr;
  TLLM_CUDA(cudaStreamEndCapture(resolve(stream), &g));
  cudaGraphExec_t ge = nullptr;
  cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) {
    set_error("cudaGraphInstantiate failed: %s (%d)", cudaGetErrorString(e),
              (int)e);
    return TLLM_ERR_CUDA;
  }
  *graph_exec = ge;
  return TLLM_OK;
}

int tllm_graph_launch(void *graph_exec, tllm_stream_t stream) {
  TLLM_CHECK_ARG(graph_exec, "graph_exec is NULL");
  TLLM_CUDA(cudaGraphLaunch(static_cast<cudaGraphExec_t>(graph_exec),
                            resolve(stream)));
  return TLLM_OK;
}

int tllm_graph_destroy(void *graph_exec) {
  if (!graph_exec) return TLLM_OK;
  TLLM_CUDA(cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(graph_exec)));
  return TLLM_OK;
}

int tllm_mem_info(size_t *free_bytes, size_t *total_bytes) {
  TLLM_CHECK_ARG(free_bytes && total_bytes, "NULL argument");
  TLLM_CUDA(cudaMemGetInfo(free_bytes, total_bytes));
  return TLLM_OK;
}

}  // extern "C"
