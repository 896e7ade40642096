// Peer-to-peer all-reduce of the tensor-parallel decode, fused into the
// kernels around it.
//
// The row-parallel projections of a KV-head-sharded model (o_proj,
// down_proj) end with partial sums that every rank needs in full; the
// reference has no multi-GPU path (its decode is batch-1 on one device,
// smollm2_triton/model.py:351-365). Here the projection's epilogue
// (tllm_linear op EPI_SCATTER) stores its partial rows straight into a
// receive slot on every rank of the group over NVLink (plain stores
// through CUDA IPC mappings), and the RMSNorm that follows
// (tllm_rmsnorm_p2p) waits for every rank's rows, sums the slots in rank
// order -- identical on every rank -- adds the sum to the residual stream
// and normalises.
//
// Every value travels as one 64-bit word: fp32 bits | call number << 32.
// A single aligned 64-bit store is seen whole or not at all, so the reader
// knows a value has arrived when its word carries the current call number:
// the writer needs no fence, no flag and no grid-wide ticket.
//
// Buffers (one cudaMalloc per rank, exported with cudaIpcGetMemHandle):
//   recv  [2][size][mmax][ncols] words   slot (parity, source rank, row)
// and a local state {calls done, reader ticket}. Call c (1, 2, ...) writes
// parity c & 1. A rank writes call c + 2 into a peer only after its own
// reader of call c + 1 has seen that peer's rows of call c + 1, which the
// peer wrote after its reader of call c had finished, so a slot is never
// overwritten while it is read. Every wait is bounded and reports through
// the device error word.
#include <cstring>

#include "common.cuh"
#include "p2p.cuh"

namespace tllm {

struct P2PHost {
  P2PDev *dev;          // device copy of the table below
  P2PDev table;
  void *base;           // this rank's exported allocation
  void *peer_base[kP2PMaxRanks];
  cudaIpcMemHandle_t handle;
  bool opened;
};

size_t p2p_recv_bytes(int size, int mmax, int ncols) {
  return (size_t)2 * size * mmax * ncols * sizeof(unsigned long long);
}

const P2PDev *p2p_table(const void *ctx, int rows, int cols) {
  if (!ctx) {
    set_error("NULL peer group");
    return nullptr;
  }
  const P2PHost *h = static_cast<const P2PHost *>(ctx);
  if (!h->opened) {
    set_error("peer group not opened (tllm_p2p_open)");
    return nullptr;
  }
  if (rows > h->table.mmax || cols > h->table.ncols || cols % 4 != 0) {
    set_error("%d x %d rows do not fit the peer slots (%d x %d, cols %% 4 == 0)",
              rows, cols, h->table.mmax, h->table.ncols);
    return nullptr;
  }
  return h->dev;
}

}  // namespace tllm

using namespace tllm;

namespace {

constexpr uint64_t kP2PWaitNs = 2000000000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

constexpr int kP2PVecPer = 4;   // float4s per thread (as the vector RMSNorm)

// The four words of columns 4i .. 4i + 3 from rank q's slot once all of
// them carry call number e (bounded wait).
__device__ __forceinline__ float4 p2p_take4(const unsigned long long *src,
                                            unsigned e, bool &ok, uint64_t t0,
                                            int *err) {
  unsigned long long a0, a1, a2, a3;
  for (uint32_t it = 0;; ++it) {
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];"
                 : "=l"(a0), "=l"(a1) : "l"(src) : "memory");
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];"
                 : "=l"(a2), "=l"(a3) : "l"(src + 2) : "memory");
    const bool here = (unsigned)(a0 >> 32) == e && (unsigned)(a1 >> 32) == e &&
                      (unsigned)(a2 >> 32) == e && (unsigned)(a3 >> 32) == e;
    if (here || !ok) break;
    // bounded: ~2 s, or 2^26 polls if the timer does not advance
    if (((it & 255) == 255 && globaltimer_ns() - t0 > kP2PWaitNs) || it == (1u << 26)) {
      ok = false;
      atomicOr(err, DEV_ERR_WAIT_TIMEOUT);
    }
  }
  return make_float4(__uint_as_float((unsigned)a0), __uint_as_float((unsigned)a1),
                     __uint_as_float((unsigned)a2), __uint_as_float((unsigned)a3));
}

// One row per block, the float4 layout and reduction order of the vector
// RMSNorm in ops.cu (blockDim.x threads, kP2PVecPer float4s each), so the
// peer path and a one-rank group give the same bits as tllm_rmsnorm_add.
__global__ void rmsnorm_p2p_kernel(float *h, const P2PDev *P, const float *w,
                                   uint16_t *ys, float *yf, size_t yplane,
                                   int planes, int N, float eps, int *err) {
  griddep_launch();
  // the projection that scatters has finished on this rank, and with it
  // this rank's reader of the previous call: state[0] is final
  griddep_wait();
  __shared__ float red[32];
  __shared__ int s_broken;
  const int m = blockIdx.x;
  const unsigned e = (unsigned)P->state[0] + 1u;
  const int par = e & 1;
  if (threadIdx.x == 0)   // after one wait has run out, stop waiting
    s_broken = *reinterpret_cast<volatile int *>(err) & DEV_ERR_WAIT_TIMEOUT;
  __syncthreads();
  bool ok = !s_broken;
  const uint64_t t0 = globaltimer_ns();
  const int n4 = N >> 2;
  float4 *h4 = reinterpret_cast<float4 *>(h + (size_t)m * N);
  float4 v[kP2PVecPer];
#pragma unroll
  for (int k = 0; k < kP2PVecPer; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < n4) {
      float4 t = h4[i];
      for (int q = 0; q < P->size; ++q) {   // rank order: identical on every rank
        const unsigned long long *src =
            P->recv_local + (((size_t)par * P->size + q) * P->mmax + m) * P->ncols + 4 * i;
        const float4 a = p2p_take4(src, e, ok, t0, err);
        t.x += a.x;
        t.y += a.y;
        t.z += a.z;
        t.w += a.w;
      }
      h4[i] = t;
      v[k] = t;
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kP2PVecPer; ++k) {
    ss = fmaf(v[k].x, v[k].x, ss);
    ss = fmaf(v[k].y, v[k].y, ss);
    ss = fmaf(v[k].z, v[k].z, ss);
    ss = fmaf(v[k].w, v[k].w, ss);
  }
  // block sum of squares (xor butterflies: every lane holds the same sum)
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  {
    const int nw = (blockDim.x + 31) >> 5;
    float t = (threadIdx.x & 31) < nw ? red[threadIdx.x & 31] : 0.f;
    for (int off = 16; off > 0; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
    ss = t;
  }
  const float rms = sqrtf(ss / (float)N + eps);
  const size_t o = (size_t)m * N;
  const float4 *w4 = reinterpret_cast<const float4 *>(w);
#pragma unroll
  for (int k = 0; k < kP2PVecPer; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i >= n4) continue;
    const float4 g = w4[i];
    const float y[4] = {(v[k].x / rms) * g.x, (v[k].y / rms) * g.y, (v[k].z / rms) * g.z,
                        (v[k].w / rms) * g.w};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if (ys)
        store_act(ys, yplane, o + 4 * (size_t)i + c, y[c], planes);
      else
        yf[o + 4 * (size_t)i + c] = y[c];
    }
  }
  // the last block to finish records the call as done (read by the next
  // scatter and reader, which run after this kernel)
  if (threadIdx.x == 0) {
    if (atomicAdd(&P->state[1], 1) == (int)gridDim.x - 1) {
      P->state[1] = 0;
      P->state[0] = (int)e;
    }
  }
}

}  // namespace

extern "C" {

int tllm_p2p_create(int size, int mmax, int ncols, void **ctx,
                    void *ipc_handle) {
  TLLM_CHECK_ARG(ctx && ipc_handle, "NULL output");
  TLLM_CHECK_ARG(size >= 1 && size <= kP2PMaxRanks, "group size %d not in [1, %d]",
                 size, kP2PMaxRanks);
  TLLM_CHECK_ARG(mmax > 0 && ncols > 0 && ncols % 4 == 0, "bad slot shape");
  P2PHost *h = new P2PHost();
  memset(h, 0, sizeof(*h));
  const size_t bytes = p2p_recv_bytes(size, mmax, ncols);
  void *base = nullptr;
  cudaError_t e = cudaMalloc(&base, bytes);
  if (e != cudaSuccess) {
    delete h;
    set_error("cudaMalloc of the peer buffers failed: %s", cudaGetErrorString(e));
    return TLLM_ERR_CUDA;
  }
  cudaMemset(base, 0, bytes);
  int *state = nullptr;
  cudaMalloc(&state, 2 * sizeof(int));
  cudaMemset(state, 0, 2 * sizeof(int));
  P2PDev *dev = nullptr;
  cudaMalloc(&dev, sizeof(P2PDev));
  e = cudaIpcGetMemHandle(&h->handle, base);
  cudaDeviceSynchronize();
  if (e != cudaSuccess || !state || !dev) {
    set_error("peer buffer setup failed: %s", cudaGetErrorString(e));
    cudaFree(base);
    delete h;
    return TLLM_ERR_CUDA;
  }
  h->base = base;
  h->dev = dev;
  h->table.size = size;
  h->table.mmax = mmax;
  h->table.ncols = ncols;
  h->table.recv_local = static_cast<unsigned long long *>(base);
  h->table.state = state;
  memcpy(ipc_handle, &h->handle, sizeof(cudaIpcMemHandle_t));
  *ctx = h;
  return TLLM_OK;
}

int tllm_p2p_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

// handles: size consecutive IPC handles (tllm_p2p_handle_bytes each), in
// rank order; this rank's own entry is ignored.
int tllm_p2p_open(void *ctx, int rank, const void *handles) {
  TLLM_CHECK_ARG(ctx && handles, "NULL argument");
  P2PHost *h = static_cast<P2PHost *>(ctx);
  P2PDev &t = h->table;
  TLLM_CHECK_ARG(rank >= 0 && rank < t.size, "rank %d not in [0, %d)", rank, t.size);
  t.rank = rank;
  for (int q = 0; q < t.size; ++q) {
    void *p = nullptr;
    if (q == rank) {
      p = h->base;
    } else {
      cudaIpcMemHandle_t hq;
      memcpy(&hq, static_cast<const char *>(handles) + q * sizeof(cudaIpcMemHandle_t),
             sizeof(hq));
      cudaError_t e = cudaIpcOpenMemHandle(&p, hq, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) {
        set_error("cudaIpcOpenMemHandle(rank %d) failed: %s", q, cudaGetErrorString(e));
        return TLLM_ERR_CUDA;
      }
      h->peer_base[q] = p;
    }
    t.peer_recv[q] = static_cast<unsigned long long *>(p);
  }
  TLLM_CUDA(cudaMemcpy(h->dev, &t, sizeof(P2PDev), cudaMemcpyHostToDevice));
  h->opened = true;
  return TLLM_OK;
}

int tllm_p2p_destroy(void *ctx) {
  if (!ctx) return TLLM_OK;
  P2PHost *h = static_cast<P2PHost *>(ctx);
  cudaDeviceSynchronize();
  for (int q = 0; q < kP2PMaxRanks; ++q)
    if (h->peer_base[q]) cudaIpcCloseMemHandle(h->peer_base[q]);
  cudaFree(h->table.state);
  cudaFree(h->dev);
  cudaFree(h->base);
  delete h;
  return TLLM_OK;
}

int tllm_rmsnorm_p2p(float *h, const void *p2p, const float *w, void *y,
                     int y_dtype, int y_plane_rows, int M, int N, float eps,
                     tllm_stream_t stream) {
  TLLM_INJECT("launch");
  TLLM_CHECK_ARG(M >= 0 && N > 0, "invalid shape");
  if (M == 0) return TLLM_OK;
  TLLM_CHECK_ARG(h && w && y, "NULL pointer");
  const P2PDev *P = p2p_table(p2p, M, N);
  if (!P) return TLLM_ERR_INVALID_ARG;
  TLLM_CHECK_ARG(y_dtype == TLLM_F32 || y_dtype == TLLM_SPLIT || y_dtype == TLLM_BF16,
                 "y_dtype must be F32, SPLIT or BF16");
  int *err = device_error_ptr();
  TLLM_CHECK_ARG(err, "device error word unavailable");
  const bool act = y_dtype != TLLM_F32;
  TLLM_CHECK_ARG(!act || y_plane_rows >= M, "y_plane_rows < M");
  // resident before the projection that scatters has finished
  // (programmatic serialization); the kernel waits for it first
  TLLM_CHECK_ARG(N % 4 == 0 && N <= 4 * kP2PVecPer * 1024, "N must be a multiple of 4, <= %d",
                 4 * kP2PVecPer * 1024);
  TLLM_CHECK_ARG((reinterpret_cast<uintptr_t>(h) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(w) & 15) == 0,
                 "h and w must be 16-byte aligned");
  int threads = ((N / 4 + kP2PVecPer - 1) / kP2PVecPer + 31) & ~31;
  if (threads < 32) threads = 32;
  TLLM_CUDA(launch_pdl(rmsnorm_p2p_kernel, dim3(M), dim3(threads), 0, resolve(stream), h, P,
                       w, act ? static_cast<uint16_t *>(y) : nullptr,
                       act ? nullptr : static_cast<float *>(y),
                       act ? (size_t)y_plane_rows * N : 0, y_dtype == TLLM_SPLIT ? 2 : 1,
                       N, eps, err));
  return TLLM_OK;
}

}  // extern "C"
