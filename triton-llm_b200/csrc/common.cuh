// Internal helpers shared by every translation unit of libtllm.so.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/tllm.h"

namespace tllm {

// Thread-local message of the last failure (read by tllm_last_error_string).
void set_error(const char *fmt, ...);
void clear_error();

// Fault injection for host-side failure tests: TLLM_FAULT_INJECT="malloc:N"
// makes the N-th tllm_malloc of the process fail (N counts from 1);
// "launch:N" makes the N-th kernel entry point fail before it launches;
// "nccl:N" makes the N-th NCCL call (unique id, init, all-reduce) fail.
bool inject_fault(const char *site);

// The library stream of the current device (created lazily).
cudaStream_t lib_stream();
inline cudaStream_t resolve(tllm_stream_t s) {
  return s ? static_cast<cudaStream_t>(s) : lib_stream();
}

inline int dtype_size(int dt) {
  switch (dt) {
    case TLLM_F32: return 4;
    case TLLM_BF16: return 2;
    case TLLM_I32: return 4;
    case TLLM_SPLIT: return 4;   // two bf16 planes
    case TLLM_BF16_TILED: return 2;
    default: return 0;
  }
}

int sm_count();  // multiprocessors of the current device (cached)
// Programmatic dependent launch of the projection kernels (TLLM_NO_PDL=1
// turns it off, for comparisons).
bool pdl_enabled();

// Device-side error word (one int per device, allocated on first use).
// Kernels receive its address and OR a code into it instead of trapping when
// a bounded wait runs out or a value read on the device is out of range; the
// host reads and clears it with tllm_device_error().
enum DeviceError : int {
  DEV_ERR_WAIT_TIMEOUT = 1,   // an mbarrier wait ran out of polls
  DEV_ERR_LEN_CLAMPED = 2,    // a device-side length exceeded its bound
  DEV_ERR_TOKEN_RANGE = 4,    // a token id outside [0, vocab)
  DEV_ERR_SMEM_ALIGN = 8,     // dynamic shared memory not 1024-byte aligned
  DEV_ERR_LAYOUT = 16,        // a launch whose ring / issuer layout is invalid
};
int *device_error_ptr();

}  // namespace tllm

struct CUtensorMap_st;
namespace tllm {
// Tensor map over a KV cache viewed as (planes, max_seq, D) with a box of
// (rows x box_inner) elements (box_inner 0 = D); swizzle128 selects the
// 128-byte swizzle (attention_decode.cu).
int make_kv_map(CUtensorMap_st *m, const void *base, int dtype, int D,
                int max_seq, long planes, int rows, int box_inner = 0,
                bool swizzle128 = false);
}  // namespace tllm

#define TLLM_CHECK_ARG(cond, ...)                 \
  do {                                            \
    if (!(cond)) {                                \
      ::tllm::set_error(__VA_ARGS__);             \
      return TLLM_ERR_INVALID_ARG;                \
    }                                             \
  } while (0)

#define TLLM_CUDA(call)                                                     \
  do {                                                                      \
    cudaError_t e_ = (call);                                                \
    if (e_ != cudaSuccess) {                                                \
      ::tllm::set_error("%s failed: %s (%d)", #call, cudaGetErrorString(e_), \
                        (int)e_);                                           \
      return TLLM_ERR_CUDA;                                                 \
    }                                                                       \
  } while (0)

// After a kernel launch: report configuration errors immediately.
#define TLLM_LAUNCH_CHECK()                                                 \
  do {                                                                      \
    cudaError_t e_ = cudaGetLastError();                                    \
    if (e_ != cudaSuccess) {                                                \
      ::tllm::set_error("kernel launch failed: %s (%d)",                    \
                        cudaGetErrorString(e_), (int)e_);                   \
      return TLLM_ERR_CUDA;                                                 \
    }                                                                       \
  } while (0)

#define TLLM_INJECT(site)                                         \
  do {                                                            \
    if (::tllm::inject_fault(site)) {                             \
      ::tllm::set_error("injected failure at %s", site);          \
      return TLLM_ERR_INJECTED;                                   \
    }                                                             \
  } while (0)

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------
namespace tllm {

__device__ __forceinline__ float bf16lo(uint32_t w) {
  return __uint_as_float(w << 16);
}
__device__ __forceinline__ float bf16hi(uint32_t w) {
  return __uint_as_float(w & 0xffff0000u);
}

// Round-to-nearest-even f32 -> bf16 bits (matches numpy's rounding used by
// the oracle's bf16 cast; NaN stays NaN).
__host__ __device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
#ifdef __CUDA_ARCH__
  uint32_t u = __float_as_uint(f);
#else
  uint32_t u;
  memcpy(&u, &f, 4);
#endif
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

// Element (n, k) of a TLLM_BF16_TILED (N, K) matrix.
__host__ __device__ __forceinline__ size_t tiled_index(size_t n, size_t k,
                                                      size_t K) {
  return ((n >> 7) * (K >> 6) + (k >> 6)) * 8192 + (n & 127) * 64 + (k & 63);
}

__host__ __device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
#ifdef __CUDA_ARCH__
  return __uint_as_float((uint32_t)h << 16);
#else
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
#endif
}

// Store v at element idx of a TLLM_SPLIT matrix whose planes are `plane`
// elements apart: hi = bf16(v), lo = bf16(v - hi).
__device__ __forceinline__ void store_split(uint16_t *base, size_t plane,
                                            size_t idx, float v) {
  const uint16_t h = f32_to_bf16_bits(v);
  base[idx] = h;
  base[plane + idx] = f32_to_bf16_bits(v - bf16_bits_to_f32(h));
}
// Activation store in the tensor-core operand format: TLLM_SPLIT (two
// planes) or TLLM_BF16 (the hi plane only).
__device__ __forceinline__ void store_act(uint16_t *base, size_t plane,
                                          size_t idx, float v, int planes) {
  const uint16_t h = f32_to_bf16_bits(v);
  base[idx] = h;
  if (planes == 2) base[plane + idx] = f32_to_bf16_bits(v - bf16_bits_to_f32(h));
}

// Load 16 bytes that are read once (bypass L1 allocation).
__device__ __forceinline__ uint4 ld_stream(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// ---- mbarrier / TMA (sm_90+ PTX, used on sm_100a) -------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after `limit` polls (each poll itself blocks for a
// hardware-defined time slice) and returns false instead of hanging.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar,
                                                  uint32_t phase,
                                                  uint32_t limit = 1u << 22) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, phase)) return true;
  return false;
}

// 3-D tiled TMA load global -> shared, completion signalled on `bar`.
__device__ __forceinline__ void tma_load_3d(void *dst, const void *tmap,
                                            uint64_t *bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_"
      "tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// 3-D tiled TMA load with an L2 eviction hint (createpolicy value).
__device__ __forceinline__ void tma_load_3d_hint(void *dst, const void *tmap,
                                                 uint64_t *bar, int c0, int c1,
                                                 int c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_"
      "tx::bytes.L2::cache_hint [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(
          smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_load_2d_hint(void *dst, const void *tmap,
                                                 uint64_t *bar, int c0, int c1,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_"
      "tx::bytes.L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(
          smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---- tcgen05 (5th-generation tensor cores, TMEM accumulators) -------------
// Shared-memory matrix descriptor of a K-major bf16 tile written by TMA with
// 128-byte swizzle: rows of 128 bytes (64 elements), 8-row groups 1024 bytes
// apart (stride byte offset), leading byte offset unused for this layout
// (set to 1), descriptor version 1 (bits 46-47), layout type 2 = 128B
// swizzle (bits 61-63). The tile base must be 1024-byte aligned; the k-th
// 16-element slice of a row starts 32 * k bytes later (start address + 2 k).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) |
         ((uint64_t)64 << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor of tcgen05.mma kind::f16: D f32 (bits 4-5 = 1),
// A and B bf16 (bits 7-9 = 1, 10-12 = 1), both K-major (bits 15, 16 = 0),
// N >> 3 in bits 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc,
                                          uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// Arrive on `bar` once every tcgen05 op issued so far by this thread is done.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
      "[%0];" ::"r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Warp-wide TMEM allocation of `ncols` columns (power of two >= 32); the
// base address is written to *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_u32(slot)),
      "r"(ncols)
      : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ void tmem_free(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(
                   taddr),
               "r"(ncols)
               : "memory");
}
// 32 consecutive fp32 columns of this thread's TMEM lane (warp-wide).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,"
      "%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,"
      "%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
        "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// 16 consecutive fp32 columns of this thread's TMEM lane (warp-wide).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,"
      "%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
        "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ---- thread-block clusters / distributed shared memory ---------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of every CTA of the cluster (like __syncthreads, cluster-wide).
__device__ __forceinline__ void cluster_sync() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// 4 consecutive fp32 at shared address `saddr` (16-byte aligned) of CTA
// `rank` of this cluster.
__device__ __forceinline__ float4 ld_dsmem_f32x4(uint32_t saddr, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(saddr), "r"(rank));
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(a)
               : "memory");
  return v;
}
// fp32 at shared address `saddr` of CTA `rank` of this cluster.
__device__ __forceinline__ float ld_dsmem_f32(uint32_t saddr, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(saddr), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
  return v;
}

// ---- programmatic dependent launch ----------------------------------------
// A kernel launched with the programmatic-serialization attribute may start
// before the previous kernel on the stream has finished; it must call
// griddep_wait() before touching anything that kernel writes or reads.
// Every kernel calls griddep_launch() once all its CTAs are resident, so a
// dependent kernel can fill the SMs freed by the last wave.
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" :::);
}

// Launch `kern` with programmatic stream serialization (unless disabled):
// its CTAs may become resident while the previous kernel on the stream is
// still running, so the kernel must call griddep_wait() before it reads or
// writes anything another kernel touches.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block,
                       size_t smem, cudaStream_t st, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Args &&>(args)...);
}

}  // namespace tllm
