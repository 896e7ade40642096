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
// "launch:N" makes the N-th kernel entry point fail before it launches.
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
    default: return 0;
  }
}

int sm_count();  // multiprocessors of the current device (cached)

// Device-side error word (one int per device, allocated on first use).
// Kernels receive its address and OR a code into it instead of trapping when
// a bounded wait runs out or a value read on the device is out of range; the
// host reads and clears it with tllm_device_error().
enum DeviceError : int {
  DEV_ERR_WAIT_TIMEOUT = 1,   // an mbarrier wait ran out of polls
  DEV_ERR_LEN_CLAMPED = 2,    // a device-side length exceeded its bound
  DEV_ERR_TOKEN_RANGE = 4,    // a token id outside [0, vocab)
  DEV_ERR_SMEM_ALIGN = 8,     // dynamic shared memory not 1024-byte aligned
};
int *device_error_ptr();

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

}  // namespace tllm
