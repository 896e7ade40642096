// Warp-level tensor-core helpers (mma.sync / ldmatrix) shared by the
// attention kernels: bf16 operands, fp32 accumulation, hi + lo bf16 splits
// of fp32 values.
#pragma once

#include "common.cuh"

namespace tllm {

// 2^x with the MUFU instruction (relative error ~2^-22; -inf -> +0).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0,
                                        uint32_t &r1, uint32_t &r2,
                                        uint32_t &r3) {
  asm volatile(
      "ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0,
                                          uint32_t &r1, uint32_t &r2,
                                          uint32_t &r3) {
  asm volatile(
      "ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4],
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// (x0, x1) -> bf16x2 with x0 in the low half (round to nearest even)
__device__ __forceinline__ uint32_t pack_bf16x2(float x0, float x1) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(x1), "f"(x0));
  return r;
}
// x = hi + lo with hi, lo bf16 pairs
__device__ __forceinline__ void split_bf16x2(float x0, float x1, uint32_t &hi,
                                             uint32_t &lo) {
  hi = pack_bf16x2(x0, x1);
  lo = pack_bf16x2(x0 - bf16lo(hi), x1 - bf16hi(hi));
}
}  // namespace tllm
