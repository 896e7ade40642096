// Projection GEMMs of the decode step, y[m, n] = sum_k x[m, k] W[n, k],
// with fused epilogues (bias, residual add, GELU, SwiGLU, RoPE + KV append).
//
// Replaces triton_llm/kernels/gemm.py:53-109 and the add / swiglu / gelu /
// apply_rope launches that follow it in the reference's decode step
// (smollm2_triton/model.py:281-365, gpt2_triton/model.py:319-361).
//
// Two kernels:
//  * linear_mma_kernel (bf16 weights): tensor cores via mma.sync m16n8k16.
//    The weight rows are the MMA M dimension (128 rows per CTA, 32 per
//    consumer warp) and the activation rows the N dimension (8..64 per
//    tile), so each weight byte is streamed from HBM once whatever the
//    batch. Weight tiles (128 x 64) and fp32 activation tiles (64 rows x 64)
//    arrive by 2-D TMA with 128-byte swizzle into a 3-stage ring; each
//    activation element is split into bf16 head + residual when it is
//    loaded into a fragment, so the product keeps ~16 mantissa bits of x.
//    K is split across CTAs when there are few weight tiles; the last CTA
//    of a tile (atomic ticket) sums the splits in fixed order and runs the
//    epilogue, so results do not depend on scheduling.
//  * linear_f32_kernel (fp32 weights, GPT-2 and the fp32 drop-in): one warp
//    per weight row, 16-byte loads along K, fp32 FMA, same epilogues.
//
// Epilogue row pairing: a thread's accumulator holds weight rows r and r+8
// of a 16-row block. SwiGLU weights are stored with gate and up rows
// interleaved in blocks of 8 (gate 8i..8i+7, up 8i..8i+7), so gate and up of
// one output sit in one thread. QKV weights are stored per head with dims
// (8b..8b+7) followed by (D/2+8b..D/2+8b+7), so the RoPE pair (d, d+D/2) of
// the reference's rotate-half (triton_llm/kernels/rope.py:49-66) sits in one
// thread and is rotated before the store.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <mutex>

#include "common.cuh"

namespace tllm {

// tma.cu
int make_map_2d(CUtensorMap *m, const void *base, int dtype, long inner,
                long outer, long stride_bytes, int box_inner, int box_outer,
                bool swizzle128);

namespace {

enum EpiOp : int {
  EPI_STORE = 0,   // out[m, n] = acc (+ bias)
  EPI_RESID = 1,   // out[m, n] = resid[m, n] + acc (+ bias)   (may alias)
  EPI_GELU = 2,    // out[m, n] = gelu_tanh(acc + bias)
  EPI_SWIGLU = 3,  // out[m, j] = silu(gate_j) * up_j  (rows interleaved by 8)
  EPI_QKV = 4,     // q / k / v heads, optional RoPE, K/V into the cache
};

struct Epilogue {
  int op;
  const float *bias;   // [N] or null (in weight-row order)
  float *out;          // [M, ld_out]
  const float *resid;  // [M, ld_out] (EPI_RESID)
  int ld_out;
  // EPI_QKV
  const float *cos, *sin;  // [max_pos, D/2] or null (no rotation)
  const int *row_seq;      // [M]: cache sequence of each activation row
  const int *row_pos;      // [M]: position of each activation row
  float *q_out;            // [M, H, D]
  void *k_cache, *v_cache; // [B, Hkv, max_seq, D]
  int kv_bf16, max_seq, H, Hkv, D;
  int *lens_out;           // optional [B]: lens_out[seq] = pos + 1
  int *err;
};

__device__ __forceinline__ float gelu_tanh(float x) {
  // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) with tanh built from
  // exp(-2|u|) as in triton_llm/kernels/gelu.py:17-28, :50-51
  const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  const float e = expf(-2.f * fabsf(u));
  const float t = (u < 0.f ? -1.f : 1.f) * (1.f - e) / (1.f + e);
  return 0.5f * x * (1.f + t);
}
__device__ __forceinline__ float silu_ref(float x) {
  // x * sigmoid(x), sigmoid from exp(-|x|) (triton_llm/kernels/swiglu.py:51-54)
  const float e = expf(-fabsf(x));
  const float sig = x >= 0.f ? 1.f / (1.f + e) : e / (1.f + e);
  return x * sig;
}

// Apply the epilogue to weight rows (r, r + 8) of one 16-row block at
// activation row m. v0 = acc(r, m), v1 = acc(r + 8, m).
__device__ __forceinline__ void epi_pair(const Epilogue &e, int N, int M,
                                         int r, int m, float v0, float v1) {
  if (m >= M) return;
  const int r1 = r + 8;
  switch (e.op) {
    case EPI_STORE:
    case EPI_RESID:
    case EPI_GELU: {
      float *o = e.out + (size_t)m * e.ld_out;
      if (r < N) {
        float a = v0 + (e.bias ? e.bias[r] : 0.f);
        if (e.op == EPI_RESID) a = e.resid[(size_t)m * e.ld_out + r] + a;
        if (e.op == EPI_GELU) a = gelu_tanh(a);
        o[r] = a;
      }
      if (r1 < N) {
        float a = v1 + (e.bias ? e.bias[r1] : 0.f);
        if (e.op == EPI_RESID) a = e.resid[(size_t)m * e.ld_out + r1] + a;
        if (e.op == EPI_GELU) a = gelu_tanh(a);
        o[r1] = a;
      }
      break;
    }
    case EPI_SWIGLU: {
      if (r1 < N) {
        const int j = (r >> 4) * 8 + (r & 7);
        e.out[(size_t)m * e.ld_out + j] = silu_ref(v0) * v1;
      }
      break;
    }
    case EPI_QKV: {
      if (r1 >= N) break;
      const int D = e.D;
      const int head = r / D;
      const int local = r - head * D;         // r is in the first 8 of a 16
      const int blk = local >> 4;
      const int d0 = blk * 8 + (local & 7);   // dim of v0; v1 is d0 + D/2
      const int d1 = d0 + D / 2;
      float x0 = v0 + (e.bias ? e.bias[r] : 0.f);
      float x1 = v1 + (e.bias ? e.bias[r1] : 0.f);
      const int pos = e.row_pos[m];
      const int seq = e.row_seq[m];
      const bool is_v = head >= e.H + e.Hkv;
      if (e.cos && !is_v) {
        // x0' = x0 c - x1 s, x1' = x0 s + x1 c with each product rounded
        // (no FMA contraction), as numpy computes rope.py:65-66
        const float c = e.cos[(size_t)pos * (D / 2) + d0];
        const float s = e.sin[(size_t)pos * (D / 2) + d0];
        const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        const float y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        x0 = y0;
        x1 = y1;
      }
      if (head < e.H) {
        float *q = e.q_out + ((size_t)m * e.H + head) * D;
        q[d0] = x0;
        q[d1] = x1;
      } else {
        const int kvh = is_v ? head - e.H - e.Hkv : head - e.H;
        if (pos < 0 || pos >= e.max_seq || seq < 0) {
          atomicOr(e.err, DEV_ERR_LEN_CLAMPED);
          break;
        }
        const size_t off =
            (((size_t)seq * e.Hkv + kvh) * e.max_seq + pos) * D;
        void *cache = is_v ? e.v_cache : e.k_cache;
        if (e.kv_bf16) {
          uint16_t *c = static_cast<uint16_t *>(cache) + off;
          c[d0] = f32_to_bf16_bits(x0);
          c[d1] = f32_to_bf16_bits(x1);
        } else {
          float *c = static_cast<float *>(cache) + off;
          c[d0] = x0;
          c[d1] = x1;
        }
        if (e.lens_out && head == e.H && local == 0) e.lens_out[seq] = pos + 1;
      }
      break;
    }
  }
}

// ------------------------------------------------------------------------
// bf16 weights, tensor cores
// ------------------------------------------------------------------------
constexpr int kLinThreads = 5 * 32;  // 4 consumer warps + 1 producer warp
constexpr int kLinBN = 128;          // weight rows per CTA
constexpr int kLinBK = 64;           // K per stage
constexpr int kLinStages = 3;

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0,
                                        uint32_t &r1, uint32_t &r2,
                                        uint32_t &r3) {
  asm volatile(
      "ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
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
__device__ __forceinline__ uint32_t pack_bf16x2(float x0, float x1) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(x1), "f"(x0));
  return r;
}
__device__ __forceinline__ void split_bf16x2(float x0, float x1, uint32_t &hi,
                                             uint32_t &lo) {
  hi = pack_bf16x2(x0, x1);
  lo = pack_bf16x2(x0 - bf16lo(hi), x1 - bf16hi(hi));
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap,
                                            uint64_t *bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_"
      "tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

struct LinParams {
  Epilogue e;
  float *partial;   // [m_tiles][S][n_tiles * 128][MT] split-K partials
  int *counters;    // [m_tiles][n_tiles]
  int M, N, K, S, k_chunks, n_tiles;
};

template <int MT>
__global__ void __launch_bounds__(kLinThreads)
    linear_mma_kernel(const LinParams p,
                      const __grid_constant__ CUtensorMap tw,
                      const __grid_constant__ CUtensorMap ta) {
  constexpr int NT = MT / 8;                       // n8 tiles of activations
  constexpr int W_BYTES = kLinBN * 128;            // 128 rows x 64 bf16
  constexpr int A_BYTES = MT * 256;                // MT rows x 64 fp32
  constexpr int STAGE = W_BYTES + A_BYTES;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + kLinStages * STAGE);
  uint64_t *empty = full + kLinStages;
  __shared__ int s_last;

  // 128-byte-swizzled TMA tiles need 1024-byte aligned stage buffers
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) atomicOr(p.e.err, DEV_ERR_SMEM_ALIGN);
    return;
  }
  const int nt = blockIdx.x;
  const int split = blockIdx.y;
  const int mt = blockIdx.z;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int per = (p.k_chunks + p.S - 1) / p.S;
  const int kc0 = split * per;
  const int kc1 = min(kc0 + per, p.k_chunks);
  const int nch = kc1 > kc0 ? kc1 - kc0 : 0;

  if (tid == 0) {
    for (int s = 0; s < kLinStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    fence_mbar_init();
  }
  __syncthreads();

  bool failed = false;
  float acc[2][NT][4];
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[a][j][e] = 0.f;

  if (warp == 4) {
    if (lane == 0) {
      for (int c = 0; c < nch; ++c) {
        const int s = c % kLinStages;
        if (c >= kLinStages &&
            !mbar_wait_bounded(&empty[s], ((c / kLinStages) - 1) & 1)) {
          failed = true;
          break;
        }
        uint8_t *st = smem + s * STAGE;
        mbar_expect_tx(&full[s], STAGE);
        const int k0 = (kc0 + c) * kLinBK;
        tma_load_2d(st, &tw, &full[s], k0, nt * kLinBN);
        tma_load_2d(st + W_BYTES, &ta, &full[s], k0, mt * MT);
        tma_load_2d(st + W_BYTES + MT * 128, &ta, &full[s], k0 + 32, mt * MT);
      }
    }
  } else {
    // ldmatrix lane addressing for the weight (A operand) 16x16 blocks
    const int w_row = (lane & 7) + ((lane >> 3) & 1) * 8;
    const int w_kof = (lane >> 4) * 8;
    const int ar = lane >> 2;        // activation row within an n8 tile
    const int ak = (lane & 3) * 2;   // k pair within a 16-k step
    for (int c = 0; c < nch; ++c) {
      const int s = c % kLinStages;
      if (!__all_sync(0xffffffffu,
                      mbar_wait_bounded(&full[s], (c / kLinStages) & 1))) {
        failed = true;
        break;
      }
      const uint8_t *wt = smem + s * STAGE;
      const uint8_t *at = wt + W_BYTES;
#pragma unroll
      for (int kk = 0; kk < kLinBK / 16; ++kk) {
        uint32_t wa[2][4];
#pragma unroll
        for (int a = 0; a < 2; ++a) {
          const int row = warp * 32 + a * 16 + w_row;
          const int chunk = kk * 2 + (w_kof >> 3);
          ldsm_x4(smem_u32(wt + row * 128 + ((chunk ^ (row & 7)) << 4)),
                  wa[a][0], wa[a][1], wa[a][2], wa[a][3]);
        }
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          const int m = j * 8 + ar;
          uint32_t bh[2], bl[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int k = kk * 16 + h * 8 + ak;      // 0..63, even
            const int box = k >> 5;
            const int chunk = (k & 31) >> 2;
            const float2 v = *reinterpret_cast<const float2 *>(
                at + box * (MT * 128) + m * 128 + ((chunk ^ (m & 7)) << 4) +
                (k & 3) * 4);
            split_bf16x2(v.x, v.y, bh[h], bl[h]);
          }
#pragma unroll
          for (int a = 0; a < 2; ++a) {
            mma_bf16(acc[a][j], wa[a], bh[0], bh[1]);
            mma_bf16(acc[a][j], wa[a], bl[0], bl[1]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
  if (failed) atomicOr(p.e.err, DEV_ERR_WAIT_TIMEOUT);
  if (warp == 4) return;

  // accumulator element (a, j, e): weight row
  //   nt*128 + warp*32 + a*16 + (lane>>2) + (e >= 2 ? 8 : 0)
  // activation row mt*MT + j*8 + (lane&3)*2 + (e & 1)
  const int row_base = nt * kLinBN + warp * 32 + (lane >> 2);
  const int m_base = mt * MT + (lane & 3) * 2;
  if (p.S > 1) {
    // write this split's partial, take a ticket, the last CTA reduces
    const size_t ldp = (size_t)p.n_tiles * kLinBN;
    float *part = p.partial + ((size_t)mt * p.S + split) * ldp * MT;
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = row_base + a * 16 + (e >= 2 ? 8 : 0);
          const int mm = j * 8 + (lane & 3) * 2 + (e & 1);
          part[(size_t)row * MT + mm] = acc[a][j][e];
        }
    __threadfence();
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (tid == 0) {
      int *ctr = p.counters + (size_t)mt * p.n_tiles + nt;
      const int ticket = atomicAdd(ctr, 1);
      s_last = (ticket == p.S - 1);
      if (s_last) *ctr = 0;
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (!s_last) return;
    __threadfence();
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = row_base + a * 16 + (e >= 2 ? 8 : 0);
          const int mm = j * 8 + (lane & 3) * 2 + (e & 1);
          float sum = 0.f;
          for (int sp = 0; sp < p.S; ++sp)  // fixed order: deterministic
            sum += __ldcg(&p.partial[(((size_t)mt * p.S + sp) * ldp + row) * MT + mm]);
          acc[a][j][e] = sum;
        }
  }
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e)
        epi_pair(p.e, p.N, p.M, row_base + a * 16, m_base + j * 8 + e,
                 acc[a][j][e], acc[a][j][e + 2]);
}

// ------------------------------------------------------------------------
// fp32 weights, CUDA cores: one warp per weight-row pair (r, r + 8)
// ------------------------------------------------------------------------
constexpr int kF32Warps = 8;

template <int MB>
__global__ void __launch_bounds__(kF32Warps * 32)
    linear_f32_kernel(const float *x, const float *w, Epilogue e, int M,
                      int N, int K, int m0) {
  const int warp = (blockIdx.x * kF32Warps) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  // pair index -> rows r (first 8 of a 16-block) and r + 8
  const int r = (warp >> 3) * 16 + (warp & 7);
  if (r >= ((N + 15) / 16) * 16) return;
  const int r1 = r + 8;
  float acc0[MB], acc1[MB];
#pragma unroll
  for (int i = 0; i < MB; ++i) acc0[i] = acc1[i] = 0.f;
  const float *w0 = w + (size_t)r * K;
  const float *w1 = w + (size_t)r1 * K;
  const bool ok0 = r < N, ok1 = r1 < N;
  for (int k = lane * 4; k < K; k += 128) {
    float4 a = ok0 ? __ldg(reinterpret_cast<const float4 *>(w0 + k))
                   : make_float4(0, 0, 0, 0);
    float4 b = ok1 ? __ldg(reinterpret_cast<const float4 *>(w1 + k))
                   : make_float4(0, 0, 0, 0);
#pragma unroll
    for (int i = 0; i < MB; ++i) {
      if (m0 + i < M) {
        const float4 xv =
            __ldg(reinterpret_cast<const float4 *>(x + (size_t)(m0 + i) * K + k));
        acc0[i] = fmaf(a.x, xv.x, acc0[i]);
        acc0[i] = fmaf(a.y, xv.y, acc0[i]);
        acc0[i] = fmaf(a.z, xv.z, acc0[i]);
        acc0[i] = fmaf(a.w, xv.w, acc0[i]);
        acc1[i] = fmaf(b.x, xv.x, acc1[i]);
        acc1[i] = fmaf(b.y, xv.y, acc1[i]);
        acc1[i] = fmaf(b.z, xv.z, acc1[i]);
        acc1[i] = fmaf(b.w, xv.w, acc1[i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < MB; ++i) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      acc0[i] += __shfl_xor_sync(0xffffffffu, acc0[i], off);
      acc1[i] += __shfl_xor_sync(0xffffffffu, acc1[i], off);
    }
  }
  if (lane < MB) {
    float v0 = 0.f, v1 = 0.f;
#pragma unroll
    for (int i = 0; i < MB; ++i)
      if (i == lane) {
        v0 = acc0[i];
        v1 = acc1[i];
      }
    epi_pair(e, N, M, r, m0 + lane, v0, v1);
  }
}

template <int MT>
int launch_mma(const LinParams &p, const CUtensorMap &tw, const CUtensorMap &ta,
               dim3 grid, cudaStream_t st) {
  const size_t smem = (size_t)kLinStages * (kLinBN * 128 + MT * 256) +
                      2 * kLinStages * sizeof(uint64_t);
  auto kern = linear_mma_kernel<MT>;
  static bool configured[64] = {};  // per instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    TLLM_CUDA(cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  kern<<<grid, kLinThreads, smem, st>>>(p, tw, ta);
  TLLM_LAUNCH_CHECK();
  return TLLM_OK;
}

int check_epilogue(const Epilogue &e, int N) {
  TLLM_CHECK_ARG(e.op >= EPI_STORE && e.op <= EPI_QKV, "bad epilogue op %d",
                 e.op);
  if (e.op == EPI_QKV) {
    TLLM_CHECK_ARG(e.D > 0 && e.D % 16 == 0, "head_dim must be a multiple of 16");
    TLLM_CHECK_ARG(N == (e.H + 2 * e.Hkv) * e.D,
                   "QKV rows (%d) != (H + 2 Hkv) * D", N);
    TLLM_CHECK_ARG(e.q_out && e.k_cache && e.v_cache && e.row_seq && e.row_pos,
                   "QKV epilogue needs q_out, caches, row_seq, row_pos");
  } else if (e.op == EPI_SWIGLU) {
    TLLM_CHECK_ARG(N % 16 == 0, "SwiGLU rows must be a multiple of 16");
    TLLM_CHECK_ARG(e.out, "NULL output");
  } else {
    TLLM_CHECK_ARG(e.out, "NULL output");
    if (e.op == EPI_RESID) TLLM_CHECK_ARG(e.resid, "residual is NULL");
  }
  return TLLM_OK;
}

}  // namespace
}  // namespace tllm

using namespace tllm;

extern "C" {

int tllm_linear_workspace(int M, int N, int K, size_t *partial_bytes,
                          size_t *counter_bytes) {
  TLLM_CHECK_ARG(partial_bytes && counter_bytes, "NULL output");
  TLLM_CHECK_ARG(M >= 0 && N >= 0 && K >= 0, "negative shape");
  const long n_tiles = (N + kLinBN - 1) / kLinBN;
  const long mt = M <= 64 ? 1 : (M + 63) / 64;
  const int mtile = M <= 8 ? 8 : M <= 16 ? 16 : M <= 32 ? 32 : 64;
  // at most 16 splits
  *partial_bytes = (size_t)mt * 16 * n_tiles * kLinBN * mtile * sizeof(float);
  *counter_bytes = (size_t)mt * n_tiles * sizeof(int32_t);
  return TLLM_OK;
}

// y = epilogue(x @ W^T); see tllm.h for the epilogue encoding.
int tllm_linear(const float *x, const void *w, int w_dtype, int M, int N,
                int K, int op, const float *bias, float *out, int ld_out,
                const float *resid, const float *cos_t, const float *sin_t,
                const int32_t *row_seq, const int32_t *row_pos, float *q_out,
                void *k_cache, void *v_cache, int kv_dtype, int max_seq,
                int n_head, int n_kv_head, int head_dim, int32_t *lens_out,
                void *partial, size_t partial_bytes, int32_t *counters,
                tllm_stream_t stream) {
  TLLM_INJECT("launch");
  TLLM_CHECK_ARG(M >= 0 && N >= 0 && K >= 0, "negative shape");
  if (M == 0 || N == 0) return TLLM_OK;
  TLLM_CHECK_ARG(x && w, "NULL input");
  TLLM_CHECK_ARG(K > 0 && K % 64 == 0 || w_dtype == TLLM_F32,
                 "bf16 linear needs K %% 64 == 0 (K=%d)", K);
  TLLM_CHECK_ARG(K % 4 == 0, "K must be a multiple of 4");
  TLLM_CHECK_ARG(((uintptr_t)x & 15) == 0 && ((uintptr_t)w & 15) == 0,
                 "x and W must be 16-byte aligned");
  Epilogue e{};
  e.op = op;
  e.bias = bias;
  e.out = out;
  e.resid = resid;
  e.ld_out = ld_out > 0 ? ld_out : (op == EPI_SWIGLU ? N / 2 : N);
  e.cos = cos_t;
  e.sin = sin_t;
  e.row_seq = row_seq;
  e.row_pos = row_pos;
  e.q_out = q_out;
  e.k_cache = k_cache;
  e.v_cache = v_cache;
  e.kv_bf16 = kv_dtype == TLLM_BF16;
  e.max_seq = max_seq;
  e.H = n_head;
  e.Hkv = n_kv_head;
  e.D = head_dim;
  e.lens_out = lens_out;
  e.err = device_error_ptr();
  TLLM_CHECK_ARG(e.err, "device error word unavailable");
  int rc = check_epilogue(e, N);
  if (rc) return rc;
  cudaStream_t st = resolve(stream);

  if (w_dtype == TLLM_F32) {
    const int pairs = ((N + 15) / 16) * 8;
    const int blocks = (pairs + kF32Warps - 1) / kF32Warps;
    for (int m0 = 0; m0 < M; m0 += 8) {
      linear_f32_kernel<8><<<blocks, kF32Warps * 32, 0, st>>>(
          x, static_cast<const float *>(w), e, M, N, K, m0);
      TLLM_LAUNCH_CHECK();
    }
    return TLLM_OK;
  }
  TLLM_CHECK_ARG(w_dtype == TLLM_BF16, "w_dtype must be F32 or BF16");

  const int MT = M <= 8 ? 8 : M <= 16 ? 16 : M <= 32 ? 32 : 64;
  const int m_tiles = (M + MT - 1) / MT;
  const int n_tiles = (N + kLinBN - 1) / kLinBN;
  const int k_chunks = K / kLinBK;
  // split K until the grid covers the device twice, >= 4 chunks per split
  int S = 1;
  const long base = (long)m_tiles * n_tiles;
  while (S < 16 && base * S < 2L * sm_count() && k_chunks / (S * 2) >= 4) S *= 2;
  if (S > 1) {
    const size_t need = (size_t)m_tiles * S * n_tiles * kLinBN * MT * sizeof(float);
    const size_t cneed = (size_t)m_tiles * n_tiles * sizeof(int32_t);
    if (!partial || !counters || partial_bytes < need || cneed == 0) S = 1;
  }
  CUtensorMap tw, ta;
  rc = make_map_2d(&tw, w, TLLM_BF16, K, N, (long)K * 2, kLinBK, kLinBN, true);
  if (rc) return rc;
  rc = make_map_2d(&ta, x, TLLM_F32, K, M, (long)K * 4, 32, MT, true);
  if (rc) return rc;
  LinParams p;
  p.e = e;
  p.partial = static_cast<float *>(partial);
  p.counters = counters;
  p.M = M;
  p.N = N;
  p.K = K;
  p.S = S;
  p.k_chunks = k_chunks;
  p.n_tiles = n_tiles;
  dim3 grid(n_tiles, S, m_tiles);
  switch (MT) {
    case 8: return launch_mma<8>(p, tw, ta, grid, st);
    case 16: return launch_mma<16>(p, tw, ta, grid, st);
    case 32: return launch_mma<32>(p, tw, ta, grid, st);
    default: return launch_mma<64>(p, tw, ta, grid, st);
  }
}

}  // extern "C"
