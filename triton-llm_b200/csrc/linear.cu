// Projection GEMMs of the decode step, y[m, n] = sum_k x[m, k] W[n, k],
// with fused epilogues (bias, residual add, GELU, SwiGLU, RoPE + KV append).
//
// Replaces triton_llm/kernels/gemm.py:53-109 and the add / swiglu / gelu /
// apply_rope launches that follow it in the reference's decode step
// (smollm2_triton/model.py:281-365, gpt2_triton/model.py:319-361).
//
// Two kernels:
//  * linear_tc_kernel (bf16 weights): 5th-generation tensor cores. Weight
//    rows are the MMA's M dimension (128 per CTA) and activation rows its N
//    dimension (16..256 per tile), so every weight byte streams from HBM
//    once whatever the batch. One thread issues the TMA loads of 128 x 64
//    weight tiles and of the activation tiles into a ring of shared-memory
//    stages; one thread issues tcgen05.mma with the fp32 accumulator in
//    TMEM and releases each stage with tcgen05.commit; after the last stage
//    the four warps read the accumulator with tcgen05.ld and run the
//    epilogue. Activations arrive in the TLLM_SPLIT format (bf16 hi and lo
//    planes): each k-slice issues one MMA for hi and one for lo, so the
//    product keeps ~16 mantissa bits of the fp32 activations while both
//    operands are bf16. K is split across CTAs when there are too few
//    weight tiles to occupy the GPU: the S CTAs of a tile form a thread-block
//    cluster, each stages its accumulator tile in shared memory, and after a
//    cluster barrier each reduces a slice of the tile over distributed shared
//    memory (ranks summed in fixed order, so results do not depend on
//    scheduling) and runs the epilogue for that slice.
//  * linear_f32_kernel (fp32 weights, GPT-2 and the fp32 drop-in): one warp
//    per weight-row pair, 16-byte loads along K, fp32 FMA, same epilogues.
//
// Epilogue row pairing: rows r and r + 8 of a 16-row block are handled by
// one thread. SwiGLU weights are stored with gate and up rows interleaved in
// blocks of 8 (gate 8i..8i+7, up 8i..8i+7), so gate and up of one output
// meet in one thread. QKV weights are stored per head with dims
// (8b..8b+7) followed by (D/2+8b..D/2+8b+7), so the RoPE pair (d, d+D/2) of
// the reference's rotate-half (triton_llm/kernels/rope.py:49-66) meets in
// one thread and is rotated before the store.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>

#include "common.cuh"

namespace tllm {

// tma.cu
int make_map_2d(CUtensorMap *m, const void *base, int dtype, long inner,
                long outer, long stride_bytes, int box_inner, int box_outer,
                bool swizzle128);
int make_map(CUtensorMap *m, const void *base, int dtype, int rank,
             const long *dims, const long *strides_bytes, const int *box,
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
  float *out;          // [M, ld_out] fp32, or null when out_split is set
  uint16_t *out_split; // TLLM_SPLIT output, planes out_plane elements apart
  size_t out_plane;
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

__device__ __forceinline__ void store_out(const Epilogue &e, size_t idx,
                                          float v) {
  if (e.out_split)
    store_split(e.out_split, e.out_plane, idx, v);
  else
    e.out[idx] = v;
}

// Apply the epilogue to weight rows (r, r + 8) of one 16-row block at
// activation row m. v0 = acc(r, m), v1 = acc(r + 8, m).
template <int OP>
__device__ __forceinline__ void epi_pair(const Epilogue &e, int N, int M,
                                         int r, int m, float v0, float v1) {
  if (m >= M) return;
  const int r1 = r + 8;
  if constexpr (OP == EPI_STORE || OP == EPI_RESID || OP == EPI_GELU) {
    const size_t o = (size_t)m * e.ld_out;
    if (r < N) {
      float a = v0 + (e.bias ? e.bias[r] : 0.f);
      if constexpr (OP == EPI_RESID) a = e.resid[o + r] + a;
      if constexpr (OP == EPI_GELU) a = gelu_tanh(a);
      store_out(e, o + r, a);
    }
    if (r1 < N) {
      float a = v1 + (e.bias ? e.bias[r1] : 0.f);
      if constexpr (OP == EPI_RESID) a = e.resid[o + r1] + a;
      if constexpr (OP == EPI_GELU) a = gelu_tanh(a);
      store_out(e, o + r1, a);
    }
  } else if constexpr (OP == EPI_SWIGLU) {
    if (r1 < N) {
      const int j = (r >> 4) * 8 + (r & 7);
      store_out(e, (size_t)m * e.ld_out + j, silu_ref(v0) * v1);
    }
  } else {  // EPI_QKV
    if (r1 >= N) return;
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
        return;
      }
      const size_t off = (((size_t)seq * e.Hkv + kvh) * e.max_seq + pos) * D;
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
  }
}

__device__ __forceinline__ void epi_pair_rt(const Epilogue &e, int N, int M,
                                            int r, int m, float v0, float v1) {
  switch (e.op) {
    case EPI_STORE: epi_pair<EPI_STORE>(e, N, M, r, m, v0, v1); break;
    case EPI_RESID: epi_pair<EPI_RESID>(e, N, M, r, m, v0, v1); break;
    case EPI_GELU: epi_pair<EPI_GELU>(e, N, M, r, m, v0, v1); break;
    case EPI_SWIGLU: epi_pair<EPI_SWIGLU>(e, N, M, r, m, v0, v1); break;
    default: epi_pair<EPI_QKV>(e, N, M, r, m, v0, v1); break;
  }
}

// ------------------------------------------------------------------------
// bf16 weights, tcgen05 tensor cores
// ------------------------------------------------------------------------
constexpr int kTcThreads = 128;       // 4 warps: TMA, MMA, then epilogue
constexpr int kTcBN = 128;            // weight rows per CTA (MMA M)
constexpr int kTcBK = 64;             // K per stage (one 128-byte row)
constexpr int kTcW = kTcBN * kTcBK * 2;  // weight tile bytes (16 KB)

constexpr int kTcMaxSplit = 8;        // portable cluster size

struct TcParams {
  Epilogue e;
  int M, N, K, S, k_chunks, n_tiles, stages;
};

__host__ __device__ constexpr int tc_stage_bytes(int MT) {
  return kTcW + 2 * MT * kTcBK * 2;
}
__host__ __device__ constexpr int tc_tmem_cols(int MT) {
  return MT < 32 ? 32 : MT;
}

template <int MT, int OP>
__global__ void __launch_bounds__(kTcThreads, 1)
    linear_tc_kernel(const TcParams p, const __grid_constant__ CUtensorMap tw,
                     const __grid_constant__ CUtensorMap tx) {
  constexpr int X_BYTES = MT * kTcBK * 2;    // one bf16 plane of the tile
  constexpr int STAGE = tc_stage_bytes(MT);
  constexpr uint32_t TCOLS = tc_tmem_cols(MT);
  constexpr uint32_t IDESC = umma_idesc_bf16(kTcBN, MT);
  extern __shared__ __align__(1024) uint8_t smem[];
  const int ST = p.stages;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + ST * STAGE);
  uint64_t *empty = full + ST;
  uint64_t *accb = empty + ST;
  __shared__ uint32_t s_tmem;
  __shared__ int s_issued, s_consumed, s_fail;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  // 128-byte-swizzled TMA tiles and UMMA descriptors need 1024-byte
  // aligned stage buffers
  if (smem_u32(smem) & 1023) {
    if (tid == 0) atomicOr(p.e.err, DEV_ERR_SMEM_ALIGN);
    return;
  }
  const int nt = blockIdx.x;
  const int split = blockIdx.y;
  const int mt = blockIdx.z;
  const int per = (p.k_chunks + p.S - 1) / p.S;
  const int kc0 = split * per;
  const int kc1 = min(kc0 + per, p.k_chunks);
  const int nch = kc1 > kc0 ? kc1 - kc0 : 0;

  if (tid == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accb, 1);
    s_issued = 0;
    s_consumed = 0;
    s_fail = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&s_tmem, TCOLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp == 0) {
    if (lane == 0) {
      // TMA producer: weights are read once (evict first), activation tiles
      // are shared by every CTA of the grid (evict last)
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      int c = 0;
      for (; c < nch; ++c) {
        const int s = c % ST;
        if (c >= ST && !mbar_wait_bounded(&empty[s], ((c / ST) - 1) & 1)) {
          s_fail = 1;
          break;
        }
        uint8_t *st = smem + s * STAGE;
        mbar_expect_tx(&full[s], STAGE);
        const int k0 = (kc0 + c) * kTcBK;
        tma_load_2d_hint(st, &tw, &full[s], k0, nt * kTcBN, pol_w);
        tma_load_3d_hint(st + kTcW, &tx, &full[s], k0, mt * MT, 0, pol_x);
        tma_load_3d_hint(st + kTcW + X_BYTES, &tx, &full[s], k0, mt * MT, 1,
                         pol_x);
      }
      s_issued = c;
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issuer: D[128 x MT] += W[128 x 16] . X[MT x 16]^T per k-slice,
      // once for the hi plane and once for the lo plane
      int c = 0;
      for (; c < nch; ++c) {
        const int s = c % ST;
        if (!mbar_wait_bounded(&full[s], (c / ST) & 1)) {
          s_fail = 1;
          break;
        }
        tc_fence_after();
        const uint32_t st = smem_u32(smem + s * STAGE);
        const uint64_t a = umma_desc_sw128(st);
        const uint64_t bh = umma_desc_sw128(st + kTcW);
        const uint64_t bl = umma_desc_sw128(st + kTcW + X_BYTES);
#pragma unroll
        for (int kk = 0; kk < kTcBK / 16; ++kk) {
          umma_bf16(tmem, a + 2 * kk, bh + 2 * kk, IDESC, (c | kk) != 0);
          umma_bf16(tmem, a + 2 * kk, bl + 2 * kk, IDESC, 1);
        }
        umma_commit(&empty[s]);   // stage free once these MMAs are done
      }
      s_consumed = c;
      umma_commit(accb);          // accumulator complete (or nothing issued)
    }
    __syncwarp();
  }

  // ---- epilogue ----
  // 1. the four warps copy the accumulator (TMEM lanes 32*warp..+31) into
  //    shared memory, column-major: tile[m * 128 + r] (the ring is free now)
  const bool acc_ok = mbar_wait_bounded(accb, 0);
  tc_fence_after();
  __syncthreads();  // s_fail / s_consumed visible
  const bool valid = acc_ok && !s_fail && nch > 0;
  float *tile = reinterpret_cast<float *>(smem);
  const int r_own = warp * 32 + lane;
  const uint32_t t_lane = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
  for (int c0 = 0; c0 < MT; c0 += 16) {
    float v[16];
    if (valid) {
      tmem_ld16(t_lane + c0, v);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) tile[(c0 + j) * kTcBN + r_own] = v[j];
  }
  // 2. every split of this tile has staged its partial
  const int S = p.S;
  if (S > 1)
    cluster_sync();
  else
    __syncthreads();
  // 3. this CTA reduces items rank, rank + S, ... of the tile: an item is
  //    one row pair (r, r + 8) at one activation column m; the splits are
  //    summed in rank order
  const int rank = S > 1 ? (int)cluster_ctarank() : 0;
  const uint32_t tile_s = smem_u32(tile);
  const int n_items = (kTcBN / 2) * MT;
#pragma unroll 2
  for (int it = rank * kTcThreads + tid; it < n_items; it += S * kTcThreads) {
    const int m = it >> 6;
    const int pr = it & 63;
    const int r = (pr >> 3) * 16 + (pr & 7);
    const int idx = m * kTcBN + r;
    float v0, v1;
    if (S == 1) {
      v0 = tile[idx];
      v1 = tile[idx + 8];
    } else {
      float a0[kTcMaxSplit], a1[kTcMaxSplit];
#pragma unroll
      for (int q = 0; q < kTcMaxSplit; ++q) {
        if (q < S) {
          a0[q] = ld_dsmem_f32(tile_s + idx * 4, q);
          a1[q] = ld_dsmem_f32(tile_s + (idx + 8) * 4, q);
        }
      }
      v0 = a0[0];
      v1 = a1[0];
#pragma unroll
      for (int q = 1; q < kTcMaxSplit; ++q) {
        if (q < S) {
          v0 += a0[q];
          v1 += a1[q];
        }
      }
    }
    epi_pair<OP>(p.e, p.N, p.M, nt * kTcBN + r, mt * MT + m, v0, v1);
  }
  if (!acc_ok || s_fail) {
    if (tid == 0) atomicOr(p.e.err, DEV_ERR_WAIT_TIMEOUT);
  }

  // teardown: the other CTAs of the cluster are done reading this tile, no
  // TMEM reads in flight, no TMA writes into this CTA's shared memory left
  // (a failed wait may have left issued stages unconsumed)
  tc_fence_before();
  if (S > 1)
    cluster_sync();
  else
    __syncthreads();
  if (tid == 0) {
    for (int c = s_consumed; c < s_issued; ++c)
      mbar_wait_bounded(&full[c % ST], (c / ST) & 1);
  }
  if (warp == 1) tmem_free(tmem, TCOLS);
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
    epi_pair_rt(e, N, M, r, m0 + lane, v0, v1);
  }
}

// ------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------
struct TcPlan {
  int MT, m_tiles, n_tiles, k_chunks, S, stages;
  size_t smem;
};

int tc_mt_for(int M) {
  return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
}

// Stages: about 100 KB of ring per CTA (two CTAs per SM), 2 to 6; the ring
// must also hold the fp32 accumulator tile staged by the epilogue.
int tc_stages_for(int MT) {
  int st = (100 * 1024) / tc_stage_bytes(MT);
  st = st < 2 ? 2 : (st > 6 ? 6 : st);
  while (st * tc_stage_bytes(MT) < kTcBN * MT * 4) ++st;
  return st;
}

size_t tc_smem_for(int MT, int stages) {
  return (size_t)stages * tc_stage_bytes(MT) +
         (2 * stages + 1) * sizeof(uint64_t);
}

TcPlan tc_plan(int M, int N, int K) {
  TcPlan pl{};
  pl.MT = tc_mt_for(M);
  pl.m_tiles = (M + pl.MT - 1) / pl.MT;
  pl.n_tiles = (N + kTcBN - 1) / kTcBN;
  pl.k_chunks = K / kTcBK;
  pl.stages = tc_stages_for(pl.MT);
  pl.smem = tc_smem_for(pl.MT, pl.stages);
  // CTAs resident at once: shared memory allows two per SM up to ~113 KB
  const int per_sm = pl.smem <= 113 * 1024 ? 2 : 1;
  const long slots = (long)per_sm * sm_count();
  const long base = (long)pl.m_tiles * pl.n_tiles;
  int S = 1;
  if (base < slots) {
    long s = slots / base;
    const long by_k = pl.k_chunks / 4;  // keep >= 4 k-chunks per split
    if (s > by_k) s = by_k;
    if (s > kTcMaxSplit) s = kTcMaxSplit;
    S = s < 1 ? 1 : (int)s;
  }
  pl.S = S;
  return pl;
}

template <int MT, int OP>
int launch_tc(const TcParams &p, const CUtensorMap &tw, const CUtensorMap &tx,
              dim3 grid, size_t smem, cudaStream_t st) {
  auto kern = linear_tc_kernel<MT, OP>;
  static bool configured[64] = {};  // per instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    TLLM_CUDA(cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = p.S;   // the splits of one weight tile
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = p.S > 1 ? 1 : 0;
  TLLM_CUDA(cudaLaunchKernelEx(&cfg, kern, p, tw, tx));
  TLLM_LAUNCH_CHECK();
  return TLLM_OK;
}

template <int MT>
int launch_tc_op(const TcParams &p, const CUtensorMap &tw,
                 const CUtensorMap &tx, dim3 grid, size_t smem,
                 cudaStream_t st) {
  switch (p.e.op) {
    case EPI_STORE: return launch_tc<MT, EPI_STORE>(p, tw, tx, grid, smem, st);
    case EPI_RESID: return launch_tc<MT, EPI_RESID>(p, tw, tx, grid, smem, st);
    case EPI_GELU: return launch_tc<MT, EPI_GELU>(p, tw, tx, grid, smem, st);
    case EPI_SWIGLU:
      return launch_tc<MT, EPI_SWIGLU>(p, tw, tx, grid, smem, st);
    default: return launch_tc<MT, EPI_QKV>(p, tw, tx, grid, smem, st);
  }
}

int check_epilogue(const Epilogue &e, int N) {
  TLLM_CHECK_ARG(e.op >= EPI_STORE && e.op <= EPI_QKV, "bad epilogue op %d",
                 e.op);
  if (e.op == EPI_QKV) {
    TLLM_CHECK_ARG(e.D > 0 && e.D % 16 == 0,
                   "head_dim must be a multiple of 16");
    TLLM_CHECK_ARG(N == (e.H + 2 * e.Hkv) * e.D,
                   "QKV rows (%d) != (H + 2 Hkv) * D", N);
    TLLM_CHECK_ARG(e.q_out && e.k_cache && e.v_cache && e.row_seq && e.row_pos,
                   "QKV epilogue needs q_out, caches, row_seq, row_pos");
  } else {
    if (e.op == EPI_SWIGLU)
      TLLM_CHECK_ARG(N % 16 == 0, "SwiGLU rows must be a multiple of 16");
    TLLM_CHECK_ARG(e.out || e.out_split, "NULL output");
    if (e.op == EPI_RESID) {
      TLLM_CHECK_ARG(e.resid, "residual is NULL");
      TLLM_CHECK_ARG(!e.out_split, "the residual output must be fp32");
    }
  }
  return TLLM_OK;
}

}  // namespace
}  // namespace tllm

using namespace tllm;

extern "C" {

int tllm_linear_workspace(int M, int N, int K, size_t *partial_bytes,
                          size_t *counter_bytes) {
  // split-K partials are reduced on chip (distributed shared memory): no
  // global scratch is needed; the entry point stays for callers that size
  // buffers generically
  TLLM_CHECK_ARG(partial_bytes && counter_bytes, "NULL output");
  TLLM_CHECK_ARG(M >= 0 && N >= 0 && K >= 0, "negative shape");
  *partial_bytes = 0;
  *counter_bytes = 0;
  return TLLM_OK;
}

// y = epilogue(x @ W^T); see tllm.h for the argument encoding.
int tllm_linear(const void *x, int x_dtype, int x_plane_rows, const void *w,
                int w_dtype, int M, int N, int K, int op, const float *bias,
                void *out, int out_dtype, int out_plane_rows, int ld_out,
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
  TLLM_CHECK_ARG(w_dtype == TLLM_F32 || w_dtype == TLLM_BF16,
                 "w_dtype must be F32 or BF16");
  TLLM_CHECK_ARG(out_dtype == TLLM_F32 || out_dtype == TLLM_SPLIT,
                 "out_dtype must be F32 or SPLIT");
  TLLM_CHECK_ARG(((uintptr_t)x & 15) == 0 && ((uintptr_t)w & 15) == 0,
                 "x and W must be 16-byte aligned");
  Epilogue e{};
  e.op = op;
  e.bias = bias;
  e.ld_out = ld_out > 0 ? ld_out : (op == EPI_SWIGLU ? N / 2 : N);
  if (out_dtype == TLLM_SPLIT) {
    TLLM_CHECK_ARG(out_plane_rows >= M, "out_plane_rows (%d) < M (%d)",
                   out_plane_rows, M);
    e.out_split = static_cast<uint16_t *>(out);
    e.out_plane = (size_t)out_plane_rows * e.ld_out;
  } else {
    e.out = static_cast<float *>(out);
  }
  e.resid = resid;
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
    TLLM_CHECK_ARG(x_dtype == TLLM_F32, "fp32 weights take fp32 activations");
    TLLM_CHECK_ARG(K % 4 == 0, "K must be a multiple of 4");
    const int pairs = ((N + 15) / 16) * 8;
    const int blocks = (pairs + kF32Warps - 1) / kF32Warps;
    for (int m0 = 0; m0 < M; m0 += 8) {
      linear_f32_kernel<8><<<blocks, kF32Warps * 32, 0, st>>>(
          static_cast<const float *>(x), static_cast<const float *>(w), e, M,
          N, K, m0);
      TLLM_LAUNCH_CHECK();
    }
    return TLLM_OK;
  }

  TLLM_CHECK_ARG(x_dtype == TLLM_SPLIT,
                 "bf16 weights take TLLM_SPLIT activations (tllm_split_bf16)");
  TLLM_CHECK_ARG(K > 0 && K % kTcBK == 0, "bf16 linear needs K %% 64 == 0 (K=%d)",
                 K);
  TLLM_CHECK_ARG(x_plane_rows >= M, "x_plane_rows (%d) < M (%d)", x_plane_rows,
                 M);
  (void)partial;
  (void)partial_bytes;
  (void)counters;
  const TcPlan pl = tc_plan(M, N, K);
  const int S = pl.S;
  CUtensorMap tw, tx;
  rc = make_map_2d(&tw, w, TLLM_BF16, K, N, (long)K * 2, kTcBK, kTcBN, true);
  if (rc) return rc;
  const long xd[3] = {K, x_plane_rows, 2};
  const long xs[2] = {(long)K * 2, (long)x_plane_rows * K * 2};
  const int xb[3] = {kTcBK, pl.MT, 1};
  rc = make_map(&tx, x, TLLM_BF16, 3, xd, xs, xb, true);
  if (rc) return rc;
  TcParams p;
  p.e = e;
  p.M = M;
  p.N = N;
  p.K = K;
  p.S = S;
  p.k_chunks = pl.k_chunks;
  p.n_tiles = pl.n_tiles;
  p.stages = pl.stages;
  dim3 grid(pl.n_tiles, S, pl.m_tiles);
  switch (pl.MT) {
    case 16: return launch_tc_op<16>(p, tw, tx, grid, pl.smem, st);
    case 32: return launch_tc_op<32>(p, tw, tx, grid, pl.smem, st);
    case 64: return launch_tc_op<64>(p, tw, tx, grid, pl.smem, st);
    case 128: return launch_tc_op<128>(p, tw, tx, grid, pl.smem, st);
    default: return launch_tc_op<256>(p, tw, tx, grid, pl.smem, st);
  }
}

}  // extern "C"
