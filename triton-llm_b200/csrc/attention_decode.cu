// Split-KV GQA decode attention for sm_100a.
//
// Computes, for every sequence b and query head h of a ragged decode batch,
//     out[b,h,:] = softmax(q[b,h,:] . K[b,kvh,:len_b,:]^T * scale) V[b,kvh,:len_b,:]
// with kvh = h / (n_head / n_kv_head) -- the math of the reference kernel
// triton_llm/kernels/attention_gqa.py:76-146 (q pre-scaled, online softmax,
// one divide at the end), restructured for B200:
//
//  * one CTA per (sequence, kv head, split of the keys); the CTA holds all
//    query heads of its KV group, so each K/V byte is read from HBM once
//    (the reference re-reads K/V once per query head);
//  * a producer warp streams K and V tiles with 3-D tiled TMA loads
//    (cp.async.bulk.tensor into this CTA only) into a 4-stage shared-memory ring
//    guarded by full/empty mbarriers; four consumer warps read 128-bit
//    vectors from shared memory;
//  * scores are reduced with warp shuffles and folded into a per-warp
//    online softmax (base-2 exponent with log2(e) folded into the q scale);
//  * splits of one (sequence, kv head) are merged by the last CTA to finish,
//    chosen by an atomic ticket (no CTA ever waits for another one).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <mutex>

#include "common.cuh"
#include "mma_sync.cuh"

namespace tllm {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();  // tma.cu

namespace {

constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kStages = 4;
constexpr int kTileBytes = 8192;  // bytes of one K tile (same for V)
constexpr int kMaxSplits = 128;
constexpr float kLog2e = 1.4426950408889634f;

template <typename T>
struct Vec;
template <>
struct Vec<float> {
  static constexpr int N = 4;
  __device__ static void unpack(const uint4 &v, float *f) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  }
};
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void unpack(const uint4 &v, float *f) {
    f[0] = bf16lo(v.x);
    f[1] = bf16hi(v.x);
    f[2] = bf16lo(v.y);
    f[3] = bf16hi(v.y);
    f[4] = bf16lo(v.z);
    f[5] = bf16hi(v.z);
    f[6] = bf16lo(v.w);
    f[7] = bf16hi(v.w);
  }
};

struct DecodeParams {
  const float *q;        // row b, head h at q + b * q_sb + h * q_sh
  float *out;            // row b, head h at out + b * o_sb + h * o_sh
  uint16_t *out_split;   // or operand-format output (TLLM_SPLIT / TLLM_BF16)
  long out_plane;        //   at the same element offsets, planes out_plane
  int out_planes;        //   elements apart, 2 or 1 planes
  const int *seq_lens;   // (B,) or null (every sequence has max_len keys)
  const int *row_seq;    // (B,) cache sequence of each row, or null (= row)
  long q_sb, q_sh, o_sb, o_sh;
  float *part_acc;       // (B, n_head, max_splits, D)
  float *part_ml;        // (B, n_head, max_splits, 2)
  int *counters;         // (B, n_y)
  int *err;              // device error word
  int n_head, n_kv, group, n_gsub;
  int n_y;               // kv heads x query-head groups (gridDim.y)
  int max_seq, max_len, chunk, max_splits;
  float qscale;          // sm_scale * log2(e)
};

__device__ __forceinline__ void store_o(const DecodeParams &p, long idx,
                                        float v) {
  if (p.out_split)
    store_act(p.out_split, (size_t)p.out_plane, (size_t)idx, v, p.out_planes);
  else
    p.out[idx] = v;
}

// Shape constants of one instantiation.
template <typename T, int D>
struct Shape {
  static constexpr int VEC = Vec<T>::N;               // elements per 16 B
  static constexpr int VPR = D / VEC;                 // vectors per row
  static constexpr int LPR = VPR < 32 ? VPR : 32;     // lanes per row
  static constexpr int NV = VPR / LPR;                // vectors per lane
  static constexpr int RPW = 32 / LPR;                // rows per warp step
  static constexpr int ROW_BYTES = D * (int)sizeof(T);
  static constexpr int TILE_ROWS = kTileBytes / ROW_BYTES;
  static constexpr int ITERS = TILE_ROWS / (kConsumerWarps * RPW);
  static_assert(VPR >= 1 && ITERS >= 1, "unsupported head_dim");
  static_assert(TILE_ROWS <= 256, "TMA box rows");
};

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

template <typename T, int D, int G>
__global__ void __launch_bounds__(kThreads)
    gqa_decode_kernel(const DecodeParams p,
                      const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv) {
  griddep_launch();
  griddep_wait();   // q, lengths and the cache come from earlier kernels
  using S = Shape<T, D>;
  extern __shared__ __align__(1024) uint8_t smem[];
  T *k_st = reinterpret_cast<T *>(smem);
  T *v_st = reinterpret_cast<T *>(smem + kStages * kTileBytes);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + 2 * kStages * kTileBytes);
  uint64_t *empty = full + kStages;
  __shared__ int s_flag;

  const int b = blockIdx.z;
  const int y = blockIdx.y;
  const int kvh = y / p.n_gsub;
  const int gsub = y - kvh * p.n_gsub;
  const int j = blockIdx.x;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  int len = p.seq_lens ? p.seq_lens[b] : p.max_len;
  len = len < 0 ? 0 : (len > p.max_seq ? p.max_seq : len);
  int n_splits = (len + p.chunk - 1) / p.chunk;
  if (n_splits < 1) n_splits = 1;
  if (n_splits > p.max_splits) {  // caller's max_len bound was too small
    if (tid == 0 && j == 0) atomicOr(p.err, DEV_ERR_LEN_CLAMPED);
    n_splits = p.max_splits;
    len = n_splits * p.chunk;
  }
  if (j >= n_splits) return;
  const int start = j * p.chunk;
  const int end = min(start + p.chunk, len);
  const int nrows = end > start ? end - start : 0;
  const int ntiles = (nrows + S::TILE_ROWS - 1) / S::TILE_ROWS;
  const int head0 = kvh * p.group + gsub * G;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
    s_flag = 0;
  }
  __syncthreads();

  bool failed = false;
  // ---------------------------------------------------------------- producer
  if (warp == kConsumerWarps) {
    if (lane == 0) {
      const int plane = (p.row_seq ? p.row_seq[b] : b) * p.n_kv + kvh;
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % kStages;
        if (t >= kStages) {
          if (!mbar_wait_bounded(&empty[s], ((t / kStages) - 1) & 1)) {
            failed = true;
            break;
          }
        }
        mbar_expect_tx(&full[s], 2 * kTileBytes);
        const int row = start + t * S::TILE_ROWS;
        tma_load_3d(k_st + s * (kTileBytes / sizeof(T)), &tmk, &full[s], 0, row,
                    plane);
        tma_load_3d(v_st + s * (kTileBytes / sizeof(T)), &tmv, &full[s], 0, row,
                    plane);
      }
    }
  }

  // ---------------------------------------------------------------- consumers
  // Per-lane state: q slice, accumulators, running max / sum per head.
  float acc[G][S::NV * S::VEC];
  float m_run[G], l_run[G];
  const int rlane = lane / S::LPR;  // row within a warp step
  const int clane = lane % S::LPR;  // vector column of this lane
  if (warp < kConsumerWarps) {
    float qr[G][S::NV * S::VEC];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float *qp = p.q + b * p.q_sb + (long)(head0 + g) * p.q_sh;
#pragma unroll
      for (int v = 0; v < S::NV; ++v) {
        const float4 *q4 =
            reinterpret_cast<const float4 *>(qp + (clane + v * S::LPR) * S::VEC);
#pragma unroll
        for (int e = 0; e < S::VEC / 4; ++e) {
          float4 t = q4[e];
          qr[g][v * S::VEC + 4 * e + 0] = t.x * p.qscale;
          qr[g][v * S::VEC + 4 * e + 1] = t.y * p.qscale;
          qr[g][v * S::VEC + 4 * e + 2] = t.z * p.qscale;
          qr[g][v * S::VEC + 4 * e + 3] = t.w * p.qscale;
        }
      }
#pragma unroll
      for (int e = 0; e < S::NV * S::VEC; ++e) acc[g][e] = 0.f;
      m_run[g] = -INFINITY;
      l_run[g] = 0.f;
    }

    for (int t = 0; t < ntiles; ++t) {
      const int s = t % kStages;
      // every lane waits (acquire); the outcome is made warp-uniform
      const bool ok =
          __all_sync(0xffffffffu, mbar_wait_bounded(&full[s], (t / kStages) & 1));
      if (!ok) {
        failed = true;
        break;
      }
      const T *kt = k_st + s * (kTileBytes / sizeof(T));
      const T *vt = v_st + s * (kTileBytes / sizeof(T));
      const int valid_rows = min(S::TILE_ROWS, nrows - t * S::TILE_ROWS);

      float sc[S::ITERS][G];
#pragma unroll
      for (int it = 0; it < S::ITERS; ++it) {
        const int r = (warp * S::ITERS + it) * S::RPW + rlane;
        float part[G];
#pragma unroll
        for (int g = 0; g < G; ++g) part[g] = 0.f;
#pragma unroll
        for (int v = 0; v < S::NV; ++v) {
          const uint4 raw = *reinterpret_cast<const uint4 *>(
              kt + r * D + (clane + v * S::LPR) * S::VEC);
          float kf[S::VEC];
          Vec<T>::unpack(raw, kf);
#pragma unroll
          for (int g = 0; g < G; ++g)
#pragma unroll
            for (int e = 0; e < S::VEC; ++e)
              part[g] = fmaf(qr[g][v * S::VEC + e], kf[e], part[g]);
        }
#pragma unroll
        for (int off = 1; off < S::LPR; off <<= 1)
#pragma unroll
          for (int g = 0; g < G; ++g)
            part[g] += __shfl_xor_sync(0xffffffffu, part[g], off);
        const bool ok = r < valid_rows;
#pragma unroll
        for (int g = 0; g < G; ++g) sc[it][g] = ok ? part[g] : -INFINITY;
      }

      // online softmax update (warp-uniform max)
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float tmax = sc[0][g];
#pragma unroll
        for (int it = 1; it < S::ITERS; ++it) tmax = fmaxf(tmax, sc[it][g]);
#pragma unroll
        for (int off = S::LPR; off < 32; off <<= 1)
          tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
        const float mnew = fmaxf(m_run[g], tmax);
        if (mnew != -INFINITY) {
          const float alpha = fast_exp2(m_run[g] - mnew);
          m_run[g] = mnew;
          l_run[g] *= alpha;
#pragma unroll
          for (int e = 0; e < S::NV * S::VEC; ++e) acc[g][e] *= alpha;
#pragma unroll
          for (int it = 0; it < S::ITERS; ++it) {
            const float pv = fast_exp2(sc[it][g] - mnew);  // exp2(-inf) = 0
            sc[it][g] = pv;
            l_run[g] += pv;
          }
        } else {
#pragma unroll
          for (int it = 0; it < S::ITERS; ++it) sc[it][g] = 0.f;
        }
      }

      // P . V
#pragma unroll
      for (int it = 0; it < S::ITERS; ++it) {
        const int r = (warp * S::ITERS + it) * S::RPW + rlane;
        if (r < valid_rows) {
#pragma unroll
          for (int v = 0; v < S::NV; ++v) {
            const uint4 raw = *reinterpret_cast<const uint4 *>(
                vt + r * D + (clane + v * S::LPR) * S::VEC);
            float vf[S::VEC];
            Vec<T>::unpack(raw, vf);
#pragma unroll
            for (int g = 0; g < G; ++g)
#pragma unroll
              for (int e = 0; e < S::VEC; ++e)
                acc[g][v * S::VEC + e] =
                    fmaf(sc[it][g], vf[e], acc[g][v * S::VEC + e]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }

    // reduce the row groups of this warp (lanes that share a column slice)
#pragma unroll
    for (int off = S::LPR; off < 32; off <<= 1)
#pragma unroll
      for (int g = 0; g < G; ++g) {
        l_run[g] += __shfl_xor_sync(0xffffffffu, l_run[g], off);
#pragma unroll
        for (int e = 0; e < S::NV * S::VEC; ++e)
          acc[g][e] += __shfl_xor_sync(0xffffffffu, acc[g][e], off);
      }
  }
  if (failed) {
    atomicOr(p.err, DEV_ERR_WAIT_TIMEOUT);
    s_flag = 1;
  }
  __syncthreads();  // all tiles consumed: the ring is free for reuse
  if (s_flag) {
    // Give in-flight copies a bounded chance to land before the CTA exits.
    if (tid == 0)
      for (int s = 0; s < kStages; ++s) mbar_wait_bounded(&full[s], 0, 1u << 12);
    return;
  }

  // ------------------------------------------- merge the 4 consumer warps
  float *w_acc = reinterpret_cast<float *>(smem);            // [4][G][D]
  float *w_m = w_acc + kConsumerWarps * G * D;               // [4][G]
  float *w_l = w_m + kConsumerWarps * G;                     // [4][G]
  if (warp < kConsumerWarps) {
    if (rlane == 0) {
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int v = 0; v < S::NV; ++v)
#pragma unroll
          for (int e = 0; e < S::VEC; ++e)
            w_acc[(warp * G + g) * D + (clane + v * S::LPR) * S::VEC + e] =
                acc[g][v * S::VEC + e];
    }
    if (lane == 0) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        w_m[warp * G + g] = m_run[g];
        w_l[warp * G + g] = l_run[g];
      }
    }
  }
  __syncthreads();

  const bool single = (n_splits == 1);
  for (int idx = tid; idx < G * D; idx += kThreads) {
    const int g = idx / D;
    const int d = idx - g * D;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) mx = fmaxf(mx, w_m[w * G + g]);
    float num = 0.f, den = 0.f;
    if (mx != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float wm = w_m[w * G + g];
        if (wm != -INFINITY) {
          const float sc = fast_exp2(wm - mx);
          num = fmaf(w_acc[(w * G + g) * D + d], sc, num);
          den = fmaf(w_l[w * G + g], sc, den);
        }
      }
    }
    const size_t row = (size_t)b * p.n_head + head0 + g;
    if (single) {
      store_o(p, b * p.o_sb + (long)(head0 + g) * p.o_sh + d, den > 0.f ? num / den : 0.f);
    } else {
      const size_t slot = row * p.max_splits + j;
      p.part_acc[slot * D + d] = num;
      if (d == 0) {
        p.part_ml[slot * 2 + 0] = mx;
        p.part_ml[slot * 2 + 1] = den;
      }
    }
  }
  if (single) return;

  // ------------------------------------ last CTA of this (b, y) merges splits
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    int *ctr = p.counters + (size_t)b * p.n_y + y;
    const int ticket = atomicAdd(ctr, 1);
    s_flag = (ticket == n_splits - 1) ? 2 : 0;
    if (s_flag) *ctr = 0;  // every other CTA has taken its ticket already
  }
  __syncthreads();
  if (s_flag != 2) return;
  __threadfence();

  float *sw = reinterpret_cast<float *>(smem);  // [G][max_splits] weights
  for (int g = warp; g < G; g += kConsumerWarps + 1) {
    const size_t base = ((size_t)b * p.n_head + head0 + g) * p.max_splits;
    float mx = -INFINITY;
    for (int s = lane; s < n_splits; s += 32)
      mx = fmaxf(mx, __ldcg(&p.part_ml[(base + s) * 2]));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float den = 0.f;
    for (int s = lane; s < n_splits; s += 32) {
      const float ms = __ldcg(&p.part_ml[(base + s) * 2]);
      const float w = (ms == -INFINITY) ? 0.f : fast_exp2(ms - mx);
      sw[g * kMaxSplits + s] = w;
      den = fmaf(__ldcg(&p.part_ml[(base + s) * 2 + 1]), w, den);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
      den += __shfl_xor_sync(0xffffffffu, den, off);
    const float inv = den > 0.f ? 1.f / den : 0.f;
    for (int s = lane; s < n_splits; s += 32) sw[g * kMaxSplits + s] *= inv;
  }
  __syncthreads();
  for (int idx = tid; idx < G * D; idx += kThreads) {
    const int g = idx / D;
    const int d = idx - g * D;
    const size_t row = (size_t)b * p.n_head + head0 + g;
    const size_t base = row * p.max_splits;
    float o = 0.f;
    for (int s = 0; s < n_splits; ++s)
      o = fmaf(sw[g * kMaxSplits + s], __ldcg(&p.part_acc[(base + s) * D + d]), o);
    store_o(p, b * p.o_sb + (long)(head0 + g) * p.o_sh + d, o);
  }
}

// --------------------------------------------------------------------------
// Tensor-core variant for bf16 caches (head_dim 64 / 128).
//
// Same decomposition, ring and split merge as above, but the products run on
// the tensor cores with mma.sync m16n8k16 (bf16 in, fp32 accumulate), with
// the keys as the M rows and the CTA's query heads as the N columns:
//   S^T (16 keys x 8 heads)  = K_w (16 x D) . Q^T      per consumer warp
//   O^T (D x 8 heads)       += V_w^T (D x 16 keys) . P^T
// where warp w of a consumer group owns keys [16 (w % 4), + 16) of every
// 64-key tile the group takes (tiles t = group mod NG); a decode
// group of G <= 8 heads (16 with two n8 blocks) fills the narrow side, so
// half the MMAs of the heads-as-rows form are spent. q and p are each split
// into a bf16 head and a bf16 residual (x = hi + lo) and both halves are
// multiplied, so scores and weights keep ~16 mantissa bits: the result
// matches fp32 arithmetic on the bf16 cache to ~1e-6 relative. K/V tiles
// arrive through TMA with 128-byte swizzle (64-dim sub-tiles of 128 B rows),
// which makes the ldmatrix reads bank-conflict free.
// --------------------------------------------------------------------------
// transpose of the 8 x 8 bf16 matrix held in the C / A fragment layout
// (lane l: row l / 4, columns 2 (l % 4), + 1)
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t r;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}


// NG consumer groups of four warps: group i takes the tiles t = i (mod NG)
// with its own online-softmax state, so NG tiles are in the consumers' hands
// at once (one group's dependent MMA / shuffle / exp chain per tile bounds a
// CTA otherwise). The ring depth is a multiple of NG, so every ring slot
// belongs to one group, which waits for that slot's fills strictly in order
// (a slot shared by two groups would let one group pass a parity wait on a
// fill two phases old while the other group's fill is still in flight).
template <int D, int NG>
struct MmaShape {
  static constexpr int KT = 64;                    // keys per tile
  static constexpr int SUB = D / 64;               // 128-byte sub-tiles per row
  static constexpr int SUB_BYTES = KT * 128;       // 8 KB
  static constexpr int TILE_BYTES = SUB * SUB_BYTES;
  static constexpr int STAGES = (D <= 64 || NG == 2) ? 4 : 3;
  static constexpr int KSTEPS = D / 16;
  static constexpr int CONSUMERS = 4 * NG;         // consumer warps
  static constexpr int THREADS = (CONSUMERS + 1) * 32;
  static constexpr size_t RING =
      2 * (size_t)STAGES * TILE_BYTES + 2 * STAGES * sizeof(uint64_t);
  static_assert(STAGES % NG == 0, "every ring slot must belong to one group");
};

// CTAs per SM the shared memory allows each instance, given to the register
// allocator as its minimum (one column block only: two need more registers).
__host__ __device__ constexpr int mma_min_blocks(int D, int QB, int NG) {
  return QB > 1 ? 1 : D <= 64 ? 3 : NG == 2 ? 1 : 2;
}

template <int D, int QB, int NG>
__global__ void __launch_bounds__(MmaShape<D, NG>::THREADS, mma_min_blocks(D, QB, NG))
    gqa_decode_mma_kernel(const DecodeParams p, const int G,
                          const __grid_constant__ CUtensorMap tmk,
                          const __grid_constant__ CUtensorMap tmv) {
  griddep_launch();
  using S = MmaShape<D, NG>;
  constexpr int NCW = S::CONSUMERS;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t *k_st = smem;
  uint8_t *v_st = smem + S::STAGES * S::TILE_BYTES;
  uint64_t *full =
      reinterpret_cast<uint64_t *>(smem + 2 * S::STAGES * S::TILE_BYTES);
  uint64_t *empty = full + S::STAGES;
  __shared__ int s_flag;
  // 128-byte-swizzled TMA tiles need 1024-byte aligned stage buffers
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) atomicOr(p.err, DEV_ERR_SMEM_ALIGN);
    return;
  }

  const int b = blockIdx.z;
  const int y = blockIdx.y;
  const int kvh = y / p.n_gsub;
  const int gsub = y - kvh * p.n_gsub;
  const int j = blockIdx.x;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int grp = warp >> 2;   // consumer group (tiles t = grp mod NG)
  const int wq = warp & 3;     // key quarter of every tile of the group

  // the barriers need nothing from earlier kernels: set them up before the
  // dependency wait
  if (tid == 0) {
    for (int s = 0; s < S::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);   // the four warps of the slot's group
    }
    fence_mbar_init();
    s_flag = 0;
  }
  __syncthreads();
  griddep_wait();   // q, lengths and the cache come from earlier kernels
  // both index loads in flight together
  const int cache_seq = p.row_seq ? p.row_seq[b] : b;
  int len = p.seq_lens ? p.seq_lens[b] : p.max_len;
  len = len < 0 ? 0 : (len > p.max_seq ? p.max_seq : len);
  const int chunk = p.chunk;
  int n_splits = (len + chunk - 1) / chunk;
  if (n_splits < 1) n_splits = 1;
  if (n_splits > p.max_splits) {
    if (tid == 0 && j == 0) atomicOr(p.err, DEV_ERR_LEN_CLAMPED);
    n_splits = p.max_splits;
    len = n_splits * chunk;
  }
  if (j >= n_splits) return;
  const int start = j * chunk;
  const int end = min(start + chunk, len);
  const int nrows = end > start ? end - start : 0;
  const int ntiles = (nrows + S::KT - 1) / S::KT;
  const int head0 = kvh * p.group + gsub * G;

  bool failed = false;
  if (warp == NCW) {
    if (lane == 0) {
      const int plane = cache_seq * p.n_kv + kvh;
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % S::STAGES;
        if (t >= S::STAGES &&
            !mbar_wait_bounded(&empty[s], ((t / S::STAGES) - 1) & 1)) {
          failed = true;
          break;
        }
        mbar_expect_tx(&full[s], 2 * S::TILE_BYTES);
        const int row = start + t * S::KT;
#pragma unroll
        for (int sub = 0; sub < S::SUB; ++sub) {
          tma_load_3d(k_st + s * S::TILE_BYTES + sub * S::SUB_BYTES, &tmk,
                      &full[s], sub * 64, row, plane);
          tma_load_3d(v_st + s * S::TILE_BYTES + sub * S::SUB_BYTES, &tmv,
                      &full[s], sub * 64, row, plane);
        }
      }
    }
  }

  // Swapped operands: the keys are the MMA's M rows and the (few) query
  // heads its N columns, so a decode group of G <= 8 heads fills an n8
  // block instead of 3 of the 16 rows of an m16 block:
  //   S^T (16 keys x 8 heads)  = K_w (16 x D) . Q^T        per consumer warp
  //   O^T (D x 8 heads)       += V_w^T (D x 16 keys) . P^T
  // C fragments hold rows r0, r0 + 8 (keys, resp. dims) and columns
  // cq, cq + 1 (heads); P^T reaches the B-operand layout by transposing its
  // two 8 x 8 blocks in registers (movmatrix).
  const int r0 = lane >> 2;
  const int cq = (lane & 3) * 2;
  float o[QB][D / 16][4];
  float m_r[QB][2], l_r[QB][2];
#pragma unroll
  for (int qb = 0; qb < QB; ++qb) {
    m_r[qb][0] = m_r[qb][1] = -INFINITY;
    l_r[qb][0] = l_r[qb][1] = 0.f;
  }
  if (warp < NCW) {
    // ---- Q^T fragments (B operand: k = dims, n = heads), scaled, hi / lo
    uint32_t qh[QB][S::KSTEPS][2], ql[QB][S::KSTEPS][2];
#pragma unroll
    for (int qb = 0; qb < QB; ++qb) {
      const int g = qb * 8 + r0;
#pragma unroll
      for (int kk = 0; kk < S::KSTEPS; ++kk) {
#pragma unroll
        for (int f = 0; f < 2; ++f) {
          const int col = kk * 16 + cq + 8 * f;
          float x0 = 0.f, x1 = 0.f;
          if (g < G) {
            const float2 v = *reinterpret_cast<const float2 *>(
                p.q + b * p.q_sb + (long)(head0 + g) * p.q_sh + col);
            x0 = v.x * p.qscale;
            x1 = v.y * p.qscale;
          }
          split_bf16x2(x0, x1, qh[qb][kk][f], ql[qb][kk][f]);
        }
      }
#pragma unroll
      for (int mb = 0; mb < D / 16; ++mb)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[qb][mb][e] = 0.f;
    }

    // ldmatrix lane addressing: K as the A operand (rows = keys), V^T as
    // the A operand via .trans (source rows = keys)
    const int a_key = wq * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
    const int a_dof = ((lane >> 4) & 1) * 8;
    const int t_key = wq * 16 + ((lane >> 4) & 1) * 8 + (lane & 7);
    const int t_dof = ((lane >> 3) & 1) * 8;

    for (int t = grp; t < ntiles; t += NG) {
      const int s = t % S::STAGES;
      const bool ok = __all_sync(
          0xffffffffu, mbar_wait_bounded(&full[s], (t / S::STAGES) & 1));
      if (!ok) {
        failed = true;
        break;
      }
      uint8_t *kt = k_st + s * S::TILE_BYTES;
      uint8_t *vt = v_st + s * S::TILE_BYTES;
      const int valid = min(S::KT, nrows - t * S::KT);

      // ---- S^T = K Q^T over this warp's 16 keys
      float sc[QB][4];
#pragma unroll
      for (int qb = 0; qb < QB; ++qb)
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[qb][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < S::KSTEPS; ++kk) {
        const int dim = kk * 16 + a_dof;
        const int sub = dim >> 6;
        const int chunk = (dim & 63) >> 3;
        const uint32_t addr = smem_u32(kt + sub * S::SUB_BYTES + a_key * 128 +
                                       ((chunk ^ (a_key & 7)) << 4));
        uint32_t ka[4];
        ldsm_x4(addr, ka[0], ka[1], ka[2], ka[3]);
#pragma unroll
        for (int qb = 0; qb < QB; ++qb) {
          mma_bf16(sc[qb], ka, qh[qb][kk][0], qh[qb][kk][1]);
          mma_bf16(sc[qb], ka, ql[qb][kk][0], ql[qb][kk][1]);
        }
      }
      const bool partial = valid < S::KT;
      if (partial) {
#pragma unroll
        for (int qb = 0; qb < QB; ++qb)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = wq * 16 + r0 + 8 * (e >> 1);
            if (key >= valid) sc[qb][e] = -INFINITY;
          }
      }

      // ---- online softmax per head (columns cq + c; keys r0, r0 + 8 here,
      //      the other 14 keys in the lanes of the same lane % 4)
      uint32_t pb[QB][4];   // P^T B fragments: hi b0, hi b1, lo b0, lo b1
#pragma unroll
      for (int qb = 0; qb < QB; ++qb) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float mx = fmaxf(sc[qb][c], sc[qb][c + 2]);
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
          const float mn = fmaxf(m_r[qb][c], mx);
          const float msafe = (mn == -INFINITY) ? 0.f : mn;
          if (mn != m_r[qb][c]) {
            const float alpha = fast_exp2(m_r[qb][c] - msafe);  // 0 when m was -inf
            l_r[qb][c] *= alpha;
#pragma unroll
            for (int mb = 0; mb < D / 16; ++mb) {
              o[qb][mb][c] *= alpha;
              o[qb][mb][c + 2] *= alpha;
            }
            m_r[qb][c] = mn;
          }
          sc[qb][c] = fast_exp2(sc[qb][c] - msafe);
          sc[qb][c + 2] = fast_exp2(sc[qb][c + 2] - msafe);
          l_r[qb][c] += sc[qb][c] + sc[qb][c + 2];
        }
        uint32_t h01, l01, h23, l23;
        split_bf16x2(sc[qb][0], sc[qb][1], h01, l01);   // keys r0
        split_bf16x2(sc[qb][2], sc[qb][3], h23, l23);   // keys r0 + 8
        pb[qb][0] = movmatrix_t(h01);
        pb[qb][1] = movmatrix_t(h23);
        pb[qb][2] = movmatrix_t(l01);
        pb[qb][3] = movmatrix_t(l23);
      }

      if (partial && wq * 16 + 16 > valid) {
        // rows past the end may hold anything (even NaN): zero this warp's
        // share of them so that 0 * row stays 0 in P . V
        for (int idx = lane; idx < 16 * S::SUB * 8; idx += 32) {
          const int key = wq * 16 + idx / (S::SUB * 8);
          const int rem = idx % (S::SUB * 8);
          if (key >= valid)
            *reinterpret_cast<uint4 *>(vt + (rem >> 3) * S::SUB_BYTES +
                                       key * 128 + ((rem & 7) << 4)) =
                make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
      }

      // ---- O^T += V^T P^T
#pragma unroll
      for (int mb = 0; mb < D / 16; ++mb) {
        const int dim = mb * 16 + t_dof;
        const int sub = dim >> 6;
        const int chunk = (dim & 63) >> 3;
        const uint32_t addr = smem_u32(vt + sub * S::SUB_BYTES + t_key * 128 +
                                       ((chunk ^ (t_key & 7)) << 4));
        uint32_t va[4];
        ldsm_x4_t(addr, va[0], va[1], va[2], va[3]);
#pragma unroll
        for (int qb = 0; qb < QB; ++qb) {
          mma_bf16(o[qb][mb], va, pb[qb][0], pb[qb][1]);
          mma_bf16(o[qb][mb], va, pb[qb][2], pb[qb][3]);
        }
      }
      if (partial) fence_proxy_async();  // generic writes before the next TMA
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    // sum the head weights over the 8 lanes of each lane % 4 (keys)
#pragma unroll
    for (int qb = 0; qb < QB; ++qb)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        l_r[qb][c] += __shfl_xor_sync(0xffffffffu, l_r[qb][c], 4);
        l_r[qb][c] += __shfl_xor_sync(0xffffffffu, l_r[qb][c], 8);
        l_r[qb][c] += __shfl_xor_sync(0xffffffffu, l_r[qb][c], 16);
      }
  }
  if (failed) {
    atomicOr(p.err, DEV_ERR_WAIT_TIMEOUT);
    s_flag = 1;
  }
  __syncthreads();
  if (s_flag) {
    if (tid == 0)
      for (int s = 0; s < S::STAGES; ++s)
        mbar_wait_bounded(&full[s], 0, 1u << 12);
    return;
  }

  // ---- merge the consumer warps (heads < G), in warp order
  float *w_acc = reinterpret_cast<float *>(smem);   // [NCW][G][D]
  float *w_m = w_acc + NCW * G * D;      // [NCW][G]
  float *w_l = w_m + NCW * G;            // [NCW][G]
  if (warp < NCW) {
#pragma unroll
    for (int qb = 0; qb < QB; ++qb) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int g = qb * 8 + cq + c;
        if (g < G) {
#pragma unroll
          for (int mb = 0; mb < D / 16; ++mb) {
            w_acc[(warp * G + g) * D + mb * 16 + r0] = o[qb][mb][c];
            w_acc[(warp * G + g) * D + mb * 16 + r0 + 8] = o[qb][mb][c + 2];
          }
          if (r0 == 0) {
            w_m[warp * G + g] = m_r[qb][c];
            w_l[warp * G + g] = l_r[qb][c];
          }
        }
      }
    }
  }
  __syncthreads();

  const bool single = (n_splits == 1);
  for (int idx = tid; idx < G * D; idx += S::THREADS) {
    const int g = idx / D;
    const int d = idx - g * D;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < NCW; ++w) mx = fmaxf(mx, w_m[w * G + g]);
    float num = 0.f, den = 0.f;
    if (mx != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NCW; ++w) {
        const float wm = w_m[w * G + g];
        if (wm != -INFINITY) {
          const float sc = fast_exp2(wm - mx);
          num = fmaf(w_acc[(w * G + g) * D + d], sc, num);
          den = fmaf(w_l[w * G + g], sc, den);
        }
      }
    }
    const size_t row = (size_t)b * p.n_head + head0 + g;
    if (single) {
      store_o(p, b * p.o_sb + (long)(head0 + g) * p.o_sh + d, den > 0.f ? num / den : 0.f);
    } else {
      const size_t slot = row * p.max_splits + j;
      p.part_acc[slot * D + d] = num;
      if (d == 0) {
        p.part_ml[slot * 2 + 0] = mx;
        p.part_ml[slot * 2 + 1] = den;
      }
    }
  }
  if (single) return;

  __threadfence();
  __syncthreads();
  if (tid == 0) {
    int *ctr = p.counters + (size_t)b * p.n_y + y;
    const int ticket = atomicAdd(ctr, 1);
    s_flag = (ticket == n_splits - 1) ? 2 : 0;
    if (s_flag) *ctr = 0;
  }
  __syncthreads();
  if (s_flag != 2) return;
  __threadfence();

  // Merge the splits of this (sequence, KV group) in split order: the
  // weights (split maxima and sums, one lane per split) and the first kPf
  // values of each thread's first output element are loaded together, so
  // a merge of up to kPf splits waits for one L2 round trip.
  constexpr int kPf = 4;
  float pre[kPf];
  if (tid < G * D) {
    const int g = tid / D;
    const int d = tid - g * D;
    const float *acc = p.part_acc + ((size_t)b * p.n_head + head0 + g) * p.max_splits * D + d;
#pragma unroll
    for (int q = 0; q < kPf; ++q) pre[q] = q < n_splits ? __ldcg(&acc[(size_t)q * D]) : 0.f;
  }
  const float2 *ml2 = reinterpret_cast<const float2 *>(p.part_ml);
  float *sw = reinterpret_cast<float *>(smem);  // [G][kMaxSplits]
  for (int g = warp; g < G; g += NCW + 1) {
    const size_t base = ((size_t)b * p.n_head + head0 + g) * p.max_splits;
    // lane l: splits l, l + 32, ...; the first one's (max, sum) is kept
    const float2 v0 = lane < n_splits ? __ldcg(&ml2[base + lane])
                                      : make_float2(-INFINITY, 0.f);
    float mx = v0.x;
    for (int s = lane + 32; s < n_splits; s += 32)
      mx = fmaxf(mx, __ldcg(&p.part_ml[(base + s) * 2]));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float den = 0.f;
    if (lane < n_splits) {
      const float w = (v0.x == -INFINITY) ? 0.f : fast_exp2(v0.x - mx);
      sw[g * kMaxSplits + lane] = w;
      den = fmaf(v0.y, w, den);
    }
    for (int s = lane + 32; s < n_splits; s += 32) {
      const float ms = __ldcg(&p.part_ml[(base + s) * 2]);
      const float w = (ms == -INFINITY) ? 0.f : fast_exp2(ms - mx);
      sw[g * kMaxSplits + s] = w;
      den = fmaf(__ldcg(&p.part_ml[(base + s) * 2 + 1]), w, den);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
      den += __shfl_xor_sync(0xffffffffu, den, off);
    const float inv = den > 0.f ? 1.f / den : 0.f;
    for (int s = lane; s < n_splits; s += 32) sw[g * kMaxSplits + s] *= inv;
  }
  __syncthreads();
  for (int idx = tid; idx < G * D; idx += S::THREADS) {
    const int g = idx / D;
    const int d = idx - g * D;
    const size_t row = (size_t)b * p.n_head + head0 + g;
    const size_t base = row * p.max_splits;
    float o2 = 0.f;
    int s0 = 0;
    if (idx == tid) {   // the prefetched first splits
#pragma unroll
      for (int q = 0; q < kPf; ++q)
        if (q < n_splits) o2 = fmaf(sw[g * kMaxSplits + q], pre[q], o2);
      s0 = n_splits < kPf ? n_splits : kPf;
    }
    for (int s = s0; s < n_splits; ++s)
      o2 = fmaf(sw[g * kMaxSplits + s], __ldcg(&p.part_acc[(base + s) * D + d]),
                o2);
    store_o(p, b * p.o_sb + (long)(head0 + g) * p.o_sh + d, o2);
  }
}

// --------------------------------------------------------------------------
// Host side
// --------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() { return tensor_map_encoder(); }

}  // namespace

// Tensor map over a KV cache viewed as (planes, max_seq, D) with a box of
// (rows x box_inner) elements; swizzle128 selects the 128-byte swizzle.
int make_kv_map(CUtensorMap *m, const void *base, int dtype, int D,
                int max_seq, long planes, int rows, int box_inner,
                bool swizzle128) {
  auto fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return TLLM_ERR_CUDA;
  }
  const int esz = dtype_size(dtype);
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)max_seq, (cuuint64_t)planes};
  cuuint64_t strides[2] = {(cuuint64_t)D * esz, (cuuint64_t)D * esz * max_seq};
  cuuint32_t box[3] = {(cuuint32_t)(box_inner > 0 ? box_inner : D),
                       (cuuint32_t)rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m,
                  dtype == TLLM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                  3, const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B
                             : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d): D=%d max_seq=%d planes=%ld",
              (int)r, D, max_seq, planes);
    return TLLM_ERR_CUDA;
  }
  return TLLM_OK;
}

namespace {

int pick_group_tile(int group) {
  for (int g = 8; g >= 1; --g)
    if (group % g == 0) return g;
  return 1;
}

int tile_rows(int dtype, int D) { return kTileBytes / (D * dtype_size(dtype)); }

template <typename T, int D, int G>
int launch_t(const DecodeParams &p, const CUtensorMap &mk, const CUtensorMap &mv,
             dim3 grid, cudaStream_t st) {
  const size_t ring = 2 * kStages * kTileBytes + 2 * kStages * sizeof(uint64_t);
  const size_t merge = (size_t)kConsumerWarps * G * (D + 2) * sizeof(float);
  const size_t sweights = (size_t)G * kMaxSplits * sizeof(float);
  size_t smem = ring;
  if (merge > smem) smem = merge;
  if (sweights > smem) smem = sweights;
  auto kern = gqa_decode_kernel<T, D, G>;
  static bool configured[64] = {};  // per instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    TLLM_CUDA(cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  TLLM_CUDA(launch_pdl(kern, grid, dim3(kThreads), smem, st, p, mk, mv));
  return TLLM_OK;
}

template <typename T, int D>
int dispatch_g(int G, const DecodeParams &p, const CUtensorMap &mk,
               const CUtensorMap &mv, dim3 grid, cudaStream_t st) {
  switch (G) {
    case 1: return launch_t<T, D, 1>(p, mk, mv, grid, st);
    case 2: return launch_t<T, D, 2>(p, mk, mv, grid, st);
    case 3: return launch_t<T, D, 3>(p, mk, mv, grid, st);
    case 4: return launch_t<T, D, 4>(p, mk, mv, grid, st);
    case 5: return launch_t<T, D, 5>(p, mk, mv, grid, st);
    case 6: return launch_t<T, D, 6>(p, mk, mv, grid, st);
    case 7: return launch_t<T, D, 7>(p, mk, mv, grid, st);
    case 8: return launch_t<T, D, 8>(p, mk, mv, grid, st);
  }
  set_error("group tile %d not built", G);
  return TLLM_ERR_UNSUPPORTED;
}

template <typename T>
int dispatch_d(int D, int G, const DecodeParams &p, const CUtensorMap &mk,
               const CUtensorMap &mv, dim3 grid, cudaStream_t st) {
  switch (D) {
    case 16: return dispatch_g<T, 16>(G, p, mk, mv, grid, st);
    case 32: return dispatch_g<T, 32>(G, p, mk, mv, grid, st);
    case 64: return dispatch_g<T, 64>(G, p, mk, mv, grid, st);
    case 128: return dispatch_g<T, 128>(G, p, mk, mv, grid, st);
    case 256: return dispatch_g<T, 256>(G, p, mk, mv, grid, st);
  }
  set_error("head_dim %d not built (16, 32, 64, 128, 256 are)", D);
  return TLLM_ERR_UNSUPPORTED;
}

// Consumer groups of the mma kernel for head_dim D and G query heads per
// CTA: two at D = 64 with G <= 8 (four ring stages either way, 71 registers,
// three CTAs per SM), one otherwise: at D = 128 two groups need four 32 KB
// stages (one CTA per SM instead of two), and two column blocks (G > 8) at
// D = 64 take 124 registers (one CTA per SM instead of three).
// TLLM_GQA_GROUPS=1 or 2 overrides the choice.
int mma_groups(int D, int G) {
  static int env = -1;
  if (env < 0) {
    const char *e = getenv("TLLM_GQA_GROUPS");
    env = e ? atoi(e) : 0;
  }
  if (env == 1 || env == 2) return env;
  return (D <= 64 && G <= 8) ? 2 : 1;
}

using MmaKern = void (*)(const DecodeParams, const int, const CUtensorMap,
                         const CUtensorMap);

// The mma kernel instance for G query heads and NG consumer groups, its
// dynamic shared memory, threads and CTAs per SM (the attribute is set once
// per device and instance).
template <int D, int NG>
int mma_kernel_setup_ng(int G, MmaKern *kern_out, size_t *smem_out,
                        int *threads_out, int *per_sm) {
  using S = MmaShape<D, NG>;
  const size_t merge = (size_t)S::CONSUMERS * G * (D + 2) * sizeof(float);
  const size_t sweights = (size_t)G * kMaxSplits * sizeof(float);
  size_t smem = S::RING;
  if (merge > smem) smem = merge;
  if (sweights > smem) smem = sweights;
  // query heads per CTA as n8 blocks of the swapped MMA
  MmaKern kern = G <= 8 ? gqa_decode_mma_kernel<D, 1, NG>
                        : gqa_decode_mma_kernel<D, 2, NG>;
  static bool configured[64][2] = {};
  static int occ[64][2] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int qi = G <= 8 ? 0 : 1;
  if (dev < 0 || dev >= 64 || !configured[dev][qi]) {
    TLLM_CUDA(cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, S::THREADS, smem) !=
        cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    if (dev >= 0 && dev < 64) {
      configured[dev][qi] = true;
      occ[dev][qi] = n;
    }
  }
  *kern_out = kern;
  *smem_out = smem;
  *threads_out = S::THREADS;
  if (per_sm) *per_sm = (dev >= 0 && dev < 64) ? occ[dev][qi] : 0;
  return TLLM_OK;
}

template <int D>
int mma_kernel_setup(int G, MmaKern *kern_out, size_t *smem_out,
                     int *threads_out, int *per_sm) {
  return mma_groups(D, G) == 2
             ? mma_kernel_setup_ng<D, 2>(G, kern_out, smem_out, threads_out, per_sm)
             : mma_kernel_setup_ng<D, 1>(G, kern_out, smem_out, threads_out, per_sm);
}

template <int D>
int launch_mma(const DecodeParams &p, int G, const CUtensorMap &mk,
               const CUtensorMap &mv, dim3 grid, cudaStream_t st) {
  MmaKern kern;
  size_t smem = 0;
  int threads = 0;
  int rc = mma_kernel_setup<D>(G, &kern, &smem, &threads, nullptr);
  if (rc) return rc;
  TLLM_CUDA(launch_pdl(kern, grid, dim3(threads), smem, st, p, G, mk, mv));
  return TLLM_OK;
}

// CTAs of the mma kernel that are resident at once on this device (0 if
// unknown).
int mma_slots(int head_dim, int G) {
  MmaKern kern;
  size_t smem = 0;
  int threads = 0, per_sm = 0;
  int rc = head_dim == 64 ? mma_kernel_setup<64>(G, &kern, &smem, &threads, &per_sm)
                          : mma_kernel_setup<128>(G, &kern, &smem, &threads, &per_sm);
  return rc ? 0 : per_sm * sm_count();
}

bool use_mma(int kv_dtype, int D) {
  static int env = -1;
  if (env < 0) {
    const char *e = getenv("TLLM_GQA_NO_MMA");
    env = (e && atoi(e) > 0) ? 1 : 0;
  }
  return !env && kv_dtype == TLLM_BF16 && (D == 64 || D == 128);
}

int pick_group_tile_mma(int group) {
  for (int g = 16; g >= 1; --g)
    if (group % g == 0) return g;
  return 1;
}

// Keys per CTA: a multiple of the tile height. Every CTA pays a fixed cost
// (first TMA round trip, the four-warp merge, the split merge) that only
// long chunks amortise, while too few CTAs leave SMs idle; on B200 the best
// chunk measured was ~3/8 of the longest sequence's tiles, between 3 and 32
// tiles (config 2: 12 of 32, config 3: 3-4 of 12, config 4: 16-32 of 128).
// With few long sequences (batch x KV-head groups small against the GPU:
// config 5 at TP = 8 has 8 sequences x 1 KV head of 32768 keys) that chunk
// leaves SMs idle, so the chunk is also capped at the size that fills ~85 %
// of one wave of resident CTAs (`slots`; 0 = unknown): 16-17 tiles there
// measured 0.66 of HBM against 0.51 with 32, while a grid just over one
// wave (12 tiles) fell to 0.48. Never more than kMaxSplits splits.
// TLLM_GQA_CHUNK_TILES (tuning) fixes the chunk for every launch.
bool chunk_env_fixed() {
  static int env = -1;
  if (env < 0) {
    const char *e = getenv("TLLM_GQA_CHUNK_TILES");
    env = (e && atoi(e) > 0) ? 1 : 0;
  }
  return env == 1;
}

int pick_chunk(int rows, int batch, int ygrid, int max_len, int slots) {
  const long tiles = (max_len + rows - 1) / rows;
  if (tiles <= 1) return rows;
  static int env_tiles = -1;
  if (env_tiles < 0) {
    const char *e = getenv("TLLM_GQA_CHUNK_TILES");
    env_tiles = e ? atoi(e) : 0;
  }
  long chunk_tiles;
  if (env_tiles > 0) {
    chunk_tiles = env_tiles;
  } else {
    chunk_tiles = (3 * tiles + 7) / 8;
    if (chunk_tiles < 3) chunk_tiles = 3;
    if (chunk_tiles > 32) chunk_tiles = 32;
    if (slots > 0) {
      const long work = (long)batch * ygrid * tiles;
      long fill = (work * 100 + 85L * slots - 1) / (85L * slots);
      if (fill < 3) fill = 3;
      if (fill < chunk_tiles) chunk_tiles = fill;
    }
  }
  long min_tiles = (tiles + kMaxSplits - 1) / kMaxSplits;
  if (chunk_tiles < min_tiles) chunk_tiles = min_tiles;
  return (int)(chunk_tiles * rows);
}

// Keys per CTA from the caller's estimate of the keys all rows read
// (`keys`: the sum of the row lengths; the host sees only max_len, which
// overstates a ragged batch): the smallest whole number of 64-key tiles c,
// at least 3 and at most the longest row, whose working CTAs, estimated as
//   ygrid * (keys / (64 c) + batch / 2)   (a row's last split is partial),
// fill at most 85 % of one wave of resident CTAs. Measured on B200 at the
// optimum chunk of each case: 8 ragged rows x 8 KV heads, 24 tiles (one
// wave: 0.78 of HBM against 0.74 with the max_len plan of 32); 16 rows,
// 48-56 tiles (0.89-0.91 against 0.76 at 32: 1.3 waves); 8 rows of 32k
// keys x 1 KV head, 17; config 2, 12. Only for batches with fewer (row, KV
// group) pairs than that target; larger ones fill the GPU at any split.
int chunk_from_keys(int rows, int batch, int ygrid, long keys, int max_len,
                    int slots, int fallback) {
  const long target = (long)slots * 85 / 100;
  if (keys <= 0 || slots <= 0 || (long)batch * ygrid >= target) return fallback;
  const long max_tiles = ((long)max_len + rows - 1) / rows;
  long lo = (max_tiles + kMaxSplits - 1) / kMaxSplits;
  if (lo < 3) lo = 3;
  if (lo >= max_tiles) return fallback;
  const double tiles = (double)keys / rows;
  for (long c = lo; c <= max_tiles; ++c)
    if ((double)ygrid * (tiles / (double)c + 0.5 * batch) <= (double)target)
      return (int)(c * rows);
  return (int)(max_tiles * rows);
}

// Validation, split selection, tensor maps and launch shared by the decode
// entry points; `err_word` is the device int that receives error codes.
//   rows = query rows (B for decode); row r reads cache sequence
//   row_seq[r] (r if null) for seq_lens[r] keys (max_len if null); q / out
//   of row r, head h live at r * q_sb + h * q_sh (resp. o_sb, o_sh);
//   cache_batch = sequences in the cache.
static int rows_impl(const float *q, long q_sb, long q_sh, const void *k_cache,
                     const void *v_cache, int kv_dtype, const int32_t *seq_lens,
                     const int32_t *row_seq, void *out, int out_dtype,
                     long out_plane_rows, long o_sb, long o_sh, int batch, int n_head, int n_kv_head, int head_dim,
                     int cache_batch, int max_seq, int max_len, float sm_scale,
                     void *partial, size_t partial_bytes, int32_t *counters,
                     int *err_word, tllm_stream_t stream, long keys_hint = 0) {
  TLLM_CHECK_ARG(batch >= 0 && n_head > 0 && n_kv_head > 0,
                 "invalid head counts n_head=%d n_kv_head=%d", n_head,
                 n_kv_head);
  TLLM_CHECK_ARG(n_head % n_kv_head == 0,
                 "n_head (%d) must be divisible by n_kv_head (%d)", n_head,
                 n_kv_head);
  TLLM_CHECK_ARG(kv_dtype == TLLM_F32 || kv_dtype == TLLM_BF16,
                 "kv_dtype must be F32 or BF16");
  TLLM_CHECK_ARG(out_dtype == TLLM_F32 || out_dtype == TLLM_SPLIT ||
                     out_dtype == TLLM_BF16,
                 "out_dtype must be F32, SPLIT or BF16");
  TLLM_CHECK_ARG(out_dtype == TLLM_F32 || out_plane_rows >= batch,
                 "out_plane_rows (%ld) < rows (%d)", out_plane_rows, batch);
  if (batch == 0) return TLLM_OK;
  TLLM_CHECK_ARG(q && out && k_cache && v_cache, "NULL tensor pointer");
  TLLM_CHECK_ARG(max_seq > 0, "max_seq must be > 0");
  TLLM_CHECK_ARG(((uintptr_t)k_cache & 15) == 0 && ((uintptr_t)v_cache & 15) == 0,
                 "KV cache must be 16-byte aligned");
  TLLM_CHECK_ARG(((uintptr_t)q & 15) == 0, "q must be 16-byte aligned");
  TLLM_CHECK_ARG(q_sb % 4 == 0 && q_sh % 4 == 0 && o_sb >= 0 && o_sh >= 0,
                 "q strides must be multiples of 4 elements");
  TLLM_CHECK_ARG(cache_batch > 0, "cache_batch must be > 0");
  if (max_len <= 0 || max_len > max_seq) max_len = max_seq;
  if (sm_scale <= 0.f) sm_scale = 1.0f / sqrtf((float)head_dim);

  const int group = n_head / n_kv_head;
  const bool mma = use_mma(kv_dtype, head_dim);
  const int G = mma ? pick_group_tile_mma(group) : pick_group_tile(group);
  const int n_gsub = group / G;
  const int rows = mma ? MmaShape<64, 1>::KT : tile_rows(kv_dtype, head_dim);
  TLLM_CHECK_ARG(rows >= 1, "head_dim %d too large", head_dim);
  const int ygrid = n_kv_head * n_gsub;
  TLLM_CHECK_ARG(ygrid <= 65535 && batch <= 65535, "grid too large");

  const int slots = mma ? mma_slots(head_dim, G) : 0;
  int chunk = pick_chunk(rows, batch, ygrid, max_len, slots);
  if (mma && keys_hint > 0 && !chunk_env_fixed())
    chunk = chunk_from_keys(rows, batch, ygrid, keys_hint, max_len, slots, chunk);
  int max_splits = (max_len + chunk - 1) / chunk;
  if (max_splits < 1) max_splits = 1;
  if (max_splits > 1) {
    // Grow the chunk until the partials fit in the caller's buffer.
    auto need = [&](int ms) {
      return (size_t)batch * n_head * ms * (head_dim + 2) * sizeof(float);
    };
    while (max_splits > 1 && need(max_splits) > partial_bytes) {
      chunk += rows;
      max_splits = (max_len + chunk - 1) / chunk;
    }
    if (max_splits > 1) {
      TLLM_CHECK_ARG(partial && counters,
                     "split-KV needs the partial and counter buffers");
      TLLM_CHECK_ARG(((uintptr_t)partial & 15) == 0, "partial misaligned");
    }
  }

  CUtensorMap mk, mv;
  int rc = make_kv_map(&mk, k_cache, kv_dtype, head_dim, max_seq,
                       (long)cache_batch * n_kv_head, rows, mma ? 64 : 0, mma);
  if (rc) return rc;
  rc = make_kv_map(&mv, v_cache, kv_dtype, head_dim, max_seq,
                   (long)cache_batch * n_kv_head, rows, mma ? 64 : 0, mma);
  if (rc) return rc;

  DecodeParams p;
  p.q = q;
  const bool act_out = out_dtype != TLLM_F32;
  p.out = act_out ? nullptr : static_cast<float *>(out);
  p.out_split = act_out ? static_cast<uint16_t *>(out) : nullptr;
  p.out_plane = act_out ? out_plane_rows * o_sb : 0;
  p.out_planes = out_dtype == TLLM_SPLIT ? 2 : 1;
  p.seq_lens = seq_lens;
  p.row_seq = row_seq;
  p.q_sb = q_sb;
  p.q_sh = q_sh;
  p.o_sb = o_sb;
  p.o_sh = o_sh;
  p.part_acc = static_cast<float *>(partial);
  p.part_ml = p.part_acc
                  ? p.part_acc + (size_t)batch * n_head * max_splits * head_dim
                  : nullptr;
  p.counters = counters;
  p.err = err_word;
  TLLM_CHECK_ARG(p.err, "device error word unavailable");
  p.n_head = n_head;
  p.n_kv = n_kv_head;
  p.group = group;
  p.n_gsub = n_gsub;
  p.max_seq = max_seq;
  p.max_len = max_len;
  p.chunk = chunk;
  p.max_splits = max_splits;
  p.qscale = sm_scale * kLog2e;

  p.n_y = ygrid;
  dim3 grid(max_splits, ygrid, batch);
  cudaStream_t st = resolve(stream);
  if (mma)
    return head_dim == 64 ? launch_mma<64>(p, G, mk, mv, grid, st)
                          : launch_mma<128>(p, G, mk, mv, grid, st);
  if (kv_dtype == TLLM_BF16)
    return dispatch_d<__nv_bfloat16>(head_dim, G, p, mk, mv, grid, st);
  return dispatch_d<float>(head_dim, G, p, mk, mv, grid, st);
}

}  // namespace
}  // namespace tllm

using namespace tllm;

extern "C" {

int tllm_gqa_decode_workspace(int batch, int n_head, int n_kv_head,
                              int head_dim, int max_seq, int kv_dtype,
                              size_t *partial_bytes, size_t *counter_bytes) {
  TLLM_CHECK_ARG(partial_bytes && counter_bytes, "NULL output pointer");
  TLLM_CHECK_ARG(batch >= 0 && n_head > 0 && n_kv_head > 0 && head_dim > 0 &&
                     max_seq >= 0,
                 "invalid shape");
  TLLM_CHECK_ARG(n_head % n_kv_head == 0,
                 "n_head (%d) must be divisible by n_kv_head (%d)", n_head,
                 n_kv_head);
  (void)kv_dtype;
  *partial_bytes =
      (size_t)batch * n_head * kMaxSplits * (head_dim + 2) * sizeof(float);
  *counter_bytes = (size_t)batch * n_head * sizeof(int32_t);
  return TLLM_OK;
}

int tllm_gqa_decode(const float *q, const void *k_cache, const void *v_cache,
                    int kv_dtype, const int32_t *seq_lens, float *out,
                    int batch, int n_head, int n_kv_head, int head_dim,
                    int max_seq, int max_len, float sm_scale, void *partial,
                    size_t partial_bytes, int32_t *counters,
                    tllm_stream_t stream) {
  TLLM_INJECT("launch");
  const long hd = (long)n_head * head_dim;
  return rows_impl(q, hd, head_dim, k_cache, v_cache, kv_dtype, seq_lens,
                   nullptr, out, TLLM_F32, 0, hd, head_dim, batch, n_head,
                   n_kv_head, head_dim, batch, max_seq, max_len, sm_scale,
                   partial, partial_bytes, counters, device_error_ptr(), stream);
}

int tllm_gqa_rows(const float *q, long q_row_stride, long q_head_stride,
                  const void *k_cache, const void *v_cache, int kv_dtype,
                  const int32_t *row_seq, const int32_t *row_len, void *out,
                  int out_dtype, long out_plane_rows, long out_row_stride,
                  long out_head_stride, int rows, int n_head, int n_kv_head,
                  int head_dim, int cache_batch, int max_seq, int max_len,
                  float sm_scale, void *partial, size_t partial_bytes,
                  int32_t *counters, tllm_stream_t stream) {
  TLLM_INJECT("launch");
  return rows_impl(q, q_row_stride, q_head_stride, k_cache, v_cache, kv_dtype,
                   row_len, row_seq, out, out_dtype, out_plane_rows,
                   out_row_stride, out_head_stride, rows, n_head, n_kv_head, head_dim, cache_batch, max_seq,
                   max_len, sm_scale, partial, partial_bytes, counters,
                   device_error_ptr(), stream);
}

int tllm_gqa_rows_hint(const float *q, long q_row_stride, long q_head_stride,
                       const void *k_cache, const void *v_cache, int kv_dtype,
                       const int32_t *row_seq, const int32_t *row_len, void *out,
                       int out_dtype, long out_plane_rows, long out_row_stride,
                       long out_head_stride, int rows, int n_head, int n_kv_head,
                       int head_dim, int cache_batch, int max_seq, int max_len,
                       float sm_scale, void *partial, size_t partial_bytes,
                       int32_t *counters, long keys_hint, tllm_stream_t stream) {
  TLLM_INJECT("launch");
  TLLM_CHECK_ARG(keys_hint >= 0, "keys_hint (%ld) must be >= 0", keys_hint);
  return rows_impl(q, q_row_stride, q_head_stride, k_cache, v_cache, kv_dtype,
                   row_len, row_seq, out, out_dtype, out_plane_rows,
                   out_row_stride, out_head_stride, rows, n_head, n_kv_head, head_dim, cache_batch, max_seq,
                   max_len, sm_scale, partial, partial_bytes, counters,
                   device_error_ptr(), stream, keys_hint);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free decode entry point.
//
// Some host programs cannot let a library allocate device memory: inference
// servers that carve all of HBM into their own arenas at start-up and
// account for every byte, plugin hosts whose memory budget forbids hidden
// allocations, and decode loops that must never block in the allocator
// (cudaMalloc/cudaFree can wait for the whole device). For them this entry
// point takes its split-KV scratch from a fixed array in device global
// memory that is part of the library image, so a call allocates nothing.
//
// Limits: the partial-result region is kNoAllocPartialBytes (8 MiB); when a
// batch would need more split partials than that, fewer, longer splits are
// used. The ticket counters cover batch * n_head <= kNoAllocMaxCounters
// (65536); larger batches are rejected with TLLM_ERR_INVALID_ARG. Every GPU
// that loads the library keeps this ~8.3 MiB until the process exits.
//
// The array is shared by every call on a device and keeps the last call's
// contents; the counters that must start at zero are cleared on the stream
// before each launch. Calls that overlap on the GPU (on different streams,
// or from several host threads) race on the array and must not be issued.
// ---------------------------------------------------------------------------
namespace tllm {
namespace {

constexpr size_t kNoAllocPartialBytes = size_t(8) << 20;
constexpr int kNoAllocMaxCounters = 65536;
constexpr size_t kNoAllocCounterOffset = kNoAllocPartialBytes;
constexpr size_t kNoAllocErrOffset =
    kNoAllocCounterOffset + size_t(kNoAllocMaxCounters) * sizeof(int32_t);
constexpr size_t kNoAllocBytes = kNoAllocErrOffset + 256;

// Scratch of tllm_gqa_decode_noalloc. In host code this name is only a
// host-side stand-in for the device array: its device address must be
// looked up with cudaGetSymbolAddress (done once per device below).
static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocBytes];

std::mutex g_noalloc_mu;
unsigned char *g_noalloc_addr[64];

// Device address of g_decode_scratch on the current device (looked up on the
// first call made while that device is current).
int noalloc_scratch(unsigned char **addr) {
  int dev = 0;
  TLLM_CUDA(cudaGetDevice(&dev));
  TLLM_CHECK_ARG(dev >= 0 && dev < 64, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void *ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_decode_scratch);
    if (e != cudaSuccess || !ptr) {
      set_error("cudaGetSymbolAddress(decode scratch) failed: %s (%d)",
                cudaGetErrorString(e), (int)e);
      return TLLM_ERR_CUDA;
    }
    g_noalloc_addr[dev] = static_cast<unsigned char *>(ptr);
  }
  *addr = g_noalloc_addr[dev];
  return TLLM_OK;
}

}  // namespace
}  // namespace tllm

extern "C" int tllm_gqa_decode_noalloc(
    const float *q, const void *k_cache, const void *v_cache, int kv_dtype,
    const int32_t *seq_lens, float *out, int batch, int n_head, int n_kv_head,
    int head_dim, int max_seq, int max_len, float sm_scale,
    tllm_stream_t stream) {
  TLLM_CHECK_ARG(batch >= 0 && n_head > 0, "invalid batch %d / n_head %d",
                 batch, n_head);
  TLLM_CHECK_ARG((long)batch * n_head <= kNoAllocMaxCounters,
                 "tllm_gqa_decode_noalloc supports batch * n_head <= %d "
                 "(got %d * %d); use tllm_gqa_decode with caller-owned scratch",
                 kNoAllocMaxCounters, batch, n_head);
  if (batch == 0) return TLLM_OK;
  unsigned char *base = nullptr;
  int rc = noalloc_scratch(&base);
  if (rc) return rc;
  int32_t *counters = reinterpret_cast<int32_t *>(base + kNoAllocCounterOffset);
  int *err_word = reinterpret_cast<int *>(base + kNoAllocErrOffset);
  cudaStream_t st = resolve(stream);
  TLLM_CUDA(cudaMemsetAsync(counters, 0, (size_t)batch * n_head * sizeof(int32_t),
                            st));
  const long hd = (long)n_head * head_dim;
  return rows_impl(q, hd, head_dim, k_cache, v_cache, kv_dtype, seq_lens,
                   nullptr, out, TLLM_F32, 0, hd, head_dim, batch, n_head,
                   n_kv_head, head_dim, batch, max_seq, max_len, sm_scale, base,
                   kNoAllocPartialBytes, counters, err_word, st);
}

// The device error word of tllm_gqa_decode_noalloc sits at the end of the
// static scratch array, so reading it allocates nothing either: the whole
// device is synchronised (the calls may have used any stream), the word is
// copied out and optionally cleared.
extern "C" int tllm_gqa_decode_noalloc_error(int *code, int reset) {
  TLLM_CHECK_ARG(code, "code is NULL");
  unsigned char *base = nullptr;
  int rc = noalloc_scratch(&base);
  if (rc) return rc;
  int *err_word = reinterpret_cast<int *>(base + kNoAllocErrOffset);
  TLLM_CUDA(cudaDeviceSynchronize());
  TLLM_CUDA(cudaMemcpy(code, err_word, sizeof(int), cudaMemcpyDeviceToHost));
  if (reset) {
    TLLM_CUDA(cudaMemset(err_word, 0, sizeof(int)));
    TLLM_CUDA(cudaDeviceSynchronize());
  }
  return TLLM_OK;
}
