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
//    (cp.async.bulk.tensor, no multicast) into a 4-stage shared-memory ring
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

namespace tllm {
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
  const float *q;        // (B, n_head, D)
  float *out;            // (B, n_head, D)
  const int *seq_lens;   // (B,) or null (every sequence has max_len keys)
  float *part_acc;       // (B, n_head, max_splits, D)
  float *part_ml;        // (B, n_head, max_splits, 2)
  int *counters;         // (B, gridDim.y)
  int *err;              // device error word
  int n_head, n_kv, group, n_gsub;
  int max_seq, max_len, chunk, max_splits;
  float qscale;          // sm_scale * log2(e)
};

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
      const int plane = b * p.n_kv + kvh;
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
      const float *qp = p.q + ((size_t)b * p.n_head + head0 + g) * D;
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
          const float alpha = exp2f(m_run[g] - mnew);
          m_run[g] = mnew;
          l_run[g] *= alpha;
#pragma unroll
          for (int e = 0; e < S::NV * S::VEC; ++e) acc[g][e] *= alpha;
#pragma unroll
          for (int it = 0; it < S::ITERS; ++it) {
            const float pv = exp2f(sc[it][g] - mnew);  // exp2(-inf) = 0
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
          const float sc = exp2f(wm - mx);
          num = fmaf(w_acc[(w * G + g) * D + d], sc, num);
          den = fmaf(w_l[w * G + g], sc, den);
        }
      }
    }
    const size_t row = (size_t)b * p.n_head + head0 + g;
    if (single) {
      p.out[row * D + d] = den > 0.f ? num / den : 0.f;
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
    int *ctr = p.counters + (size_t)b * gridDim.y + y;
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
      const float w = (ms == -INFINITY) ? 0.f : exp2f(ms - mx);
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
    p.out[row * D + d] = o;
  }
}

// --------------------------------------------------------------------------
// Host side
// --------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr,
                                cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// Tensor map over a KV cache viewed as (planes, max_seq, D) with a box of
// (rows x D) elements.
int make_kv_map(CUtensorMap *m, const void *base, int dtype, int D,
                int max_seq, long planes, int rows) {
  auto fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return TLLM_ERR_CUDA;
  }
  const int esz = dtype_size(dtype);
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)max_seq, (cuuint64_t)planes};
  cuuint64_t strides[2] = {(cuuint64_t)D * esz, (cuuint64_t)D * esz * max_seq};
  cuuint32_t box[3] = {(cuuint32_t)D, (cuuint32_t)rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m,
                  dtype == TLLM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                  3, const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d): D=%d max_seq=%d planes=%ld",
              (int)r, D, max_seq, planes);
    return TLLM_ERR_CUDA;
  }
  return TLLM_OK;
}

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
  kern<<<grid, kThreads, smem, st>>>(p, mk, mv);
  TLLM_LAUNCH_CHECK();
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
    case 32: return dispatch_g<T, 32>(G, p, mk, mv, grid, st);
    case 64: return dispatch_g<T, 64>(G, p, mk, mv, grid, st);
    case 128: return dispatch_g<T, 128>(G, p, mk, mv, grid, st);
    case 256: return dispatch_g<T, 256>(G, p, mk, mv, grid, st);
  }
  set_error("head_dim %d not built (32, 64, 128, 256 are)", D);
  return TLLM_ERR_UNSUPPORTED;
}

// Keys per CTA: a multiple of the tile height chosen so that the launch has
// roughly `target` CTAs doing work, never more than kMaxSplits splits.
int pick_chunk(int rows, int batch, int ygrid, int max_len) {
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
    // The average sequence is taken as half of max_len (ragged batches).
    const long target = 4L * sm_count();
    const long pairs = (long)batch * ygrid;
    long want_splits = (target + pairs - 1) / pairs;  // per (b, y) at max_len
    if (want_splits < 1) want_splits = 1;
    want_splits *= 2;
    chunk_tiles = (tiles + want_splits - 1) / want_splits;
    if (chunk_tiles < 2) chunk_tiles = 2;
  }
  long min_tiles = (tiles + kMaxSplits - 1) / kMaxSplits;
  if (chunk_tiles < min_tiles) chunk_tiles = min_tiles;
  return (int)(chunk_tiles * rows);
}

// Validation, split selection, tensor maps and launch shared by the decode
// entry points; `err_word` is the device int that receives error codes.
static int decode_impl(const float *q, const void *k_cache, const void *v_cache,
                       int kv_dtype, const int32_t *seq_lens, float *out,
                       int batch, int n_head, int n_kv_head, int head_dim,
                       int max_seq, int max_len, float sm_scale, void *partial,
                       size_t partial_bytes, int32_t *counters, int *err_word,
                       tllm_stream_t stream) {
  TLLM_CHECK_ARG(batch >= 0 && n_head > 0 && n_kv_head > 0,
                 "invalid head counts n_head=%d n_kv_head=%d", n_head,
                 n_kv_head);
  TLLM_CHECK_ARG(n_head % n_kv_head == 0,
                 "n_head (%d) must be divisible by n_kv_head (%d)", n_head,
                 n_kv_head);
  TLLM_CHECK_ARG(kv_dtype == TLLM_F32 || kv_dtype == TLLM_BF16,
                 "kv_dtype must be F32 or BF16");
  if (batch == 0) return TLLM_OK;
  TLLM_CHECK_ARG(q && out && k_cache && v_cache, "NULL tensor pointer");
  TLLM_CHECK_ARG(max_seq > 0, "max_seq must be > 0");
  TLLM_CHECK_ARG(((uintptr_t)k_cache & 15) == 0 && ((uintptr_t)v_cache & 15) == 0,
                 "KV cache must be 16-byte aligned");
  TLLM_CHECK_ARG(((uintptr_t)q & 15) == 0, "q must be 16-byte aligned");
  if (max_len <= 0 || max_len > max_seq) max_len = max_seq;
  if (sm_scale <= 0.f) sm_scale = 1.0f / sqrtf((float)head_dim);

  const int group = n_head / n_kv_head;
  const int G = pick_group_tile(group);
  const int n_gsub = group / G;
  const int rows = tile_rows(kv_dtype, head_dim);
  TLLM_CHECK_ARG(rows >= 1, "head_dim %d too large", head_dim);
  const int ygrid = n_kv_head * n_gsub;
  TLLM_CHECK_ARG(ygrid <= 65535 && batch <= 65535, "grid too large");

  int chunk = pick_chunk(rows, batch, ygrid, max_len);
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
                       (long)batch * n_kv_head, rows);
  if (rc) return rc;
  rc = make_kv_map(&mv, v_cache, kv_dtype, head_dim, max_seq,
                   (long)batch * n_kv_head, rows);
  if (rc) return rc;

  DecodeParams p;
  p.q = q;
  p.out = out;
  p.seq_lens = seq_lens;
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

  dim3 grid(max_splits, ygrid, batch);
  cudaStream_t st = resolve(stream);
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
  return decode_impl(q, k_cache, v_cache, kv_dtype, seq_lens, out, batch,
                     n_head, n_kv_head, head_dim, max_seq, max_len, sm_scale,
                     partial, partial_bytes, counters, device_error_ptr(),
                     stream);
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
  return decode_impl(q, k_cache, v_cache, kv_dtype, seq_lens, out, batch,
                     n_head, n_kv_head, head_dim, max_seq, max_len, sm_scale,
                     base, kNoAllocPartialBytes, counters, err_word, st);
}
