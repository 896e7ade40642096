// Causal GQA prefill attention over the preallocated KV cache, for sm_100a.
//
// The prompt rows of a prefill attend the cache of their own sequence up to
// and including their own position:
//     out[r, h, :] = softmax(q[r, h, :] . K[seq, kvh, :pos_r + 1, :]^T * scale)
//                    V[seq, kvh, :pos_r + 1, :],      kvh = h / (H / Hkv)
// the causal branch of the reference's attention_gqa
// (triton_llm/kernels/attention_gqa.py:97-119: query i of seq_q sees keys
// j <= seq_k - seq_q + i; q pre-scaled, online softmax, one divide at the
// end) as the SmolLM2 prefill calls it (smollm2_triton/model.py:318-348,
// attention at :341-343), here over the cache the QKV epilogue has just
// written, for every prompt of a batch at once.
//
// Work is cut into blocks of up to 64 consecutive rows of one sequence
// (consecutive positions), described by the caller: (first row, rows,
// cache sequence, first position). One CTA = (block, query head): a producer
// warp streams 64-key K and V tiles of the block's KV head by TMA (128-byte
// swizzle) into a ring guarded by full / empty mbarriers, up to the block's
// last position; four consumer warps own 16 query rows each and compute, with
// mma.sync m16n8k16 (bf16 in, fp32 accumulate), S = Q K^T and O += P V in
// the FlashAttention-2 arrangement (the P fragments are the S accumulators,
// no shared-memory round trip). Q and P are split into bf16 hi + lo, so the
// products keep ~16 mantissa bits against the exact bf16 cache, as in the
// decode kernel. The causal mask is applied only on tiles that cross a
// warp's diagonal; tiles past a warp's last row are waited on and released
// without work. Output fp32 or in the projection operand format.
#include <cuda.h>

#include <cmath>

#include "common.cuh"
#include "mma_sync.cuh"

namespace tllm {
namespace {

constexpr int kPfWarps = 4;                   // consumer warps, 16 rows each
constexpr int kPfThreads = (kPfWarps + 1) * 32;
constexpr int kPfRows = kPfWarps * 16;        // query rows per block
constexpr int kPfKT = 64;                     // keys per tile
constexpr float kPfLog2e = 1.4426950408889634f;

template <int D>
struct PfShape {
  static constexpr int SUB = D / 64;             // 128-byte sub-tiles per key
  static constexpr int SUB_BYTES = kPfKT * 128;  // 8 KB
  static constexpr int TILE_BYTES = SUB * SUB_BYTES;
  static constexpr int STAGES = D <= 64 ? 4 : 3;
  static constexpr int KSTEPS = D / 16;
  static constexpr size_t SMEM = 2 * (size_t)STAGES * TILE_BYTES;
};

struct PrefillParams {
  const float *q;       // row r, head h at q + r * q_sr + h * q_sh
  long q_sr, q_sh;
  float *out;           // fp32 output, or
  uint16_t *out_act;    // operand-format output (planes out_plane apart)
  long out_plane;
  int out_planes;
  long o_sr, o_sh;
  const int4 *blocks;   // (first row, rows, cache sequence, first position)
  int *err;
  int n_head, n_kv, group, max_seq, cache_batch;
  float qscale;         // sm_scale * log2(e)
};

__device__ __forceinline__ void pf_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

template <int D>
__global__ void __launch_bounds__(kPfThreads)
    gqa_prefill_kernel(const PrefillParams p,
                       const __grid_constant__ CUtensorMap tmk,
                       const __grid_constant__ CUtensorMap tmv) {
  griddep_launch();
  griddep_wait();   // q and the cache rows come from the QKV projection
  using S = PfShape<D>;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t *k_st = smem;
  uint8_t *v_st = smem + S::STAGES * S::TILE_BYTES;
  __shared__ uint64_t full[S::STAGES], empty[S::STAGES];
  __shared__ int s_fail;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  if (smem_u32(smem) & 1023) {
    if (tid == 0) atomicOr(p.err, DEV_ERR_SMEM_ALIGN);
    return;
  }
  const int4 bd = p.blocks[blockIdx.x];
  const int row0 = bd.x, nrows = bd.y, seq = bd.z, pos0 = bd.w;
  if (nrows < 1 || nrows > kPfRows || pos0 < 0 || pos0 + nrows > p.max_seq ||
      seq < 0 || seq >= p.cache_batch || row0 < 0) {
    if (tid == 0) atomicOr(p.err, DEV_ERR_LEN_CLAMPED);
    return;
  }
  const int h = blockIdx.y;
  const int kvh = h / p.group;
  const int maxpos = pos0 + nrows - 1;
  const int ntiles = maxpos / kPfKT + 1;

  if (tid == 0) {
    for (int s = 0; s < S::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kPfWarps);
    }
    fence_mbar_init();
    s_fail = 0;
  }
  __syncthreads();

  bool failed = false;
  if (warp == kPfWarps) {
    if (lane == 0) {
      const int plane = seq * p.n_kv + kvh;
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % S::STAGES;
        if (t >= S::STAGES &&
            !mbar_wait_bounded(&empty[s], ((t / S::STAGES) - 1) & 1)) {
          failed = true;
          break;
        }
        mbar_expect_tx(&full[s], 2 * S::TILE_BYTES);
#pragma unroll
        for (int sub = 0; sub < S::SUB; ++sub) {
          tma_load_3d(k_st + s * S::TILE_BYTES + sub * S::SUB_BYTES, &tmk,
                      &full[s], sub * 64, t * kPfKT, plane);
          tma_load_3d(v_st + s * S::TILE_BYTES + sub * S::SUB_BYTES, &tmv,
                      &full[s], sub * 64, t * kPfKT, plane);
        }
      }
    }
  } else {
    // rows r0 and r0 + 8 of this warp's 16; columns 2c, 2c + 1 of each n8
    const int r0 = lane >> 2;
    const int c2 = (lane & 3) * 2;
    const int wrow = warp * 16;                 // first local row of the warp
    const int wrows = min(16, nrows - wrow);    // valid rows (may be <= 0)
    const int wmin = pos0 + wrow;               // position of local row 0
    const int wmax = pos0 + wrow + wrows - 1;   // last valid position
    const bool ok0 = r0 < wrows, ok1 = r0 + 8 < wrows;
    const int pos_r0 = wmin + r0, pos_r1 = wmin + r0 + 8;

    // ---- Q A-fragments (rows = positions, k = dims), scaled, hi / lo
    uint32_t qh[S::KSTEPS][4], ql[S::KSTEPS][4];
    {
      const float *q0 = p.q + (long)(row0 + wrow + r0) * p.q_sr + (long)h * p.q_sh;
      const float *q1 = q0 + 8 * p.q_sr;
#pragma unroll
      for (int kk = 0; kk < S::KSTEPS; ++kk) {
#pragma unroll
        for (int f = 0; f < 2; ++f) {          // dims kk*16 + 8f + c2, + 1
          const int col = kk * 16 + 8 * f + c2;
          float2 a = make_float2(0.f, 0.f), b = make_float2(0.f, 0.f);
          if (ok0) a = *reinterpret_cast<const float2 *>(q0 + col);
          if (ok1) b = *reinterpret_cast<const float2 *>(q1 + col);
          split_bf16x2(a.x * p.qscale, a.y * p.qscale, qh[kk][2 * f], ql[kk][2 * f]);
          split_bf16x2(b.x * p.qscale, b.y * p.qscale, qh[kk][2 * f + 1],
                       ql[kk][2 * f + 1]);
        }
      }
    }
    float o[D / 8][4];
#pragma unroll
    for (int n = 0; n < D / 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[n][e] = 0.f;
    float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};

    // ldmatrix lane addressing (matrix l / 8, row l % 8):
    //  K (B operand of S, rows = keys): matrices (keys +0 / +8) x (dims +0 / +8)
    const int kb_key = ((lane >> 4) & 1) * 8 + (lane & 7);
    const int kb_dof = ((lane >> 3) & 1) * 8;
    //  V (B operand of O via .trans, rows = keys): (keys +0 / +8) x (dims +0 / +8)
    const int vb_key = ((lane >> 3) & 1) * 8 + (lane & 7);
    const int vb_dof = ((lane >> 4) & 1) * 8;

    for (int t = 0; t < ntiles; ++t) {
      const int s = t % S::STAGES;
      const bool got = __all_sync(
          0xffffffffu, mbar_wait_bounded(&full[s], (t / S::STAGES) & 1));
      if (!got) {
        failed = true;
        break;
      }
      const int key0 = t * kPfKT;
      if (wrows > 0 && key0 <= wmax) {
        const uint8_t *kt = k_st + s * S::TILE_BYTES;
        const uint8_t *vt = v_st + s * S::TILE_BYTES;
        // ---- S = Q K^T (16 rows x 64 keys)
        float sc[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) sc[n][e] = 0.f;
#pragma unroll
        for (int kk = 0; kk < S::KSTEPS; ++kk) {
          const int dim = kk * 16 + kb_dof;
          const int sub = dim >> 6;
          const int chunk = (dim & 63) >> 3;
#pragma unroll
          for (int np = 0; np < 4; ++np) {
            const int key = np * 16 + kb_key;
            const uint32_t addr = smem_u32(kt + sub * S::SUB_BYTES + key * 128 +
                                           ((chunk ^ (key & 7)) << 4));
            uint32_t b[4];
            ldsm_x4(addr, b[0], b[1], b[2], b[3]);
            mma_bf16(sc[2 * np], qh[kk], b[0], b[1]);
            mma_bf16(sc[2 * np], ql[kk], b[0], b[1]);
            mma_bf16(sc[2 * np + 1], qh[kk], b[2], b[3]);
            mma_bf16(sc[2 * np + 1], ql[kk], b[2], b[3]);
          }
        }
        // ---- causal mask where the tile crosses this warp's diagonal
        if (key0 + kPfKT - 1 > wmin || !ok0 || !ok1) {
#pragma unroll
          for (int n = 0; n < 8; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int key = key0 + n * 8 + c2 + (e & 1);
              const bool vis = (e < 2) ? (ok0 && key <= pos_r0) : (ok1 && key <= pos_r1);
              if (!vis) sc[n][e] = -INFINITY;
            }
        }
        // ---- online softmax (base 2) of rows r0 (e = 0, 1), r0 + 8 (e = 2, 3)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          float mx = -INFINITY;
#pragma unroll
          for (int n = 0; n < 8; ++n)
            mx = fmaxf(mx, fmaxf(sc[n][2 * hr], sc[n][2 * hr + 1]));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
          const float mn = fmaxf(m_r[hr], mx);
          const float msafe = (mn == -INFINITY) ? 0.f : mn;
          if (mn != m_r[hr]) {
            const float alpha = fast_exp2(m_r[hr] - msafe);   // 0 when m was -inf
            l_r[hr] *= alpha;
#pragma unroll
            for (int n = 0; n < D / 8; ++n) {
              o[n][2 * hr] *= alpha;
              o[n][2 * hr + 1] *= alpha;
            }
            m_r[hr] = mn;
          }
#pragma unroll
          for (int n = 0; n < 8; ++n) {
            sc[n][2 * hr] = fast_exp2(sc[n][2 * hr] - msafe);
            sc[n][2 * hr + 1] = fast_exp2(sc[n][2 * hr + 1] - msafe);
            l_r[hr] += sc[n][2 * hr] + sc[n][2 * hr + 1];
          }
        }
        // ---- O += P V: P's A fragments are the S accumulators of key
        //      blocks 2ks, 2ks + 1 (hi + lo)
        const bool tail = key0 + kPfKT - 1 > maxpos;   // keys past the block
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          uint32_t ph[4], pl[4];
          split_bf16x2(sc[2 * ks][0], sc[2 * ks][1], ph[0], pl[0]);
          split_bf16x2(sc[2 * ks][2], sc[2 * ks][3], ph[1], pl[1]);
          split_bf16x2(sc[2 * ks + 1][0], sc[2 * ks + 1][1], ph[2], pl[2]);
          split_bf16x2(sc[2 * ks + 1][2], sc[2 * ks + 1][3], ph[3], pl[3]);
          const int key = ks * 16 + vb_key;
#pragma unroll
          for (int nd = 0; nd < D / 16; ++nd) {
            const int dim = nd * 16 + vb_dof;
            const int sub = dim >> 6;
            const int chunk = (dim & 63) >> 3;
            const uint32_t addr = smem_u32(vt + sub * S::SUB_BYTES + key * 128 +
                                           ((chunk ^ (key & 7)) << 4));
            uint32_t b[4];
            ldsm_x4_t(addr, b[0], b[1], b[2], b[3]);
            if (tail) {
              // V rows past the block's last position were not written by
              // this prefill (they may hold anything, even NaN): zero them so
              // that 0 * row stays 0. b0 / b2 hold keys 2c, 2c + 1 of the
              // step, b1 / b3 keys 8 + 2c, 8 + 2c + 1 (low / high halves).
              const int kb = key0 + ks * 16 + c2;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int k_lo = kb + ((i & 1) ? 8 : 0);
                uint32_t m = 0xffffffffu;
                if (k_lo > maxpos) m &= 0xffff0000u;
                if (k_lo + 1 > maxpos) m &= 0x0000ffffu;
                b[i] &= m;
              }
            }
            mma_bf16(o[2 * nd], ph, b[0], b[1]);
            mma_bf16(o[2 * nd], pl, b[0], b[1]);
            mma_bf16(o[2 * nd + 1], ph, b[2], b[3]);
            mma_bf16(o[2 * nd + 1], pl, b[2], b[3]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) pf_arrive(&empty[s]);
    }
    // ---- normalise and store rows r0, r0 + 8
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      l_r[hr] += __shfl_xor_sync(0xffffffffu, l_r[hr], 1);
      l_r[hr] += __shfl_xor_sync(0xffffffffu, l_r[hr], 2);
    }
    if (!failed) {
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        if (!(hr ? ok1 : ok0)) continue;
        const float inv = l_r[hr] > 0.f ? 1.f / l_r[hr] : 0.f;
        const long base = (long)(row0 + wrow + r0 + 8 * hr) * p.o_sr + (long)h * p.o_sh;
#pragma unroll
        for (int n = 0; n < D / 8; ++n) {
          const long idx = base + n * 8 + c2;
          const float v0 = o[n][2 * hr] * inv, v1 = o[n][2 * hr + 1] * inv;
          if (p.out_act) {
            store_act(p.out_act, (size_t)p.out_plane, (size_t)idx, v0, p.out_planes);
            store_act(p.out_act, (size_t)p.out_plane, (size_t)idx + 1, v1, p.out_planes);
          } else {
            p.out[idx] = v0;
            p.out[idx + 1] = v1;
          }
        }
      }
    }
  }
  if (failed) {
    atomicOr(p.err, DEV_ERR_WAIT_TIMEOUT);
    s_fail = 1;
  }
  __syncthreads();
  if (s_fail && tid == 0) {
    // a failed wait may have left loads in flight: wait (bounded) for the
    // last fill of every stage before the shared memory goes away
    for (int t = ntiles > S::STAGES ? ntiles - S::STAGES : 0; t < ntiles; ++t)
      mbar_wait_bounded(&full[t % S::STAGES], (t / S::STAGES) & 1, 1u << 12);
  }
}

template <int D>
int launch_prefill(const PrefillParams &p, const CUtensorMap &mk,
                   const CUtensorMap &mv, int n_blocks, cudaStream_t st) {
  using S = PfShape<D>;
  auto kern = gqa_prefill_kernel<D>;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    // + 1 KB so the kernel can align its stage buffers to 1024 bytes
    TLLM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)S::SMEM + 1024));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_blocks, p.n_head, 1);
  cfg.blockDim = dim3(kPfThreads);
  cfg.dynamicSmemBytes = S::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  TLLM_CUDA(cudaLaunchKernelEx(&cfg, kern, p, mk, mv));
  TLLM_LAUNCH_CHECK();
  return TLLM_OK;
}

}  // namespace
}  // namespace tllm

using namespace tllm;

extern "C" int tllm_gqa_prefill(
    const float *q, long q_row_stride, long q_head_stride, const void *k_cache,
    const void *v_cache, int kv_dtype, const int32_t *blocks, int n_blocks,
    void *out, int out_dtype, long out_plane_rows, long out_row_stride,
    long out_head_stride, int n_head, int n_kv_head, int head_dim,
    int cache_batch, int max_seq, float sm_scale, tllm_stream_t stream) {
  TLLM_INJECT("launch");
  TLLM_CHECK_ARG(n_blocks >= 0, "negative block count");
  if (n_blocks == 0) return TLLM_OK;
  TLLM_CHECK_ARG(n_head > 0 && n_kv_head > 0 && n_head % n_kv_head == 0,
                 "n_head (%d) must be a positive multiple of n_kv_head (%d)",
                 n_head, n_kv_head);
  TLLM_CHECK_ARG(n_head <= 65535 && n_blocks <= (1 << 30), "grid too large");
  TLLM_CHECK_ARG(q && out && k_cache && v_cache && blocks, "NULL pointer");
  TLLM_CHECK_ARG(max_seq > 0 && cache_batch > 0, "max_seq and cache_batch must be > 0");
  if (kv_dtype != TLLM_BF16 || (head_dim != 64 && head_dim != 128)) {
    set_error("tllm_gqa_prefill supports bf16 caches with head_dim 64 or 128 "
              "(got dtype %d, head_dim %d); use tllm_gqa_rows", kv_dtype, head_dim);
    return TLLM_ERR_UNSUPPORTED;
  }
  TLLM_CHECK_ARG(out_dtype == TLLM_F32 || out_dtype == TLLM_SPLIT ||
                     out_dtype == TLLM_BF16,
                 "out_dtype must be F32, SPLIT or BF16");
  TLLM_CHECK_ARG(((uintptr_t)k_cache & 15) == 0 && ((uintptr_t)v_cache & 15) == 0 &&
                     ((uintptr_t)blocks & 15) == 0,
                 "caches and the block table must be 16-byte aligned");
  TLLM_CHECK_ARG(((uintptr_t)q & 7) == 0 && q_row_stride % 2 == 0 &&
                     q_head_stride % 2 == 0 && out_row_stride % 2 == 0 &&
                     out_head_stride % 2 == 0,
                 "q must be 8-byte aligned and the strides even");
  PrefillParams p{};
  p.q = q;
  p.q_sr = q_row_stride;
  p.q_sh = q_head_stride;
  if (out_dtype == TLLM_F32) {
    p.out = static_cast<float *>(out);
  } else {
    p.out_act = static_cast<uint16_t *>(out);
    p.out_plane = out_plane_rows * out_row_stride;
    p.out_planes = out_dtype == TLLM_SPLIT ? 2 : 1;
  }
  p.o_sr = out_row_stride;
  p.o_sh = out_head_stride;
  p.blocks = reinterpret_cast<const int4 *>(blocks);
  p.err = device_error_ptr();
  TLLM_CHECK_ARG(p.err, "device error word unavailable");
  p.n_head = n_head;
  p.n_kv = n_kv_head;
  p.group = n_head / n_kv_head;
  p.max_seq = max_seq;
  p.cache_batch = cache_batch;
  if (sm_scale <= 0.f) sm_scale = 1.0f / sqrtf((float)head_dim);
  p.qscale = sm_scale * kPfLog2e;
  CUtensorMap mk, mv;
  int rc = make_kv_map(&mk, k_cache, kv_dtype, head_dim, max_seq,
                       (long)cache_batch * n_kv_head, kPfKT, 64, true);
  if (rc) return rc;
  rc = make_kv_map(&mv, v_cache, kv_dtype, head_dim, max_seq,
                   (long)cache_batch * n_kv_head, kPfKT, 64, true);
  if (rc) return rc;
  cudaStream_t st = resolve(stream);
  return head_dim == 64 ? launch_prefill<64>(p, mk, mv, n_blocks, st)
                        : launch_prefill<128>(p, mk, mv, n_blocks, st);
}
