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
//    epilogue. Activations arrive as bf16 (TLLM_BF16, one MMA per k-slice)
//    or in the TLLM_SPLIT format (bf16 hi and lo planes, one MMA for each:
//    the product keeps ~16 mantissa bits of the fp32 activations while both
//    operands are bf16). K is split across CTAs when there are too few
//    weight tiles to occupy the GPU: the S CTAs of a tile form a thread-block
//    cluster, each stages its accumulator tile in shared memory, and after a
//    cluster barrier each reduces a slice of the tile over distributed shared
//    memory (ranks summed in fixed order, so results do not depend on
//    scheduling) and runs the epilogue for that slice.
//  * linear_f32_kernel (fp32 weights, GPT-2 and the fp32 drop-in): one warp
//    per (weight-row pair, K slice), 16-byte streaming loads along K with
//    two batches in flight per lane, fp32 FMA, same epilogues.
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
#include <cstdlib>

#include "common.cuh"
#include "p2p.cuh"

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
  EPI_SCATTER = 5, // partial rows into every rank's receive slot (p2p.cu)
};

struct Epilogue {
  int op;
  const float *bias;   // [N] or null (in weight-row order)
  float *out;          // [M, ld_out] fp32, or null when out_split is set
  uint16_t *out_split; // bf16 operand-format output (TLLM_SPLIT or TLLM_BF16)
  size_t out_plane;    //   planes out_plane elements apart
  int out_planes;      //   2 (SPLIT) or 1 (BF16)
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
  // EPI_SCATTER
  const P2PDev *p2p;
  // RMSNorm folded into the neighbouring projections (tcgen05 kernel only).
  // Producer (EPI_RESID): besides out, fx[m, n] = out[m, n] * fx_w[n] in
  // operand format and ss_out[tile * ss_ld + m] = sum of out[m, n]^2 over
  // each 128-column weight tile.
  // Consumer (EPI_STORE / EPI_SWIGLU / EPI_QKV): row m of the product divided
  // by sqrt(sum_{p < ss_parts} ss_in[p * ss_ld + m] / ss_cols + eps).
  const float *fx_w;
  uint16_t *fx;
  size_t fx_plane;
  int fx_planes;
  float *ss_out;
  const float *ss_in;
  int ss_parts, ss_cols, ss_ld;
  float ss_eps;
};

// sqrt(mean of squares + eps) of activation rows m0 .. m0 + rows - 1 from
// the producer's partial sums, into s_rms[0 .. rows), computed by the nthr
// threads t = 0 .. nthr - 1 (whole warps): T threads per row (a power of two
// <= 32, as many as the threads allow) each add the parts j, j + T, ... in
// order, then a fixed butterfly -- deterministic, and every row's loads are
// in flight at once.
__device__ __forceinline__ void fold_rms_rows(const Epilogue &e, int m0, int rows,
                                              int M, float *s_rms, int t, int nthr) {
  int T = 1;
  while (T < 32 && T * 2 * rows <= nthr) T *= 2;
  const int per_pass = nthr / T;
  for (int base = 0; base < rows; base += per_pass) {
    const int rl = base + t / T;
    const int j = t % T;
    const int m = m0 + rl;
    float acc = 0.f;
    if (rl < rows && m < M) {
      // eight loads in flight per round, added in part order
      for (int p0 = j; p0 < e.ss_parts; p0 += 8 * T) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int pp = p0 + u * T;
          v[u] = pp < e.ss_parts ? e.ss_in[(size_t)pp * e.ss_ld + m] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) acc += v[u];
      }
    }
    for (int o = T / 2; o >= 1; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (j == 0 && rl < rows)
      s_rms[rl] = m < M ? sqrtf(acc / (float)e.ss_cols + e.ss_eps) : 1.f;
  }
}

__device__ __forceinline__ float gelu_tanh(float x) {
  // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) with tanh built from
  // exp(-2|u|) as in triton_llm/kernels/gelu.py:17-28, :50-51
  const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  const float e = expf(-2.f * fabsf(u));
  const float t = (u < 0.f ? -1.f : 1.f) * (1.f - e) / (1.f + e);
  return 0.5f * x * (1.f + t);
}
__device__ __forceinline__ float silu_ref(float x) {
  // x * sigmoid(x), sigmoid from exp(-|x|) (triton_llm/kernels/swiglu.py:51-54):
  // 1 / (1 + e) for x >= 0 (the correctly rounded reciprocal, equal to the
  // IEEE quotient), e / (1 + e) as e times it for x < 0 (within 1 ulp); no
  // division, so the epilogue's many independent evaluations overlap
  const float e = expf(-fabsf(x));
  const float r = __frcp_rn(1.f + e);
  const float sig = x >= 0.f ? r : e * r;
  return x * sig;
}

__device__ __forceinline__ void store_out(const Epilogue &e, size_t idx,
                                          float v) {
  if (e.out_split)
    store_act(e.out_split, e.out_plane, idx, v, e.out_planes);
  else
    e.out[idx] = v;
}

// Two adjacent outputs idx, idx + 1 (idx even) with one store per plane.
__device__ __forceinline__ void store_out2(const Epilogue &e, size_t idx,
                                           float a0, float a1) {
  if (e.out_split) {
    const uint16_t h0 = f32_to_bf16_bits(a0), h1 = f32_to_bf16_bits(a1);
    *reinterpret_cast<uint32_t *>(e.out_split + idx) = (uint32_t)h0 | ((uint32_t)h1 << 16);
    if (e.out_planes == 2) {
      const uint16_t l0 = f32_to_bf16_bits(a0 - bf16_bits_to_f32(h0));
      const uint16_t l1 = f32_to_bf16_bits(a1 - bf16_bits_to_f32(h1));
      *reinterpret_cast<uint32_t *>(e.out_split + e.out_plane + idx) =
          (uint32_t)l0 | ((uint32_t)l1 << 16);
    }
  } else {
    *reinterpret_cast<float2 *>(e.out + idx) = make_float2(a0, a1);
  }
}

// Where weight row r of a QKV projection goes (r is the first row of a
// pair r, r + 8): head, dims d0 and d1 = d0 + D/2 within the head.
struct QkvGeom {
  int head, local, d0, d1;
  bool is_q, is_v;
};
__device__ __forceinline__ QkvGeom qkv_geom(const Epilogue &e, int r) {
  QkvGeom g;
  const int D = e.D;
  g.head = r / D;
  g.local = r - g.head * D;                      // in the first 8 of a 16
  g.d0 = (g.local >> 4) * 8 + (g.local & 7);
  g.d1 = g.d0 + D / 2;
  g.is_q = g.head < e.H;
  g.is_v = g.head >= e.H + e.Hkv;
  return g;
}
// x0' = x0 c - x1 s, x1' = x0 s + x1 c with each product rounded (no FMA
// contraction), as numpy computes rope.py:65-66
__device__ __forceinline__ void rope_pair(float c, float s, float &x0, float &x1) {
  const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
  const float y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
  x0 = y0;
  x1 = y1;
}
// q heads to q_out (M, H, D); k / v heads into the caches at (seq, pos)
__device__ __forceinline__ void qkv_store(const Epilogue &e, const QkvGeom &g,
                                          int m, int pos, int seq, float x0,
                                          float x1) {
  const int D = e.D;
  if (g.is_q) {
    float *q = e.q_out + ((size_t)m * e.H + g.head) * D;
    q[g.d0] = x0;
    q[g.d1] = x1;
    return;
  }
  const int kvh = g.is_v ? g.head - e.H - e.Hkv : g.head - e.H;
  if (pos < 0 || pos >= e.max_seq || seq < 0) {
    atomicOr(e.err, DEV_ERR_LEN_CLAMPED);
    return;
  }
  const size_t off = (((size_t)seq * e.Hkv + kvh) * e.max_seq + pos) * D;
  void *cache = g.is_v ? e.v_cache : e.k_cache;
  if (e.kv_bf16) {
    uint16_t *c = static_cast<uint16_t *>(cache) + off;
    c[g.d0] = f32_to_bf16_bits(x0);
    c[g.d1] = f32_to_bf16_bits(x1);
  } else {
    float *c = static_cast<float *>(cache) + off;
    c[g.d0] = x0;
    c[g.d1] = x1;
  }
  if (e.lens_out && g.head == e.H && g.local == 0) e.lens_out[seq] = pos + 1;
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
    const QkvGeom g = qkv_geom(e, r);
    float x0 = v0 + (e.bias ? e.bias[r] : 0.f);
    float x1 = v1 + (e.bias ? e.bias[r1] : 0.f);
    const int pos = e.row_pos[m];
    const int seq = e.row_seq[m];
    if (e.cos && !g.is_v && pos >= 0 && pos < e.max_seq)
      rope_pair(e.cos[(size_t)pos * (e.D / 2) + g.d0],
                e.sin[(size_t)pos * (e.D / 2) + g.d0], x0, x1);
    qkv_store(e, g, m, pos, seq, x0, x1);
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
// 8 warps: warps 0-3 stream and issue (one thread each), all 8 share the
// epilogue, where a single warp per scheduler would leave the latency of
// TMEM, distributed shared memory and global accesses exposed
constexpr int kTcWarps = 8;
constexpr int kTcThreads = kTcWarps * 32;
// Epilogue rows a warp finishes at once. The epilogue runs once per CTA and
// launch, after other kernels have used the SM, so its code comes from a
// cold instruction cache: one row at a time (and the split ranks in a loop)
// keeps it short. Measured at config 4 against four rows at a time: +10 %
// tokens/s at 8 rows per GPU, +4 % at 32, +1.4 % at 64.
constexpr int kTcRB = 1;
// MMA-issuing threads: 4 (warps 1, 3, 5, 7, two per odd scheduler), 2 when
// four accumulators of the tile do not fit in TMEM's 512 columns. Issuer i
// takes the chunks c = i (mod issuers), so each ring depth is a multiple of
// the issuer count: every ring slot then belongs to one issuer, which waits
// for the slot's fills strictly in order (an issuer may otherwise run a whole
// ring ahead of another and pass a parity wait on a fill two phases old).
constexpr int kTcMaxIssuers = 4;
__host__ __device__ constexpr int tc_issuer_index(int warp) {
  return warp == 1 ? 0 : warp == 3 ? 1 : warp == 5 ? 2 : warp == 7 ? 3
       : kTcMaxIssuers;
}
constexpr int kTcBN = 128;            // weight rows per CTA (MMA M)
constexpr int kTcBK = 64;             // K per stage (one 128-byte row)
constexpr int kTcW = kTcBN * kTcBK * 2;  // weight tile bytes (16 KB)
constexpr int kTcMaxSplit = 8;        // portable cluster size
constexpr int kTcMaxWS = 12;          // weight ring stages (at most)
constexpr int kTcMaxXS = 8;           // activation ring stages (at most)

struct TcParams {
  Epilogue e;
  int M, N, K, S, k_chunks, n_tiles, wstages, xstages;
  int nacc;      // independent TMEM accumulators (a multiple of issuers)
  int issuers;   // MMA-issuing threads (2 or 4; divides both ring depths)
  uint32_t tcols;  // TMEM columns allocated (power of two >= 32)
  int w_tiled;   // TLLM_BF16_TILED weights: tile (nt, kc) = rows
                 // (nt * k_chunks + kc) * 128 .. +127 of a (., 64) view
};

// one activation stage: the bf16 planes (1 or 2) of an MT x 64 tile
__host__ __device__ constexpr int tc_x_bytes(int MT, int PL) {
  return PL * MT * kTcBK * 2;
}
// activation ring depth (default): up to 8 stages in at most 128 KB

// TMEM accumulators: one per MMA-issuing thread by default (the epilogue
// sums them in fixed order); TLLM_LINEAR_NACC (even) gives each issuer more,
// rotated over the MMAs of a chunk.
__host__ __device__ constexpr int tc_nacc(int) { return 2; }

// Weight tiles and activation tiles travel in two rings: the weights are
// the HBM stream (a deep ring keeps many bytes in flight per SM), the
// activation tiles are L2 hits shared by every CTA (a 2-stage ring suffices).
// The producer of the weight ring starts before the previous kernel has
// finished (programmatic dependent launch); the activation producer waits
// for it.
template <int MT, int OP, int PL>
__global__ void __launch_bounds__(kTcThreads, 1)
    linear_tc_kernel(const TcParams p, const __grid_constant__ CUtensorMap tw,
                     const __grid_constant__ CUtensorMap tx) {
  constexpr int X_PLANE = MT * kTcBK * 2;    // one bf16 plane of the tile
  constexpr int X_BYTES = tc_x_bytes(MT, PL);
  const uint32_t TCOLS = p.tcols;
  const int NACC = p.nacc;
  const int NI = p.issuers;
  constexpr uint32_t IDESC = umma_idesc_bf16(kTcBN, MT);
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint64_t wfull[kTcMaxWS], wempty[kTcMaxWS];
  const int kTcXS = p.xstages;
  __shared__ uint64_t xfull[kTcMaxXS], xempty[kTcMaxXS], accb[1];
  __shared__ uint32_t s_tmem;
  __shared__ int s_wissued, s_xissued, s_fail;
  __shared__ int s_empty_acc[kTcMaxIssuers];   // an issuer whose accumulators were never written
  __shared__ unsigned s_epoch;     // EPI_SCATTER: this call's number
  __shared__ float s_rms[MT];      // folded RMSNorm: rms of each activation row
  const int WS = p.wstages;
  uint8_t *wring = smem;
  uint8_t *xring = smem + WS * kTcW;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  // 128-byte-swizzled TMA tiles and UMMA descriptors need 1024-byte
  // aligned stage buffers
  if (smem_u32(smem) & 1023) {
    if (tid == 0) atomicOr(p.e.err, DEV_ERR_SMEM_ALIGN);
    return;
  }
  // every ring slot must belong to one MMA issuer (the host plans it so)
  if (WS % NI != 0 || p.xstages % NI != 0 || NI > kTcMaxIssuers) {
    if (tid == 0) atomicOr(p.e.err, DEV_ERR_LAYOUT);
    return;
  }
  griddep_launch();
  const int nt = blockIdx.x;
  const int split = blockIdx.y;
  const int mt = blockIdx.z;
  const int per = (p.k_chunks + p.S - 1) / p.S;
  const int kc0 = split * per;
  const int kc1 = min(kc0 + per, p.k_chunks);
  const int nch = kc1 > kc0 ? kc1 - kc0 : 0;

  if (tid == 0) {
    for (int s = 0; s < WS; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 1);
    }
    for (int s = 0; s < kTcXS; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);
    }
    mbar_init(accb, NI);   // one arrival per MMA issuer
    s_wissued = 0;
    s_xissued = 0;
    s_fail = 0;
    for (int i = 0; i < kTcMaxIssuers; ++i) s_empty_acc[i] = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&s_tmem, TCOLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp == 0) {
    if (lane == 0) {
      // weight producer: read once, evict first; needs nothing from the
      // previous kernel
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tw) : "memory");
      const uint64_t pol = l2_policy_evict_first();
      int c = 0;
      for (; c < nch; ++c) {
        const int s = c % WS;
        if (c >= WS && !mbar_wait_bounded(&wempty[s], ((c / WS) - 1) & 1)) {
          s_fail = 1;
          break;
        }
        mbar_expect_tx(&wfull[s], kTcW);
        if (p.w_tiled)
          tma_load_2d_hint(wring + s * kTcW, &tw, &wfull[s], 0,
                           (nt * p.k_chunks + kc0 + c) * kTcBN, pol);
        else
          tma_load_2d_hint(wring + s * kTcW, &tw, &wfull[s], (kc0 + c) * kTcBK,
                           nt * kTcBN, pol);
      }
      s_wissued = c;
    }
    __syncwarp();
  } else if (warp == 2) {
    if (lane == 0) {
      // activation producer: the tiles are written by the previous kernel
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tx) : "memory");
      const uint64_t pol = l2_policy_evict_last();
      griddep_wait();
      int c = 0;
      for (; c < nch; ++c) {
        const int s = c % kTcXS;
        if (c >= kTcXS &&
            !mbar_wait_bounded(&xempty[s], ((c / kTcXS) - 1) & 1)) {
          s_fail = 1;
          break;
        }
        uint8_t *st = xring + s * X_BYTES;
        const int k0 = (kc0 + c) * kTcBK;
        mbar_expect_tx(&xfull[s], X_BYTES);
        tma_load_3d_hint(st, &tx, &xfull[s], k0, mt * MT, 0, pol);
        if (PL == 2)
          tma_load_3d_hint(st + X_PLANE, &tx, &xfull[s], k0, mt * MT, 1, pol);
      }
      s_xissued = c;
    }
    __syncwarp();
  } else if (tc_issuer_index(warp) < NI) {
    if (lane == 0) {
      // MMA issuers: NI threads (warps 1, 3, 5, 7, 4, 6 in that order,
      // spread over the four schedulers) take k-chunks in turn, each with
      // its own share of the accumulators, so one thread's barrier waits and
      // MMA issue overlap the others'. Per chunk and plane:
      // D[128 x MT] += W[128 x 16] . X[MT x 16]^T for each k-slice.
      const int who = tc_issuer_index(warp);
      const int nacc = NACC / NI;                   // accumulators per issuer
      const uint32_t tacc = tmem + who * nacc * MT;
      int c = who;
      bool first = true;
      for (; c < nch; c += NI) {
        const int ws = c % WS;
        const int xs = c % kTcXS;
        if (!mbar_wait_bounded(&wfull[ws], (c / WS) & 1) ||
            !mbar_wait_bounded(&xfull[xs], (c / kTcXS) & 1)) {
          s_fail = 1;
          break;
        }
        tc_fence_after();
        const uint64_t a = umma_desc_sw128(smem_u32(wring + ws * kTcW));
        const uint32_t xa = smem_u32(xring + xs * X_BYTES);
        const uint64_t bh = umma_desc_sw128(xa);
        const uint64_t bl = umma_desc_sw128(xa + X_PLANE);
#pragma unroll
        for (int j = 0; j < PL * (kTcBK / 16); ++j) {
          const int kk = j / PL;        // k-slice
          const int acc = j % nacc;     // accumulator of this MMA
          // the first MMA into an accumulator initialises it
          const uint32_t accumulate = (!first || j >= nacc) ? 1u : 0u;
          umma_bf16(tacc + acc * MT, a + 2 * kk,
                    ((PL == 2 && (j & 1)) ? bl : bh) + 2 * kk, IDESC, accumulate);
        }
        umma_commit(&wempty[ws]);   // slots free once these MMAs are done
        umma_commit(&xempty[xs]);
        first = false;
      }
      // an issuer that got no chunk zeroes its accumulators by marking them
      if (first) s_empty_acc[who] = 1;
      umma_commit(accb);            // this issuer's MMAs complete
    }
    __syncwarp();
  } else if ((warp == 4 || warp == 6) && p.e.ss_in) {
    // folded RMSNorm consumer: warps 4 and 6 (idle in the main loop) sum
    // the producer's partials of this tile's activation rows
    griddep_wait();
    fold_rms_rows(p.e, mt * MT, MT, p.M, s_rms, (warp == 4 ? 0 : 32) + lane, 64);
  }

  // ---- epilogue ----
  // 1. the four warps copy the accumulator (TMEM lanes 32*warp..+31) into
  //    shared memory, column-major: tile[m * 128 + r] (the rings are free)
  const bool acc_ok = mbar_wait_bounded(accb, 0);
  tc_fence_after();
  griddep_wait();   // the epilogue reads / writes buffers of earlier kernels
  if constexpr (OP == EPI_SCATTER) {
    // calls completed so far (this rank's reader of the previous call has
    // finished): this call's number
    if (tid == 0)
      s_epoch = (unsigned)*reinterpret_cast<volatile const int *>(&p.e.p2p->state[0]) + 1u;
  }
  __syncthreads();  // s_fail visible
  const bool valid = acc_ok && !s_fail && nch > 0;
  float *tile = reinterpret_cast<float *>(smem);
  // a warp reads the TMEM lane quarter warp % 4; warps w and w + 4 take
  // alternate column chunks
  const int r_own = (warp & 3) * 32 + lane;
  const uint32_t t_lane = tmem + ((uint32_t)((warp & 3) * 32) << 16);
  // 32 columns per TMEM load (16 for the narrowest tile), one wait each
  constexpr int CW = MT >= 32 ? 32 : 16;
#pragma unroll 1
  for (int c0 = (warp >> 2) * CW; c0 < MT; c0 += 2 * CW) {
    float v[CW];
#pragma unroll
    for (int j = 0; j < CW; ++j) v[j] = 0.f;
    if (valid) {
      const int nacc = NACC / NI;
#pragma unroll 1
      for (int acc = 0; acc < NACC; ++acc) {   // fixed order: deterministic
        if (s_empty_acc[acc / nacc]) continue;
        float u[CW];
        if constexpr (CW == 32)
          tmem_ld32(t_lane + acc * MT + c0, u);
        else
          tmem_ld16(t_lane + acc * MT + c0, u);
#pragma unroll
        for (int j = 0; j < CW; ++j) v[j] += u[j];
      }
    }
#pragma unroll
    for (int j = 0; j < CW; ++j) tile[(c0 + j) * kTcBN + r_own] = v[j];
  }
  // 2. every split of this tile has staged its partial
  const int S = p.S;
  if (S > 1)
    cluster_sync();
  else
    __syncthreads();
  // 3. this CTA finishes activation rows m = rank, rank + S, ... of the
  //    tile, one warp per row: the splits are summed in rank order and the
  //    epilogue stores whole output rows (lane l covers weight rows
  //    4l .. 4l + 3 of the tile)
  const int rank = S > 1 ? (int)cluster_ctarank() : 0;
  const uint32_t tile_s = smem_u32(tile);
  const int row0 = nt * kTcBN;
#pragma unroll 1
  for (int mlb = rank + warp * S; mlb < MT; mlb += kTcWarps * S * kTcRB) {
    int mrow[kTcRB];
    bool in_tile[kTcRB], ok[kTcRB];
#pragma unroll
    for (int i = 0; i < kTcRB; ++i) {
      const int ml = mlb + i * kTcWarps * S;
      mrow[i] = mt * MT + ml;
      in_tile[i] = ml < MT;
      ok[i] = in_tile[i] && mrow[i] < p.M;
    }
    if constexpr (OP == EPI_SCATTER || OP == EPI_STORE || OP == EPI_RESID ||
                  OP == EPI_GELU) {
      // lane l: weight rows 4l .. 4l + 3 of the tile, every row of the group
      const int r4 = lane * 4;
      const int n = row0 + r4;
      float4 v[kTcRB];
#pragma unroll
      for (int i = 0; i < kTcRB; ++i) {
        const int ml = mlb + i * kTcWarps * S;
        v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (!in_tile[i]) continue;
        if (S == 1) {
          v[i] = *reinterpret_cast<const float4 *>(&tile[ml * kTcBN + r4]);
        } else {
#pragma unroll 1
          for (int q = 0; q < kTcMaxSplit; ++q) {
            if (q < S) {
              const float4 u = ld_dsmem_f32x4(tile_s + (ml * kTcBN + r4) * 4, q);
              v[i].x += u.x;
              v[i].y += u.y;
              v[i].z += u.z;
              v[i].w += u.w;
            }
          }
        }
      }
      if constexpr (OP == EPI_SCATTER) {
        // each value with this call's number, as 64-bit words, into this
        // rank's slot on every rank
        const P2PDev *P = p.e.p2p;
        const unsigned ep = s_epoch;
        if (n < p.N) {
#pragma unroll
          for (int i = 0; i < kTcRB; ++i) {
            if (!ok[i]) continue;
            const size_t off =
                (((size_t)(ep & 1) * P->size + P->rank) * P->mmax + mrow[i]) * P->ncols + n;
            const unsigned long long w0 = p2p_word(v[i].x, ep), w1 = p2p_word(v[i].y, ep);
            const unsigned long long w2 = p2p_word(v[i].z, ep), w3 = p2p_word(v[i].w, ep);
            for (int q = 0; q < P->size; ++q) {
              unsigned long long *d = P->peer_recv[q] + off;
              asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(d), "l"(w0),
                           "l"(w1) : "memory");
              asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(d + 2),
                           "l"(w2), "l"(w3) : "memory");
            }
          }
        }
      } else {
        const Epilogue &e = p.e;
        const bool full = n + 3 < p.N;
        float fw[4] = {0.f, 0.f, 0.f, 0.f};   // folded producer: next norm weight
        if (OP == EPI_RESID && e.ss_out) {
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if (n + k < p.N) fw[k] = e.fx_w[n + k];
        }
        float bias[4] = {0.f, 0.f, 0.f, 0.f};
        if (e.bias) {
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if (n + k < p.N) bias[k] = e.bias[n + k];
        }
        // residual rows of the whole group before the first use
        float rv[kTcRB][4];
#pragma unroll
        for (int i = 0; i < kTcRB; ++i) {
#pragma unroll
          for (int k = 0; k < 4; ++k) rv[i][k] = 0.f;
          if constexpr (OP == EPI_RESID) {
            const size_t o = (size_t)mrow[i] * e.ld_out + n;
            if (!ok[i]) continue;
            if (full && (o & 3) == 0) {
              const float4 t = *reinterpret_cast<const float4 *>(&e.resid[o]);
              rv[i][0] = t.x;
              rv[i][1] = t.y;
              rv[i][2] = t.z;
              rv[i][3] = t.w;
            } else {
#pragma unroll
              for (int k = 0; k < 4; ++k)
                if (n + k < p.N) rv[i][k] = e.resid[o + k];
            }
          }
        }
#pragma unroll
        for (int i = 0; i < kTcRB; ++i) {
          if (!ok[i]) continue;   // uniform over the warp (one row per i)
          const size_t o = (size_t)mrow[i] * e.ld_out + n;
          float a[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
          if (OP == EPI_STORE && e.ss_in) {
            const float rms = s_rms[mrow[i] - mt * MT];
#pragma unroll
            for (int k = 0; k < 4; ++k) a[k] = a[k] / rms;
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            if (e.bias) a[k] += bias[k];
            if constexpr (OP == EPI_RESID) a[k] = rv[i][k] + a[k];
            if constexpr (OP == EPI_GELU) a[k] = gelu_tanh(a[k]);
          }
          if (full && !e.out_split && ((o & 3) == 0)) {
            *reinterpret_cast<float4 *>(&e.out[o]) = make_float4(a[0], a[1], a[2], a[3]);
          } else {
#pragma unroll
            for (int k = 0; k < 4; ++k)
              if (n + k < p.N) store_out(e, o + k, a[k]);
          }
          if (OP == EPI_RESID && e.ss_out) {
            // the next RMSNorm, folded: h * w as its projection's operand and
            // the sum of squares of h over this tile's 128 columns (the warp
            // holds the whole row of the tile)
            float sq = 0.f;
            if (full && (o & 3) == 0 && (e.fx_plane & 3) == 0) {
              // four adjacent operand values: one 8-byte store per plane
              uint32_t hi[2], lo[2];
#pragma unroll
              for (int k = 0; k < 4; k += 2) {
                const float f0 = a[k] * fw[k], f1 = a[k + 1] * fw[k + 1];
                const uint16_t h0 = f32_to_bf16_bits(f0), h1 = f32_to_bf16_bits(f1);
                hi[k / 2] = (uint32_t)h0 | ((uint32_t)h1 << 16);
                lo[k / 2] = (uint32_t)f32_to_bf16_bits(f0 - bf16_bits_to_f32(h0)) |
                            ((uint32_t)f32_to_bf16_bits(f1 - bf16_bits_to_f32(h1)) << 16);
                sq = fmaf(a[k], a[k], sq);
                sq = fmaf(a[k + 1], a[k + 1], sq);
              }
              *reinterpret_cast<uint2 *>(e.fx + o) = make_uint2(hi[0], hi[1]);
              if (e.fx_planes == 2)
                *reinterpret_cast<uint2 *>(e.fx + e.fx_plane + o) = make_uint2(lo[0], lo[1]);
            } else {
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                if (n + k < p.N) {
                  store_act(e.fx, e.fx_plane, o + k, a[k] * fw[k], e.fx_planes);
                  sq = fmaf(a[k], a[k], sq);
                }
              }
            }
#pragma unroll
            for (int sh = 1; sh < 32; sh <<= 1) sq += __shfl_xor_sync(0xffffffffu, sq, sh);
            if (lane == 0) e.ss_out[(size_t)nt * e.ss_ld + mrow[i]] = sq;
          }
        }
      }
    } else {
      // SwiGLU / QKV combine weight rows r and r + 8 of each 16-row block:
      // lane l takes row pairs 2l and 2l + 1 of the 64 in this tile row
      const Epilogue &e = p.e;
      int rr[2];
      bool live[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int pr = lane * 2 + h;
        rr[h] = (pr >> 3) * 16 + (pr & 7);
        live[h] = row0 + rr[h] + 8 < p.N;
      }
      float v0[kTcRB][2], v1[kTcRB][2];
#pragma unroll
      for (int i = 0; i < kTcRB; ++i) {
        const int ml = mlb + i * kTcWarps * S;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          v0[i][h] = 0.f;
          v1[i][h] = 0.f;
          if (!in_tile[i]) continue;
          const int r = rr[h];
          if (S == 1) {
            v0[i][h] = tile[ml * kTcBN + r];
            v1[i][h] = tile[ml * kTcBN + r + 8];
          } else {
#pragma unroll 1
            for (int q = 0; q < kTcMaxSplit; ++q) {
              if (q < S) {
                v0[i][h] += ld_dsmem_f32(tile_s + (ml * kTcBN + r) * 4, q);
                v1[i][h] += ld_dsmem_f32(tile_s + (ml * kTcBN + r + 8) * 4, q);
              }
            }
          }
        }
      }
      if (p.e.ss_in) {
#pragma unroll
        for (int i = 0; i < kTcRB; ++i) {
          if (!in_tile[i]) continue;
          const float rms = s_rms[mlb + i * kTcWarps * S];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            v0[i][h] = v0[i][h] / rms;
            v1[i][h] = v1[i][h] / rms;
          }
        }
      }
      if constexpr (OP == EPI_SWIGLU) {
        // pairs 2l and 2l + 1 give adjacent outputs j0, j0 + 1
        const int r = row0 + rr[0];
        const int j0 = (r >> 4) * 8 + (r & 7);
        const bool pack =
            e.out_split ? ((reinterpret_cast<uintptr_t>(e.out_split) & 3) == 0 &&
                           (e.out_plane & 1) == 0)
                        : (reinterpret_cast<uintptr_t>(e.out) & 7) == 0;
        float a[kTcRB][2];
#pragma unroll
        for (int i = 0; i < kTcRB; ++i)
#pragma unroll
          for (int h = 0; h < 2; ++h) a[i][h] = silu_ref(v0[i][h]) * v1[i][h];
#pragma unroll
        for (int i = 0; i < kTcRB; ++i) {
          if (!ok[i]) continue;
          const size_t o = (size_t)mrow[i] * e.ld_out + j0;
          if (pack && live[0] && live[1] && (o & 1) == 0) {
            store_out2(e, o, a[i][0], a[i][1]);
          } else {
#pragma unroll
            for (int h = 0; h < 2; ++h)
              if (live[h]) store_out(e, o + h, a[i][h]);
          }
        }
      } else {  // EPI_QKV
        QkvGeom g[2];
        float b0[2], b1[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = row0 + rr[h];
          g[h] = qkv_geom(e, r);
          b0[h] = (e.bias && live[h]) ? e.bias[r] : 0.f;
          b1[h] = (e.bias && live[h]) ? e.bias[r + 8] : 0.f;
        }
        int pos[kTcRB], seq[kTcRB];
#pragma unroll
        for (int i = 0; i < kTcRB; ++i) {
          pos[i] = ok[i] ? e.row_pos[mrow[i]] : -1;
          seq[i] = ok[i] ? e.row_seq[mrow[i]] : -1;
        }
        float cs[kTcRB][2], sn[kTcRB][2];
#pragma unroll
        for (int i = 0; i < kTcRB; ++i) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            cs[i][h] = 1.f;
            sn[i][h] = 0.f;
            if (ok[i] && live[h] && e.cos && !g[h].is_v && pos[i] >= 0 &&
                pos[i] < e.max_seq) {
              const size_t t = (size_t)pos[i] * (e.D / 2) + g[h].d0;
              cs[i][h] = e.cos[t];
              sn[i][h] = e.sin[t];
            }
          }
        }
#pragma unroll
        for (int i = 0; i < kTcRB; ++i) {
          if (!ok[i]) continue;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (!live[h]) continue;
            float x0 = v0[i][h] + b0[h];
            float x1 = v1[i][h] + b1[h];
            if (e.cos && !g[h].is_v && pos[i] >= 0 && pos[i] < e.max_seq)
              rope_pair(cs[i][h], sn[i][h], x0, x1);
            qkv_store(e, g[h], mrow[i], pos[i], seq[i], x0, x1);
          }
        }
      }
    }
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
  if (tid == 0 && (s_fail || !acc_ok)) {
    // a failed wait may have left fills in flight: wait (bounded) for the
    // last fill issued into every slot; without a failure every issued
    // fill was consumed
    for (int c = s_wissued > WS ? s_wissued - WS : 0; c < s_wissued; ++c)
      mbar_wait_bounded(&wfull[c % WS], (c / WS) & 1);
    for (int c = s_xissued > kTcXS ? s_xissued - kTcXS : 0; c < s_xissued; ++c)
      mbar_wait_bounded(&xfull[c % kTcXS], (c / kTcXS) & 1);
  }
  if (warp == 1) tmem_free(tmem, TCOLS);
}

// ------------------------------------------------------------------------
// fp32 weights, CUDA cores: a warp per (weight-row pair (r, r + 8), K slice)
// ------------------------------------------------------------------------
constexpr int kF32Warps = 8;
constexpr int kF32U = 4;   // float4 loads of each row in flight per lane and batch

__device__ __forceinline__ float4 f32_ld4(const float *p) {
  const uint4 u = ld_stream(p);
  return make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z),
                     __uint_as_float(u.w));
}

// A CTA takes kF32Warps / KS row pairs; the KS warps of a pair stream KS
// consecutive K slices (multiples of 128 floats), each lane keeping two
// batches of kF32U float4 loads per row in flight (the batch being summed
// and the next one). The first batch is issued before the wait for the
// previous kernel (weights do not depend on it). The KS partial sums of a
// pair are added in slice order through shared memory.
template <int MB, int KS>
__global__ void __launch_bounds__(kF32Warps * 32)
    linear_f32_kernel(const float *x, const float *w, Epilogue e, int M,
                      int N, int K, int m0) {
  constexpr int PPC = kF32Warps / KS;
  __shared__ float s_part[kF32Warps][2][MB];
  griddep_launch();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int slice = warp % KS;
  const int pair = blockIdx.x * PPC + warp / KS;
  // pair index -> rows r (first 8 of a 16-block) and r + 8
  const int r = (pair >> 3) * 16 + (pair & 7);
  const bool live = r < ((N + 15) / 16) * 16;
  const int r1 = r + 8;
  const bool ok0 = live && r < N, ok1 = live && r1 < N;
  const int steps = (K + 127) / 128;            // warp-wide float4 rows
  const int per = (steps + KS - 1) / KS;
  const int kb = slice * per * 128;
  const int ke = min(K, kb + per * 128);
  const float *w0 = w + (size_t)(ok0 ? r : 0) * K;
  const float *w1 = w + (size_t)(ok1 ? r1 : 0) * K;
  float acc0[MB], acc1[MB];
#pragma unroll
  for (int i = 0; i < MB; ++i) acc0[i] = acc1[i] = 0.f;
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 a[kF32U], b[kF32U];
  int k0 = kb + lane * 4;
#pragma unroll
  for (int u = 0; u < kF32U; ++u) {
    const int k = k0 + u * 128;
    a[u] = ok0 && k < ke ? f32_ld4(w0 + k) : z;
    b[u] = ok1 && k < ke ? f32_ld4(w1 + k) : z;
  }
  griddep_wait();   // x and the epilogue's inputs come from earlier kernels
  for (; k0 < ke; k0 += 128 * kF32U) {
    float4 ca[kF32U], cb[kF32U];
#pragma unroll
    for (int u = 0; u < kF32U; ++u) {
      ca[u] = a[u];
      cb[u] = b[u];
    }
    const int kn = k0 + 128 * kF32U;
#pragma unroll
    for (int u = 0; u < kF32U; ++u) {
      const int k = kn + u * 128;
      a[u] = ok0 && k < ke ? f32_ld4(w0 + k) : z;
      b[u] = ok1 && k < ke ? f32_ld4(w1 + k) : z;
    }
#pragma unroll
    for (int u = 0; u < kF32U; ++u) {
      const int k = k0 + u * 128;
      if (k < ke) {
#pragma unroll
        for (int i = 0; i < MB; ++i) {
          if (m0 + i < M) {
            const float4 xv =
                __ldg(reinterpret_cast<const float4 *>(x + (size_t)(m0 + i) * K + k));
            acc0[i] = fmaf(ca[u].x, xv.x, acc0[i]);
            acc0[i] = fmaf(ca[u].y, xv.y, acc0[i]);
            acc0[i] = fmaf(ca[u].z, xv.z, acc0[i]);
            acc0[i] = fmaf(ca[u].w, xv.w, acc0[i]);
            acc1[i] = fmaf(cb[u].x, xv.x, acc1[i]);
            acc1[i] = fmaf(cb[u].y, xv.y, acc1[i]);
            acc1[i] = fmaf(cb[u].z, xv.z, acc1[i]);
            acc1[i] = fmaf(cb[u].w, xv.w, acc1[i]);
          }
        }
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
  if constexpr (KS > 1) {
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < MB; ++i) {
        s_part[warp][0][i] = acc0[i];
        s_part[warp][1][i] = acc1[i];
      }
    }
    __syncthreads();
    if (slice != 0 || !live) return;
    if (lane < MB) {
      float v0 = 0.f, v1 = 0.f;
#pragma unroll
      for (int s = 0; s < KS; ++s) {
        v0 += s_part[warp + s][0][lane];
        v1 += s_part[warp + s][1][lane];
      }
      epi_pair_rt(e, N, M, r, m0 + lane, v0, v1);
    }
  } else {
    if (!live) return;
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
}

template <int MB>
cudaError_t f32_launch(int KS, int blocks, cudaStream_t st, const float *x, const float *w,
               const Epilogue &e, int M, int N, int K, int m0) {
  const dim3 grid(blocks), block(kF32Warps * 32);
  switch (KS) {
    case 1: return launch_pdl(linear_f32_kernel<MB, 1>, grid, block, 0, st, x, w, e, M, N, K, m0);
    case 2: return launch_pdl(linear_f32_kernel<MB, 2>, grid, block, 0, st, x, w, e, M, N, K, m0);
    case 4: return launch_pdl(linear_f32_kernel<MB, 4>, grid, block, 0, st, x, w, e, M, N, K, m0);
    default: return launch_pdl(linear_f32_kernel<MB, 8>, grid, block, 0, st, x, w, e, M, N, K, m0);
  }
}

// ------------------------------------------------------------------------
// bf16 weights, small batches: mma.sync skinny GEMM
// ------------------------------------------------------------------------
// At decode batch sizes a projection is a weight stream with a few
// activation rows: this kernel has none of the tcgen05 kernel's set-up
// (tensor maps, TMEM, rings, clusters). A warp owns one 16-row weight block
// over one K slice; per 32-k step each lane loads 16 bytes of rows r and
// r + 8 (r = lane / 4) straight from HBM into registers and 16 bytes of each
// of its activation rows (L1 hits), and issues two m16n8k16 MMAs per 8
// activation rows. The k order inside a step is permuted the same way for
// both operands (lane q = lane % 4 supplies logical k {2q, 2q+1, 2q+8,
// 2q+9} of MMA j from physical k 8q + 4j .. 8q + 4j + 3), so every operand
// fragment is one contiguous 16-byte load and the dot products are
// unchanged. The accumulator gives each lane rows r and r + 8 at
// activation rows 2q and 2q + 1 of each 8-row block -- the row pairing of
// the shared epilogue. The KS slices of a block are added in slice order
// through shared memory.
constexpr int kSkWarps = 8;
// 32-k steps per load batch (two batches in flight): U = 4 for long K
// slices; 2 when a warp's slice has at most 8 steps -- the kernel then runs
// its loop body once or twice, from a cold instruction cache, and the
// shorter body measured +3.9 % tokens/s at config 3
constexpr int kSkSmallSlice = 8;

__device__ __forceinline__ void sk_mma(float (&c)[4], uint32_t a0, uint32_t a1,
                                       uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
  // no side effects besides c: not volatile, so loads may be scheduled
  // across it
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, "
      "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 16 bytes of weight row n at k (k % 8 == 0, inside one 64-wide chunk)
__device__ __forceinline__ const uint16_t *sk_w(const uint16_t *w, bool tiled, int kc,
                                                int K, int n, int k) {
  return tiled ? w + ((((size_t)(n >> 7) * kc + (k >> 6)) << 7) + (n & 127)) * kTcBK +
                     (k & 63)
               : w + (size_t)n * K + k;
}

// Epilogue of one lane's accumulators: weight rows r and r + 8, activation
// rows b * 8 + 2q + t (t = 0, 1) for the blocks b in `bmask`; v[b] holds
// {c0, c1, c2, c3} = {(r, t=0), (r, t=1), (r+8, t=0), (r+8, t=1)}. Same
// arithmetic as epi_pair, but every load an op needs (residual rows,
// positions, RoPE tables) is issued before the first store: the stores may
// alias the loads (in-place residual), so per-row code would wait out one
// memory round trip per row.
template <int NB>
__device__ __forceinline__ void sk_epilogue(const Epilogue &e, int N, int M, int r, int q,
                                            const float (&v)[NB][4], unsigned bmask) {
  const int r1 = r + 8;
  const bool ok0 = r < N, ok1 = r1 < N;
  bool okm[NB][2];
  int mm[NB][2];
#pragma unroll
  for (int b = 0; b < NB; ++b)
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      mm[b][t] = b * 8 + 2 * q + t;
      okm[b][t] = ((bmask >> b) & 1) && mm[b][t] < M;
    }
  const int op = e.op;
  if (op == EPI_STORE || op == EPI_RESID || op == EPI_GELU) {
    const float b0 = e.bias && ok0 ? e.bias[r] : 0.f;
    const float b1 = e.bias && ok1 ? e.bias[r1] : 0.f;
    float rv[NB][2][2];
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const size_t o = (size_t)mm[b][t] * e.ld_out;
        const bool ld = op == EPI_RESID && okm[b][t];
        rv[b][t][0] = ld && ok0 ? e.resid[o + r] : 0.f;
        rv[b][t][1] = ld && ok1 ? e.resid[o + r1] : 0.f;
      }
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        if (!okm[b][t]) continue;
        const size_t o = (size_t)mm[b][t] * e.ld_out;
        float a0 = v[b][t] + b0, a1 = v[b][2 + t] + b1;
        if (op == EPI_RESID) {
          a0 = rv[b][t][0] + a0;
          a1 = rv[b][t][1] + a1;
        } else if (op == EPI_GELU) {
          a0 = gelu_tanh(a0);
          a1 = gelu_tanh(a1);
        }
        if (ok0) store_out(e, o + r, a0);
        if (ok1) store_out(e, o + r1, a1);
      }
  } else if (op == EPI_SWIGLU) {
    if (!ok1) return;
    const int j = (r >> 4) * 8 + (r & 7);
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int t = 0; t < 2; ++t)
        if (okm[b][t])
          store_out(e, (size_t)mm[b][t] * e.ld_out + j, silu_ref(v[b][t]) * v[b][2 + t]);
  } else {  // EPI_QKV
    if (!ok1) return;
    const QkvGeom g = qkv_geom(e, r);
    const float b0 = e.bias ? e.bias[r] : 0.f;
    const float b1 = e.bias ? e.bias[r1] : 0.f;
    int pos[NB][2], seq[NB][2];
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        pos[b][t] = okm[b][t] ? e.row_pos[mm[b][t]] : -1;
        seq[b][t] = okm[b][t] ? e.row_seq[mm[b][t]] : -1;
      }
    const bool rot = e.cos && !g.is_v;
    float cs[NB][2], sn[NB][2];
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int ps = pos[b][t];
        const bool in = rot && okm[b][t] && ps >= 0 && ps < e.max_seq;
        const size_t ti = (size_t)(in ? ps : 0) * (e.D / 2) + g.d0;
        cs[b][t] = in ? e.cos[ti] : 1.f;
        sn[b][t] = in ? e.sin[ti] : 0.f;
      }
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        if (!okm[b][t]) continue;
        float x0 = v[b][t] + b0, x1 = v[b][2 + t] + b1;
        const int ps = pos[b][t];
        if (rot && ps >= 0 && ps < e.max_seq) rope_pair(cs[b][t], sn[b][t], x0, x1);
        qkv_store(e, g, mm[b][t], ps, seq[b][t], x0, x1);
      }
  }
}

template <int MT, int PL, int KS, int kSkU>
__global__ void __launch_bounds__(kSkWarps * 32)
    linear_mma_kernel(const uint16_t *x, int x_plane_rows, const uint16_t *w, int tiled,
                      Epilogue e, int M, int N, int K) {
  constexpr int NB = MT / 8;                // 8-row activation blocks
  constexpr int RB = kSkWarps / KS;         // weight blocks per CTA
  __shared__ float s_part[KS > 1 ? kSkWarps : 1][NB * 4][32];
  griddep_launch();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int slice = warp % KS;
  const int row0 = (blockIdx.x * RB + warp / KS) * 16;
  const bool live = row0 < N;
  const int g = lane >> 2, q = lane & 3;
  const int ra = row0 + g;
  // tiled weights are padded with zero rows to a multiple of 128; rows of
  // plain weights past N are clamped (their sums are never stored)
  const int na = tiled ? ra : min(ra, N - 1);
  const int nb8 = tiled ? ra + 8 : min(ra + 8, N - 1);
  const int kc = K >> 6;
  const int steps = K >> 5;
  const int per = (steps + KS - 1) / KS;
  const int s0 = live ? slice * per : 0;
  const int s1 = live ? min(steps, s0 + per) : 0;
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  uint4 wa[kSkU], wb[kSkU];
#pragma unroll
  for (int u = 0; u < kSkU; ++u) {
    const int k = (s0 + u) * 32 + q * 8;
    const bool in = s0 + u < s1;
    wa[u] = in ? ld_stream(sk_w(w, tiled, kc, K, na, k)) : z;
    wb[u] = in ? ld_stream(sk_w(w, tiled, kc, K, nb8, k)) : z;
  }
  griddep_wait();   // the activations and the epilogue's inputs
  float acc[NB][4];
#pragma unroll
  for (int b = 0; b < NB; ++b)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[b][i] = 0.f;
  const uint16_t *xr[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) xr[b] = x + (size_t)min(b * 8 + g, M - 1) * K + q * 8;
  const size_t xplane = (size_t)x_plane_rows * K;
  for (int s = s0; s < s1; s += kSkU) {
    uint4 ca[kSkU], cb[kSkU];
#pragma unroll
    for (int u = 0; u < kSkU; ++u) {
      ca[u] = wa[u];
      cb[u] = wb[u];
    }
#pragma unroll
    for (int u = 0; u < kSkU; ++u) {
      const int sn = s + kSkU + u;
      const int k = sn * 32 + q * 8;
      const bool in = sn < s1;
      wa[u] = in ? ld_stream(sk_w(w, tiled, kc, K, na, k)) : z;
      wb[u] = in ? ld_stream(sk_w(w, tiled, kc, K, nb8, k)) : z;
    }
    // the activation fragments of the whole batch first (L1/L2 hits, one
    // round trip), then the MMAs
    uint4 xv[kSkU][PL][NB];
#pragma unroll
    for (int u = 0; u < kSkU; ++u) {
      const int k = min(s + u, s1 - 1) * 32;
#pragma unroll
      for (int pl = 0; pl < PL; ++pl)
#pragma unroll
        for (int b = 0; b < NB; ++b)
          xv[u][pl][b] = __ldg(reinterpret_cast<const uint4 *>(xr[b] + pl * xplane + k));
    }
#pragma unroll
    for (int u = 0; u < kSkU; ++u) {
      if (s + u < s1) {
#pragma unroll
        for (int pl = 0; pl < PL; ++pl) {
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            sk_mma(acc[b], ca[u].x, cb[u].x, ca[u].y, cb[u].y, xv[u][pl][b].x, xv[u][pl][b].y);
            sk_mma(acc[b], ca[u].z, cb[u].z, ca[u].w, cb[u].w, xv[u][pl][b].z, xv[u][pl][b].w);
          }
        }
      }
    }
  }
  unsigned bmask = (1u << NB) - 1;
  if constexpr (KS > 1) {
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int i = 0; i < 4; ++i) s_part[warp][b * 4 + i][lane] = acc[b][i];
    __syncthreads();
    if (!live) return;
    // the KS warps of a block share its epilogue: slice s finishes the
    // activation blocks b = s (mod KS), each summed over the slices in order
    const int w0 = warp - slice;
    bmask = 0;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      if (b % KS != slice) continue;
      bmask |= 1u << b;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float t = 0.f;
#pragma unroll
        for (int sl = 0; sl < KS; ++sl) t += s_part[w0 + sl][b * 4 + i][lane];
        acc[b][i] = t;
      }
    }
    if (!bmask) return;
  } else {
    if (!live) return;
  }
  sk_epilogue<NB>(e, N, M, ra, q, acc, bmask);
}

template <int MT, int PL, int U>
cudaError_t sk_launch_u(int KS, dim3 grid, cudaStream_t st, const uint16_t *x, int xr,
                        const uint16_t *w, int tiled, const Epilogue &e, int M, int N,
                        int K) {
  const dim3 block(kSkWarps * 32);
  switch (KS) {
    case 1: return launch_pdl(linear_mma_kernel<MT, PL, 1, U>, grid, block, 0, st, x, xr, w, tiled, e, M, N, K);
    case 2: return launch_pdl(linear_mma_kernel<MT, PL, 2, U>, grid, block, 0, st, x, xr, w, tiled, e, M, N, K);
    case 4: return launch_pdl(linear_mma_kernel<MT, PL, 4, U>, grid, block, 0, st, x, xr, w, tiled, e, M, N, K);
    default: return launch_pdl(linear_mma_kernel<MT, PL, 8, U>, grid, block, 0, st, x, xr, w, tiled, e, M, N, K);
  }
}

template <int MT, int PL>
cudaError_t sk_launch(int KS, dim3 grid, cudaStream_t st, const uint16_t *x, int xr,
                      const uint16_t *w, int tiled, const Epilogue &e, int M, int N, int K) {
  const int steps = K >> 5;
  const int per = (steps + KS - 1) / KS;   // 32-k steps in a warp's slice
  return per <= kSkSmallSlice
             ? sk_launch_u<MT, PL, 2>(KS, grid, st, x, xr, w, tiled, e, M, N, K)
             : sk_launch_u<MT, PL, 4>(KS, grid, st, x, xr, w, tiled, e, M, N, K);
}

// Largest weight matrix the skinny kernel takes (TLLM_SKINNY_MAX_MB, in
// MiB, overrides): below it a projection is bound by latency, where the
// tcgen05 kernel's set-up costs most; above it the tcgen05 kernel's deep
// TMA ring streams HBM better.
size_t sk_max_bytes() {
  const char *sv = getenv("TLLM_SKINNY_MAX_MB");
  const long v = sv && sv[0] ? atol(sv) : 8;
  return (size_t)(v < 0 ? 0 : v) << 20;
}

// Largest batch the skinny kernel takes (TLLM_SKINNY_MAX_M overrides: 0
// sends every bf16 projection to the tcgen05 kernel, at most 32).
int sk_max_m() {
  const char *sv = getenv("TLLM_SKINNY_MAX_M");
  const int v = sv && sv[0] ? atoi(sv) : 32;
  return v < 0 ? 0 : (v > 32 ? 32 : v);
}

// ------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------
struct TcPlan {
  int MT, PL, m_tiles, n_tiles, k_chunks, S, wstages;
  size_t smem;
};

int tc_mt_for(int M) {
  return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
}

int env_int(const char *name, int dflt) {
  const char *v = getenv(name);
  return v && v[0] ? atoi(v) : dflt;
}

// Activation ring depth (TLLM_LINEAR_XS overrides, for tuning).
int tc_issuers_for(int MT, int PL) {
  static const int forced = env_int("TLLM_LINEAR_ISSUERS", 0);
  int ni = forced == 2 || forced == 4 ? forced : kTcMaxIssuers;
  // one accumulator of MT columns per issuer in TMEM's 512 columns, and
  // two activation stages per issuer must leave room for the weight ring
  if (ni * MT > 512 || ni * tc_x_bytes(MT, PL) > 64 * 1024) ni = 2;
  return ni;
}

// a ring depth rounded down to a multiple of the issuer count
int tc_ring_for_issuers(int depth, int MT, int PL) {
  const int ni = tc_issuers_for(MT, PL);
  depth -= depth % ni;
  return depth < ni ? ni : depth;
}

static int tc_ring_budget() {
  static const int budget_kb = env_int("TLLM_LINEAR_RING_KB", 224);
  return budget_kb * 1024;
}

// Activation ring depth: the deepest multiple of the issuer count (<= 8)
// that leaves >= 8 weight stages; the activation tiles are L2 hits, so two
// stages per issuer keep its next tile on the way.
int tc_xs_for(int MT, int PL) {
  static const int forced = env_int("TLLM_LINEAR_XS", 0);
  if (forced >= 2 && forced <= kTcMaxXS) return tc_ring_for_issuers(forced, MT, PL);
  const int ni = tc_issuers_for(MT, PL);
  const int xb = tc_x_bytes(MT, PL);
  int xs = kTcMaxXS - kTcMaxXS % ni;
  while (xs > ni && (tc_ring_budget() - xs * xb) / kTcW < 8) xs -= ni;
  return xs;
}

// Weight ring depth: one CTA per SM with ~224 KB of rings (the activation
// ring first); the rings also hold the fp32 accumulator tile staged by the
// epilogue.
int tc_wstages_for(int MT, int PL) {
  static const int forced = [] {  // TLLM_LINEAR_WS: ring depth for tuning
    const char *v = getenv("TLLM_LINEAR_WS");
    return v ? atoi(v) : 0;
  }();
  if (forced >= 2 && forced <= kTcMaxWS) return tc_ring_for_issuers(forced, MT, PL);
  const int xb = tc_xs_for(MT, PL) * tc_x_bytes(MT, PL);
  int ws = (tc_ring_budget() - xb) / kTcW;
  ws = ws < 2 ? 2 : (ws > kTcMaxWS ? kTcMaxWS : ws);
  return tc_ring_for_issuers(ws, MT, PL);
}

size_t tc_smem_for(int MT, int PL, int wstages) {
  const size_t rings =
      (size_t)wstages * kTcW + (size_t)tc_xs_for(MT, PL) * tc_x_bytes(MT, PL);
  // the epilogue stages the fp32 accumulator tile (MT x 128) in the rings
  const size_t tile = (size_t)MT * kTcBN * 4;
  return rings > tile ? rings : tile;
}

template <int MT, int OP, int PL>
int configure_tc() {
  auto kern = linear_tc_kernel<MT, OP, PL>;
  static bool configured[64] = {};  // per instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    TLLM_CUDA(cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 225 * 1024));
    TLLM_CUDA(cudaFuncSetAttribute(
        kern, cudaFuncAttributePreferredSharedMemoryCarveout,
        cudaSharedmemCarveoutMaxShared));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  return TLLM_OK;
}

int tc_cluster_policy() {   // TLLM_LINEAR_CLUSTER_POLICY: 1 spread, 2 balance
  static const int pol = [] {
    const char *v = getenv("TLLM_LINEAR_CLUSTER_POLICY");
    return v ? atoi(v) : 2;
  }();
  return pol;
}

// Clusters of S CTAs resident at once (cached per device and S).
template <int MT, int PL>
int tc_active_clusters(int S, size_t smem) {
  static int cached[64][kTcMaxSplit + 1] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && cached[dev][S]) return cached[dev][S] - 1;
  int n = 0;
  if (configure_tc<MT, EPI_STORE, PL>() == TLLM_OK) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, S, 1);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = S;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeClusterSchedulingPolicyPreference;
    attr[1].val.clusterSchedulingPolicyPreference =
        tc_cluster_policy() == 1 ? cudaClusterSchedulingPolicySpread
                                 : cudaClusterSchedulingPolicyLoadBalancing;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (cudaOccupancyMaxActiveClusters(&n, linear_tc_kernel<MT, EPI_STORE, PL>,
                                       &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
  }
  if (dev >= 0 && dev < 64) cached[dev][S] = n + 1;
  return n;
}

// CTAs that can run at once with S splits: one CTA per SM (the rings take
// ~224 KB of shared memory); clusters of S CTAs as the device places them.
int tc_active_ctas(int MT, int PL, int S, size_t smem) {
  static const int per_sm = env_int("TLLM_LINEAR_PER_SM", 0);
  if (per_sm > 0) return per_sm * sm_count();
  if (S == 1) return sm_count();
  int c = 0;
  if (PL == 2) {
    switch (MT) {
      case 16: c = tc_active_clusters<16, 2>(S, smem); break;
      case 32: c = tc_active_clusters<32, 2>(S, smem); break;
      case 64: c = tc_active_clusters<64, 2>(S, smem); break;
      case 128: c = tc_active_clusters<128, 2>(S, smem); break;
      default: c = tc_active_clusters<256, 2>(S, smem); break;
    }
  } else {
    switch (MT) {
      case 16: c = tc_active_clusters<16, 1>(S, smem); break;
      case 32: c = tc_active_clusters<32, 1>(S, smem); break;
      case 64: c = tc_active_clusters<64, 1>(S, smem); break;
      case 128: c = tc_active_clusters<128, 1>(S, smem); break;
      default: c = tc_active_clusters<256, 1>(S, smem); break;
    }
  }
  return c * S;
}

TcPlan tc_plan(int M, int N, int K, int PL) {
  TcPlan pl{};
  pl.MT = tc_mt_for(M);
  pl.PL = PL;
  pl.m_tiles = (M + pl.MT - 1) / pl.MT;
  pl.n_tiles = (N + kTcBN - 1) / kTcBN;
  pl.k_chunks = K / kTcBK;
  pl.wstages = tc_wstages_for(pl.MT, PL);
  pl.smem = tc_smem_for(pl.MT, PL, pl.wstages);
  // the largest split count (cluster size) whose whole grid is resident at
  // once, keeping >= 4 k-chunks per split
  const long base = (long)pl.m_tiles * pl.n_tiles;
  int s_max = pl.k_chunks / 4;
  if (s_max > kTcMaxSplit) s_max = kTcMaxSplit;
  int S = 1;
  for (int s = s_max; s >= 2; --s) {
    if (base * s <= tc_active_ctas(pl.MT, PL, s, pl.smem)) {
      S = s;
      break;
    }
  }
  pl.S = S;
  return pl;
}

template <int MT, int OP, int PL>
int launch_tc(const TcParams &p, const CUtensorMap &tw, const CUtensorMap &tx,
              dim3 grid, size_t smem, cudaStream_t st) {
  auto kern = linear_tc_kernel<MT, OP, PL>;
  int rc = configure_tc<MT, OP, PL>();
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[3];
  int na = 0;
  if (p.S > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = p.S;   // the splits of one weight tile
    attr[na].val.clusterDim.z = 1;
    ++na;
    attr[na].id = cudaLaunchAttributeClusterSchedulingPolicyPreference;
    attr[na].val.clusterSchedulingPolicyPreference =
        tc_cluster_policy() == 1 ? cudaClusterSchedulingPolicySpread
                                 : cudaClusterSchedulingPolicyLoadBalancing;
    ++na;
  }
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  TLLM_CUDA(cudaLaunchKernelEx(&cfg, kern, p, tw, tx));
  TLLM_LAUNCH_CHECK();
  return TLLM_OK;
}

template <int MT, int PL>
int launch_tc_op(const TcParams &p, const CUtensorMap &tw,
                 const CUtensorMap &tx, dim3 grid, size_t smem,
                 cudaStream_t st) {
  switch (p.e.op) {
    case EPI_STORE:
      return launch_tc<MT, EPI_STORE, PL>(p, tw, tx, grid, smem, st);
    case EPI_RESID:
      return launch_tc<MT, EPI_RESID, PL>(p, tw, tx, grid, smem, st);
    case EPI_GELU:
      return launch_tc<MT, EPI_GELU, PL>(p, tw, tx, grid, smem, st);
    case EPI_SWIGLU:
      return launch_tc<MT, EPI_SWIGLU, PL>(p, tw, tx, grid, smem, st);
    case EPI_SCATTER:
      return launch_tc<MT, EPI_SCATTER, PL>(p, tw, tx, grid, smem, st);
    default: return launch_tc<MT, EPI_QKV, PL>(p, tw, tx, grid, smem, st);
  }
}

template <int PL>
int launch_tc_mt(const TcParams &p, int MT, const CUtensorMap &tw,
                 const CUtensorMap &tx, dim3 grid, size_t smem,
                 cudaStream_t st) {
  switch (MT) {
    case 16: return launch_tc_op<16, PL>(p, tw, tx, grid, smem, st);
    case 32: return launch_tc_op<32, PL>(p, tw, tx, grid, smem, st);
    case 64: return launch_tc_op<64, PL>(p, tw, tx, grid, smem, st);
    case 128: return launch_tc_op<128, PL>(p, tw, tx, grid, smem, st);
    default: return launch_tc_op<256, PL>(p, tw, tx, grid, smem, st);
  }
}

int check_epilogue(const Epilogue &e, int N) {
  TLLM_CHECK_ARG(e.op >= EPI_STORE && e.op <= EPI_SCATTER, "bad epilogue op %d",
                 e.op);
  if (e.op == EPI_SCATTER) {
    TLLM_CHECK_ARG(e.p2p, "EPI_SCATTER needs a peer group (tllm_p2p_create)");
    TLLM_CHECK_ARG(!e.bias, "EPI_SCATTER takes no bias");
  } else if (e.op == EPI_QKV) {
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

int tllm_linear_fold_parts(int M, int N, int K, int *parts) {
  // a folded call always runs on the tensor-core kernel: one part per
  // 128-column weight tile
  TLLM_CHECK_ARG(parts, "NULL output");
  TLLM_CHECK_ARG(M > 0 && N > 0 && K > 0, "M, N, K must be > 0");
  *parts = (N + kTcBN - 1) / kTcBN;
  return TLLM_OK;
}

int tllm_linear_plan(int M, int N, int K, int x_dtype, int *plan) {
  TLLM_CHECK_ARG(plan, "NULL output");
  TLLM_CHECK_ARG(M > 0 && N > 0 && K >= kTcBK && K % kTcBK == 0,
                 "plan needs M, N > 0 and K a positive multiple of 64");
  TLLM_CHECK_ARG(x_dtype == TLLM_SPLIT || x_dtype == TLLM_BF16,
                 "x_dtype must be SPLIT or BF16");
  const int PL = x_dtype == TLLM_SPLIT ? 2 : 1;
  const TcPlan pl = tc_plan(M, N, K, PL);
  plan[0] = pl.MT;
  plan[1] = pl.m_tiles;
  plan[2] = pl.n_tiles;
  plan[3] = pl.S;
  plan[4] = pl.wstages;
  plan[5] = (int)pl.smem;
  plan[6] = tc_xs_for(pl.MT, PL);
  plan[7] = tc_active_ctas(pl.MT, PL, pl.S, pl.smem);
  return TLLM_OK;
}

int tllm_linear_folded(const void *x, int x_dtype, int x_plane_rows, const void *w,
                       int w_dtype, int M, int N, int K, int op, const float *bias,
                       void *out, int out_dtype, int out_plane_rows, int ld_out,
                       const float *resid, const float *cos_t, const float *sin_t,
                       const int32_t *row_seq, const int32_t *row_pos, float *q_out,
                       void *k_cache, void *v_cache, int kv_dtype, int max_seq,
                       int n_head, int n_kv_head, int head_dim, int32_t *lens_out,
                       const void *p2p, void *partial, size_t partial_bytes,
                       int32_t *counters, const tllm_norm_fold *fold,
                       tllm_stream_t stream);

// y = epilogue(x @ W^T); see tllm.h for the argument encoding.
int tllm_linear(const void *x, int x_dtype, int x_plane_rows, const void *w,
                int w_dtype, int M, int N, int K, int op, const float *bias,
                void *out, int out_dtype, int out_plane_rows, int ld_out,
                const float *resid, const float *cos_t, const float *sin_t,
                const int32_t *row_seq, const int32_t *row_pos, float *q_out,
                void *k_cache, void *v_cache, int kv_dtype, int max_seq,
                int n_head, int n_kv_head, int head_dim, int32_t *lens_out,
                const void *p2p, void *partial, size_t partial_bytes,
                int32_t *counters, tllm_stream_t stream) {
  return tllm_linear_folded(x, x_dtype, x_plane_rows, w, w_dtype, M, N, K, op, bias,
                            out, out_dtype, out_plane_rows, ld_out, resid, cos_t,
                            sin_t, row_seq, row_pos, q_out, k_cache, v_cache,
                            kv_dtype, max_seq, n_head, n_kv_head, head_dim,
                            lens_out, p2p, partial, partial_bytes, counters,
                            nullptr, stream);
}

// tllm_linear with a folded RMSNorm on either side (fold may be NULL).
int tllm_linear_folded(const void *x, int x_dtype, int x_plane_rows, const void *w,
                       int w_dtype, int M, int N, int K, int op, const float *bias,
                       void *out, int out_dtype, int out_plane_rows, int ld_out,
                       const float *resid, const float *cos_t, const float *sin_t,
                       const int32_t *row_seq, const int32_t *row_pos, float *q_out,
                       void *k_cache, void *v_cache, int kv_dtype, int max_seq,
                       int n_head, int n_kv_head, int head_dim, int32_t *lens_out,
                       const void *p2p, void *partial, size_t partial_bytes,
                       int32_t *counters, const tllm_norm_fold *fold,
                       tllm_stream_t stream) {
  TLLM_INJECT("launch");
  TLLM_CHECK_ARG(M >= 0 && N >= 0 && K >= 0, "negative shape");
  if (M == 0 || N == 0) return TLLM_OK;
  TLLM_CHECK_ARG(x && w, "NULL input");
  TLLM_CHECK_ARG(w_dtype == TLLM_F32 || w_dtype == TLLM_BF16 ||
                     w_dtype == TLLM_BF16_TILED,
                 "w_dtype must be F32, BF16 or BF16_TILED");
  TLLM_CHECK_ARG(out_dtype == TLLM_F32 || out_dtype == TLLM_SPLIT ||
                     out_dtype == TLLM_BF16,
                 "out_dtype must be F32, SPLIT or BF16");
  TLLM_CHECK_ARG(((uintptr_t)x & 15) == 0 && ((uintptr_t)w & 15) == 0,
                 "x and W must be 16-byte aligned");
  Epilogue e{};
  e.op = op;
  e.bias = bias;
  e.ld_out = ld_out > 0 ? ld_out : (op == EPI_SWIGLU ? N / 2 : N);
  if (out_dtype != TLLM_F32) {
    TLLM_CHECK_ARG(out_plane_rows >= M, "out_plane_rows (%d) < M (%d)",
                   out_plane_rows, M);
    e.out_split = static_cast<uint16_t *>(out);
    e.out_plane = (size_t)out_plane_rows * e.ld_out;
    e.out_planes = out_dtype == TLLM_SPLIT ? 2 : 1;
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
  if (op == EPI_SCATTER) {
    e.p2p = p2p_table(p2p, M, N);
    if (!e.p2p) return TLLM_ERR_INVALID_ARG;
  }
  e.err = device_error_ptr();
  TLLM_CHECK_ARG(e.err, "device error word unavailable");
  if (fold && fold->ss_out) {   // producer of the next norm's operand
    TLLM_CHECK_ARG(op == EPI_RESID, "a folded-norm producer must use op RESID");
    TLLM_CHECK_ARG(fold->next_norm_w && fold->fx, "folded norm: NULL weight or operand");
    TLLM_CHECK_ARG(fold->fx_dtype == TLLM_SPLIT || fold->fx_dtype == TLLM_BF16,
                   "folded norm: operand dtype SPLIT or BF16");
    TLLM_CHECK_ARG(fold->fx_plane_rows >= M && fold->ss_ld >= M,
                   "folded norm: fx_plane_rows / ss_ld < M");
    TLLM_CHECK_ARG(e.ld_out == N, "folded norm: the residual rows must be dense");
    e.fx_w = fold->next_norm_w;
    e.fx = static_cast<uint16_t *>(fold->fx);
    e.fx_plane = (size_t)fold->fx_plane_rows * N;
    e.fx_planes = fold->fx_dtype == TLLM_SPLIT ? 2 : 1;
    e.ss_out = fold->ss_out;
    e.ss_ld = fold->ss_ld;
  }
  if (fold && fold->ss_in) {    // consumer: rows scaled by 1 / rms
    TLLM_CHECK_ARG(op == EPI_STORE || op == EPI_SWIGLU || op == EPI_QKV,
                   "a folded-norm consumer must use op STORE, SWIGLU or QKV");
    TLLM_CHECK_ARG(fold->ss_parts > 0 && fold->ss_cols > 0 && fold->ss_ld >= M,
                   "folded norm: ss_parts, ss_cols > 0 and ss_ld >= M");
    TLLM_CHECK_ARG(w_dtype != TLLM_F32, "folded norm needs bf16 weights");
    e.ss_in = fold->ss_in;
    e.ss_parts = fold->ss_parts;
    e.ss_cols = fold->ss_cols;
    e.ss_ld = fold->ss_ld;
    e.ss_eps = fold->eps;
  }
  if (fold && (fold->ss_out || fold->ss_in))
    TLLM_CHECK_ARG(w_dtype != TLLM_F32, "folded norm needs bf16 weights");
  int rc = check_epilogue(e, N);
  if (rc) return rc;
  cudaStream_t st = resolve(stream);

  if (w_dtype == TLLM_F32) {
    TLLM_CHECK_ARG(op != EPI_SCATTER, "EPI_SCATTER needs bf16 weights");
    TLLM_CHECK_ARG(x_dtype == TLLM_F32, "fp32 weights take fp32 activations");
    TLLM_CHECK_ARG(K % 4 == 0, "K must be a multiple of 4");
    const int pairs = ((N + 15) / 16) * 8;
    // K slices per pair: enough warps for two CTAs of 8 on every SM, each
    // slice at least one warp-wide row of 128 floats
    int KS = 1;
    while (KS < kF32Warps && (long)pairs * KS < 2L * kF32Warps * sm_count() &&
           2 * KS * 128 <= K)
      KS *= 2;
    const int blocks = (pairs * KS + kF32Warps - 1) / kF32Warps;
    const float *xf = static_cast<const float *>(x);
    const float *wf = static_cast<const float *>(w);
    for (int m0 = 0; m0 < M; m0 += 8) {
      TLLM_CUDA(M - m0 == 1 ? f32_launch<1>(KS, blocks, st, xf, wf, e, M, N, K, m0)
                            : f32_launch<8>(KS, blocks, st, xf, wf, e, M, N, K, m0));
    }
    return TLLM_OK;
  }

  TLLM_CHECK_ARG(x_dtype == TLLM_SPLIT || x_dtype == TLLM_BF16,
                 "bf16 weights take TLLM_SPLIT or TLLM_BF16 activations "
                 "(tllm_split_bf16)");
  const int PL = x_dtype == TLLM_SPLIT ? 2 : 1;
  TLLM_CHECK_ARG(K > 0 && K % kTcBK == 0, "bf16 linear needs K %% 64 == 0 (K=%d)",
                 K);
  TLLM_CHECK_ARG(x_plane_rows >= M, "x_plane_rows (%d) < M (%d)", x_plane_rows,
                 M);
  (void)partial;
  (void)partial_bytes;
  (void)counters;
  // the skinny kernel has no folded-norm epilogues: folded calls take the
  // tensor-core kernel, whose idle warps sum the partials during the stream
  const bool folded = e.ss_in || e.ss_out;
  if (op != EPI_SCATTER && !folded && M <= sk_max_m() &&
      (size_t)N * K * 2 <= sk_max_bytes()) {
    // K slices per 16-row block: enough warps for two CTAs of 8 on every
    // SM, at least one 32-k step each
    const int blocks16 = (N + 15) / 16;
    int KS = 1;
    while (KS < kSkWarps && (long)blocks16 * KS < 2L * kSkWarps * sm_count() &&
           2 * KS <= K / 32)
      KS *= 2;
    const int RB = kSkWarps / KS;
    const dim3 grid((blocks16 + RB - 1) / RB);
    const uint16_t *xb = static_cast<const uint16_t *>(x);
    const uint16_t *wb = static_cast<const uint16_t *>(w);
    const int tl = w_dtype == TLLM_BF16_TILED;
    cudaError_t ce;
    if (M <= 8)
      ce = PL == 1 ? sk_launch<8, 1>(KS, grid, st, xb, x_plane_rows, wb, tl, e, M, N, K)
                   : sk_launch<8, 2>(KS, grid, st, xb, x_plane_rows, wb, tl, e, M, N, K);
    else if (M <= 16)
      ce = PL == 1 ? sk_launch<16, 1>(KS, grid, st, xb, x_plane_rows, wb, tl, e, M, N, K)
                   : sk_launch<16, 2>(KS, grid, st, xb, x_plane_rows, wb, tl, e, M, N, K);
    else
      ce = PL == 1 ? sk_launch<32, 1>(KS, grid, st, xb, x_plane_rows, wb, tl, e, M, N, K)
                   : sk_launch<32, 2>(KS, grid, st, xb, x_plane_rows, wb, tl, e, M, N, K);
    TLLM_CUDA(ce);
    return TLLM_OK;
  }
  const TcPlan pl = tc_plan(M, N, K, PL);
  const int S = pl.S;
  CUtensorMap tw, tx;
  const bool tiled = w_dtype == TLLM_BF16_TILED;
  if (tiled)  // (n_tiles * k_chunks * 128, 64) rows of 128 bytes
    rc = make_map_2d(&tw, w, TLLM_BF16, kTcBK,
                     (long)pl.n_tiles * pl.k_chunks * kTcBN, kTcBK * 2, kTcBK,
                     kTcBN, true);
  else
    rc = make_map_2d(&tw, w, TLLM_BF16, K, N, (long)K * 2, kTcBK, kTcBN, true);
  if (rc) return rc;
  const long xd[3] = {K, x_plane_rows, PL};
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
  p.wstages = pl.wstages;
  p.xstages = tc_xs_for(pl.MT, PL);
  {
    static const int forced = env_int("TLLM_LINEAR_NACC", 0);
    // MMA issuers, each with its own accumulators (>= 1 each, 512 TMEM
    // columns in all)
    const int ni = tc_issuers_for(pl.MT, PL);
    int nacc = forced > 0 ? forced : tc_nacc(pl.MT);
    if (nacc > ni * PL * (kTcBK / 16)) nacc = ni * PL * (kTcBK / 16);
    while (nacc > ni && nacc * pl.MT > 512) nacc -= ni;
    nacc = nacc < ni ? ni : nacc - nacc % ni;
    uint32_t cols = 32;
    while (cols < (uint32_t)(nacc * pl.MT)) cols <<= 1;
    p.nacc = nacc;
    p.issuers = ni;
    p.tcols = cols;
  }
  p.w_tiled = tiled ? 1 : 0;
  dim3 grid(pl.n_tiles, S, pl.m_tiles);
  if (PL == 2) return launch_tc_mt<2>(p, pl.MT, tw, tx, grid, pl.smem, st);
  return launch_tc_mt<1>(p, pl.MT, tw, tx, grid, pl.smem, st);
}

}  // extern "C"
