// Persistent decode MLP block: one cooperative launch per layer computes
//
//   h  += attn . Wo^T                       (o_proj + residual)
//   x   = RMSNorm(h) * ln_w                 (bf16 operand of gate/up)
//   act = silu(x . Wg^T) * (x . Wu^T)       (gate/up + SwiGLU, bf16)
//   h  += act . Wd^T                        (down_proj + residual)
//
// which the layer-by-layer path runs as four launches (smollm2_triton/
// model.py:344-357 in the reference: o GEMM, add, rms_norm, gate/up GEMMs,
// swiglu, down GEMM, add). At decode sizes every launch of the projection
// kernel pays a fixed cost -- pipeline fill, epilogue, the wait for the
// previous grid's last CTA -- comparable to its weight stream; here one CTA
// per SM streams the weights of all three GEMMs through one ring without a
// break, and the phases meet at grid barriers.
//
// Work split: each GEMM's 128-row weight tiles are split along k into S
// equal pieces, S the most that keeps tiles x S within the grid, one piece
// per CTA (with more tiles than CTAs, S = 1 and a CTA takes whole tiles
// c, c + grid, ...). The S CTAs of a tile write their fp32 partials to
// global memory, wait for one another (all CTAs are resident: a
// cooperative launch), and each finishes rows m = split, split + S, ... of
// the tile, adding the S partials in split order (fixed, so results do not
// depend on timing) -- the distributed reduction that a cluster does in
// shared memory.
//
// Roles (12 warps): warp 0 lane 0 streams weight tiles (TMA, evict-first),
// warp 2 lane 0 streams activation tiles (after the grid barrier that makes
// them valid), warps 1, 3, 5, 7 lane 0 issue tcgen05.mma on the chunks
// c = i (mod 4) of the CTA's chunk sequence into their own accumulators
// (TMEM holds two segments' accumulators, so a segment's MMAs overlap the
// previous segment's epilogue), warps 8-11 run the epilogues and the norm.
// Every wait is bounded and reports through the device error word.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>

#include "common.cuh"

namespace tllm {

int make_map_2d(CUtensorMap *m, const void *base, int dtype, long inner,
                long outer, long stride_bytes, int box_inner, int box_outer,
                bool swizzle128);
int make_map(CUtensorMap *m, const void *base, int dtype, int rank,
             const long *dims, const long *strides_bytes, const int *box,
             bool swizzle128);

namespace {

constexpr int kMlWarps = 12;
constexpr int kMlThreads = kMlWarps * 32;
constexpr int kMlBN = 128;                 // weight rows per tile (MMA M)
constexpr int kMlBK = 64;                  // k per chunk
constexpr int kMlW = kMlBN * kMlBK * 2;    // 16 KB weight tile
constexpr int kMlWS = 8;                   // weight ring (multiple of issuers)
constexpr int kMlXS = 8;                   // activation ring (multiple of issuers)
constexpr int kMlNI = 4;                   // MMA issuers
constexpr int kMlEpi = 8;                  // first epilogue warp (4 warps)
constexpr int kMlMaxM = 64;
constexpr uint64_t kMlWaitNs = 2000000000ull;

struct MlPhase {
  int n_tiles, k_chunks;
  int splits;          // S: k pieces per tile (every piece non-empty)
  int per;             // chunks per piece (the last may have fewer)
  int active;          // n_tiles * S CTAs have a piece (S > 1)
  float *partial;      // [n_tiles][S][MT][128] (S > 1)
  // [n_tiles] pieces written, monotonic over launches (each adds S); zero
  // when the workspace is made
  unsigned long long *arrive;
};

struct MlParams {
  MlPhase ph[3];       // o, gate/up, down
  int M, hidden, ffn;
  float *h;            // (M, hidden) fp32, in place
  const float *ln_w;   // (hidden)
  float eps;
  uint16_t *x;         // (., hidden) bf16 operand rows
  uint16_t *act;       // (., ffn) bf16 operand rows
  float *rss;          // [o tiles][64] row sums of squares per o tile
  unsigned long long *bar;   // grid barrier arrivals, monotonic (3 G a launch)
  int *err;
};

__device__ __forceinline__ uint64_t ml_now() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void ml_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ unsigned long long ml_ld_acquire64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ml_add_release64(unsigned long long *p) {
  unsigned long long old;
  asm volatile("atom.release.gpu.global.add.u64 %0, [%1], 1;" : "=l"(old) : "l"(p) : "memory");
  return old;
}
// generic-proxy writes before later TMA (async-proxy) reads of them
__device__ __forceinline__ void ml_fence_proxy_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void ml_named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ bool ml_broken(const int *err) {
  return (*reinterpret_cast<const volatile int *>(err) & DEV_ERR_WAIT_TIMEOUT) != 0;
}

// Grid barriers: one monotonic 64-bit arrival counter. A launch starts with
// it at a multiple of 3 G (every launch adds exactly 3 G arrivals), and its
// barrier k (1..3) is complete once the counter reaches base + k G. An
// arrival is one release add by a CTA's leader after its CTA's writes of
// the phase; a CTA arrives at barrier k + 1 only after it has seen barrier
// k complete.
__device__ __forceinline__ void ml_grid_arrive(unsigned long long *bar) {
  asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(bar) : "memory");
}
// Bounded wait until the arrival counter reaches `target`.
__device__ bool ml_grid_wait(const unsigned long long *bar, unsigned long long target, int *err) {
  if (ml_broken(err)) return false;
  const uint64_t t0 = ml_now();
  for (uint32_t it = 0;; ++it) {
    if (ml_ld_acquire64(bar) >= target) return true;
    if (((it & 63) == 63 && ml_now() - t0 > kMlWaitNs) || it == (1u << 26)) {
      atomicOr(err, DEV_ERR_WAIT_TIMEOUT);
      return false;
    }
  }
}

// This CTA's pieces of one phase: with S > 1 at most one (tile c / S,
// split c % S); with S == 1 the whole tiles c, c + G, c + 2G, ...
struct MlSegs {
  int tile, split_, S, G, n_tiles, per, kc;
  bool one;
  __device__ MlSegs(const MlPhase &ph, int c, int grid)
      : S(ph.splits), G(grid), n_tiles(ph.n_tiles), per(ph.per), kc(ph.k_chunks) {
    one = S > 1;
    tile = one ? (c < ph.active ? c / S : n_tiles) : c;
    split_ = one && c < ph.active ? c - (c / S) * S : 0;
  }
  __device__ bool next(int &t, int &k0, int &n) {
    if (tile >= n_tiles) return false;
    t = tile;
    k0 = split_ * per;
    n = min(per, kc - k0);
    tile = one ? n_tiles : tile + G;
    return true;
  }
};

// 1 / d for d in [1, 2]: the hardware approximation refined by one
// Newton-Raphson step, r' = r + r (1 - d r); no special cases to branch on
__device__ __forceinline__ float ml_rcp(float d) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
  return fmaf(r, fmaf(-d, r, 1.f), r);
}
__device__ __forceinline__ float ml_silu(float x) {
  // x * sigmoid(x), sigmoid from exp(-|x|) (triton_llm/kernels/swiglu.py:51-54)
  const float e = expf(-fabsf(x));
  const float r = ml_rcp(1.f + e);
  return x * (x >= 0.f ? r : e * r);
}

template <int MT>
__global__ void __launch_bounds__(kMlThreads, 1)
    mlp_kernel(const MlParams p, const __grid_constant__ CUtensorMap tw0,
               const __grid_constant__ CUtensorMap tw1,
               const __grid_constant__ CUtensorMap tw2,
               const __grid_constant__ CUtensorMap tx0,
               const __grid_constant__ CUtensorMap tx1,
               const __grid_constant__ CUtensorMap tx2) {
  constexpr int X_BYTES = MT * kMlBK * 2;
  constexpr uint32_t TCOLS = 2 * kMlNI * MT;   // two segments' accumulators
  constexpr uint32_t IDESC = umma_idesc_bf16(kMlBN, MT);
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint64_t wfull[kMlWS], wempty[kMlWS], xfull[kMlXS], xempty[kMlXS];
  __shared__ uint64_t accf[2], acce[2];
  __shared__ uint32_t s_tmem;
  __shared__ unsigned long long s_base;
  __shared__ int s_fail;
  __shared__ float s_red[4][kMlMaxM];
  __shared__ float s_rms[kMlMaxM];
  uint8_t *wring = smem;
  uint8_t *xring = smem + kMlWS * kMlW;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int G = gridDim.x;
  const int me = blockIdx.x;
  if (smem_u32(smem) & 1023) {
    if (tid == 0) atomicOr(p.err, DEV_ERR_SMEM_ALIGN);
    return;
  }
  griddep_launch();
  if (tid == 0) {
    for (int s = 0; s < kMlWS; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 1);
    }
    for (int s = 0; s < kMlXS; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], kMlNI);   // one arrival per issuer
      mbar_init(&acce[b], 1);       // the epilogue leader
    }
    s_fail = 0;
    // barrier 1 cannot complete before this CTA arrives, so the counter is
    // below base + G: rounding down to a multiple of 3 G gives the base
    const unsigned long long c = ml_ld_acquire64(p.bar);
    s_base = c - c % (3ull * (unsigned)G);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&s_tmem, TCOLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  const unsigned long long base = s_base;
  const unsigned long long G64 = (unsigned)G;

  if (warp == 0) {
    if (lane == 0) {
      // ---- weight producer: all three GEMMs, one ring, no breaks
      const uint64_t pol = l2_policy_evict_first();
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tw0) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tw1) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tw2) : "memory");
      long g = 0;
      bool ok = true;
      for (int ph = 0; ph < 3 && ok; ++ph) {
        const CUtensorMap *tw = ph == 0 ? &tw0 : (ph == 1 ? &tw1 : &tw2);
        MlSegs segs(p.ph[ph], me, G);
        int tile, k0, n;
        while (ok && segs.next(tile, k0, n)) {
          for (int j = 0; j < n; ++j, ++g) {
            const int s = (int)(g % kMlWS);
            if (g >= kMlWS && !mbar_wait_bounded(&wempty[s], (int)((g / kMlWS) - 1) & 1)) {
              ok = false;
              break;
            }
            mbar_expect_tx(&wfull[s], kMlW);
            tma_load_2d_hint(wring + s * kMlW, tw, &wfull[s], 0,
                             ((long)tile * p.ph[ph].k_chunks + k0 + j) * kMlBN, pol);
          }
        }
      }
      if (!ok) s_fail = 1;
    }
    __syncwarp();
  } else if (warp == 2) {
    if (lane == 0) {
      // ---- activation producer: attn (written by the previous kernel),
      //      then x after the norm barrier, act after the gate/up barrier
      const uint64_t pol = l2_policy_evict_last();
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tx0) : "memory");
      griddep_wait();
      long g = 0;
      bool ok = true;
      for (int ph = 0; ph < 3 && ok; ++ph) {
        if (ph > 0) {
          // gate/up reads x (ready at barrier 2), down reads act (barrier 3)
          if (!ml_grid_wait(p.bar, base + (ph == 1 ? 2 : 3) * G64, p.err)) {
            ok = false;
            break;
          }
          ml_fence_proxy_global();
        }
        const CUtensorMap *tx = ph == 0 ? &tx0 : (ph == 1 ? &tx1 : &tx2);
        MlSegs segs(p.ph[ph], me, G);
        int tile, k0, n;
        while (ok && segs.next(tile, k0, n)) {
          for (int j = 0; j < n; ++j, ++g) {
            const int s = (int)(g % kMlXS);
            if (g >= kMlXS && !mbar_wait_bounded(&xempty[s], (int)((g / kMlXS) - 1) & 1)) {
              ok = false;
              break;
            }
            mbar_expect_tx(&xfull[s], X_BYTES);
            tma_load_3d_hint(xring + s * X_BYTES, tx, &xfull[s], (k0 + j) * kMlBK, 0, 0, pol);
          }
        }
      }
      if (!ok) s_fail = 1;
    }
    __syncwarp();
  } else if (warp < 8 && (warp & 1)) {
    if (lane == 0) {
      // ---- MMA issuer `who`: chunks g = who (mod 4) of the CTA's sequence
      const int who = warp >> 1;
      long g = 0;
      int seg = 0;
      bool ok = true;
      for (int ph = 0; ph < 3; ++ph) {
        MlSegs segs(p.ph[ph], me, G);
        int tile, k0, n;
        while (segs.next(tile, k0, n)) {
          const int buf = seg & 1;
          const int use = seg >> 1;
          // the epilogue has read this buffer's previous segment
          if (ok && use > 0 && !mbar_wait_bounded(&acce[buf], (use - 1) & 1)) ok = false;
          tc_fence_after();
          const uint32_t tacc = tmem + (uint32_t)((buf * kMlNI + who) * MT);
          bool first = true;
          for (int j = 0; j < n; ++j) {
            const long gc = g + j;
            if ((int)(gc % kMlNI) != who) continue;
            const int ws = (int)(gc % kMlWS);
            const int xs = (int)(gc % kMlXS);
            if (!ok || !mbar_wait_bounded(&wfull[ws], (int)(gc / kMlWS) & 1) ||
                !mbar_wait_bounded(&xfull[xs], (int)(gc / kMlXS) & 1)) {
              ok = false;
              continue;   // keep the arrival counts balanced
            }
            tc_fence_after();
            const uint64_t a = umma_desc_sw128(smem_u32(wring + ws * kMlW));
            const uint64_t bx = umma_desc_sw128(smem_u32(xring + xs * X_BYTES));
#pragma unroll
            for (int kk = 0; kk < kMlBK / 16; ++kk)
              umma_bf16(tacc, a + 2 * kk, bx + 2 * kk, IDESC, (first && kk == 0) ? 0u : 1u);
            umma_commit(&wempty[ws]);
            umma_commit(&xempty[xs]);
            first = false;
          }
          g += n;
          if (!first)
            umma_commit(&accf[buf]);
          else
            ml_arrive(&accf[buf]);
          ++seg;
        }
      }
      if (!ok) s_fail = 1;
    }
    __syncwarp();
  } else if (warp >= kMlEpi) {
    // ---- epilogue warps: TMEM lane quarter ew = weight rows 32 ew .. + 31
    const int ew = warp - kMlEpi;
    const int r = ew * 32 + lane;          // weight row within the tile
    const int et = ew * 32 + lane;         // epilogue thread 0..127
    const bool leader = ew == 0 && lane == 0;
    const uint32_t t_lane = tmem + ((uint32_t)(ew * 32) << 16);
    griddep_wait();   // h and the earlier kernels' outputs
    long g = 0;
    int seg = 0;
    for (int ph = 0; ph < 3; ++ph) {
      const MlPhase &P = p.ph[ph];
      MlSegs segs(P, me, G);
      int tile, k0, n;
      while (segs.next(tile, k0, n)) {
        const int buf = seg & 1;
        const int use = seg >> 1;
        const bool ok = !ml_broken(p.err) && mbar_wait_bounded(&accf[buf], use & 1);
        tc_fence_after();
        float v[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) v[m] = 0.f;
        if (ok) {
#pragma unroll 1
          for (int i = 0; i < kMlNI; ++i) {
            // issuer i wrote this buffer iff it had a chunk in the segment
            const int first_i = (int)(((i - g) % kMlNI + kMlNI) % kMlNI);
            if (first_i >= n) continue;
            const uint32_t col = (uint32_t)((buf * kMlNI + i) * MT);
#pragma unroll
            for (int c0 = 0; c0 < MT; c0 += (MT >= 32 ? 32 : 16)) {
              if constexpr (MT >= 32) {
                float u[32];
                tmem_ld32(t_lane + col + c0, u);
#pragma unroll
                for (int j = 0; j < 32; ++j) v[c0 + j] += u[j];
              } else {
                float u[16];
                tmem_ld16(t_lane + col + c0, u);
#pragma unroll
                for (int j = 0; j < 16; ++j) v[c0 + j] += u[j];
              }
            }
          }
        }
        tc_fence_before();
        ml_named_sync(1, 128);
        if (leader) ml_arrive(&acce[buf]);   // buffer free for segment seg + 2
        g += n;
        ++seg;

        const int S = P.splits;
        const int split = S > 1 ? me - tile * S : 0;   // this CTA's piece
        // rows this CTA finishes: m_i = split + S i for i < nr (every row
        // below M when S == 1); from here on v[i] holds row m_i. The row
        // loops run over every i with clamped load addresses and only the
        // stores predicated, so the loads of a batch are in flight together
        // (a branch per row would wait out one L2 round trip per row).
        const int lim = min(MT, p.M);
        const int nr = split < lim ? (lim - split + S - 1) / S : 0;
        constexpr int H = MT / 2;   // rows per batch; S >= 2 leaves at most H
        if (S > 1) {
          float *part = P.partial + (((size_t)tile * S + split) * MT) * kMlBN + r;
#pragma unroll
          for (int m = 0; m < MT; ++m) part[(size_t)m * kMlBN] = v[m];
          ml_named_sync(1, 128);
          if (leader) {
            // the tile's counter holds a multiple of S before this launch
            // and S more after it: wait for the next multiple (bounded)
            const unsigned long long old = ml_add_release64(&P.arrive[tile]);
            const unsigned long long want = old - old % (unsigned)S + (unsigned)S;
            const uint64_t t0 = ml_now();
            for (uint32_t it = 0;; ++it) {
              if (ml_ld_acquire64(&P.arrive[tile]) >= want) break;
              if (ml_broken(p.err) ||
                  ((it & 63) == 63 && ml_now() - t0 > kMlWaitNs) || it == (1u << 26)) {
                atomicOr(p.err, DEV_ERR_WAIT_TIMEOUT);
                break;
              }
            }
          }
          ml_named_sync(1, 128);
          // the rows of this slice, summed over the pieces in split order
          const float *src = P.partial + ((size_t)tile * S * MT) * kMlBN + r;
#pragma unroll
          for (int i = 0; i < MT; ++i) v[i] = 0.f;
#pragma unroll 1
          for (int q = 0; q < S; ++q) {
            const float *pq = src + (size_t)q * MT * kMlBN;
#pragma unroll
            for (int i = 0; i < H; ++i)
              v[i] += __ldcg(pq + (size_t)min(split + S * i, MT - 1) * kMlBN);
          }
        }
        // ---- epilogue of this CTA's rows of the tile
        const int n0 = tile * kMlBN;
        if (ph == 1) {
          // SwiGLU: rows R (first 8 of a 16-block) and R + 8 pair up
          const int R = n0 + r;
          const bool head = (lane & 8) == 0;
          const int j = (R >> 4) * 8 + (R & 7);
          // rows i and i + 1 go together: lane L (gate) finishes row i and
          // lane L + 8 (up) row i + 1, one exchange and one silu each
#pragma unroll
          for (int hb = 0; hb < 2; ++hb) {
            if (hb * H >= nr) break;
#pragma unroll
            for (int k = 0; k < H; k += 2) {
              const int i0 = hb * H + k;
              const float t = __shfl_xor_sync(0xffffffffu, head ? v[i0 + 1] : v[i0], 8);
              const float gate = head ? v[i0] : t;
              const float up = head ? t : v[i0 + 1];
              const int i = head ? i0 : i0 + 1;
              const float a = ml_silu(gate) * up;
              if (i < nr) p.act[(size_t)(split + S * i) * p.ffn + j] = f32_to_bf16_bits(a);
            }
          }
        } else {
          // residual: h[m][n0 + r] += acc (o, down); loads first (other CTAs
          // wrote h: L2, not L1), then the stores
          float *hcol = p.h + n0 + r;
#pragma unroll
          for (int hb = 0; hb < 2; ++hb) {
            if (hb * H >= nr) break;
            float hv[H];
#pragma unroll
            for (int k = 0; k < H; ++k)
              hv[k] = __ldcg(hcol + (size_t)min(split + S * (hb * H + k), lim - 1) * p.hidden);
#pragma unroll
            for (int k = 0; k < H; ++k) {
              const int i = hb * H + k;
              v[i] += hv[k];
              if (i < nr) hcol[(size_t)(split + S * i) * p.hidden] = v[i];
            }
          }
          if (ph == 0) {
            // row sums of squares of the new h over this tile's columns
#pragma unroll
            for (int hb = 0; hb < 2; ++hb) {
              if (hb * H >= nr) break;
#pragma unroll
              for (int k = 0; k < H; ++k) {
                const int i = hb * H + k;
                float sq = v[i] * v[i];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1)
                  sq += __shfl_xor_sync(0xffffffffu, sq, off);
                if (lane == 0 && i < nr) s_red[ew][split + S * i] = sq;
              }
            }
            ml_named_sync(1, 128);
            if (et < lim && et >= split && (et - split) % S == 0)
              p.rss[(size_t)tile * kMlMaxM + et] =
                  ((s_red[0][et] + s_red[1][et]) + s_red[2][et]) + s_red[3][et];
            ml_named_sync(1, 128);
          }
        }
      }
      // ---- end of phase
      if (ph == 2) break;
      if (ph == 1) ml_fence_proxy_global();   // act is read by TMA after barrier 3
      ml_named_sync(1, 128);
      if (leader) {
        // a CTA without a gate/up piece gets here before barrier 2 is
        // complete; its arrival must not count toward barrier 2
        if (ph == 1) ml_grid_wait(p.bar, base + 2 * G64, p.err);
        ml_grid_arrive(p.bar);   // barrier 1 (after o) / 3 (after gate/up)
      }
      if (ph == 0) {
        // ---- RMSNorm of the complete h rows: x = (h / rms) * w (bf16)
        if (leader) ml_grid_wait(p.bar, base + G64, p.err);
        ml_named_sync(1, 128);
        if (et < p.M) {
          float ss = 0.f;
          for (int t = 0; t < p.ph[0].n_tiles; ++t) ss += __ldcg(&p.rss[(size_t)t * kMlMaxM + et]);
          s_rms[et] = sqrtf(ss / (float)p.hidden + p.eps);
        }
        ml_named_sync(1, 128);
        const int n4 = p.hidden >> 2;
        const long total4 = (long)p.M * n4;
        for (long i = (long)me * 128 + et; i < total4; i += (long)G * 128) {
          const int m = (int)(i / n4);
          const int c4 = (int)(i - (long)m * n4);
          const float4 hv = __ldcg(reinterpret_cast<const float4 *>(p.h + (size_t)m * p.hidden) + c4);
          const float4 wv = reinterpret_cast<const float4 *>(p.ln_w)[c4];
          const float rms = s_rms[m];
          const uint32_t lo = (uint32_t)f32_to_bf16_bits((hv.x / rms) * wv.x) |
                              ((uint32_t)f32_to_bf16_bits((hv.y / rms) * wv.y) << 16);
          const uint32_t hi = (uint32_t)f32_to_bf16_bits((hv.z / rms) * wv.z) |
                              ((uint32_t)f32_to_bf16_bits((hv.w / rms) * wv.w) << 16);
          *reinterpret_cast<uint2 *>(p.x + (size_t)m * p.hidden + 4 * (size_t)c4) = make_uint2(lo, hi);
        }
        ml_fence_proxy_global();   // x is read by TMA after barrier 2
        ml_named_sync(1, 128);
        if (leader) ml_grid_arrive(p.bar);   // barrier 2
      }
    }
  }

  // ---- teardown
  tc_fence_before();
  __syncthreads();
  if (s_fail && tid == 0) atomicOr(p.err, DEV_ERR_WAIT_TIMEOUT);
  if (warp == 1) tmem_free(tmem, TCOLS);
}

int ml_mt_for(int M) { return M <= 16 ? 16 : (M <= 32 ? 32 : 64); }

struct MlLayout {
  int G, MT;
  int tiles[3], kc[3], splits[3], per[3];
  size_t off_bar, off_rss, off_count[3], off_part[3], bytes;
};

int ml_grid() {
  static int g[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && g[dev]) return g[dev];
  const int n = sm_count();
  if (dev >= 0 && dev < 64) g[dev] = n;
  return n;
}

MlLayout ml_layout(int M, int attn_dim, int hidden, int ffn) {
  MlLayout L{};
  L.G = ml_grid();
  L.MT = ml_mt_for(M);
  const int N[3] = {hidden, 2 * ffn, hidden};
  const int K[3] = {attn_dim, hidden, ffn};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~(size_t)255;
    return o;
  };
  L.off_bar = take(256);
  L.off_rss = take((size_t)(hidden / kMlBN) * kMlMaxM * sizeof(float));
  for (int i = 0; i < 3; ++i) {
    L.tiles[i] = N[i] / kMlBN;
    L.kc[i] = K[i] / kMlBK;
    // the most k pieces per tile that keep tiles x pieces within the grid,
    // none of them empty
    int S = L.G / L.tiles[i];
    if (S < 1) S = 1;
    if (S > L.kc[i]) S = L.kc[i];
    int per = (L.kc[i] + S - 1) / S;
    while (S > 1 && (S - 1) * per >= L.kc[i]) {
      --S;
      per = (L.kc[i] + S - 1) / S;
    }
    L.splits[i] = S;
    L.per[i] = per;
    L.off_count[i] = take((size_t)L.tiles[i] * sizeof(unsigned long long));
  }
  for (int i = 0; i < 3; ++i)
    L.off_part[i] = L.splits[i] > 1
                        ? take((size_t)L.tiles[i] * L.splits[i] * L.MT * kMlBN * sizeof(float))
                        : 0;
  L.bytes = off;
  return L;
}

template <int MT>
int ml_launch(const MlParams &p, const CUtensorMap (&tw)[3], const CUtensorMap (&tx)[3],
              int G, cudaStream_t st) {
  auto kern = mlp_kernel<MT>;
  const size_t smem = (size_t)kMlWS * kMlW + (size_t)kMlXS * MT * kMlBK * 2;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    TLLM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int per_sm = 0;
    TLLM_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kMlThreads, smem));
    if (per_sm < 1) {
      set_error("the MLP block kernel does not fit on an SM");
      return TLLM_ERR_UNSUPPORTED;
    }
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(kMlThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  // the grid barriers need every CTA resident at once
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  TLLM_CUDA(cudaLaunchKernelEx(&cfg, kern, p, tw[0], tw[1], tw[2], tx[0], tx[1], tx[2]));
  return TLLM_OK;
}

}  // namespace
}  // namespace tllm

using namespace tllm;

extern "C" {

int tllm_mlp_workspace(int M, int attn_dim, int hidden, int ffn, size_t *bytes) {
  TLLM_CHECK_ARG(bytes, "NULL output");
  TLLM_CHECK_ARG(M > 0 && M <= kMlMaxM, "M must be in [1, %d]", kMlMaxM);
  TLLM_CHECK_ARG(hidden > 0 && hidden % kMlBN == 0, "hidden must be a multiple of 128");
  TLLM_CHECK_ARG(attn_dim > 0 && attn_dim % kMlBK == 0, "attn_dim must be a multiple of 64");
  TLLM_CHECK_ARG(ffn > 0 && ffn % kMlBK == 0, "ffn must be a multiple of 64");
  *bytes = ml_layout(M, attn_dim, hidden, ffn).bytes;
  return TLLM_OK;
}

int tllm_mlp(const void *attn, int attn_plane_rows, const void *w_o, float *h,
             const float *ln_w, float eps, void *x, int x_plane_rows,
             const void *w_gu, void *act, int act_plane_rows, const void *w_down,
             int M, int attn_dim, int hidden, int ffn, void *workspace,
             size_t workspace_bytes, tllm_stream_t stream) {
  TLLM_INJECT("launch");
  TLLM_CHECK_ARG(M >= 0, "negative M");
  if (M == 0) return TLLM_OK;
  size_t need = 0;
  int rc = tllm_mlp_workspace(M, attn_dim, hidden, ffn, &need);
  if (rc) return rc;
  TLLM_CHECK_ARG(attn && w_o && h && ln_w && x && w_gu && act && w_down && workspace,
                 "NULL pointer");
  TLLM_CHECK_ARG(workspace_bytes >= need, "workspace of %zu bytes, %zu needed",
                 workspace_bytes, need);
  TLLM_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
                 "workspace must be 256-byte aligned");
  TLLM_CHECK_ARG(attn_plane_rows >= M && x_plane_rows >= M && act_plane_rows >= M,
                 "operand buffers need >= M rows");
  TLLM_CHECK_ARG((reinterpret_cast<uintptr_t>(h) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(ln_w) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(x) & 15) == 0,
                 "h, ln_w and x must be 16-byte aligned");
  int *err = device_error_ptr();
  TLLM_CHECK_ARG(err, "device error word unavailable");
  const MlLayout L = ml_layout(M, attn_dim, hidden, ffn);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  MlParams p;
  const void *W[3] = {w_o, w_gu, w_down};
  for (int i = 0; i < 3; ++i) {
    p.ph[i].n_tiles = L.tiles[i];
    p.ph[i].k_chunks = L.kc[i];
    p.ph[i].splits = L.splits[i];
    p.ph[i].per = L.per[i];
    p.ph[i].active = L.tiles[i] * L.splits[i];
    p.ph[i].partial = L.splits[i] > 1 ? reinterpret_cast<float *>(ws + L.off_part[i]) : nullptr;
    p.ph[i].arrive = reinterpret_cast<unsigned long long *>(ws + L.off_count[i]);
  }
  p.M = M;
  p.hidden = hidden;
  p.ffn = ffn;
  p.h = h;
  p.ln_w = ln_w;
  p.eps = eps;
  p.x = static_cast<uint16_t *>(x);
  p.act = static_cast<uint16_t *>(act);
  p.rss = reinterpret_cast<float *>(ws + L.off_rss);
  p.bar = reinterpret_cast<unsigned long long *>(ws + L.off_bar);
  p.err = err;
  // weights: tiled bf16, (tiles * k_chunks * 128, 64) rows of 128 bytes
  CUtensorMap tw[3], tx[3];
  for (int i = 0; i < 3; ++i) {
    rc = make_map_2d(&tw[i], W[i], TLLM_BF16, kMlBK, (long)L.tiles[i] * L.kc[i] * kMlBN,
                     kMlBK * 2, kMlBK, kMlBN, true);
    if (rc) return rc;
  }
  const void *X[3] = {attn, x, act};
  const long XK[3] = {attn_dim, hidden, ffn};
  const long XR[3] = {attn_plane_rows, x_plane_rows, act_plane_rows};
  for (int i = 0; i < 3; ++i) {
    const long d[3] = {XK[i], XR[i], 1};
    const long s[2] = {XK[i] * 2, XR[i] * XK[i] * 2};
    const int b[3] = {kMlBK, L.MT, 1};
    rc = make_map(&tx[i], X[i], TLLM_BF16, 3, d, s, b, true);
    if (rc) return rc;
  }
  cudaStream_t st = resolve(stream);
  switch (L.MT) {
    case 16: return ml_launch<16>(p, tw, tx, L.G, st);
    case 32: return ml_launch<32>(p, tw, tx, L.G, st);
    default: return ml_launch<64>(p, tw, tx, L.G, st);
  }
}

}  // extern "C"
