// Temperature / top-k sampling of the next token on the device.
//
// The reference samples on the host (smollm2_triton/model.py:566-584):
//   scaled = logits / T; probs = exp(scaled - max(scaled)) (float32, then
//   float64); probs /= sum(probs); with top_k > 0 the top_k largest probs are
//   kept (np.argpartition) and renormalised; then np.random.choice(V, p=probs)
//   -- NumPy draws one uniform u = random_sample() and returns the index of
//   the first entry of cdf = cumsum(p) / cdf[-1] that exceeds u.
// Here the caller draws the same u from the same NumPy generator (the random
// stream is consumed exactly as by the reference) and passes it in; the
// device does the rest, so only the 8-byte uniform and the 4-byte token
// cross the bus instead of the (V,) logits.
//
// One CTA of 1024 threads per row. The normalisations cancel in the cdf
// ratio, so p_i = (double) expf(x_i / T - max) for kept i and the sample is
// the first i (index order) whose cumulative weight / total exceeds u.
//
// top_k keeps the k largest logits (x -> exp(x / T - max) does not decrease
// for T > 0, so they are k most probable entries); among logits equal to the
// k-th largest the lowest indices are kept (np.argpartition leaves the choice
// among equal probabilities open). The threshold is the k-th largest
// order-preserving 32-bit key of the float32 logits, found by radix select:
// the first 12-bit digit from a histogram built in the same pass as the
// maximum; the entries in the threshold's digit bin (a few thousand for
// normally spread logits at V = 128K) are then compacted into shared memory
// and the remaining 20 bits selected there. A bin larger than the shared
// buffer (many equal logits) selects the remaining digits over the row.
//
// Passes over the row: max (+ histogram), compaction (top_k only), chunk
// sums. A chunk is 256 consecutive entries read by one warp, 32 consecutive
// floats per load; the chunk sums are scanned in index order to find the
// chunk where the cdf crosses u, and one warp walks that chunk in order.
#include "common.cuh"

namespace tllm {
namespace {

constexpr int kSmThreads = 1024;
constexpr int kSmWarps = kSmThreads / 32;
constexpr int kChunk = 256;                   // entries per chunk (8 per lane)
constexpr int kMaxChunks = 2 * kSmThreads;    // V <= 524288
constexpr int kBins = 4096;                   // first digit: 12 bits
constexpr int kCandCap = 8192;                // compacted entries
constexpr int kLoads = 8;                     // row loads in flight per thread
constexpr size_t kSampleSmem =
    kMaxChunks * sizeof(double) + kBins * sizeof(int) +
    kCandCap * (sizeof(uint32_t) + sizeof(int));

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

template <typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, Op op, T *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = red[lane];
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

// Exclusive prefix sum over the block in thread order; *total gets the sum.
template <typename T>
__device__ __forceinline__ T block_exclusive_scan(T v, T *sh, T *total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) sh[warp] = x;
  __syncthreads();
  if (warp == 0) {
    T w = sh[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const T y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    sh[lane] = w;   // inclusive over warps
  }
  __syncthreads();
  const T before = (warp > 0 ? sh[warp - 1] : T(0)) + x - v;
  *total = sh[kSmWarps - 1];
  return before;
}

// hist[digit] += 1 for every lane with digit < nbins. A warp whose lanes
// all hold one digit (equal logits) adds once. All 32 lanes must call it.
__device__ __forceinline__ void hist_add(int *hist, uint32_t digit, uint32_t nbins) {
  const uint32_t d0 = __shfl_sync(0xffffffffu, digit, 0);
  if (__all_sync(0xffffffffu, digit == d0)) {
    if ((threadIdx.x & 31) == 0 && d0 < nbins) atomicAdd(&hist[d0], 32);
  } else if (digit < nbins) {
    atomicAdd(&hist[digit], 1);
  }
}

struct SelectState {
  uint32_t prefix;   // the threshold's digits chosen so far
  int krem;          // how many entries equal to the prefix are still wanted
  int eq;            // entries whose digits so far equal the prefix
};

// After a histogram of nb bins over the entries matching st->prefix: the bin
// b holding the krem-th largest (bins ranked from the top, parallel over the
// block); st->prefix |= b << shift, st->krem -= the count above b.
__device__ void find_bin(const int *hist, int nb, int shift, SelectState *st,
                         int *sh_int) {
  const int per = nb > kSmThreads ? nb / kSmThreads : 1;
  const int r0 = threadIdx.x * per;   // ranks from the top bin
  const int krem = st->krem;
  const uint32_t prefix = st->prefix;
  int local = 0;
  for (int r = r0; r < r0 + per && r < nb; ++r) local += hist[nb - 1 - r];
  int tot = 0;
  int above = block_exclusive_scan(local, sh_int, &tot);
  if (above < krem && krem <= above + local) {
    for (int r = r0; r < r0 + per && r < nb; ++r) {
      const int b = nb - 1 - r;
      if (above + hist[b] >= krem) {
        st->prefix = prefix | ((uint32_t)b << shift);
        st->krem = krem - above;
        st->eq = hist[b];
        break;
      }
      above += hist[b];
    }
  }
  __syncthreads();
}

// Radix select of the st->krem-th largest key among the entries src(i, &key)
// accepts for i in [0, n) whose bits under `mask` equal st->prefix: `passes`
// digits of `bits` bits from `shift` down, histograms in hist.
template <typename Src>
__device__ void radix_select(const Src &src, int n, uint32_t mask, int shift, int bits,
                             int passes, int *hist, SelectState *st, int *sh_int) {
  const int tid = threadIdx.x;
  for (int p = 0; p < passes; ++p, shift -= bits) {
    const uint32_t nb = 1u << bits;
    for (int b = tid; b < (int)nb; b += kSmThreads) hist[b] = 0;
    __syncthreads();
    const uint32_t prefix = st->prefix;
    const int iters = (n + kSmThreads - 1) / kSmThreads;
    for (int it = 0; it < iters; ++it) {
      uint32_t key = 0;
      const bool ok = src(it * kSmThreads + tid, key) && (key & mask) == prefix;
      hist_add(hist, ok ? (key >> shift) & (nb - 1) : nb, nb);
    }
    __syncthreads();
    find_bin(hist, (int)nb, shift, st, sh_int);
    mask |= (nb - 1) << shift;
  }
}

__global__ void __launch_bounds__(kSmThreads)
    sample_kernel(const float *logits, int V, int ld, float temperature, int top_k,
                  const double *u, int *ids, int *pos_inc) {
  extern __shared__ __align__(16) unsigned char smem[];
  double *s_chunk = reinterpret_cast<double *>(smem);
  int *s_hist = reinterpret_cast<int *>(s_chunk + kMaxChunks);
  uint32_t *s_ckey = reinterpret_cast<uint32_t *>(s_hist + kBins);
  int *s_cidx = reinterpret_cast<int *>(s_ckey + kCandCap);
  __shared__ float s_redf[32];
  __shared__ double s_redd[32];
  __shared__ int s_redi[32];
  __shared__ SelectState s_sel;
  __shared__ int s_ncand, s_last, s_cross, s_pick;
  __shared__ double s_cbefore;

  griddep_wait();   // the logits come from the lm_head launch before
  griddep_launch();
  const int row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float *x = logits + (size_t)row * ld;
  const float T = temperature;
  const bool use_k = top_k > 0 && top_k < V;

  // ---- pass 1: max of the logits (rounding x / T is monotonic in x, so it
  // gives the scaled maximum) and, for top_k, the histogram of the keys'
  // top 12 bits
  if (use_k)
    for (int b = tid; b < kBins; b += kSmThreads) s_hist[b] = 0;
  if (tid == 0) {
    s_last = -1;
    s_cross = 0x7fffffff;
    s_pick = -1;
    s_ncand = 0;
    s_sel.prefix = 0;
    s_sel.krem = top_k;
    s_sel.eq = 0;
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int base = 0; base < V; base += kSmThreads * kLoads) {
    float v[kLoads];
#pragma unroll
    for (int b = 0; b < kLoads; ++b) {
      const int i = base + b * kSmThreads + tid;
      v[b] = i < V ? __ldg(x + i) : -INFINITY;
    }
#pragma unroll
    for (int b = 0; b < kLoads; ++b) {
      mx = fmaxf(mx, v[b]);
      if (use_k)
        hist_add(s_hist, base + b * kSmThreads + tid < V ? order_key(v[b]) >> 20 : kBins,
                 kBins);
    }
  }
  mx = __fdiv_rn(block_reduce(mx, [](float a, float b) { return fmaxf(a, b); }, s_redf), T);

  // ---- the k-th largest key (thr) and the largest kept index among keys
  // equal to it (idx_cut)
  uint32_t thr = 0;
  int idx_cut = 0x7fffffff;
  if (use_k) {
    find_bin(s_hist, kBins, 20, &s_sel, s_redi);
    const uint32_t b1 = s_sel.prefix >> 20;
    const bool compact = s_sel.eq <= kCandCap;
    if (compact) {
      // the threshold bin's entries -> shared memory (warp-aggregated slots)
      for (int base = 0; base < V; base += kSmThreads * kLoads) {
        float v[kLoads];
#pragma unroll
        for (int b = 0; b < kLoads; ++b) {
          const int i = base + b * kSmThreads + tid;
          v[b] = i < V ? __ldg(x + i) : 0.f;
        }
#pragma unroll
        for (int b = 0; b < kLoads; ++b) {
          const int i = base + b * kSmThreads + tid;
          const uint32_t key = order_key(v[b]);
          const bool take = i < V && (key >> 20) == b1;
          const unsigned bal = __ballot_sync(0xffffffffu, take);
          int slot0 = 0;
          if (lane == 0 && bal) slot0 = atomicAdd(&s_ncand, __popc(bal));
          const int slot = __shfl_sync(0xffffffffu, slot0, 0) +
                           __popc(bal & ((1u << lane) - 1));
          if (take && slot < kCandCap) {   // slot < the bin's count <= kCandCap
            s_ckey[slot] = key;
            s_cidx[slot] = i;
          }
        }
      }
      __syncthreads();
      const int nc = s_ncand;
      radix_select([&](int j, uint32_t &key) {
        if (j >= nc) return false;
        key = s_ckey[j];
        return true;
      }, nc, 0xFFF00000u, 10, 10, 2, s_hist, &s_sel, s_redi);
    } else {
      radix_select([&](int i, uint32_t &key) {
        if (i >= V) return false;
        key = order_key(x[i]);
        return true;
      }, V, 0xFFF00000u, 10, 10, 2, s_hist, &s_sel, s_redi);
    }
    thr = s_sel.prefix;
    const int k_eq = s_sel.krem;
    if (s_sel.eq > k_eq) {
      // ties at the threshold: keep the k_eq lowest indices, i.e. the k_eq
      // largest of ~index among the entries equal to thr
      __syncthreads();
      if (tid == 0) {
        s_sel.prefix = 0;
        s_sel.krem = k_eq;
      }
      __syncthreads();
      if (compact) {
        const int nc = s_ncand;
        auto src = [&](int j, uint32_t &key) {
          if (j >= nc || s_ckey[j] != thr) return false;
          key = ~(uint32_t)s_cidx[j];
          return true;
        };
        radix_select(src, nc, 0u, 20, 12, 1, s_hist, &s_sel, s_redi);
        radix_select(src, nc, 0xFFF00000u, 10, 10, 2, s_hist, &s_sel, s_redi);
      } else {
        auto src = [&](int i, uint32_t &key) {
          if (i >= V || order_key(x[i]) != thr) return false;
          key = ~(uint32_t)i;
          return true;
        };
        radix_select(src, V, 0u, 20, 12, 1, s_hist, &s_sel, s_redi);
        radix_select(src, V, 0xFFF00000u, 10, 10, 2, s_hist, &s_sel, s_redi);
      }
      idx_cut = (int)~s_sel.prefix;
    }
  }
  auto kept = [&](float v, int i) {
    if (!use_k) return true;
    const uint32_t key = order_key(v);
    return key > thr || (key == thr && i <= idx_cut);
  };

  // ---- chunk sums of the kept weights (a warp per chunk, 32 consecutive
  // floats per load) and the last index with a positive weight
  const int nchunks = (V + kChunk - 1) / kChunk;
  int last = -1;
  for (int c = warp; c < nchunks; c += kSmWarps) {
    float v[kChunk / 32];
#pragma unroll
    for (int j = 0; j < kChunk / 32; ++j) {
      const int i = c * kChunk + j * 32 + lane;
      v[j] = i < V ? __ldg(x + i) : 0.f;
    }
    double s = 0.0;
#pragma unroll
    for (int j = 0; j < kChunk / 32; ++j) {
      const int i = c * kChunk + j * 32 + lane;
      if (i < V && kept(v[j], i)) {
        const float p = expf(__fdiv_rn(v[j], T) - mx);
        s += (double)p;
        if (p > 0.f) last = i;
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) s_chunk[c] = s;
  }
  if (last >= 0) atomicMax(&s_last, last);
  __syncthreads();

  // ---- scan of the chunk sums (two per thread, index order): the lowest
  // chunk whose cumulative weight crosses u
  const int c0 = 2 * tid;
  const double a0 = c0 < nchunks ? s_chunk[c0] : 0.0;
  const double a1 = c0 + 1 < nchunks ? s_chunk[c0 + 1] : 0.0;
  double total = 0.0;
  const double before = block_exclusive_scan(a0 + a1, s_redd, &total);
  const double uu = u[row];
  const bool crosses = (before + a0 + a1) / total > uu && !(before / total > uu);
  const bool first = (before + a0) / total > uu;
  if (crosses) atomicMin(&s_cross, first ? c0 : c0 + 1);
  __syncthreads();
  if (crosses && s_cross == (first ? c0 : c0 + 1)) s_cbefore = first ? before : before + a0;
  __syncthreads();

  // ---- warp 0 walks the crossing chunk in index order
  if (warp == 0 && s_cross != 0x7fffffff) {
    const int c = s_cross;
    double cum = s_cbefore;
    int pick = -1, lastpos = -1;
    for (int j = 0; j < kChunk / 32 && pick < 0; ++j) {
      const int i = c * kChunk + j * 32 + lane;
      double p = 0.0;
      if (i < V) {
        const float v = x[i];
        if (kept(v, i)) p = (double)expf(__fdiv_rn(v, T) - mx);
      }
      double incl = p;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const double y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const unsigned hit = __ballot_sync(0xffffffffu, p > 0.0 && (cum + incl) / total > uu);
      const unsigned pos = __ballot_sync(0xffffffffu, p > 0.0);
      if (hit) pick = c * kChunk + j * 32 + __ffs(hit) - 1;
      if (pos) lastpos = c * kChunk + j * 32 + 31 - __clz(pos);
      cum += __shfl_sync(0xffffffffu, incl, 31);
    }
    // the walk's sums round apart from the scanned ones: a chunk that
    // crosses u by the scan but not by the walk yields its last positive entry
    if (lane == 0) s_pick = pick >= 0 ? pick : lastpos;
  }
  __syncthreads();
  if (tid == 0) {
    // u at or above the last boundary after rounding: the last index with a
    // positive weight (where the reference's cdf first reaches 1)
    const int pick = s_pick >= 0 ? s_pick : max(s_last, 0);
    ids[row] = pick;
    if (pos_inc) pos_inc[row] += 1;
  }
}

}  // namespace
}  // namespace tllm

using namespace tllm;

extern "C" int tllm_sample(const float *logits, int M, int V, int ld,
                           float temperature, int top_k, const double *u,
                           int32_t *ids, int32_t *pos_inc, tllm_stream_t stream) {
  TLLM_INJECT("launch");
  TLLM_CHECK_ARG(M >= 0 && V > 0, "invalid shape");
  TLLM_CHECK_ARG(V <= kMaxChunks * kChunk, "V = %d exceeds %d", V, kMaxChunks * kChunk);
  if (M == 0) return TLLM_OK;
  TLLM_CHECK_ARG(logits && u && ids, "NULL pointer");
  TLLM_CHECK_ARG(ld == 0 || ld >= V, "row stride %d < V = %d", ld, V);
  TLLM_CHECK_ARG(temperature > 1e-6f, "temperature must be > 1e-6 (use tllm_argmax)");
  TLLM_CHECK_ARG(top_k >= 0, "top_k must be non-negative");
  TLLM_CHECK_ARG(((uintptr_t)u & 7) == 0, "u must be 8-byte aligned");
  static int configured = -1;
  int dev = 0;
  TLLM_CUDA(cudaGetDevice(&dev));
  if (configured != dev) {
    TLLM_CUDA(cudaFuncSetAttribute(sample_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)kSampleSmem));
    configured = dev;
  }
  TLLM_CUDA(launch_pdl(sample_kernel, dim3(M), dim3(kSmThreads), kSampleSmem,
                       resolve(stream), logits, V, ld > 0 ? ld : V, temperature,
                       top_k, u, (int *)ids, (int *)pos_inc));
  TLLM_LAUNCH_CHECK();
  return TLLM_OK;
}
