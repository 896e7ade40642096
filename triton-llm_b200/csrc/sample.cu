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
// ratio, so p_i = (double) expf(scaled_i - max) for kept i and the sample is
// the first i (index order) with cumsum_i / sum > u. top_k keeps the k
// largest logits (x -> exp(x / T - max) is monotonic for T > 0, so they are
// the k most probable): their threshold is the k-th largest of the
// order-preserving 32-bit keys of the float32 logits, found by a four-pass
// radix select (8 bits per pass, histograms in shared memory); among logits
// equal to the threshold the lowest indices are kept (np.argpartition leaves
// the choice among equal probabilities open). Each thread owns a contiguous
// run of indices, so the float64 prefix sums follow index order.
#include "common.cuh"

namespace tllm {
namespace {

constexpr int kSmThreads = 1024;
constexpr int kSmWarps = kSmThreads / 32;

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

__global__ void __launch_bounds__(kSmThreads)
    sample_kernel(const float *logits, int V, int ld, float temperature, int top_k,
                  const double *u, int *ids, int *pos_inc) {
  __shared__ float s_redf[32];
  __shared__ double s_redd[32];
  __shared__ int s_redi[32];
  __shared__ int s_hist[256];
  __shared__ uint32_t s_prefix;
  __shared__ int s_krem;
  __shared__ int s_pick, s_last;
  griddep_wait();   // the logits come from the lm_head launch before
  griddep_launch();
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const float *x = logits + (size_t)row * ld;
  const float T = temperature;

  // ---- max of the scaled logits: rounding x / T is monotonic in x, so it
  // is the scaled maximum of x
  float mx = -INFINITY;
  for (int i = tid; i < V; i += kSmThreads) mx = fmaxf(mx, x[i]);
  mx = __fdiv_rn(block_reduce(mx, [](float a, float b) { return fmaxf(a, b); }, s_redf), T);

  // ---- top-k threshold key (radix select of the k-th largest key)
  const bool use_k = top_k > 0 && top_k < V;
  uint32_t thr = 0;
  int k_eq = 0;       // how many keys equal to thr are kept
  if (use_k) {
    if (tid == 0) {
      s_prefix = 0;
      s_krem = top_k;
    }
    uint32_t mask = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = tid; b < 256; b += kSmThreads) s_hist[b] = 0;
      __syncthreads();
      const uint32_t prefix = s_prefix;
      for (int i = tid; i < V; i += kSmThreads) {
        const uint32_t key = order_key(x[i]);
        if ((key & mask) == prefix) atomicAdd(&s_hist[(key >> shift) & 0xFF], 1);
      }
      __syncthreads();
      if (tid == 0) {
        int krem = s_krem, above = 0, b = 255;
        for (; b > 0; --b) {
          if (above + s_hist[b] >= krem) break;
          above += s_hist[b];
        }
        s_prefix = prefix | ((uint32_t)b << shift);
        s_krem = krem - above;
      }
      __syncthreads();
      mask |= 0xFFu << shift;
    }
    thr = s_prefix;
    k_eq = s_krem;
  }

  // ---- this thread's contiguous run of indices: kept weights and sum
  const int per = (V + kSmThreads - 1) / kSmThreads;
  const int i0 = tid * per;
  const int i1 = min(V, i0 + per);
  int n_eq = 0;
  if (use_k)
    for (int i = i0; i < i1; ++i) n_eq += order_key(x[i]) == thr;
  int eq_total = 0;
  int eq_before = use_k ? block_exclusive_scan(n_eq, s_redi, &eq_total) : 0;
  double local = 0.0;
  int last = -1;      // last index of the run with a positive kept weight
  {
    int eq_seen = eq_before;
    for (int i = i0; i < i1; ++i) {
      bool keep = true;
      if (use_k) {
        const uint32_t key = order_key(x[i]);
        keep = key > thr || (key == thr && eq_seen++ < k_eq);
      }
      if (!keep) continue;
      const float p = expf(__fdiv_rn(x[i], T) - mx);
      local += (double)p;
      if (p > 0.f) last = i;
    }
  }
  double total = 0.0;
  const double before = block_exclusive_scan(local, s_redd, &total);

  // ---- the first index whose cumulative weight / total exceeds u: the
  // thread whose run crosses u walks it again. Its running sum rounds apart
  // from the scanned one, so a run that crosses u by the scan but not by the
  // walk yields its last positive index. Zero weights never cross.
  if (tid == 0) {
    s_pick = 0x7fffffff;
    s_last = -1;
  }
  __syncthreads();
  const double uu = u[row];
  if (last >= 0) atomicMax(&s_last, last);
  if ((before + local) / total > uu && !(before / total > uu)) {
    double c = before;
    int eq_seen = eq_before;
    int pick = last;
    for (int i = i0; i < i1; ++i) {
      if (use_k) {
        const uint32_t key = order_key(x[i]);
        if (!(key > thr || (key == thr && eq_seen++ < k_eq))) continue;
      }
      c += (double)expf(__fdiv_rn(x[i], T) - mx);
      if (c / total > uu) {
        pick = i;
        break;
      }
    }
    if (pick >= 0) atomicMin(&s_pick, pick);
  }
  __syncthreads();
  if (tid == 0) {
    // u at or above the last boundary after rounding: the last index with a
    // positive weight (where the reference's cdf first reaches 1)
    const int pick = s_pick != 0x7fffffff ? s_pick : max(s_last, 0);
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
  if (M == 0) return TLLM_OK;
  TLLM_CHECK_ARG(logits && u && ids, "NULL pointer");
  TLLM_CHECK_ARG(temperature > 1e-6f, "temperature must be > 1e-6 (use tllm_argmax)");
  TLLM_CHECK_ARG(top_k >= 0, "top_k must be non-negative");
  TLLM_CHECK_ARG(((uintptr_t)u & 7) == 0, "u must be 8-byte aligned");
  TLLM_CUDA(launch_pdl(sample_kernel, dim3(M), dim3(kSmThreads), 0, resolve(stream),
                       logits, V, ld > 0 ? ld : V, temperature, top_k, u,
                       (int *)ids, (int *)pos_inc));
  TLLM_LAUNCH_CHECK();
  return TLLM_OK;
}
