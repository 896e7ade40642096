/*
 * tllm.h -- C ABI of libtllm.so, the sm_100a decode hot path of triton-llm.
 *
 * Every entry point takes plain device pointers, element counts, a dtype enum
 * and an optional stream (NULL = the library's stream for the current device).
 * No entry point allocates device memory except the tllm_malloc* family: the
 * caller (Python's triton_llm.gpu, or the model's workspace) owns all buffers,
 * including the scratch buffers some kernels need.
 *
 * Every function returns a tllm_status (0 = success). On failure the
 * thread-local message is available from tllm_last_error_string().
 *
 * Reference interfaces replaced (paths are inside ziliangpeng/triton-llm):
 *   runtime  -> triton_llm/gpu.py:114-131 (cudaMalloc/cudaFree/cudaMemcpy
 *               through ctypes), gpu.py:230-263 (allocate/to_device/
 *               to_host/synchronize), gpu.py:179-181 (check_error)
 *   kernels  -> triton_llm/kernels/*.py wrappers, cited per function below.
 */
#ifndef TLLM_H_
#define TLLM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void *tllm_stream_t; /* a cudaStream_t; NULL = library stream */

typedef enum {
  TLLM_OK = 0,
  TLLM_ERR_INVALID_ARG = 1, /* bad shape / size / pointer: Python ValueError */
  TLLM_ERR_CUDA = 2,        /* CUDA runtime error: Python RuntimeError */
  TLLM_ERR_UNSUPPORTED = 3, /* valid but not built (e.g. head_dim 24) */
  TLLM_ERR_NO_DEVICE = 4,   /* no CUDA device visible */
  TLLM_ERR_NCCL = 5,        /* NCCL failure or NCCL library missing */
  TLLM_ERR_TIMEOUT = 6,     /* a bounded wait ran out */
  TLLM_ERR_INJECTED = 7     /* failure injected through TLLM_FAULT_INJECT */
} tllm_status;

typedef enum {
  TLLM_F32 = 0,
  TLLM_BF16 = 1,
  TLLM_I32 = 2,
  /* An fp32 activation matrix stored as two bf16 planes of `plane_rows`
   * rows each: hi = bf16(x) in plane 0, lo = bf16(x - hi) in plane 1, so
   * hi + lo keeps ~16 mantissa bits of x. This is the operand format of the
   * tensor-core projections; the kernels that produce their inputs (norms,
   * attention, the SwiGLU / GELU epilogues) can write it directly. */
  TLLM_SPLIT = 3,
  /* A bf16 weight matrix (N, K) stored as contiguous 128 x 64 tiles so that
   * every tile the projection streams is one 16 KB block of HBM: tile
   * (n / 128, k / 64) starts at element ((n / 128) * (K / 64) + k / 64) * 8192
   * and holds its 128 rows of 64 elements row-major. N is padded to a
   * multiple of 128 with zero rows. K % 64 == 0. */
  TLLM_BF16_TILED = 4
} tllm_dtype;

/* ------------------------------------------------------------------------ */
/* Runtime: devices, streams, memory (replaces triton_llm/gpu.py)            */
/* ------------------------------------------------------------------------ */

/* Message of the last failing call on this thread ("" if none). */
const char *tllm_last_error_string(void);
/* Library version, e.g. 100 for 0.1.0. */
int tllm_version(void);

int tllm_device_count(int *count);
int tllm_set_device(int device);
int tllm_get_device(int *device);
/* The library stream of the current device (created on first use). */
int tllm_get_stream(tllm_stream_t *stream);

/* gpu.py:230-236 allocate(): stream-ordered pool allocation on the library
 * stream (cudaMallocAsync); the pool keeps freed memory for reuse. */
int tllm_malloc(void **ptr, size_t nbytes);
/* gpu.py:194-200 DeviceTensor.__del__: stream-ordered free. */
int tllm_free(void *ptr);
/* Plain cudaMalloc/cudaFree for buffers that other devices map. */
int tllm_malloc_static(void **ptr, size_t nbytes);
int tllm_free_static(void *ptr);
/* Page-locked host memory for the end-to-end copies. */
int tllm_host_alloc(void **ptr, size_t nbytes);
int tllm_host_free(void *ptr);

/* gpu.py:215-224 from_numpy / gpu.py:202-213 to_numpy: the copy is queued
 * on the library stream and the call returns once it is complete. */
int tllm_memcpy_h2d(void *dst, const void *src, size_t nbytes);
int tllm_memcpy_d2h(void *dst, const void *src, size_t nbytes);
int tllm_memcpy_d2d(void *dst, const void *src, size_t nbytes);
/* Asynchronous variants on `stream` (host side must be pinned to overlap). */
int tllm_memcpy_h2d_async(void *dst, const void *src, size_t nbytes,
                          tllm_stream_t stream);
int tllm_memcpy_d2h_async(void *dst, const void *src, size_t nbytes,
                          tllm_stream_t stream);
int tllm_memset(void *ptr, int value, size_t nbytes, tllm_stream_t stream);
/* gpu.py:252-263 synchronize(): waits for the library stream. */
int tllm_synchronize(void);
int tllm_stream_synchronize(tllm_stream_t stream);
int tllm_device_synchronize(void);

/* Stream and event helpers for timing and overlap. */
int tllm_stream_create(tllm_stream_t *stream);
int tllm_stream_destroy(tllm_stream_t stream);
int tllm_event_create(void **event);
int tllm_event_destroy(void *event);
int tllm_event_record(void *event, tllm_stream_t stream);
int tllm_event_elapsed_ms(void *start, void *end, float *ms);
int tllm_stream_wait_event(tllm_stream_t stream, void *event);

/* Device-side error word of the current device (bit set: 1 = a bounded
 * wait ran out, 2 = a device-side length exceeded its bound, 4 = a token id
 * was out of range, 8 = dynamic shared memory misaligned, 16 = a projection
 * launch with an invalid pipeline layout). Waits for the library stream
 * first; reset != 0 clears the word. Kernels report through it instead of
 * trapping. */
int tllm_device_error(int *code, int reset);

/* CUDA graphs of the library's work (decode steps are replayed as graphs so
 * that host launch cost leaves the critical path). Capture is thread-local:
 * every tllm_* call made by this thread on `stream` between begin and end is
 * recorded, not executed. */
int tllm_graph_capture_begin(tllm_stream_t stream);
int tllm_graph_capture_end(tllm_stream_t stream, void **graph_exec);
int tllm_graph_launch(void *graph_exec, tllm_stream_t stream);
int tllm_graph_destroy(void *graph_exec);

/* Memory info of the current device (bytes). */
int tllm_mem_info(size_t *free_bytes, size_t *total_bytes);

/* ------------------------------------------------------------------------ */
/* Attention                                                                 */
/* ------------------------------------------------------------------------ */

/*
 * Split-KV GQA decode attention over a preallocated KV cache.
 *
 * Replaces triton_llm/kernels/attention_gqa.py:149-269 (attention_gqa) on
 * its decode path (seq_q == 1, causal=False, as called from
 * smollm2_triton/model.py:310-314), batched over B independent sequences.
 *
 *   q        (B, n_head, head_dim) f32
 *   k_cache  (B, n_kv_head, max_seq, head_dim) kv_dtype
 *   v_cache  (B, n_kv_head, max_seq, head_dim) kv_dtype
 *   seq_lens (B,) int32 on the device: keys to attend for each sequence
 *            (0 <= seq_lens[b] <= max_seq; 0 yields a zero output row)
 *   out      (B, n_head, head_dim) f32
 *   head h reads kv head h / (n_head / n_kv_head) (attention_gqa.py:76).
 *   sm_scale <= 0 selects 1/sqrt(head_dim) (attention_gqa.py:235-236).
 *   max_len  host-side upper bound on max(seq_lens); it sizes the split
 *            grid (values above max_seq are clamped).
 *
 * Scratch (caller owned, see tllm_gqa_decode_workspace):
 *   partial   f32 buffer of `partial_bytes`
 *   counters  int32 (B * n_kv_head) zero-filled once; every call leaves
 *             them at zero again.
 */
int tllm_gqa_decode_workspace(int batch, int n_head, int n_kv_head,
                              int head_dim, int max_seq, int kv_dtype,
                              size_t *partial_bytes, size_t *counter_bytes);
int tllm_gqa_decode(const float *q, const void *k_cache, const void *v_cache,
                    int kv_dtype, const int32_t *seq_lens, float *out,
                    int batch, int n_head, int n_kv_head, int head_dim,
                    int max_seq, int max_len, float sm_scale, void *partial,
                    size_t partial_bytes, int32_t *counters,
                    tllm_stream_t stream);

/*
 * Causal GQA prefill attention over the preallocated cache. Replaces the
 * prefill attention of smollm2_triton/model.py:318-348 (attention_gqa with
 * causal=True at :341-343; mask of triton_llm/kernels/attention_gqa.py:
 * 97-119) for every prompt of a batch in one launch. blocks holds n_blocks
 * rows of four int32 (16-byte aligned): first row, rows (1..64), cache
 * sequence, first position; row first_row + i is the query at position
 * first_position + i and attends cache rows [0, first_position + i] of that
 * sequence (its K/V must already be in the cache: the QKV epilogue writes
 * them). Rows of a block are consecutive positions of one sequence; a
 * prompt of L rows takes ceil(L / 64) blocks. q / out as for tllm_gqa_rows.
 * bf16 caches with head_dim 64 or 128 (else TLLM_ERR_UNSUPPORTED: use
 * tllm_gqa_rows). A block that is out of range (rows, positions past
 * max_seq, sequence past cache_batch) is skipped and sets bit 2 of the
 * device error word. No scratch.
 */
int tllm_gqa_prefill(const float *q, long q_row_stride, long q_head_stride,
                     const void *k_cache, const void *v_cache, int kv_dtype,
                     const int32_t *blocks, int n_blocks, void *out,
                     int out_dtype, long out_plane_rows, long out_row_stride,
                     long out_head_stride, int n_head, int n_kv_head,
                     int head_dim, int cache_batch, int max_seq,
                     float sm_scale, tllm_stream_t stream);

/*
 * GQA attention for query rows that each read a prefix of one cached
 * sequence: row r attends to the first row_len[r] cache rows of sequence
 * row_seq[r] (row_seq NULL: sequence r). q and out of (row r, head h) are at
 * r * *_row_stride + h * *_head_stride elements. Used for the prefill
 * (causal: row_len = position + 1) and for the reference's flat layout
 * (Q as (n_head * seq_q, d_k) is row stride d_k, head stride seq_q * d_k).
 * out_dtype F32 writes fp32; TLLM_SPLIT / TLLM_BF16 write the bf16 planes
 * at the same element offsets, planes out_plane_rows * out_row_stride
 * elements apart (the operand formats of tllm_linear). Replaces
 * triton_llm/kernels/attention_gqa.py:149-269 (causal branch) and the
 * prefill attention of smollm2_triton/model.py:341-343. Scratch as for
 * tllm_gqa_decode with batch = rows.
 */
int tllm_gqa_rows(const float *q, long q_row_stride, long q_head_stride,
                  const void *k_cache, const void *v_cache, int kv_dtype,
                  const int32_t *row_seq, const int32_t *row_len, void *out,
                  int out_dtype, long out_plane_rows, long out_row_stride,
                  long out_head_stride, int rows, int n_head, int n_kv_head,
                  int head_dim, int cache_batch, int max_seq, int max_len,
                  float sm_scale, void *partial, size_t partial_bytes,
                  int32_t *counters, tllm_stream_t stream);
/* tllm_gqa_rows with the caller's estimate of the keys the rows read in
 * all (keys_hint: the sum of row_len at launch; 0 = unknown). The split of
 * each row's keys over CTAs is then planned from that total instead of
 * from max_len alone, which for a small ragged batch (fewer row x KV-group
 * pairs than ~85 % of the resident CTAs) gives longer or shorter splits
 * that fill one wave of the GPU. Results are correct for any hint; only the
 * split boundaries (and so the fp32 rounding of the merge) follow it. Used
 * by the decode step of smollm2_triton/engine.py, whose lengths are known
 * on the host when the step's graph is captured. Replaces the same
 * reference interface as tllm_gqa_rows (triton_llm/kernels/attention_gqa.py:149-269). */
int tllm_gqa_rows_hint(const float *q, long q_row_stride, long q_head_stride,
                       const void *k_cache, const void *v_cache, int kv_dtype,
                       const int32_t *row_seq, const int32_t *row_len, void *out,
                       int out_dtype, long out_plane_rows, long out_row_stride,
                       long out_head_stride, int rows, int n_head, int n_kv_head,
                       int head_dim, int cache_batch, int max_seq, int max_len,
                       float sm_scale, void *partial, size_t partial_bytes,
                       int32_t *counters, long keys_hint, tllm_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Projections (GEMM with fused epilogues)                                   */
/* ------------------------------------------------------------------------ */

/*
 * y = epilogue(x @ W^T) for x (M, K) and W (N, K). Replaces
 * triton_llm/kernels/gemm.py:53-109 plus the add / swiglu / gelu /
 * apply_rope calls that follow it in smollm2_triton/model.py:281-365 and
 * gpt2_triton/model.py:319-361.
 *
 * w_dtype BF16 or BF16_TILED: tensor-core path; x is TLLM_BF16 (one
 *   bf16 plane) or TLLM_SPLIT (hi and lo planes, ~16 mantissa bits), planes
 *   of x_plane_rows >= M rows (see tllm_split_bf16), K % 64 == 0.
 *   BF16_TILED streams each weight tile as one 16 KB block. M <= 32 on a
 *   matrix of at most 8 MiB (environment TLLM_SKINNY_MAX_M,
 *   TLLM_SKINNY_MAX_MB; every op but SCATTER) runs the decode kernel
 *   (mma.sync, weights streamed straight into registers, no set-up); other
 *   shapes run the tcgen05 kernel (TMA ring, TMEM accumulators, split-K
 *   over a cluster). The two agree to fp32 summation order.
 * w_dtype F32 : CUDA-core fp32 path; x must be F32 (M, K), K % 4 == 0.
 * out_dtype F32, TLLM_SPLIT or TLLM_BF16 (planes of out_plane_rows rows of
 *   ld_out); op RESID needs F32.
 *
 * op 0 STORE : out[m, n] = acc (+ bias[n])
 * op 1 RESID : out[m, n] = resid[m, n] + acc (+ bias[n]); resid may be out
 * op 2 GELU  : out[m, n] = gelu_tanh(acc + bias[n])   (gelu.py:17-28, :50-51)
 * op 3 SWIGLU: W rows are gate/up interleaved in blocks of 8;
 *              out[m, j] = silu(gate_j) * up_j        (swiglu.py:51-56)
 * op 4 QKV   : W rows are the q, k, v heads (n_head + 2 n_kv_head heads of
 *              head_dim rows), each head stored as blocks of 8 dims
 *              (8b..8b+7, D/2+8b..D/2+8b+7). Row m is token row_pos[m] of
 *              cache sequence row_seq[m]: q heads (rotated if cos_t != NULL)
 *              go to q_out (M, n_head, D); k heads (rotated) and v heads are
 *              written into the caches (B, n_kv_head, max_seq, D) at
 *              row_pos[m] (rope.py:49-66 + smollm2_triton/model.py:296-302);
 *              if lens_out != NULL, lens_out[row_seq[m]] = row_pos[m] + 1.
 * op 5 SCATTER: row m of acc goes to the receive slot of this rank on every
 *              rank of the peer group p2p (tllm_p2p_create), over NVLink,
 *              each value tagged with the call's number in one 64-bit word.
 *              M <= the group's rows, N <= its columns, no bias, out unused.
 *              tllm_rmsnorm_p2p completes the all-reduce. No counterpart in
 *              the reference (single-GPU); it replaces the all-reduce of a
 *              row-parallel o_proj / down_proj.
 * Scratch for split-K: tllm_linear_workspace; counters zero-filled once
 * (the kernel leaves them at zero).
 */
/*
 * RMSNorm folded into the projections on either side of it
 * (kernels/rms_norm.py:50-55: y = x / sqrt(sum(x^2) / N + eps) * w, then
 * y @ W). Since sum_k W[n, k] (x_k / r) w_k = (sum_k W[n, k] x_k w_k) / r
 * for a per-row r, the norm weight goes on the operand and the row scale
 * after the product:
 *   producer (op RESID, the projection that writes x): also stores
 *     fx[m, n] = out[m, n] * next_norm_w[n] in operand format (fx_dtype
 *     TLLM_SPLIT or TLLM_BF16, planes fx_plane_rows rows apart, rows of N)
 *     and ss_out[p * ss_ld + m] = sum of out[m, n]^2 over column part p
 *     (the 128-column weight tiles: tllm_linear_fold_parts gives their
 *     number); a folded call always runs on the tensor-core kernel;
 *   consumer (op STORE, SWIGLU or QKV, the projection that reads fx):
 *     divides row m of the product by
 *     sqrt(sum_{p < ss_parts} ss_in[p * ss_ld + m] / ss_cols + eps)
 *     before bias, SwiGLU or RoPE.
 * The norm's own launch disappears. bf16 weights only. No counterpart in the
 * reference (it launches rms_norm between the GEMMs).
 */
typedef struct {
  const float *next_norm_w;  /* producer */
  void *fx;
  int fx_dtype;
  int fx_plane_rows;
  float *ss_out;
  const float *ss_in;        /* consumer */
  int ss_parts;
  int ss_cols;
  float eps;
  int ss_ld;                 /* both: row stride of the partials (>= M) */
} tllm_norm_fold;

/* Partial sums per row that a folded-norm producer tllm_linear(M, N, K,
 * bf16 weights, op RESID) writes: its consumers' ss_parts. */
int tllm_linear_fold_parts(int M, int N, int K, int *parts);

int tllm_linear_workspace(int M, int N, int K, size_t *partial_bytes,
                          size_t *counter_bytes);
/* Launch plan of the bf16 path for (M, N, K) and activation format x_dtype
 * (SPLIT or BF16): plan[0..7] = activation tile width, activation tiles,
 * 128-row weight tiles, K splits (cluster size), weight ring stages, dynamic
 * shared memory bytes, activation ring stages, CTAs resident at once. */
int tllm_linear_plan(int M, int N, int K, int x_dtype, int *plan);
int tllm_linear(const void *x, int x_dtype, int x_plane_rows, const void *w,
                int w_dtype, int M, int N, int K, int op, const float *bias,
                void *out, int out_dtype, int out_plane_rows, int ld_out,
                const float *resid, const float *cos_t, const float *sin_t,
                const int32_t *row_seq, const int32_t *row_pos, float *q_out,
                void *k_cache, void *v_cache, int kv_dtype, int max_seq,
                int n_head, int n_kv_head, int head_dim, int32_t *lens_out,
                const void *p2p, void *partial, size_t partial_bytes,
                int32_t *counters, tllm_stream_t stream);
/* tllm_linear with a folded RMSNorm (tllm_norm_fold above; NULL = none). */
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

/*
 * The decode MLP half of a Llama-style layer in one persistent launch (no
 * counterpart in the reference, which runs it as o GEMM, add, rms_norm,
 * gate/up GEMMs, swiglu, down GEMM and add: smollm2_triton/model.py:344-357):
 *   h   += attn . Wo^T
 *   x    = RMSNorm(h) * ln_w            (eps; the norm before the MLP)
 *   act  = silu(x . Wg^T) * (x . Wu^T)
 *   h   += act . Wd^T
 * attn, x and act are TLLM_BF16 operand buffers (one plane of
 * *_plane_rows >= M rows of attn_dim, hidden and ffn values); x and act are
 * overwritten with the norm and SwiGLU outputs. Weights TLLM_BF16_TILED: Wo
 * (hidden, attn_dim), Wgu (2 ffn, hidden) with gate/up rows interleaved in
 * blocks of 8 as for op SWIGLU of tllm_linear, Wd (hidden, ffn). h fp32
 * (M, hidden), in place. M <= 64, hidden % 128 == 0, attn_dim % 64 == 0,
 * ffn % 64 == 0. One CTA per SM, launched cooperatively; the three GEMMs
 * share one weight stream split evenly over the SMs, and the phases meet at
 * grid barriers. workspace: tllm_mlp_workspace bytes, 256-byte aligned,
 * zero-filled before the first call; its barrier and per-tile counters
 * only grow (each call adds a fixed amount), so they stay valid across
 * calls and graph replays without a reset. Calls that overlap on the GPU
 * must not share one, and after a call that set the device error word
 * (a bounded wait gave up) it must be zero-filled again.
 */
int tllm_mlp_workspace(int M, int attn_dim, int hidden, int ffn,
                       size_t *bytes);
int tllm_mlp(const void *attn, int attn_plane_rows, const void *w_o, float *h,
             const float *ln_w, float eps, void *x, int x_plane_rows,
             const void *w_gu, void *act, int act_plane_rows,
             const void *w_down, int M, int attn_dim, int hidden, int ffn,
             void *workspace, size_t workspace_bytes, tllm_stream_t stream);

/* C = A @ B, fp32, A (M, K), B (K, N) row-major: the reference's weight
 * layout (triton_llm/kernels/gemm.py:53-109). */
int tllm_gemm_f32(const float *a, const float *b, float *c, int M, int N,
                  int K, tllm_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Norms, embedding, sampling, elementwise                                   */
/* ------------------------------------------------------------------------ */

/* triton_llm/kernels/rms_norm.py:68-115: y = (x / sqrt(mean(x^2) + eps)) * w
 * y_dtype F32 (M, N), or TLLM_SPLIT / TLLM_BF16 with planes of y_plane_rows
 * rows (the projection operand formats). */
int tllm_rmsnorm(const float *x, const float *w, void *y, int y_dtype,
                 int y_plane_rows, int M, int N, float eps,
                 tllm_stream_t stream);
/* h += add in place, then y = RMSNorm(h): the residual add of a row-sharded
 * projection (its all-reduced partial sums) fused into the next norm
 * (smollm2_triton/model.py:351-357: add, then rms_norm). Output as for
 * tllm_rmsnorm. */
int tllm_rmsnorm_add(float *h, const float *add, const float *w, void *y,
                     int y_dtype, int y_plane_rows, int M, int N, float eps,
                     tllm_stream_t stream);

/*
 * Peer-to-peer all-reduce of a tensor-parallel group, one rank per GPU
 * (no counterpart in the reference, whose decode runs on one device).
 * Each rank allocates receive slots [2][size][rows][cols] of 64-bit words
 * (fp32 bits | call number << 32) and exports them as a CUDA IPC handle
 * (tllm_p2p_handle_bytes bytes); after exchanging the handles (any host
 * channel), tllm_p2p_open maps every peer's slots. A projection with op
 * SCATTER writes its partial rows into every rank's slot; tllm_rmsnorm_p2p
 * then waits (bounded, ~2 s, device error bit 1) until every word carries
 * the current call number, adds the slots in rank order to h (identical on
 * every rank), and normalises: h += sum_q part_q; y = RMSNorm(h). Calls
 * alternate between two slot sets, so consecutive SCATTER / rmsnorm_p2p
 * pairs need no barrier. All ranks must issue the same sequence of pairs.
 */
int tllm_p2p_handle_bytes(void);
int tllm_p2p_create(int size, int rows, int cols, void **ctx, void *ipc_handle);
int tllm_p2p_open(void *ctx, int rank, const void *handles);
int tllm_p2p_destroy(void *ctx);
int tllm_rmsnorm_p2p(float *h, const void *p2p, const float *w, void *y,
                     int y_dtype, int y_plane_rows, int M, int N, float eps,
                     tllm_stream_t stream);

/*
 * NCCL all-reduce of a tensor-parallel group (no counterpart in the
 * reference, which runs on one device; its roadmap defers tensor
 * parallelism, ROADMAP.md:121). NCCL is loaded on first use (libnccl.so.2,
 * or TLLM_NCCL_LIB); TLLM_ERR_NCCL when it is missing. Rank 0 makes a
 * unique id (tllm_nccl_unique_id_bytes bytes) and the caller hands it to
 * every rank over its own host channel; each rank then calls
 * tllm_nccl_init with its device current. Communicators are non-blocking:
 * init, an all-reduce that cannot be enqueued at once, and destroy are
 * polled for at most timeout_ms (<= 0: 120 s), after which the
 * communicator is aborted and TLLM_ERR_TIMEOUT returned -- a rank that
 * never joins or has died ends its peers' waits with an error, not a hang.
 * tllm_nccl_all_reduce sums `count` F32 or BF16 elements of `buf` in place
 * over the group, ordered on `stream` (NULL = library stream); it may be
 * captured in a CUDA graph. tllm_nccl_check reports the communicator's
 * asynchronous state (0 = healthy, 7 = in progress, other = an ncclResult_t
 * error) for a host-side health check between steps.
 */
int tllm_nccl_version(int *version);
int tllm_nccl_unique_id_bytes(void);
int tllm_nccl_unique_id(void *id);
int tllm_nccl_init(void **comm, int size, int rank, const void *id,
                   int timeout_ms);
int tllm_nccl_all_reduce(void *comm, void *buf, size_t count, int dtype,
                         tllm_stream_t stream, int timeout_ms);
int tllm_nccl_check(void *comm, int *state);
int tllm_nccl_destroy(void *comm, int timeout_ms);
int tllm_nccl_abort(void *comm);
/* triton_llm/kernels/layernorm.py:79-152 (two-pass mean / variance);
 * output as for tllm_rmsnorm. */
int tllm_layernorm(const float *x, const float *gamma, const float *beta,
                   void *y, int y_dtype, int y_plane_rows, int M, int N,
                   float eps, tllm_stream_t stream);
/* fp32 (rows, cols) -> the projection operand format: y_dtype TLLM_SPLIT
 * (hi and lo planes) or TLLM_BF16 (one plane), planes of plane_rows >= rows
 * rows. No counterpart in the reference (its activations stay fp32). */
int tllm_split_bf16(const float *x, void *y, int y_dtype, int rows, int cols,
                    int plane_rows, tllm_stream_t stream);
/* out[m] = wte[ids[m]] (+ wpe[pos[m]] if wpe): triton_llm/kernels/
 * embedding.py:98-187 and smollm2_triton/model.py:547-560. Out-of-range ids
 * give a zero row and set bit 4 of the device error word. */
int tllm_embedding(const int32_t *ids, const void *wte, int wte_dtype,
                   const float *wpe, const int32_t *pos, float *out, int M,
                   int n_embd, int vocab, int max_pos, tllm_stream_t stream);
/* ids[m] = first argmax of logits[m, :V] (smollm2_triton/model.py:583);
 * pos_inc[m] += 1 when pos_inc != NULL. ld = row stride (0: V). */
int tllm_argmax(const float *logits, int M, int V, int ld, int32_t *ids,
                int32_t *pos_inc, tllm_stream_t stream);
/* Temperature / top-k sample of each row (smollm2_triton/model.py:566-582):
 * ids[m] = the first index i (index order) whose cumulative weight
 * exp(logits[m,i]/T - max) / sum exceeds u[m], over the top_k largest
 * entries when 0 < top_k < V (ties at the threshold keep the lowest indices),
 * else over all V. u[m] in [0, 1) is the uniform the reference's
 * np.random.choice draws (random_sample()); the caller draws it from the same
 * generator so the random stream is consumed as the reference consumes it.
 * temperature must be > 1e-6 (the reference takes argmax below that: call
 * tllm_argmax). pos_inc[m] += 1 when pos_inc != NULL; ld = row stride (0: V).
 * u is device memory, 8-byte aligned. */
int tllm_sample(const float *logits, int M, int V, int ld, float temperature,
                int top_k, const double *u, int32_t *ids, int32_t *pos_inc,
                tllm_stream_t stream);
/* triton_llm/kernels/rope.py:153-222: in-place rotate-half RoPE of x
 * (n_rows, d), row r at position (r % seq_len) + position_offset, tables
 * (max_seq, d/2) f32. */
int tllm_rope(float *x, const float *cos_t, const float *sin_t, int n_rows,
              int d, int seq_len, int position_offset, tllm_stream_t stream);
/* op 0: out = silu(a) * b (swiglu.py:70-119); op 1: out = a + b
 * (add.py:54-95); op 2: out = gelu_tanh(a) (gelu.py:56-83). */
int tllm_elementwise(int op, const float *a, const float *b, float *out,
                     long n, tllm_stream_t stream);
/* Row softmax (triton_llm/kernels/softmax.py:105-180). */
int tllm_softmax(const float *x, float *y, int M, int N, tllm_stream_t stream);

/* Synthetic data on the device: element i = (sum of four 16-bit hashes of
 * (seed, i) - 131070) * std / (65536 / sqrt(3)), mean 0, standard deviation
 * std (bf16: rounded to nearest even). Used for random-init weights and
 * prefilled KV contexts in benchmarks. */
int tllm_fill_random(void *ptr, int dtype, long n, uint64_t seed, float std,
                     tllm_stream_t stream);

/*
 * Allocation-free variant of tllm_gqa_decode. It has no counterpart in the
 * reference; it exists for callers that cannot let a library allocate device
 * memory (servers that own all of HBM through their own arenas, hosts whose
 * memory accounting forbids hidden allocations, decode loops that must never
 * block in cudaMalloc). Same arguments and results as tllm_gqa_decode, minus
 * the scratch buffers: the split-KV partials and counters live in a fixed
 * ~8.3 MiB device array inside libtllm.so (8 MiB of partials; when more
 * would be needed the batch is cut into fewer, longer splits). Limit: batch *
 * n_head <= 65536, larger batches fail with TLLM_ERR_INVALID_ARG. The first
 * call on a device looks up the array's device address
 * (cudaGetSymbolAddress); make that first call before any stream capture.
 * All calls on a device share the array and it keeps the last call's data:
 * calls that overlap on the GPU race and must not be issued. Device-side
 * error codes of these calls are kept in the same array, not in the word
 * read by tllm_device_error: read them with tllm_gqa_decode_noalloc_error.
 */
int tllm_gqa_decode_noalloc(const float *q, const void *k_cache,
                            const void *v_cache, int kv_dtype,
                            const int32_t *seq_lens, float *out, int batch,
                            int n_head, int n_kv_head, int head_dim,
                            int max_seq, int max_len, float sm_scale,
                            tllm_stream_t stream);

/* Device-side error bits raised by tllm_gqa_decode_noalloc calls on the
 * current device since the last reset, with the bit values of
 * tllm_device_error: 1 = a bounded wait ran out (the output is then
 * incomplete), 2 = a sequence length above max_len (it was clamped). Waits
 * for the whole device, copies the word out (allocating nothing) and clears
 * it when reset != 0. No counterpart in the reference (it belongs to
 * tllm_gqa_decode_noalloc). */
int tllm_gqa_decode_noalloc_error(int *code, int reset);

#ifdef __cplusplus
}
#endif

#endif /* TLLM_H_ */
