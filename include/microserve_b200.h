/*
 * microserve_b200.h -- C ABI of the B200 (sm_100a) speculative-decoding step.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), launches asynchronously on that stream and returns an
 * int status: 0 = ok, otherwise one of MS_ERR_*.  ms_last_error() returns a
 * human-readable message for the most recent failure on the calling thread.
 * No entry point allocates device memory unless its comment says so; callers
 * own every buffer (weights, K/V pools, block tables, logits, outputs).
 *
 * The Python layer (the microserve_b200 package) binds these with ctypes and keeps
 * the reference's Python API: each declaration cites the reference function
 * (path inside the MicroServe project, file:line) whose arithmetic it takes
 * over.
 */
#ifndef MICROSERVE_B200_H_
#define MICROSERVE_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MS_API __attribute__((visibility("default")))
#else
#define MS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes and dtypes ------------------------------------------ */
#define MS_OK 0
#define MS_ERR_INVALID 1     /* bad argument (null pointer, size, alignment) */
#define MS_ERR_CUDA 2        /* a CUDA runtime call or launch failed         */
#define MS_ERR_UNSUPPORTED 3 /* shape/dtype combination not compiled         */
#define MS_ERR_TOO_LARGE 4   /* size beyond a documented fixed maximum       */

#define MS_DTYPE_F32 0
#define MS_DTYPE_BF16 1

/* Philox lanes: which uniform of a request's draw step a kernel consumes.
 * A draw step is one engine iteration the request takes part in. */
#define MS_LANE_SAMPLE 0        /* plain (non-speculative) sample, lane 0   */
#define MS_LANE_DRAFT 0         /* draft proposal j uses lane j             */
#define MS_LANE_ACCEPT 64       /* accept roll for proposal i: lane 64 + i  */
#define MS_LANE_RESAMPLE 128    /* residual / bonus draw                    */

/* ---- library info -------------------------------------------------------- */
MS_API int ms_version(void);
MS_API const char* ms_last_error(void);
/* Number of kernels this library has launched since load (all threads). */
MS_API uint64_t ms_launch_count(void);
/* Device-side error word written by bounds checks on metadata (block ids,
 * slots, token ids).  Reads and clears it (synchronous copy on `stream`). */
MS_API int ms_device_error(void* stream, int32_t* out_code);
/* Live timing of one kernel class (1 GEMM, 2 attention, 3 sampling,
 * 4 accept, 5 norm): until stop, every launch of that class is bracketed by
 * CUDA events on its stream.  stop() waits for the last launch and returns
 * the summed device time and the number of launches.  Not for use inside
 * stream capture.  No reference counterpart (measurement support). */
MS_API int ms_profile_start(int kernel_class);
MS_API int ms_profile_stop(double* total_ms, int64_t* launches);

/* ---- sampling ------------------------------------------------------------ */
/* Per-request sampling parameters (device array).  temperature == 0 means
 * greedy (reference config.py:124 SamplingConfig.greedy); top_k <= 0 and
 * top_p >= 1 disable those filters (reference sampling.py:25-51). */
typedef struct {
  float temperature;
  float top_p;
  int32_t top_k;
  int32_t pad_;
  uint64_t seed; /* Philox4x32-10 key (the request generator's seed) */
  uint64_t step; /* Philox counter: the request's draw-step index    */
} ms_sampling_params;

/* Statistics of one processed logits row: p_i = x_i >= thresh ?
 * exp(x_i - max) / z : 0 with x = logits / temperature.  For a greedy row
 * argmax is set and the distribution is one-hot. */
typedef struct {
  float max;
  float thresh;
  float z;
  int32_t argmax;
} ms_row_stats;

/* Philox4x32-10 uniforms in [0,1): out[i] = u(seed[i], step[i], lane). */
MS_API int ms_philox_uniforms(const uint64_t* seeds, const uint64_t* steps, int n,
                       int lane, float* out, void* stream);

/* Draw one token per row of `logits` (row r at logits + r*row_stride):
 * temperature -> top-k -> top-p -> softmax -> inverse-CDF draw with the
 * Philox uniform of (params[pidx[r]], lane); greedy rows take the argmax.
 * Replaces reference sampling.py:54-92 (process_logits, probs_from_logits,
 * sample_from_probs, sample).  Optional outputs (nullable):
 *   probs (n_rows x vocab): the exact distribution drawn from;
 *   stats: per-row ms_row_stats;
 *   scatter_dst[scatter_idx[r]] = token (a second copy of the token).
 * Vocabularies up to 40,960 take one CTA per row; larger ones a
 * thread-block cluster of 4 or 8 CTAs per row (ms_spec_accept likewise,
 * per request, when draft_stats is given). */
MS_API int ms_sample(const float* logits, int64_t row_stride, int n_rows, int vocab,
              const ms_sampling_params* params, const int32_t* pidx, int lane,
              int32_t* tokens, float* probs, ms_row_stats* stats,
              int32_t* scatter_dst, const int32_t* scatter_idx, void* stream);

/* Fused accept / resample / bonus for B requests with gamma proposals each
 * (reference speculative.py:44-86 verify_proposals, applied as in
 * speculative.py:191-202).  Target side: (B*(gamma+1)) rows of logits,
 * row b*(gamma+1)+i, processed with params[b] (probs_from_logits,
 * sampling.py:64).  Draft side is position-major, as the draft passes
 * produce it: row, stats and proposal of (request b, position i) are at
 * index i*B + b.  One of:
 *   draft_stats != NULL: rows of draft logits plus their ms_row_stats;
 *   draft_probs_mode == 0: rows of draft logits, stats computed here;
 *   draft_probs_mode == 1: rows already hold probabilities.
 * Accept test: u < min(1, p[x] / max(q[x], 1e-10)) with u = lane
 * MS_LANE_ACCEPT+i; first reject draws from normalise(max(0, p - q)) (p if
 * the residual mass is <= 1e-9) with lane MS_LANE_RESAMPLE; all accepted
 * draws the bonus from p[gamma].
 * Outputs: out_tokens (B x (gamma+1)): accepted prefix then the extra token;
 * out_num_accepted (B). */
MS_API int ms_spec_accept(const float* target_logits, int64_t target_stride,
                   const float* draft_rows, int64_t draft_stride,
                   const ms_row_stats* draft_stats, int draft_probs_mode,
                   const int32_t* proposals, const ms_sampling_params* params,
                   int n_requests, int gamma, int vocab, int32_t* out_tokens,
                   int32_t* out_num_accepted, void* stream);

/* The draft side of the next speculative round, planned on the device from
 * this round's results, so the next round's draft passes can start before
 * the host reads them: build_paged_batch + PagedKVCache.append for the
 * draft cache (reference batching.py:19-63, cache.py:159-171) after the
 * rollback of SpeculativeDecoder._rollback (speculative.py:213-226).
 * Inputs per request b: out_tokens (B x (gamma+1)) and num_accepted (B)
 * from ms_spec_accept; n_tok[b], its token count before this round;
 * last_tok[b], its last token before this round; draft_tables (B x
 * table_width block ids) covering n_tok[b] + 2*gamma tokens; params_in
 * (B).  Output: `chain` (ms_spec_chain_size ints), laid out as
 *   ids0[2B] pos0[2B] slots0[2B] q_start0[B+1] ctx0[B] q_lens0[B] rows0[B]
 *   pos[(gamma-1)B] slots[(gamma-1)B] ctx[(gamma-1)B] q_start1[B+1] ones[B]
 *   verify_ids[B(gamma+1)]:
 * draft pass 0 takes each request's last two tokens (2B rows, logits from
 * row 2b+1; the first row's K/V goes to a spare reserved slot when it is
 * already cached), pass j >= 1 one token per request at pos[(j-1)B+b];
 * verify_ids[b(gamma+1)] is the next verify pass's first token (the
 * proposals are scattered after it).  params_out = params_in with step + 1
 * (may alias params_in).  Slots outside the tables set the device error
 * word and are written as -1. */
MS_API int64_t ms_spec_chain_size(int n_requests, int gamma);
MS_API int ms_spec_chain_plan(const int32_t* out_tokens, const int32_t* num_accepted,
                              const int32_t* n_tok, const int32_t* last_tok,
                              const int32_t* draft_tables, int table_width, int block_size,
                              int num_blocks, const ms_sampling_params* params_in,
                              int n_requests, int gamma, int32_t* chain,
                              ms_sampling_params* params_out, void* stream);

/* verify_proposals on probability rows (reference speculative.py:44-86)
 * with explicit uniforms: accept_u (gamma x B, position-major), draw_u (B).
 * Target rows b*(gamma+1)+i; draft rows and proposals at i*B+b. */
MS_API int ms_verify_probs(const float* target_probs, const float* draft_probs,
                    const int32_t* proposals, const float* accept_u,
                    const float* draw_u, int n_requests, int gamma, int vocab,
                    int32_t* out_tokens, int32_t* out_num_accepted,
                    void* stream);

/* ---- paged KV cache ------------------------------------------------------ */
/* Pool layout (per layer): [num_blocks][n_kv_heads][block_size][d_head];
 * logical slot s = block * block_size + offset (reference cache.py:1-12). */
typedef struct {
  int32_t n_layers;
  int32_t num_blocks;
  int32_t block_size;
  int32_t n_kv_heads;
  int32_t d_head;
  int32_t dtype;
  void* const* k_pool; /* host array [n_layers] of device pointers */
  void* const* v_pool;
} ms_kv_cache;

/* Host-side block-table bookkeeping (no GPU work).  The table is a dense
 * int32 array, `stride` entries per row; row r holds ntok[r] tokens in
 * nblk[r] blocks.  Rows of one call must be distinct.
 *
 * Blocks that appending counts[i] tokens to rows[i] takes beyond the blocks
 * each row holds, summed; *max_blocks (nullable) = the widest row after it
 * (reference cache.py:148-153 PagedKVCache.blocks_needed, over a batch). */
MS_API int64_t ms_host_blocks_needed(const int64_t* rows, const int64_t* counts, int n,
                                     const int64_t* ntok, const int32_t* nblk,
                                     int block_size, int64_t* max_blocks);

/* Append counts[i] tokens to rows[i]: the rows take the n_blocks new
 * `blocks` in batch order, and out_slots receives the slot of every new
 * token, row by row (reference cache.py:155-171 PagedKVCache.append, over a
 * batch).  Checks the whole batch before changing anything. */
MS_API int ms_host_append(const int64_t* rows, const int64_t* counts, int n, int64_t* ntok,
                          int32_t* nblk, int32_t* table, int64_t stride, int block_size,
                          const int32_t* blocks, int64_t n_blocks, int64_t* out_slots);

/* Shrink rows[i] to num_tokens[i] tokens; the blocks past each new end go
 * to out_blocks, row by row in table order.  Returns their number, -1 if a
 * row would grow, -2 for bad sizes or too small an out_blocks; nothing
 * changes on an error (reference cache.py:210-222 PagedKVCache.truncate,
 * over a batch). */
MS_API int64_t ms_host_truncate(const int64_t* rows, const int64_t* num_tokens, int n,
                                int64_t* ntok, int32_t* nblk, const int32_t* table,
                                int64_t stride, int block_size, int32_t* out_blocks,
                                int64_t out_capacity);

/* Scatter (T, n_kv_heads, d_head) float keys/values into one layer's pools
 * at `slots` (reference cache.py:225-234 PagedKVCache.write). */
MS_API int ms_kv_write(const ms_kv_cache* cache, int layer, const int32_t* slots,
                int n_tokens, const float* keys, const float* values,
                void* stream);

/* Gather (B, max_context, n_kv_heads, d_head) float K/V through padded
 * block tables (reference cache.py:255-272 PagedKVCache.gather). */
MS_API int ms_kv_gather(const ms_kv_cache* cache, int layer,
                 const int32_t* block_tables, int n_seqs, int max_blocks,
                 int max_context, float* keys, float* values, void* stream);

/* ---- model forward ------------------------------------------------------- */
/* Pre-norm RMSNorm / RoPE / SwiGLU decoder with tied embeddings (reference
 * model.py:265-354) and grouped-query attention (n_kv_heads <= n_heads).
 * Weights are row-major `out x in` (torch Linear layout) in `dtype`; norm
 * weights and the RoPE tables are float32.  w_qkv stacks q, k, v rows;
 * w_gate_up interleaves gate and up in groups of 8 rows
 * (rows 16g..16g+7 = gate 8g..8g+7, rows 16g+8..16g+15 = up 8g..8g+7). */
typedef struct {
  int32_t vocab_size;
  int32_t d_model;
  int32_t n_layers;
  int32_t n_heads;
  int32_t n_kv_heads;
  int32_t d_head;
  int32_t d_ff;
  int32_t max_seq_len;
  int32_t dtype;
  float norm_eps;
  const void* embed;      /* (vocab, d) -- also the lm_head              */
  const float* final_norm;
  const float* rope_cos;  /* (max_seq_len, d_head/2) float32              */
  const float* rope_sin;
  const float* const* attn_norm; /* host arrays [n_layers] of device ptrs */
  const void* const* w_qkv;      /* ((n_heads+2*n_kv_heads)*d_head, d)    */
  const void* const* w_o;        /* (d, n_heads*d_head)                   */
  const float* const* ffn_norm;
  const void* const* w_gate_up;  /* (2*d_ff, d), interleaved as above     */
  const void* const* w_down;     /* (d, d_ff)                             */
} ms_model;

/* One flattened paged batch (reference model.py:33-45 PagedBatch): n_seqs
 * sequences, sequence b owns tokens [q_start[b], q_start[b+1]) of the flat
 * arrays.  context_lens[b] counts every token cached for b after this pass's
 * writes.  All pointers are device int32. */
typedef struct {
  int32_t n_tokens;
  int32_t n_seqs;
  int32_t max_blocks;  /* row stride of block_tables */
  int32_t max_q_len;
  int32_t max_context; /* max of context_lens; 0 = unknown (bounded by the table) */
  int32_t reserved_;
  const int32_t* input_ids;
  const int32_t* positions;
  const int32_t* slot_mapping;
  const int32_t* q_start;      /* (n_seqs + 1) */
  const int32_t* context_lens; /* (n_seqs)     */
  const int32_t* block_tables; /* (n_seqs, max_blocks) */
} ms_batch;

/* Bytes of scratch ms_forward needs for up to max_tokens tokens and
 * max_logit_rows logits rows. */
MS_API size_t ms_forward_workspace_size(const ms_model* model, int max_tokens,
                                 int max_logit_rows);

/* Paged forward (reference model.py:339-354 Transformer.forward_paged):
 * writes this pass's K/V into `cache` and float32 logits for the flat rows
 * listed in logit_rows (n_logit_rows of them; NULL = every token, in order)
 * into logits (row r at logits + r*logits_row_stride; 0 means vocab). */
MS_API int ms_forward(const ms_model* model, const ms_kv_cache* cache,
               const ms_batch* batch, const int32_t* logit_rows,
               int n_logit_rows, float* logits, int64_t logits_row_stride,
               void* workspace, size_t workspace_bytes, void* stream);

/* ms_forward without a caller-provided workspace.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory (a
 * host that reaches this library only through an FFI and has no CUDA
 * allocator of its own, or a running serving loop that must not call
 * cudaMalloc).  Its scratch is an array compiled into the library, 16 MiB
 * per device, held by every GPU that loads the library until exit; a batch
 * whose workspace (ms_forward_workspace_size) exceeds it is rejected with
 * MS_ERR_TOO_LARGE before anything is launched.  The first call on a device
 * looks up the array's device address (make it before any stream capture).
 * All calls on a device share the array, so calls that overlap on the GPU
 * race; nothing in it needs clearing between calls.  Arguments and results
 * are those of ms_forward. */
MS_API int ms_forward_static_scratch(const ms_model* model,
                                     const ms_kv_cache* cache,
                                     const ms_batch* batch,
                                     const int32_t* logit_rows,
                                     int n_logit_rows, float* logits,
                                     int64_t logits_row_stride, void* stream);

/* ---- building blocks, exported for tests and for callers that compose
 *      their own forward ---------------------------------------------- */
/* y[r] = x[r] * rsqrt(mean(x[r]^2) + eps) * w  (reference model.py:77-79);
 * x float32, y in `dtype`; rows optionally gathered through row_idx. */
MS_API int ms_rmsnorm(const float* x, const float* w, void* y, const int32_t* row_idx,
               int n_rows, int dim, float eps, int dtype, void* stream);

/* C[m, n] = sum_k A[m, k] * B[n, k] in float32 accumulation (torch Linear).
 * epilogue 0: C = acc (C in c_dtype); 1: C(float) = R(float) + acc;
 * 2: SwiGLU on interleaved gate/up groups of 8, C has N/2 columns.
 * A and B are dense row-major; C (and R) rows are ldc elements apart
 * (0 = dense). */
MS_API int ms_gemm(const void* A, const void* B, void* C, const float* R, int M,
            int N, int K, int64_t ldc, int ab_dtype, int c_dtype,
            int epilogue, void* stream);

/* Which tensor-core GEMM ms_gemm and ms_forward use: 0 = chosen by shape
 * (the default), 1 = one CTA per 128 x 256 tile, 2 = CTA pairs on two SMs
 * (tcgen05 cta_group::2, 256 x 256 tiles) wherever the shape allows.  No
 * reference counterpart: a switch for measurements and tests.  Process-wide. */
MS_API int ms_gemm_set_policy(int policy);

/* Scratch bytes the tensor-core attention would use for split-KV partials on
 * this batch.  ms_forward uses workspace bytes past
 * ms_forward_workspace_size() for them; with fewer it runs one KV range per
 * tile (same results, less parallelism).  No reference counterpart. */
MS_API size_t ms_attention_scratch_size(const ms_kv_cache* cache, int n_heads,
                                        const ms_batch* batch);

/* Paged attention over one layer: q (T, n_heads, d_head) in `dtype`, causal
 * by absolute position (key j visible to a query at position p iff j <= p;
 * reference model.py:200-221), output (T, n_heads*d_head) in `dtype`. */
MS_API int ms_paged_attention(const void* q, const ms_kv_cache* cache, int layer,
                       const ms_batch* batch, int n_heads, void* out,
                       void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MICROSERVE_B200_H_ */
