// Host-side launchers shared by forward.cu.
#pragma once
#include "common.cuh"

namespace ms {

// w_const: w holds a model's weights, which no kernel on the stream writes
// (the kernel reads it before waiting for its predecessor).
int rmsnorm(const float* x, const float* w, void* y, const int32_t* row_idx, int n_rows, int dim,
            float eps, int dtype, cudaStream_t s, bool w_const = false);
int embed_rmsnorm(const void* embed, const int32_t* ids, int n_tokens, int vocab, int dim,
                  const float* w, float eps, float* x, void* y, int dtype, cudaStream_t s);
int rope_kv_write(void* qkv, const int32_t* positions, const int32_t* slots, const float* cos_t,
                  const float* sin_t, int max_pos, int n_tokens, int hq, int hkv, int dh,
                  const ms_kv_cache& cache, int layer, int dtype, cudaStream_t s);
int validate_cache(const ms_kv_cache* c, int layer);
// Paged attention (attention.cu).  q: token t's head h at q + t*q_stride +
// h*dh; out: (T, hq*dh).
// `scratch` (may be null) holds split-KV partials for the tensor-core path.
// `seq_order` (may be null): the order in which sequences are scheduled (a
// permutation of 0..n_seqs-1, longest context first, from attn_seq_order).
int paged_attention(const void* q, int q_stride, const ms_kv_cache& cache, int layer,
                    const ms_batch& batch, int hq, void* out, void* scratch, size_t scratch_bytes,
                    cudaStream_t s, const int32_t* seq_order = nullptr);

// order[r] = the sequence with the r-th longest context (ties by index), so
// the attention grid starts the longest sequences first and the short ones
// fill the last wave.  Scheduling order only: every output is unchanged.
int attn_seq_order(const int32_t* context_lens, int n_seqs, int32_t* order, cudaStream_t s);

}  // namespace ms
