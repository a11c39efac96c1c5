// Tensor-core paged attention (attention_tc.cu).
#pragma once
#include "common.cuh"

namespace ms {

bool attn_tc_supported(const ms_kv_cache& c, int hq);
// Row tiles, KV ranges and range length for a batch.
void attn_tc_plan(int max_q_len, int group, int max_context, int n_seqs, int hkv, int* row_tiles,
                  int* n_splits, int* split_len);
size_t attn_tc_scratch_bytes(int n_seqs, int hkv, int dh, int row_tiles, int n_splits);
// Uses split-KV when `scratch_bytes` holds the partials, else one range per tile.
int paged_attention_tc(const void* q, int q_stride, const ms_kv_cache& c, int layer,
                       const ms_batch& bt, int hq, void* out, int max_context, void* scratch,
                       size_t scratch_bytes, cudaStream_t s);

// TMA-fed variant (attention_tma.cu) for power-of-two block sizes 8..64.
bool attn_tma_supported(const ms_kv_cache& c, int hq);
int paged_attention_tma(const void* q, int q_stride, const ms_kv_cache& c, int layer,
                        const ms_batch& bt, int hq, void* out, int max_context, void* scratch,
                        size_t scratch_bytes, cudaStream_t s, const int32_t* seq_order);

}  // namespace ms
