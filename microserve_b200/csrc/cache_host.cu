// Host-side bookkeeping of the paged KV cache: the per-sequence arithmetic of
// PagedKVCache.blocks_needed_many / append_many / truncate_many over the
// dense block table (reference cache.py:148-171, :206-222), one pass over the
// batch instead of some thirty numpy calls per round.
//
// The block free list stays with the Python allocator: it hands the new blocks
// to ms_host_append in the order sequences take them and gets the blocks that
// ms_host_truncate releases back, in table order, so block ids come and go in
// the reference's order.  Nothing here touches the GPU.
#include "common.cuh"

extern "C" int64_t ms_host_blocks_needed(const int64_t* rows, const int64_t* counts, int n,
                                         const int64_t* ntok, const int32_t* nblk,
                                         int block_size, int64_t* max_blocks) {
  int64_t total = 0, widest = 0;
  for (int i = 0; i < n; ++i) {
    const int64_t r = rows[i];
    const int64_t want = (ntok[r] + counts[i] + block_size - 1) / block_size;
    const int64_t have = nblk[r];
    const int64_t need = want > have ? want - have : 0;
    total += need;
    if (have + need > widest) widest = have + need;
  }
  if (max_blocks) *max_blocks = widest;
  return total;
}

extern "C" int ms_host_append(const int64_t* rows, const int64_t* counts, int n, int64_t* ntok,
                              int32_t* nblk, int32_t* table, int64_t stride, int block_size,
                              const int32_t* blocks, int64_t n_blocks, int64_t* out_slots) {
  MS_REQUIRE(n >= 0 && block_size > 0 && stride > 0, "ms_host_append: bad sizes");
  // Check the whole batch first: nothing changes unless every row fits.
  int64_t total = 0;
  for (int i = 0; i < n; ++i) {
    const int64_t r = rows[i];
    MS_REQUIRE(counts[i] >= 0, "ms_host_append: negative count");
    const int64_t want = (ntok[r] + counts[i] + block_size - 1) / block_size;
    MS_REQUIRE(want <= stride, "ms_host_append: row %lld needs %lld blocks, the table has %lld",
               (long long)r, (long long)want, (long long)stride);
    if (want > nblk[r]) total += want - nblk[r];
  }
  MS_REQUIRE(total == n_blocks, "ms_host_append: %lld new blocks needed, %lld given",
             (long long)total, (long long)n_blocks);
  int64_t b = 0, s = 0;
  for (int i = 0; i < n; ++i) {
    const int64_t r = rows[i];
    int32_t* row = table + r * stride;
    const int64_t first = ntok[r], last = first + counts[i];
    const int64_t want = (last + block_size - 1) / block_size;
    for (int64_t c = nblk[r]; c < want; ++c) row[c] = blocks[b++];
    if (want > nblk[r]) nblk[r] = (int32_t)want;
    for (int64_t p = first; p < last; ++p)
      out_slots[s++] = (int64_t)row[p / block_size] * block_size + p % block_size;
    ntok[r] = last;
  }
  return MS_OK;
}

extern "C" int64_t ms_host_truncate(const int64_t* rows, const int64_t* num_tokens, int n,
                                    int64_t* ntok, int32_t* nblk, const int32_t* table,
                                    int64_t stride, int block_size, int32_t* out_blocks,
                                    int64_t out_capacity) {
  if (n < 0 || block_size <= 0) return -2;
  // Check the whole batch first: nothing changes unless every row can shrink.
  int64_t drop = 0;
  for (int i = 0; i < n; ++i) {
    const int64_t r = rows[i];
    if (num_tokens[i] < 0 || num_tokens[i] > ntok[r]) return -1;  // would grow
    const int64_t keep = (num_tokens[i] + block_size - 1) / block_size;
    if (keep < nblk[r]) drop += nblk[r] - keep;
  }
  if (drop > out_capacity) return -2;
  int64_t k = 0;
  for (int i = 0; i < n; ++i) {
    const int64_t r = rows[i];
    const int64_t keep = (num_tokens[i] + block_size - 1) / block_size;
    const int32_t* row = table + r * stride;
    for (int64_t c = keep; c < nblk[r]; ++c) out_blocks[k++] = row[c];
    if (keep < nblk[r]) nblk[r] = (int32_t)keep;
    ntok[r] = num_tokens[i];
  }
  return k;
}
