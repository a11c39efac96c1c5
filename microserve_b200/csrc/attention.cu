// Paged attention, CUDA-core path: varlen queries, causal by absolute
// position, grouped-query heads, K/V read through the block table inside the
// kernel (never materialised, unlike reference cache.py:255-272).
//
// One CTA per (query-row tile, kv head, sequence).  A sequence's query rows
// are (token t, head-in-group h) pairs, r = t * group + h, so all query heads
// that share a kv head read each K/V chunk once.  Keys stream through shared
// memory 32 at a time; each warp keeps an online softmax (running max, sum,
// accumulator) for up to kRowsPerWarp rows.
#include <cfloat>

#include "attention_tc.cuh"
#include "common.cuh"
#include "model_kernels.cuh"

namespace ms {
namespace {

constexpr int kWarps = 8;
constexpr int kChunk = 32;
// Rows per warp: 4 for d_head <= 64, 2 for 128 (static shared memory < 48 KB).
template <int DH> constexpr int rows_per_warp() { return DH <= 64 ? 4 : 2; }

template <typename T, int DH>
__global__ void __launch_bounds__(kWarps * 32)
    attn_simt_kernel(const T* __restrict__ q, int q_stride, const T* __restrict__ kpool,
                     const T* __restrict__ vpool, const int32_t* __restrict__ q_start,
                     const int32_t* __restrict__ context_lens, const int32_t* __restrict__ positions,
                     const int32_t* __restrict__ tables, int max_blocks, int bs, int num_blocks,
                     int hq, int hkv, float scale, T* __restrict__ out, int* __restrict__ err) {
  pdl_enter();
  // Lane l owns output dims l, l+32, ...; for d_head < 32 lanes >= DH idle.
  constexpr int PER_LANE = DH >= 32 ? DH / 32 : 1;
  constexpr int kRowsPerWarp = rows_per_warp<DH>();
  constexpr int kRowsPerCta = kWarps * kRowsPerWarp;
  __shared__ float Qs[kRowsPerCta][DH];
  __shared__ float Ks[kChunk][DH + 1];
  __shared__ float Vs[kChunk][DH];
  __shared__ int rowpos[kRowsPerCta];

  const int b = blockIdx.z, g = blockIdx.y, tile = blockIdx.x;
  const int group = hq / hkv;
  const int t0 = q_start[b], qlen = q_start[b + 1] - t0;
  const int nrows = qlen * group;
  const int r0 = tile * kRowsPerCta;
  if (r0 >= nrows) return;
  const int nr = min(kRowsPerCta, nrows - r0);
  const int ctx = context_lens[b];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  // Stage the tile's query rows (float) and their positions.
  for (int idx = threadIdx.x; idx < kRowsPerCta * DH; idx += blockDim.x) {
    const int r = idx / DH, d = idx - r * DH;
    float v = 0.f;
    if (r < nr) {
      const int rr = r0 + r, t = rr / group, h = g * group + rr % group;
      v = to_f(q[(int64_t)(t0 + t) * q_stride + h * DH + d]);
    }
    Qs[r][d] = v;
  }
  int kmax = 0;
  for (int r = threadIdx.x; r < kRowsPerCta; r += blockDim.x) {
    int p = -1;
    if (r < nr) p = positions[t0 + (r0 + r) / group];
    rowpos[r] = p;
  }
  __syncthreads();
  for (int r = 0; r < nr; ++r) kmax = max(kmax, rowpos[r] + 1);
  kmax = min(kmax, ctx);

  float m[kRowsPerWarp], l[kRowsPerWarp], acc[kRowsPerWarp][PER_LANE];
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int e = 0; e < PER_LANE; ++e) acc[i][e] = 0.f;
  }

  const int32_t* table = tables + (int64_t)b * max_blocks;
  for (int j0 = 0; j0 < kmax; j0 += kChunk) {
    __syncthreads();
    for (int idx = threadIdx.x; idx < kChunk * DH; idx += blockDim.x) {
      const int kk = idx / DH, d = idx - kk * DH;
      const int j = j0 + kk;
      float kv = 0.f, vv = 0.f;
      if (j < kmax) {
        int blk = table[j / bs];
        if (blk < 0 || blk >= num_blocks) {
          raise_device_error(err, kErrBlock);
          blk = 0;
        }
        const int64_t o = (((int64_t)blk * hkv + g) * bs + (j % bs)) * DH + d;
        kv = to_f(kpool[o]);
        vv = to_f(vpool[o]);
      }
      Ks[kk][d] = kv;
      Vs[kk][d] = vv;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
      const int r = warp + i * kWarps;
      if (r >= nr) continue;
      const int pos = rowpos[r];
      float s = 0.f;
#pragma unroll 8
      for (int d = 0; d < DH; ++d) s = fmaf(Qs[r][d], Ks[lane][d], s);
      s *= scale;
      const int j = j0 + lane;
      const bool valid = j < kmax && j <= pos;
      s = valid ? s : -INFINITY;
      const float cmax = warp_max(s);
      const float mn = fmaxf(m[i], cmax);
      if (mn == -INFINITY) continue;
      const float alpha = m[i] == -INFINITY ? 0.f : expf(m[i] - mn);
      const float p = valid ? expf(s - mn) : 0.f;
      l[i] = l[i] * alpha + warp_sum(p);
#pragma unroll
      for (int e = 0; e < PER_LANE; ++e) acc[i][e] *= alpha;
#pragma unroll 4
      for (int kk = 0; kk < kChunk; ++kk) {
        const float pk = __shfl_sync(0xffffffffu, p, kk);
#pragma unroll
        for (int e = 0; e < PER_LANE; ++e)
          if (DH >= 32 || lane < DH) acc[i][e] = fmaf(pk, Vs[kk][lane + 32 * e], acc[i][e]);
      }
      m[i] = mn;
    }
  }
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const int r = warp + i * kWarps;
    if (r >= nr) continue;
    const int rr = r0 + r, t = rr / group, h = g * group + rr % group;
    const float inv = l[i] > 0.f ? 1.f / l[i] : 0.f;
    T* o = out + ((int64_t)(t0 + t) * hq + h) * DH;
#pragma unroll
    for (int e = 0; e < PER_LANE; ++e)
      if (DH >= 32 || lane < DH) o[lane + 32 * e] = from_f<T>(acc[i][e] * inv);
  }
}

template <typename T, int DH>
int launch_attn(const void* q, int q_stride, const ms_kv_cache& c, int layer, const ms_batch& bt,
                int hq, void* out, cudaStream_t s) {
  const int group = hq / c.n_kv_heads;
  const int tiles = ceil_div(bt.max_q_len * group, kWarps * rows_per_warp<DH>());
  dim3 grid(tiles, c.n_kv_heads, bt.n_seqs);
  const float scale = 1.f / sqrtf((float)DH);
  launch_pdl(attn_simt_kernel<T, DH>, grid, kWarps * 32, 0, s,
      static_cast<const T*>(q), q_stride, static_cast<const T*>(c.k_pool[layer]),
      static_cast<const T*>(c.v_pool[layer]), bt.q_start, bt.context_lens, bt.positions,
      bt.block_tables, bt.max_blocks, c.block_size, c.num_blocks, hq, c.n_kv_heads, scale,
      static_cast<T*>(out), device_error_word());
  return check_launch("attn_simt_kernel");
}

template <typename T>
int attn_by_dh(const void* q, int q_stride, const ms_kv_cache& c, int layer, const ms_batch& bt,
               int hq, void* out, cudaStream_t s) {
  switch (c.d_head) {
    case 8: return launch_attn<T, 8>(q, q_stride, c, layer, bt, hq, out, s);
    case 16: return launch_attn<T, 16>(q, q_stride, c, layer, bt, hq, out, s);
    case 32: return launch_attn<T, 32>(q, q_stride, c, layer, bt, hq, out, s);
    case 64: return launch_attn<T, 64>(q, q_stride, c, layer, bt, hq, out, s);
    case 128: return launch_attn<T, 128>(q, q_stride, c, layer, bt, hq, out, s);
    default: return fail(MS_ERR_UNSUPPORTED, "paged_attention: d_head %d (8/16/32/64/128)", c.d_head);
  }
}

}  // namespace

int paged_attention(const void* q, int q_stride, const ms_kv_cache& c, int layer,
                    const ms_batch& bt, int hq, void* out, void* scratch, size_t scratch_bytes,
                    cudaStream_t s, const int32_t* seq_order) {
  if (bt.n_seqs == 0 || bt.n_tokens == 0) return MS_OK;
  if (hq % c.n_kv_heads != 0)
    return fail(MS_ERR_INVALID, "paged_attention: n_heads %d not a multiple of n_kv_heads %d", hq,
                c.n_kv_heads);
  if (bt.max_q_len <= 0) return fail(MS_ERR_INVALID, "paged_attention: max_q_len must be > 0");
  ProfScope prof(kClsAttention, s);
  if (attn_tc_supported(c, hq) && q_stride % 8 == 0) {
    const int table_bound = bt.max_blocks * c.block_size;
    const int max_ctx = bt.max_context > 0 ? min(bt.max_context, table_bound) : table_bound;
    if (attn_tma_supported(c, hq))
      return paged_attention_tma(q, q_stride, c, layer, bt, hq, out, max_ctx, scratch,
                                 scratch_bytes, s, seq_order);
    return paged_attention_tc(q, q_stride, c, layer, bt, hq, out, max_ctx, scratch, scratch_bytes,
                              s);
  }
  if (c.dtype == MS_DTYPE_F32) return attn_by_dh<float>(q, q_stride, c, layer, bt, hq, out, s);
  if (c.dtype == MS_DTYPE_BF16)
    return attn_by_dh<__nv_bfloat16>(q, q_stride, c, layer, bt, hq, out, s);
  return fail(MS_ERR_UNSUPPORTED, "paged_attention: dtype %d", c.dtype);
}

namespace {

constexpr int kOrderThreads = 256;
constexpr int kOrderTile = 2048;

// Rank of sequence b under (context length descending, index ascending): a
// strict total order, so the ranks are a permutation and each order[] slot is
// written exactly once.
__global__ void __launch_bounds__(kOrderThreads)
    seq_order_kernel(const int32_t* __restrict__ ctx, int n, int32_t* __restrict__ order) {
  pdl_enter();
  __shared__ int keys[kOrderTile];
  const int b = blockIdx.x * kOrderThreads + threadIdx.x;
  const int kb = b < n ? ctx[b] : 0;
  int rank = 0;
  for (int base = 0; base < n; base += kOrderTile) {
    const int cnt = min(kOrderTile, n - base);
    __syncthreads();
    for (int i = threadIdx.x; i < cnt; i += kOrderThreads) keys[i] = ctx[base + i];
    __syncthreads();
    if (b < n) {
      for (int i = 0; i < cnt; ++i) {
        const int kc = keys[i];
        rank += (kc > kb) | ((kc == kb) & (base + i < b));
      }
    }
  }
  if (b < n) order[rank] = b;
}

}  // namespace

int attn_seq_order(const int32_t* context_lens, int n_seqs, int32_t* order, cudaStream_t s) {
  if (n_seqs <= 0) return MS_OK;
  launch_pdl(seq_order_kernel, (n_seqs + kOrderThreads - 1) / kOrderThreads, kOrderThreads, 0, s,
      context_lens, n_seqs, order);
  return check_launch("seq_order_kernel");
}

}  // namespace ms

using namespace ms;

extern "C" int ms_paged_attention(const void* q, const ms_kv_cache* cache, int layer,
                                  const ms_batch* batch, int n_heads, void* out, void* stream) {
  MS_TRY(validate_cache(cache, layer));
  MS_REQUIRE(batch != nullptr && q && out, "ms_paged_attention: null pointer");
  MS_REQUIRE(batch->q_start && batch->context_lens && batch->positions && batch->block_tables,
             "ms_paged_attention: batch has null arrays");
  return paged_attention(q, n_heads * cache->d_head, *cache, layer, *batch, n_heads, out, nullptr,
                         0, as_stream(stream));
}

extern "C" size_t ms_attention_scratch_size(const ms_kv_cache* cache, int n_heads,
                                            const ms_batch* batch) {
  if (cache == nullptr || batch == nullptr || n_heads <= 0 || cache->n_kv_heads <= 0) return 0;
  if (!attn_tc_supported(*cache, n_heads) || batch->n_seqs <= 0 || batch->max_q_len <= 0) return 0;
  const int table_bound = batch->max_blocks * cache->block_size;
  const int max_ctx =
      batch->max_context > 0 ? min(batch->max_context, table_bound) : table_bound;
  int row_tiles = 0, n_splits = 1, split_len = 0;
  attn_tc_plan(batch->max_q_len, n_heads / cache->n_kv_heads, max_ctx, batch->n_seqs,
               cache->n_kv_heads, &row_tiles, &n_splits, &split_len);
  return attn_tc_scratch_bytes(batch->n_seqs, cache->n_kv_heads, cache->d_head, row_tiles,
                               n_splits);
}
