// The paged forward pass (reference model.py:339-354), as a sequence of
// launches on one stream:
//   embed+norm -> L x [QKV GEMM -> RoPE+KV write -> attention -> O GEMM+res
//                     -> norm -> gate/up GEMM+SwiGLU -> down GEMM+res -> norm]
//   -> final norm on the requested rows -> tied lm_head GEMM (float32 logits)
// The residual stream stays float32; GEMM inputs are in the model dtype.
#include "common.cuh"
#include "gemm.cuh"
#include "model_kernels.cuh"

namespace ms {
namespace {

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct Workspace {
  float* x;      // (T, d) float32 residual stream
  void* xn;      // (T, d) normalised activations
  void* qkv;     // (T, (hq + 2 hkv) dh)
  void* attn;    // (T, hq dh)
  void* h;       // (T, d_ff)
  void* xl;      // (R, d) final-normed logit rows
  int32_t* order;  // (T) attention schedule order of the sequences
  size_t bytes;
};

Workspace carve(const ms_model& m, int T, int R, unsigned char* base) {
  const size_t es = m.dtype == MS_DTYPE_BF16 ? 2 : 4;
  const size_t qkv_w = (size_t)(m.n_heads + 2 * m.n_kv_heads) * m.d_head;
  Workspace w{};
  size_t off = 0;
  auto take = [&](size_t n) {
    unsigned char* p = base ? base + off : nullptr;
    off += align256(n);
    return p;
  };
  w.x = reinterpret_cast<float*>(take((size_t)T * m.d_model * 4));
  w.xn = take((size_t)T * m.d_model * es);
  w.qkv = take((size_t)T * qkv_w * es);
  w.attn = take((size_t)T * m.n_heads * m.d_head * es);
  w.h = take((size_t)T * m.d_ff * es);
  w.xl = take((size_t)(R > 0 ? R : 1) * m.d_model * es);
  w.order = reinterpret_cast<int32_t*>(take((size_t)(T > 0 ? T : 1) * 4));
  w.bytes = off;
  return w;
}

int validate_model(const ms_model* m) {
  MS_REQUIRE(m != nullptr, "null ms_model");
  MS_REQUIRE(m->vocab_size > 0 && m->d_model > 0 && m->n_layers > 0 && m->n_heads > 0 &&
                 m->n_kv_heads > 0 && m->d_head > 0 && m->d_ff > 0,
             "ms_model: non-positive dimension");
  MS_REQUIRE(m->n_heads % m->n_kv_heads == 0, "ms_model: n_heads %% n_kv_heads != 0");
  MS_REQUIRE(m->d_ff % 8 == 0, "ms_model: d_ff must be a multiple of 8 (got %d)", m->d_ff);
  MS_REQUIRE(m->d_head % 2 == 0, "ms_model: odd d_head");
  MS_REQUIRE(m->dtype == MS_DTYPE_F32 || m->dtype == MS_DTYPE_BF16, "ms_model: dtype %d", m->dtype);
  MS_REQUIRE(m->embed && m->final_norm && m->rope_cos && m->rope_sin && m->attn_norm && m->w_qkv &&
                 m->w_o && m->ffn_norm && m->w_gate_up && m->w_down,
             "ms_model: null weight pointer");
  return MS_OK;
}

}  // namespace
}  // namespace ms

using namespace ms;

extern "C" size_t ms_forward_workspace_size(const ms_model* model, int max_tokens,
                                            int max_logit_rows) {
  if (model == nullptr || max_tokens < 0) return 0;
  return carve(*model, max_tokens, max_logit_rows, nullptr).bytes;
}

extern "C" int ms_forward(const ms_model* model, const ms_kv_cache* cache, const ms_batch* batch,
                          const int32_t* logit_rows, int n_logit_rows, float* logits,
                          int64_t logits_row_stride, void* workspace, size_t workspace_bytes,
                          void* stream) {
  MS_TRY(validate_model(model));
  MS_TRY(validate_cache(cache, 0));
  MS_REQUIRE(batch != nullptr, "ms_forward: null batch");
  const ms_model& m = *model;
  const ms_kv_cache& c = *cache;
  const ms_batch& bt = *batch;
  MS_REQUIRE(c.n_layers == m.n_layers && c.n_kv_heads == m.n_kv_heads && c.d_head == m.d_head &&
                 c.dtype == m.dtype,
             "ms_forward: cache geometry does not match the model");
  MS_REQUIRE(bt.n_tokens >= 0 && bt.n_seqs >= 0, "ms_forward: bad batch sizes");
  if (bt.n_tokens == 0) return MS_OK;
  MS_REQUIRE(bt.input_ids && bt.positions && bt.slot_mapping && bt.q_start && bt.context_lens &&
                 bt.block_tables,
             "ms_forward: batch has null arrays");
  const int T = bt.n_tokens;
  const int R = logit_rows ? n_logit_rows : T;
  MS_REQUIRE(R >= 0 && (R == 0 || logits), "ms_forward: logits output missing");
  const Workspace w = carve(m, T, R, static_cast<unsigned char*>(workspace));
  MS_REQUIRE(workspace != nullptr && workspace_bytes >= w.bytes,
             "ms_forward: workspace too small (%zu < %zu)", workspace_bytes, w.bytes);
  cudaStream_t s = as_stream(stream);
  const int d = m.d_model, hq = m.n_heads, hkv = m.n_kv_heads, dh = m.d_head;
  const int qkv_w = (hq + 2 * hkv) * dh;
  const int dt = m.dtype;
  // workspace past the carve is scratch for the attention's split-KV partials
  void* attn_scratch = static_cast<unsigned char*>(workspace) + w.bytes;
  const size_t attn_scratch_bytes = workspace_bytes - w.bytes;

  // Longest sequences first in every layer's attention grid (one sort per pass).
  const int32_t* order = nullptr;
  if (bt.n_seqs > 1 && bt.n_seqs <= T) {
    MS_TRY(attn_seq_order(bt.context_lens, bt.n_seqs, w.order, s));
    order = w.order;
  }
  MS_TRY(embed_rmsnorm(m.embed, bt.input_ids, T, m.vocab_size, d, m.attn_norm[0], m.norm_eps, w.x,
                       w.xn, dt, s));
  for (int l = 0; l < m.n_layers; ++l) {
    // q, k, v projection with RoPE and the cache write in the GEMM's epilogue
    // (bf16 tensor-core shapes), else the projection and then rope_kv_write.
    int rc = MS_ERR_UNSUPPORTED;
    if (dt == MS_DTYPE_BF16) {
      const RopeKv rk{bt.positions, bt.slot_mapping, m.rope_cos, m.rope_sin, m.max_seq_len, hq,
                      hkv, dh, c.block_size, c.num_blocks,
                      static_cast<__nv_bfloat16*>(c.k_pool[l]),
                      static_cast<__nv_bfloat16*>(c.v_pool[l])};
      rc = gemm_qkv_rope(w.xn, m.w_qkv[l], w.qkv, T, qkv_w, d, rk, s, true);
    }
    if (rc == MS_ERR_UNSUPPORTED) {
      MS_TRY(gemm_dispatch(w.xn, m.w_qkv[l], w.qkv, nullptr, T, qkv_w, d, 0, dt, dt, kEpiStore, s,
                           true));
      MS_TRY(rope_kv_write(w.qkv, bt.positions, bt.slot_mapping, m.rope_cos, m.rope_sin,
                           m.max_seq_len, T, hq, hkv, dh, c, l, dt, s));
    } else {
      MS_TRY(rc);
    }
    // q occupies the first hq*dh columns of each qkv row.
    MS_TRY(paged_attention(w.qkv, qkv_w, c, l, bt, hq, w.attn, attn_scratch, attn_scratch_bytes,
                           s, order));
    MS_TRY(gemm_dispatch(w.attn, m.w_o[l], w.x, w.x, T, d, hq * dh, 0, dt, MS_DTYPE_F32,
                         kEpiResidual, s, true));
    MS_TRY(rmsnorm(w.x, m.ffn_norm[l], w.xn, nullptr, T, d, m.norm_eps, dt, s, true));
    MS_TRY(gemm_dispatch(w.xn, m.w_gate_up[l], w.h, nullptr, T, 2 * m.d_ff, d, 0, dt, dt,
                         kEpiSwiGLU, s, true));
    MS_TRY(gemm_dispatch(w.h, m.w_down[l], w.x, w.x, T, d, m.d_ff, 0, dt, MS_DTYPE_F32,
                         kEpiResidual, s, true));
    if (l + 1 < m.n_layers)
      MS_TRY(rmsnorm(w.x, m.attn_norm[l + 1], w.xn, nullptr, T, d, m.norm_eps, dt, s, true));
  }
  if (R == 0) return MS_OK;
  MS_TRY(rmsnorm(w.x, m.final_norm, w.xl, logit_rows, R, d, m.norm_eps, dt, s, true));
  MS_REQUIRE(logits_row_stride == 0 || logits_row_stride >= m.vocab_size,
             "ms_forward: logits_row_stride < vocab");
  return gemm_dispatch(w.xl, m.embed, logits, nullptr, R, m.vocab_size, d, logits_row_stride, dt,
                       MS_DTYPE_F32, kEpiStore, s, true);
}
