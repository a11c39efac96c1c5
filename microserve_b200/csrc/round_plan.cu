// The draft side of the next speculative round, planned on the device from
// this round's accepted counts: what build_paged_batch + PagedKVCache.append
// produce for the draft cache on the host (reference batching.py:19-63,
// cache.py:159-171), after the rollback arithmetic of
// SpeculativeDecoder._rollback (speculative.py:213-226).  Launched right
// after the accept kernel, it lets the next round's draft passes start
// before the host has read this round's results.
//
// Per request b, with T = its token count before this round and n its
// accepted count, the sequence then holds T + n + 1 tokens; the target has
// T + n of them cached and the draft min(T + G - 1, T + n).  The next
// round's draft pass 0 takes the last two tokens (positions T+n-1, T+n):
// when n < G the first is already in the draft cache, so its K/V goes to a
// spare slot of the request's own reserved capacity (position T + 2G - 1,
// never read before a later pass writes it) and the cache keeps the value
// the earlier pass computed; when n == G both are new.  Two rows per
// request keep the batch shape (2B rows) fixed, so the host launches the
// passes without knowing n.  Passes j = 1..G-1 take one token at position
// T + n + j.  The verify batch's first token per request is the emitted
// token at T + n; the samplers scatter the proposals after it.  Sampling
// parameters advance one round (step + 1).
//
// The draft block tables must cover T + 2G tokens per request (the caller
// reserves the blocks); slots outside them, and block ids outside the pool,
// set the device error word and become -1 (the forward skips them).
#include "common.cuh"

namespace ms {
namespace {

struct ChainOut {
  int32_t *ids0, *pos0, *slots0, *qs0, *ctx0, *ql0, *rows0;
  int32_t *pos, *slots, *ctx;  // (G-1) x B, pass-major
  int32_t *unit_qs, *ones;
  int32_t* idsv;  // B x (G+1), request-major
};

__global__ void chain_plan_kernel(const int32_t* out_tokens, const int32_t* nacc,
                                  const int32_t* n_tok, const int32_t* last_tok,
                                  const int32_t* table, int width, int bs, int num_blocks,
                                  const ms_sampling_params* params_in, int B, int G, ChainOut o,
                                  ms_sampling_params* params_out, int* err) {
  pdl_enter();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b > B) return;
  if (b == B) {
    o.qs0[B] = 2 * B;
    o.unit_qs[B] = B;
    return;
  }
  int n = nacc[b];
  if (n < 0 || n > G) {
    raise_device_error(err, kErrToken);
    n = 0;
  }
  const int T = n_tok[b];
  const int32_t* e = out_tokens + (int64_t)b * (G + 1);
  const int32_t* row = table + (int64_t)b * width;
  auto slot = [&](int p) -> int32_t {
    const int c = p / bs;
    if (p < 0 || c >= width) {
      raise_device_error(err, kErrSlot);
      return -1;
    }
    const int blk = row[c];
    if (blk < 0 || blk >= num_blocks) {
      raise_device_error(err, kErrBlock);
      return -1;
    }
    return blk * bs + p % bs;
  };
  const int ntok = T + n + 1;
  const int tok_a = n >= 1 ? e[n - 1] : last_tok[b];
  const int tok_b = e[n];
  o.ids0[2 * b] = tok_a;
  o.ids0[2 * b + 1] = tok_b;
  o.pos0[2 * b] = ntok - 2;
  o.pos0[2 * b + 1] = ntok - 1;
  o.slots0[2 * b] = slot(n == G ? ntok - 2 : T + 2 * G - 1);
  o.slots0[2 * b + 1] = slot(ntok - 1);
  o.qs0[b] = 2 * b;
  o.ctx0[b] = ntok;
  o.ql0[b] = 2;
  o.rows0[b] = 2 * b + 1;
  for (int j = 1; j < G; ++j) {
    const int64_t k = (int64_t)(j - 1) * B + b;
    o.pos[k] = ntok + j - 1;
    o.slots[k] = slot(ntok + j - 1);
    o.ctx[k] = ntok + j;
  }
  o.unit_qs[b] = b;
  o.ones[b] = 1;
  o.idsv[(int64_t)b * (G + 1)] = tok_b;
  ms_sampling_params p = params_in[b];
  p.step += 1;
  params_out[b] = p;
}

}  // namespace
}  // namespace ms

extern "C" int64_t ms_spec_chain_size(int n_requests, int gamma) {
  if (n_requests < 1 || gamma < 1) return -1;
  const int64_t B = n_requests, G = gamma;
  return 6 * B + (B + 1) + 3 * B + 3 * (G - 1) * B + (B + 1) + B + (G + 1) * B;
}

extern "C" int ms_spec_chain_plan(const int32_t* out_tokens, const int32_t* num_accepted,
                                  const int32_t* n_tok, const int32_t* last_tok,
                                  const int32_t* draft_tables, int table_width, int block_size,
                                  int num_blocks, const ms_sampling_params* params_in,
                                  int n_requests, int gamma, int32_t* chain,
                                  ms_sampling_params* params_out, void* stream) {
  using namespace ms;
  MS_REQUIRE(n_requests >= 1 && gamma >= 1, "ms_spec_chain_plan: bad sizes");
  MS_REQUIRE(table_width >= 1 && block_size >= 1 && num_blocks >= 1,
             "ms_spec_chain_plan: bad table geometry");
  MS_REQUIRE(out_tokens && num_accepted && n_tok && last_tok && draft_tables && params_in &&
                 chain && params_out,
             "ms_spec_chain_plan: null pointer");
  const int64_t B = n_requests, G = gamma;
  int32_t* p = chain;
  ChainOut o;
  o.ids0 = p, p += 2 * B;
  o.pos0 = p, p += 2 * B;
  o.slots0 = p, p += 2 * B;
  o.qs0 = p, p += B + 1;
  o.ctx0 = p, p += B;
  o.ql0 = p, p += B;
  o.rows0 = p, p += B;
  o.pos = p, p += (G - 1) * B;
  o.slots = p, p += (G - 1) * B;
  o.ctx = p, p += (G - 1) * B;
  o.unit_qs = p, p += B + 1;
  o.ones = p, p += B;
  o.idsv = p;
  int* err = device_error_word();
  MS_REQUIRE(err != nullptr, "ms_spec_chain_plan: device error word unavailable");
  const int threads = 256;
  const int blocks = (int)((B + 1 + threads - 1) / threads);
  launch_pdl(chain_plan_kernel, dim3(blocks), dim3(threads), 0,
             static_cast<cudaStream_t>(stream), out_tokens, num_accepted, n_tok, last_tok,
             draft_tables, table_width, block_size, num_blocks, params_in, n_requests, gamma, o,
             params_out, err);
  return check_launch("chain_plan_kernel");
}
