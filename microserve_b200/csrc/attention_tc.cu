// Paged attention on the tensor cores for bf16 caches (mma.sync m16n8k16).
//
// Work unit: (row tile, kv head, sequence, KV split).  A sequence's query rows
// are (token t, head-in-group h) pairs, r = t * group + h, so the query heads
// sharing a kv head (GQA) form one M dimension and every K/V byte is read
// once per row tile: 5 verify tokens x 8 heads = 40 rows for the 1.1B model,
// 6 x 4 = 24 for the 8B shape.  Four warps each own 16 query rows.
//
// Per 64-key chunk: all threads cp.async the chunk's K and V rows (each key
// row found through the block table) into a 3-stage (d_head 64) or 2-stage
// (d_head 128) shared-memory ring; each warp computes S = Q K^T with
// ldmatrix + mma, applies the causal mask (key j visible to a query at
// absolute position p iff j <= p, reference model.py:214-218), updates an
// online softmax in registers, and accumulates O += P V (P re-packed from
// the S accumulators, V through ldmatrix.trans).
//
// Long contexts are split into KV ranges of `split_len` keys; a sequence
// with one range writes its normalised output directly, otherwise each
// range writes (O, max, sum) partials and attn_combine_kernel merges them.
#include <cfloat>

#include "attention_tc.cuh"
#include "model_kernels.cuh"

namespace ms {
namespace {

constexpr int kRows = 64;    // query rows per CTA (4 warps x 16)
constexpr int kChunk = 64;   // keys per pipeline stage
constexpr int kThreads = 128;
constexpr float kLog2e = 1.4426950408889634f;

template <int DH> struct AttnCfg {
  static constexpr int kStages = DH <= 64 ? 3 : 2;
  static constexpr int kLd = DH + 8;  // padded row (elements): conflict-free ldmatrix
  static constexpr int kTileBytes = kChunk * kLd * 2;
  static constexpr int kSmem = kRows * kLd * 2 + kStages * 2 * kTileBytes + kRows * 4;
};

__device__ __forceinline__ uint32_t s_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldm_x4(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c,
                                       uint32_t& d) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
               : "r"(addr));
}
__device__ __forceinline__ void ldm_x4_t(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c,
                                         uint32_t& d) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

struct AttnArgs {
  const __nv_bfloat16* q;
  int q_stride;
  const __nv_bfloat16* kpool;
  const __nv_bfloat16* vpool;
  const int32_t* q_start;
  const int32_t* context_lens;
  const int32_t* positions;
  const int32_t* tables;
  int max_blocks, bs, num_blocks, hq, hkv, row_tiles, n_splits, split_len;
  float scale_log2;
  __nv_bfloat16* out;
  float* part_o;   // [B][hkv][row_tiles][n_splits][kRows][DH]
  float* part_ml;  // [B][hkv][row_tiles][n_splits][kRows][2]
  int* err;
};

template <int DH>
__global__ void __launch_bounds__(kThreads) attn_tc_kernel(AttnArgs a) {
  pdl_enter();
  using Cfg = AttnCfg<DH>;
  constexpr int LD = Cfg::kLd;
  constexpr int NT = DH / 8;  // n8 tiles of the output
  extern __shared__ __align__(128) unsigned char smem[];
  __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* KV = Qs + kRows * LD;  // stages x {K, V} x [kChunk][LD]
  int* rowpos = reinterpret_cast<int*>(KV + Cfg::kStages * 2 * kChunk * LD);

  const int split = blockIdx.x % a.n_splits, rt = blockIdx.x / a.n_splits;
  const int g = blockIdx.y, b = blockIdx.z;
  const int group = a.hq / a.hkv;
  const int t0 = a.q_start[b], qlen = a.q_start[b + 1] - t0;
  const int nrows = qlen * group;
  const int r0 = rt * kRows;
  if (r0 >= nrows) return;
  const int nr = min(kRows, nrows - r0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // rows: positions and the key range this tile can see
  for (int r = threadIdx.x; r < kRows; r += kThreads)
    rowpos[r] = r < nr ? a.positions[t0 + (r0 + r) / group] : -1;
  __syncthreads();
  int kmax = 0;
  for (int r = 0; r < nr; ++r) kmax = max(kmax, rowpos[r] + 1);
  kmax = min(kmax, a.context_lens[b]);
  const int splits_here = max(1, (kmax + a.split_len - 1) / a.split_len);
  if (split >= splits_here) return;
  const int kbeg = split * a.split_len;
  const int kend = min(kmax, kbeg + a.split_len);

  // stage Q (zero rows past nr)
  for (int idx = threadIdx.x; idx < kRows * (DH / 8); idx += kThreads) {
    const int r = idx / (DH / 8), c = (idx % (DH / 8)) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < nr) {
      const int rr = r0 + r, t = rr / group, h = g * group + rr % group;
      v = *reinterpret_cast<const uint4*>(a.q + (int64_t)(t0 + t) * a.q_stride + h * DH + c);
    }
    *reinterpret_cast<uint4*>(Qs + r * LD + c) = v;
  }

  const int32_t* table = a.tables + (int64_t)b * a.max_blocks;
  const int64_t head_stride = (int64_t)a.bs * DH;
  auto load_chunk = [&](int j0, int stage) {
    __nv_bfloat16* Kd = KV + stage * 2 * kChunk * LD;
    __nv_bfloat16* Vd = Kd + kChunk * LD;
    constexpr int SEGS = DH / 8;  // 16-byte segments per key row
    for (int idx = threadIdx.x; idx < kChunk * SEGS; idx += kThreads) {
      const int kk = idx / SEGS, c = (idx % SEGS) * 8;
      const int j = j0 + kk;
      const bool valid = j < kend;
      int64_t off = 0;
      if (valid) {
        int blk = table[j / a.bs];
        if (blk < 0 || blk >= a.num_blocks) {
          raise_device_error(a.err, kErrBlock);
          blk = 0;
        }
        off = ((int64_t)blk * a.hkv + g) * head_stride + (int64_t)(j % a.bs) * DH + c;
      }
      cp_async16(s_addr(Kd + kk * LD + c), a.kpool + off, valid);
      cp_async16(s_addr(Vd + kk * LD + c), a.vpool + off, valid);
    }
  };

  const int nchunks = (kend - kbeg + kChunk - 1) / kChunk;
#pragma unroll
  for (int s = 0; s < Cfg::kStages - 1; ++s) {
    if (s < nchunks) load_chunk(kbeg + s * kChunk, s);
    cp_commit();
  }

  // per-thread rows of this warp's 16-row slice: lane/4 and lane/4 + 8
  const int wr = warp * 16;
  const int ra = wr + (lane >> 2), rb = ra + 8;
  const int pos_a = rowpos[ra], pos_b = rowpos[rb];
  const bool warp_live = wr < nr;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  float o[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  for (int ch = 0; ch < nchunks; ++ch) {
    const int pre = ch + Cfg::kStages - 1;
    if (pre < nchunks) load_chunk(kbeg + pre * kChunk, pre % Cfg::kStages);
    cp_commit();
    cp_wait<Cfg::kStages - 1>();
    __syncthreads();
    if (warp_live) {
      const __nv_bfloat16* Ks = KV + (ch % Cfg::kStages) * 2 * kChunk * LD;
      const __nv_bfloat16* Vs = Ks + kChunk * LD;
      // S = Q K^T : 16 rows x 64 keys = 8 n8 tiles
      float s[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
      for (int k0 = 0; k0 < DH; k0 += 16) {
        uint32_t a0, a1, a2, a3;
        ldm_x4(s_addr(Qs + (wr + (lane & 15)) * LD + k0 + (lane >> 4) * 8), a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < 8; nt += 2) {
          uint32_t b0, b1, b2, b3;
          const int key = nt * 8 + (lane & 7) + ((lane >> 4) << 3);
          ldm_x4(s_addr(Ks + key * LD + k0 + ((lane >> 3) & 1) * 8), b0, b1, b2, b3);
          mma_bf16(s[nt], a0, a1, a2, a3, b0, b1);
          mma_bf16(s[nt + 1], a0, a1, a2, a3, b2, b3);
        }
      }
      // mask, online softmax (base-2 exponentials of scaled scores)
      const int jbase = kbeg + ch * kChunk + 2 * (lane & 3);
      float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int j = jbase + nt * 8 + e;
          const bool va = j < kend && j <= pos_a, vb = j < kend && j <= pos_b;
          s[nt][e] = va ? s[nt][e] * a.scale_log2 : -INFINITY;
          s[nt][2 + e] = vb ? s[nt][2 + e] * a.scale_log2 : -INFINITY;
          mx_a = fmaxf(mx_a, s[nt][e]);
          mx_b = fmaxf(mx_b, s[nt][2 + e]);
        }
      }
#pragma unroll
      for (int o_ = 1; o_ <= 2; o_ <<= 1) {
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, o_));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, o_));
      }
      const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
      const float al_a = mn_a == -INFINITY ? 1.f : exp2f(m_a - mn_a);
      const float al_b = mn_b == -INFINITY ? 1.f : exp2f(m_b - mn_b);
      float ps_a = 0.f, ps_b = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          s[nt][e] = mn_a == -INFINITY ? 0.f : exp2f(s[nt][e] - mn_a);
          s[nt][2 + e] = mn_b == -INFINITY ? 0.f : exp2f(s[nt][2 + e] - mn_b);
          ps_a += s[nt][e];
          ps_b += s[nt][2 + e];
        }
      }
      l_a = l_a * al_a + ps_a;
      l_b = l_b * al_b + ps_b;
      m_a = mn_a;
      m_b = mn_b;
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        o[i][0] *= al_a;
        o[i][1] *= al_a;
        o[i][2] *= al_b;
        o[i][3] *= al_b;
      }
      // O += P V : P (16 x 64 keys) as four k16 A-fragments
#pragma unroll
      for (int kt = 0; kt < 4; ++kt) {
        const uint32_t p0 = pack2(s[2 * kt][0], s[2 * kt][1]);
        const uint32_t p1 = pack2(s[2 * kt][2], s[2 * kt][3]);
        const uint32_t p2 = pack2(s[2 * kt + 1][0], s[2 * kt + 1][1]);
        const uint32_t p3 = pack2(s[2 * kt + 1][2], s[2 * kt + 1][3]);
#pragma unroll
        for (int nt = 0; nt < NT; nt += 2) {
          uint32_t b0, b1, b2, b3;
          const int key = kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          ldm_x4_t(s_addr(Vs + key * LD + nt * 8 + (lane >> 4) * 8), b0, b1, b2, b3);
          mma_bf16(o[nt], p0, p1, p2, p3, b0, b1);
          mma_bf16(o[nt + 1], p0, p1, p2, p3, b2, b3);
        }
      }
    }
    __syncthreads();
  }
  cp_wait<0>();
  if (!warp_live) return;

  // row sums across the quad
#pragma unroll
  for (int o_ = 1; o_ <= 2; o_ <<= 1) {
    l_a += __shfl_xor_sync(0xffffffffu, l_a, o_);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, o_);
  }
  const int col = 2 * (lane & 3);
  if (splits_here == 1) {
    const float ia = l_a > 0.f ? 1.f / l_a : 0.f, ib = l_b > 0.f ? 1.f / l_b : 0.f;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = half ? rb : ra;
      if (r >= nr) continue;
      const int rr = r0 + r, t = rr / group, h = g * group + rr % group;
      __nv_bfloat16* dst = a.out + ((int64_t)(t0 + t) * a.hq + h) * DH + col;
      const float inv = half ? ib : ia;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        *reinterpret_cast<uint32_t*>(dst + nt * 8) =
            pack2(o[nt][2 * half] * inv, o[nt][2 * half + 1] * inv);
    }
  } else {
    const int64_t unit = (((int64_t)b * a.hkv + g) * a.row_tiles + rt) * a.n_splits + split;
    float* po = a.part_o + unit * kRows * DH;
    float* pml = a.part_ml + unit * kRows * 2;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = half ? rb : ra;
      if (r >= nr) continue;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        *reinterpret_cast<float2*>(po + r * DH + nt * 8 + col) =
            make_float2(o[nt][2 * half], o[nt][2 * half + 1]);
      if ((lane & 3) == 0) {
        pml[r * 2] = half ? m_b : m_a;
        pml[r * 2 + 1] = half ? l_b : l_a;
      }
    }
  }
}

// Merge the split partials of sequences with more than one KV range.
template <int DH>
__global__ void attn_combine_kernel(AttnArgs a) {
  pdl_enter();
  const int rt = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int group = a.hq / a.hkv;
  const int t0 = a.q_start[b], qlen = a.q_start[b + 1] - t0;
  const int nrows = qlen * group;
  const int r0 = rt * kRows;
  if (r0 >= nrows) return;
  const int nr = min(kRows, nrows - r0);
  int kmax = 0;
  for (int r = 0; r < nr; ++r) kmax = max(kmax, a.positions[t0 + (r0 + r) / group] + 1);
  kmax = min(kmax, a.context_lens[b]);
  const int splits = max(1, (kmax + a.split_len - 1) / a.split_len);
  if (splits == 1) return;
  const int64_t unit0 = (((int64_t)b * a.hkv + g) * a.row_tiles + rt) * a.n_splits;
  for (int idx = threadIdx.x; idx < nr * DH; idx += blockDim.x) {
    const int r = idx / DH, d = idx % DH;
    float mx = -INFINITY;
    for (int s = 0; s < splits; ++s) mx = fmaxf(mx, a.part_ml[((unit0 + s) * kRows + r) * 2]);
    float l = 0.f, acc = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float ms = a.part_ml[((unit0 + s) * kRows + r) * 2];
      const float w = ms == -INFINITY ? 0.f : exp2f(ms - mx);
      l += w * a.part_ml[((unit0 + s) * kRows + r) * 2 + 1];
      acc += w * a.part_o[(unit0 + s) * kRows * DH + r * DH + d];
    }
    const int rr = r0 + r, t = rr / group, h = g * group + rr % group;
    a.out[((int64_t)(t0 + t) * a.hq + h) * DH + d] = __float2bfloat16_rn(l > 0.f ? acc / l : 0.f);
  }
}

template <int DH>
int launch(AttnArgs& a, int n_seqs, cudaStream_t s) {
  using Cfg = AttnCfg<DH>;
  // the shared-memory opt-in is per device
  static uint64_t attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set & (1ull << (dev & 63)))) {
    const cudaError_t e = cudaFuncSetAttribute(
        attn_tc_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
    if (e != cudaSuccess) return fail(MS_ERR_CUDA, "attn_tc: smem attribute: %s", cudaGetErrorString(e));
    attr_set |= 1ull << (dev & 63);
  }
  dim3 grid(a.row_tiles * a.n_splits, a.hkv, n_seqs);
  launch_pdl(attn_tc_kernel<DH>, grid, kThreads, Cfg::kSmem, s, a);
  MS_TRY(check_launch("attn_tc_kernel"));
  if (a.n_splits > 1) {
    launch_pdl(attn_combine_kernel<DH>, dim3(a.row_tiles, a.hkv, n_seqs), 256, 0, s, a);
    MS_TRY(check_launch("attn_combine_kernel"));
  }
  return MS_OK;
}

}  // namespace

bool attn_tc_supported(const ms_kv_cache& c, int hq) {
  return c.dtype == MS_DTYPE_BF16 && (c.d_head == 64 || c.d_head == 128) && hq % c.n_kv_heads == 0;
}

size_t attn_tc_scratch_bytes(int n_seqs, int hkv, int dh, int row_tiles, int n_splits) {
  if (n_splits <= 1) return 0;
  const size_t units = (size_t)n_seqs * hkv * row_tiles * n_splits;
  return units * kRows * dh * sizeof(float) + units * kRows * 2 * sizeof(float) + 256;
}

void attn_tc_plan(int max_q_len, int group, int max_context, int n_seqs, int hkv, int* row_tiles,
                  int* n_splits, int* split_len) {
  *row_tiles = (max_q_len * group + kRows - 1) / kRows;
  // Split the KV range only when the (sequence, kv head, row tile) units do
  // not fill one wave (148 SMs x 3 resident CTAs): a split costs a partials
  // round trip and a combine launch, which a full grid does not recover.
  // At least 256 keys per range; ranges are whole 64-key chunks.
  const int units = n_seqs * hkv * *row_tiles;
  const int wave = 148 * 3;
  int splits = units < wave ? (2 * wave + units - 1) / units : 1;
  const int by_len = (max_context + 255) / 256;
  splits = max(1, min(splits, min(by_len, 32)));
  int len = (max_context + splits - 1) / splits;
  len = ((len + kChunk - 1) / kChunk) * kChunk;
  if (len <= 0) len = kChunk;
  *n_splits = (max_context + len - 1) / len;
  if (*n_splits < 1) *n_splits = 1;
  *split_len = len;
}

int paged_attention_tc(const void* q, int q_stride, const ms_kv_cache& c, int layer,
                       const ms_batch& bt, int hq, void* out, int max_context, void* scratch,
                       size_t scratch_bytes, cudaStream_t s) {
  AttnArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_stride = q_stride;
  a.kpool = static_cast<const __nv_bfloat16*>(c.k_pool[layer]);
  a.vpool = static_cast<const __nv_bfloat16*>(c.v_pool[layer]);
  a.q_start = bt.q_start;
  a.context_lens = bt.context_lens;
  a.positions = bt.positions;
  a.tables = bt.block_tables;
  a.max_blocks = bt.max_blocks;
  a.bs = c.block_size;
  a.num_blocks = c.num_blocks;
  a.hq = hq;
  a.hkv = c.n_kv_heads;
  attn_tc_plan(bt.max_q_len, hq / c.n_kv_heads, max_context, bt.n_seqs, c.n_kv_heads, &a.row_tiles,
               &a.n_splits, &a.split_len);
  a.scale_log2 = kLog2e / sqrtf((float)c.d_head);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.err = device_error_word();
  const size_t need = attn_tc_scratch_bytes(bt.n_seqs, c.n_kv_heads, c.d_head, a.row_tiles,
                                            a.n_splits);
  if (need > scratch_bytes) {
    // not enough scratch for partials: one KV range per tile
    a.n_splits = 1;
    a.split_len = ((max_context + kChunk - 1) / kChunk) * kChunk;
    if (a.split_len <= 0) a.split_len = kChunk;
  } else if (need > 0) {
    const size_t units = (size_t)bt.n_seqs * a.hkv * a.row_tiles * a.n_splits;
    a.part_o = static_cast<float*>(scratch);
    a.part_ml = a.part_o + units * kRows * c.d_head;
  }
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15 || q_stride % 8)
    return fail(MS_ERR_INVALID, "attn_tc: q/out must be 16-byte aligned");
  if (c.d_head == 64) return launch<64>(a, bt.n_seqs, s);
  return launch<128>(a, bt.n_seqs, s);
}

}  // namespace ms
