// Paged attention for bf16 caches with TMA tile loads (sm_100a).
//
// One CTA per (64-row query tile, kv head, sequence, KV range); the GQA query
// heads of a kv head share the tile (row r = token * group + head-in-group),
// so every K/V byte of a range is read once per kv head.
//   producer warp, lane 0: for each chunk of kCh keys, looks up the chunk's
//                  blocks in the block table (staged in shared memory) and
//                  issues one 2-D TMA load per (block, kv head, 64-column
//                  half) of K and of V into a kStages-deep ring, 128-byte
//                  swizzled, completing on the stage's "full" mbarrier;
//   consumer warps: warp w owns m-tile (w % MTP) of the query rows and key
//                  slice (w / MTP) of every chunk, KW keys wide.  Per slice:
//                  S = Q K^T and O += P V with ldmatrix (swizzle-aware
//                  addresses) + mma.sync m16n8k16 bf16, online softmax in
//                  base 2; then arrive on the stage's "empty" barrier.
// The layout is picked at launch from the batch's widest row tile.  For dh 64
// (and dh 128 up to 32 rows) each warp takes a whole 64-key chunk of one
// m-tile, so the CTA is as narrow as its rows (1-4 consumer warps) and 3-6
// CTAs share an SM; wider dh-128 tiles split each chunk's keys over the warps
// that the m-tiles leave.
// When a chunk is split over several warps, their (max, sum, O) states are
// merged through shared memory at the end, with the same rescaling the
// cross-CTA split-KV combine uses.
// The pools are viewed as 2-D tensors [num_blocks * n_kv_heads * block_size
// rows][d_head columns]; a (block, kv head) tile is block_size consecutive
// rows.  No multicast; only this GPU's memory is read.  Every mbarrier wait
// is bounded and reports kErrTimeout through the device error word.
#include <cuda.h>

#include <cfloat>
#include <mutex>
#include <unordered_map>

#include "attention_tc.cuh"
#include "model_kernels.cuh"

namespace ms {
namespace {

constexpr int kRows = 64;
constexpr float kLog2e = 1.4426950408889634f;
constexpr long long kWaitCycles = 1ll << 32;
constexpr int kErrTimeout = 5;
constexpr int kErrRows = 6;  // a row tile wider than the launch's slice layout covers
constexpr int kTblCap = 64;  // block-table entries staged per refill (multiple of 16)

// One launch layout: CHK keys per ring stage, NS stages, NW consumer warps,
// each owning one 16-row m-tile and a KW-key slice of every chunk.  The Q
// tile holds the rows those m-tiles cover, so a decode layout (one m-tile)
// keeps 2 KB of Q instead of 9 KB and more CTAs fit on an SM.
template <int DH, int KW, int NW, int NS, int CHK>
struct TmaCfg {
  static constexpr int kCh = CHK;                   // keys per stage
  static constexpr int kWarps = NW;                 // consumer warps
  static constexpr int kKS = CHK / KW;              // key slices per chunk
  static constexpr int kMTP = NW / kKS;             // m-tiles the warps cover
  static constexpr int kQRows = kMTP * 16;
  static constexpr int kThreads = (kWarps + 1) * 32;
  static constexpr int kHalves = DH / 64;           // 128-byte column halves
  static constexpr int kStages = NS;
  static constexpr int kTileBytes = kCh * DH * 2;   // one operand, one chunk
  static constexpr int kStageBytes = 2 * kTileBytes;  // K + V
  static constexpr int kLdQ = DH + 8;
  static constexpr int kQBytes = kQRows * kLdQ * 2;
  static constexpr int kLdPart = DH + 8;            // merge buffer row stride (floats)
  static constexpr int kPartBytes = kWarps * 16 * (kLdPart * 4 + 8);
  static_assert(KW % 16 == 0 && CHK % KW == 0 && NW % kKS == 0 && kQRows <= kRows,
                "slice layout");
  static_assert(kKS == 1 || kPartBytes <= kStages * kStageBytes, "merge buffer must fit in the ring");
  static_assert(kTblCap % (kCh / 8) == 0, "table refill must hold whole chunks");
  static constexpr int kSmem =
      1024 + kStages * kStageBytes + kQBytes + kRows * 4 + 128 + kTblCap * 4;
};
// Default layout (wide row tiles): 8 (dh 64) or 4 (dh 128) consumer warps,
// 3 or 2 stages of 128 or 64 keys, 2 CTAs per SM.
template <int DH> struct TmaDefault {
  static constexpr int kCh = DH == 64 ? 128 : 64;
  static constexpr int kWarps = DH == 64 ? 8 : 4;
  static constexpr int kStages = DH == 64 ? 3 : 2;
};
__device__ __forceinline__ uint32_t s_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) {
      *abort_flag = 1;
      atomicCAS(err, 0, kErrTimeout);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
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
// 2^x by the SFU's ex2.approx (ftz): 2^-inf = +0; arguments here are <= 0.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
__device__ __forceinline__ void consumer_sync(int threads) {
  asm volatile("bar.sync 1, %0;" ::"r"(threads) : "memory");
}
// Named barrier 1 over the consumer warps; true when `pred` holds in any of them.
__device__ __forceinline__ bool consumer_any(int threads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(threads)
      : "memory");
  return r != 0;
}

// Address of the 16-byte chunk `c` (0 .. dh/8-1) of key row `k` (0..CH-1) in
// a swizzled operand tile: half c/8, row k of 128 bytes, chunk (c%8) ^ (k%8).
template <int CH>
__device__ __forceinline__ uint32_t tile_addr(uint32_t tile, int k, int c) {
  return tile + (uint32_t)((c >> 3) * (CH * 128) + k * 128 + (((c & 7) ^ (k & 7)) << 4));
}

struct TmaArgs {
  const __nv_bfloat16* q;
  int q_stride;
  const int32_t* q_start;
  const int32_t* context_lens;
  const int32_t* positions;
  const int32_t* tables;
  const int32_t* seq_order;  // null: sequence b is grid column b
  int max_blocks, bs, log2_bs, num_blocks, hq, hkv, row_tiles, n_splits, split_len;
  float scale_log2;
  __nv_bfloat16* out;
  float* part_o;
  float* part_ml;
  int* err;
};

template <int DH, int KW, int NWARPS, int NSTAGES, int MINB, int CHK>
__global__ void __launch_bounds__(TmaCfg<DH, KW, NWARPS, NSTAGES, CHK>::kThreads, MINB)
    attn_tma_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                    TmaArgs a) {
  pdl_enter();
  using Cfg = TmaCfg<DH, KW, NWARPS, NSTAGES, CHK>;
  constexpr int S = Cfg::kStages;
  constexpr int CH = Cfg::kCh;
  constexpr int NW = Cfg::kWarps;
  constexpr int NT = DH / 8;
  constexpr int LDQ = Cfg::kLdQ;
  constexpr int KS = CH / KW;   // key slices per chunk
  constexpr int MTP = NW / KS;  // m-tiles the consumer warps cover
  static_assert(KW % 16 == 0 && CH % KW == 0 && NW % KS == 0 && MTP * 16 <= kRows, "slice layout");
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = s_addr(smem_raw);
  unsigned char* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  const uint32_t stage0 = s_addr(smem);
  __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(smem + S * Cfg::kStageBytes);
  int* rowpos = reinterpret_cast<int*>(smem + S * Cfg::kStageBytes + Cfg::kQBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(rowpos + kRows);
  const uint32_t full0 = s_addr(bars), empty0 = full0 + 8 * S;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * S);
  int* tbl = reinterpret_cast<int*>(smem + S * Cfg::kStageBytes + Cfg::kQBytes + kRows * 4 + 128);

  const int split = blockIdx.x % a.n_splits, rt = blockIdx.x / a.n_splits;
  const int g = blockIdx.y, b = a.seq_order ? a.seq_order[blockIdx.z] : blockIdx.z;
  const int group = a.hq / a.hkv;
  // independent loads issued together: the query range, the context length
  const int t0 = a.q_start[b], qlen = a.q_start[b + 1] - t0;
  const int ctx_len = a.context_lens[b];
  const int nrows = qlen * group;
  const int r0 = rt * kRows;
  if (r0 >= nrows) return;
  const int nr = min(kRows, nrows - r0);
  if (nr > MTP * 16) {
    if (threadIdx.x == 0) atomicCAS(a.err, 0, kErrRows);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The producer's first block-table slice, read while the row positions
  // load (its start depends only on the split): no extra round trip later.
  const int32_t* table = a.tables + (int64_t)b * a.max_blocks;
  const int first_blk = (split * a.split_len) >> a.log2_bs;
  int tbl_pre[kTblCap / 32];
  if (warp == NW) {
#pragma unroll
    for (int j = 0; j < kTblCap / 32; ++j) {
      const int i = first_blk + lane + 32 * j;
      tbl_pre[j] = i < a.max_blocks ? table[i] : 0;
    }
  }

  for (int r = threadIdx.x; r < kRows; r += Cfg::kThreads)
    rowpos[r] = r < nr ? a.positions[t0 + (r0 + r) / group] : -1;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, NW);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  // Stage tiles start zeroed: key rows a chunk never loads must hold finite
  // values (their probabilities are 0, and 0 * NaN would poison O).
  for (int i = threadIdx.x; i < S * Cfg::kStageBytes / 16; i += Cfg::kThreads)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // zeros before TMA writes
  __syncthreads();

  int kmax = 0, minpos = INT_MAX;
  for (int r = 0; r < nr; ++r) {
    kmax = max(kmax, rowpos[r] + 1);
    minpos = min(minpos, rowpos[r]);
  }
  kmax = min(kmax, ctx_len);
  const int splits_here = max(1, (kmax + a.split_len - 1) / a.split_len);
  if (split >= splits_here) return;
  const int kbeg = split * a.split_len;
  const int kend = min(kmax, kbeg + a.split_len);
  const int nchunks = (kend - kbeg + CH - 1) / CH;
  // Keys below jfree are visible to every row of the tile: no mask needed.
  const int jfree = min(kend, minpos + 1);

  if (warp == NW) {
    // ---- producer: block-table slice staged in smem, one lane issues TMA ----
    const int bpc = CH >> a.log2_bs;  // blocks per chunk
    const int n_blk = (kend - kbeg + a.bs - 1) >> a.log2_bs;
    int issued = 0;
    bool stop = false;
    for (int base = 0; base < n_blk && !stop; base += kTblCap) {
      const int cnt = min(kTblCap, n_blk - base);
      __syncwarp();
#pragma unroll
      for (int j = 0; j < kTblCap / 32; ++j) {
        const int i = lane + 32 * j;
        if (i >= cnt) break;
        int blk = base == 0 ? tbl_pre[j] : table[first_blk + base + i];
        if (blk < 0 || blk >= a.num_blocks) {
          atomicCAS(a.err, 0, (int)kErrBlock);
          blk = 0;
        }
        tbl[i] = blk;
      }
      __syncwarp();
      if (lane == 0) {
        const int ch_end = min(nchunks, (base + cnt + bpc - 1) / bpc);
        for (int ch = base / bpc; ch < ch_end; ++ch) {
          const int s = ch % S;
          if (ch >= S && !mbar_wait(empty0 + 8 * s, ((ch / S) - 1) & 1, abort_flag, a.err)) {
            stop = true;
            break;
          }
          const int j0 = kbeg + ch * CH;
          const int nb = (min(kend, j0 + CH) - j0 + a.bs - 1) >> a.log2_bs;
          mbar_expect_tx(full0 + 8 * s, (uint32_t)(nb * a.bs * DH * 2 * 2));
          const uint32_t kdst = stage0 + s * Cfg::kStageBytes;
          const uint32_t vdst = kdst + Cfg::kTileBytes;
          const int t0b = ch * bpc - base;
          for (int i = 0; i < nb; ++i) {
            const int y = (tbl[t0b + i] * a.hkv + g) * a.bs;
            const uint32_t off = (uint32_t)(i * a.bs * 128);
#pragma unroll
            for (int h = 0; h < Cfg::kHalves; ++h) {
              tma_load_2d(kdst + h * CH * 128 + off, &kmap, full0 + 8 * s, h * 64, y);
              tma_load_2d(vdst + h * CH * 128 + off, &vmap, full0 + 8 * s, h * 64, y);
            }
          }
          ++issued;
        }
      }
      stop = __shfl_sync(0xffffffffu, stop ? 1 : 0, 0) != 0;
    }
    if (lane == 0 && *abort_flag) {
      const long long t0c = clock64();
      for (int ch = issued > S ? issued - S : 0; ch < issued; ++ch)
        while (!mbar_try_wait(full0 + 8 * (ch % S), (ch / S) & 1) && clock64() - t0c < kWaitCycles) {
        }
    }
    return;
  }

  // ---- consumers ----
  const int mi = warp % MTP, si = warp / MTP;
  const int wr = mi * 16, kof = si * KW;
  const int ra = wr + (lane >> 2), rb = ra + 8;
  const int pos_a = rowpos[ra], pos_b = rowpos[rb];
  const bool live = wr < nr;
  // The Q rows of this warp's m-tile (zero past nr), loaded while the
  // producer's first TMA loads are already in flight: only this warp reads
  // them (warps that share an m-tile write the same bytes).
  if (live) {
    for (int idx = lane; idx < 16 * (DH / 8); idx += 32) {
      const int r = wr + idx / (DH / 8), c = (idx % (DH / 8)) * 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r < nr) {
        const int rr = r0 + r, t = rr / group, h = g * group + rr % group;
        v = *reinterpret_cast<const uint4*>(a.q + (int64_t)(t0 + t) * a.q_stride + h * DH + c);
      }
      *reinterpret_cast<uint4*>(Qs + r * LDQ + c) = v;
    }
    __syncwarp();
  }
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  float o[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  // Q fragments stay in registers for the narrow slices; the 64-key slice
  // (more live accumulators) re-reads them from shared memory per chunk.
  constexpr bool kQRegs = KW <= 32;
  const uint32_t q_lane = s_addr(Qs + (wr + (lane & 15)) * LDQ + (lane >> 4) * 8);
  uint32_t qf[kQRegs ? DH / 16 : 1][4];
  if constexpr (kQRegs) {
#pragma unroll
    for (int k = 0; k < DH / 16; ++k)
      ldm_x4(q_lane + k * 32, qf[k][0], qf[k][1], qf[k][2], qf[k][3]);
  }

  bool ok = true;
  for (int ch = 0; ch < nchunks && ok; ++ch) {
    const int s = ch % S;
    ok = mbar_wait(full0 + 8 * s, (ch / S) & 1, abort_flag, a.err);
    if (!ok) break;
    const int jlo = kbeg + ch * CH + kof;  // first key of this warp's slice
    if (live && jlo < kend) {
      const uint32_t Kt = stage0 + s * Cfg::kStageBytes;
      const uint32_t Vt = Kt + Cfg::kTileBytes;
      float sc[KW / 8][4];
#pragma unroll
      for (int i = 0; i < KW / 8; ++i) sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = 0.f;
#pragma unroll
      for (int k = 0; k < DH / 16; ++k) {
        uint32_t a0, a1, a2, a3;
        if constexpr (kQRegs) {
          a0 = qf[k][0];
          a1 = qf[k][1];
          a2 = qf[k][2];
          a3 = qf[k][3];
        } else {
          ldm_x4(q_lane + k * 32, a0, a1, a2, a3);
        }
        // The k-step's K fragments are all loaded before its MMAs: the
        // loads and MMAs stay in program order, so interleaving them would
        // expose each ldmatrix latency (verify 75.6 -> 73.0 us).
        uint32_t kb[KW / 16][4];
#pragma unroll
        for (int p = 0; p < KW / 16; ++p) {
          const int key = kof + p * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int c = 2 * k + ((lane >> 3) & 1);
          ldm_x4(tile_addr<CH>(Kt, key, c), kb[p][0], kb[p][1], kb[p][2], kb[p][3]);
        }
#pragma unroll
        for (int p = 0; p < KW / 16; ++p) {
          mma_bf16(sc[2 * p], a0, a1, a2, a3, kb[p][0], kb[p][1]);
          mma_bf16(sc[2 * p + 1], a0, a1, a2, a3, kb[p][2], kb[p][3]);
        }
      }
      // Raw scores: the scale is positive, so it commutes with the max and
      // folds into the exponent's FMA; masked scores are -inf.
      float mx_a = -INFINITY, mx_b = -INFINITY;
      if (jlo + KW <= jfree) {
#pragma unroll
        for (int nt = 0; nt < KW / 8; ++nt) {
          mx_a = fmaxf(mx_a, fmaxf(sc[nt][0], sc[nt][1]));
          mx_b = fmaxf(mx_b, fmaxf(sc[nt][2], sc[nt][3]));
        }
      } else {
        const int jbase = jlo + 2 * (lane & 3);
#pragma unroll
        for (int nt = 0; nt < KW / 8; ++nt) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int j = jbase + nt * 8 + e;
            const bool va = j < kend && j <= pos_a, vb = j < kend && j <= pos_b;
            sc[nt][e] = va ? sc[nt][e] : -INFINITY;
            sc[nt][2 + e] = vb ? sc[nt][2 + e] : -INFINITY;
            mx_a = fmaxf(mx_a, sc[nt][e]);
            mx_b = fmaxf(mx_b, sc[nt][2 + e]);
          }
        }
      }
#pragma unroll
      for (int o_ = 1; o_ <= 2; o_ <<= 1) {
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, o_));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, o_));
      }
      const float mn_a = fmaxf(m_a, mx_a * a.scale_log2), mn_b = fmaxf(m_b, mx_b * a.scale_log2);
      const bool grow_a = mn_a > m_a, grow_b = mn_b > m_b;
      const float al_a = grow_a ? (m_a == -INFINITY ? 0.f : fast_exp2(m_a - mn_a)) : 1.f;
      const float al_b = grow_b ? (m_b == -INFINITY ? 0.f : fast_exp2(m_b - mn_b)) : 1.f;
      const float sub_a = mn_a == -INFINITY ? 0.f : mn_a;
      const float sub_b = mn_b == -INFINITY ? 0.f : mn_b;
      float ps_a0 = 0.f, ps_a1 = 0.f, ps_b0 = 0.f, ps_b1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < KW / 8; ++nt) {
        sc[nt][0] = fast_exp2(fmaf(sc[nt][0], a.scale_log2, -sub_a));
        sc[nt][1] = fast_exp2(fmaf(sc[nt][1], a.scale_log2, -sub_a));
        sc[nt][2] = fast_exp2(fmaf(sc[nt][2], a.scale_log2, -sub_b));
        sc[nt][3] = fast_exp2(fmaf(sc[nt][3], a.scale_log2, -sub_b));
        ps_a0 += sc[nt][0];
        ps_a1 += sc[nt][1];
        ps_b0 += sc[nt][2];
        ps_b1 += sc[nt][3];
      }
      l_a = l_a * al_a + (ps_a0 + ps_a1);
      l_b = l_b * al_b + (ps_b0 + ps_b1);
      m_a = mn_a;
      m_b = mn_b;
      // O is rescaled only when a row's maximum grew (exact: alpha is 1 else)
      if (__any_sync(0xffffffffu, grow_a || grow_b)) {
#pragma unroll
        for (int i = 0; i < NT; ++i) {
          o[i][0] *= al_a;
          o[i][1] *= al_a;
          o[i][2] *= al_b;
          o[i][3] *= al_b;
        }
      }
#pragma unroll
      for (int kt = 0; kt < KW / 16; ++kt) {
        const uint32_t p0 = pack2(sc[2 * kt][0], sc[2 * kt][1]);
        const uint32_t p1 = pack2(sc[2 * kt][2], sc[2 * kt][3]);
        const uint32_t p2 = pack2(sc[2 * kt + 1][0], sc[2 * kt + 1][1]);
        const uint32_t p3 = pack2(sc[2 * kt + 1][2], sc[2 * kt + 1][3]);
        const int key = kof + kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        uint32_t vb[NT / 2][4];  // V fragments likewise before the MMAs
#pragma unroll
        for (int p = 0; p < NT / 2; ++p)
          ldm_x4_t(tile_addr<CH>(Vt, key, 2 * p + (lane >> 4)), vb[p][0], vb[p][1], vb[p][2],
                   vb[p][3]);
#pragma unroll
        for (int p = 0; p < NT / 2; ++p) {
          mma_bf16(o[2 * p], p0, p1, p2, p3, vb[p][0], vb[p][1]);
          mma_bf16(o[2 * p + 1], p0, p1, p2, p3, vb[p][2], vb[p][3]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8 * s);
  }
#pragma unroll
  for (int o_ = 1; o_ <= 2; o_ <<= 1) {
    l_a += __shfl_xor_sync(0xffffffffu, l_a, o_);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, o_);
  }
  const int col = 2 * (lane & 3);

  if constexpr (KS == 1) {
    if (!live || !ok) return;
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
  } else {
    // ---- merge the KS key slices of each row through the (drained) ring ----
    // Every slice has finished reading the ring; leave together if any wait
    // gave up (bar.red makes the decision uniform across the consumers).
    if (consumer_any(NW * 32, !ok || *abort_flag)) return;
    constexpr int LP = Cfg::kLdPart;
    float* part = reinterpret_cast<float*>(smem);
    float2* pml = reinterpret_cast<float2*>(part + NW * 16 * LP);
    if (live) {
      // partial row p = si * (MTP * 16) + r, for tile row r = wr + (0..15)
      const int pa = si * (MTP * 16) + ra, pb = pa + 8;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        *reinterpret_cast<float2*>(part + pa * LP + nt * 8 + col) = make_float2(o[nt][0], o[nt][1]);
        *reinterpret_cast<float2*>(part + pb * LP + nt * 8 + col) = make_float2(o[nt][2], o[nt][3]);
      }
      if ((lane & 3) == 0) {
        pml[pa] = make_float2(m_a, l_a);
        pml[pb] = make_float2(m_b, l_b);
      }
    }
    consumer_sync(NW * 32);
    const int64_t unit = (((int64_t)b * a.hkv + g) * a.row_tiles + rt) * a.n_splits + split;
    for (int idx = threadIdx.x; idx < nr * DH; idx += NW * 32) {
      const int r = idx / DH, d = idx % DH;
      float mx = -INFINITY;
#pragma unroll
      for (int k = 0; k < KS; ++k) mx = fmaxf(mx, pml[k * (MTP * 16) + r].x);
      float l = 0.f, acc = 0.f;
#pragma unroll
      for (int k = 0; k < KS; ++k) {
        const float2 ml = pml[k * (MTP * 16) + r];
        const float w = ml.x == -INFINITY ? 0.f : exp2f(ml.x - mx);
        l += w * ml.y;
        acc += w * part[(k * (MTP * 16) + r) * LP + d];
      }
      if (splits_here == 1) {
        const int rr = r0 + r, t = rr / group, h = g * group + rr % group;
        a.out[((int64_t)(t0 + t) * a.hq + h) * DH + d] = __float2bfloat16_rn(l > 0.f ? acc / l : 0.f);
      } else {
        a.part_o[unit * kRows * DH + r * DH + d] = acc;
        if (d == 0) {
          a.part_ml[unit * kRows * 2 + r * 2] = mx;
          a.part_ml[unit * kRows * 2 + r * 2 + 1] = l;
        }
      }
    }
  }
}

// ---- host ----------------------------------------------------------------------
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                              const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                              const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

struct PoolKey {
  const void* ptr;
  int64_t rows;
  int dh, bs, dev;
  bool operator==(const PoolKey& o) const {
    return ptr == o.ptr && rows == o.rows && dh == o.dh && bs == o.bs && dev == o.dev;
  }
};
struct PoolKeyHash {
  size_t operator()(const PoolKey& k) const {
    return std::hash<const void*>()(k.ptr) ^ ((size_t)k.rows << 7) ^ ((size_t)k.dh << 40) ^
           ((size_t)k.bs << 50) ^ ((size_t)k.dev << 58);
  }
};

// The pool as [rows][dh] bf16 with (64 x block_size) boxes, 128-byte swizzle.
int pool_map(const void* pool, int64_t rows, int dh, int bs, CUtensorMap* out) {
  static std::mutex mu;
  static std::unordered_map<PoolKey, CUtensorMap, PoolKeyHash> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const PoolKey key{pool, rows, dh, bs, dev};
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return MS_OK;
  }
  EncodeFn enc = encode_fn();
  if (!enc) return fail(MS_ERR_CUDA, "attn_tma: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)dh, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)dh * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)bs};
  const cuuint32_t estr[2] = {1, 1};
  CUtensorMap map;
  const CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(pool), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MS_ERR_CUDA, "attn_tma: tensor map encode failed (%d)", (int)r);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, map);
  *out = map;
  return MS_OK;
}

__global__ void attn_tma_combine_kernel(TmaArgs a, int dh) {
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
  for (int idx = threadIdx.x; idx < nr * dh; idx += blockDim.x) {
    const int r = idx / dh, d = idx % dh;
    float mx = -INFINITY;
    for (int s = 0; s < splits; ++s) mx = fmaxf(mx, a.part_ml[((unit0 + s) * kRows + r) * 2]);
    float l = 0.f, acc = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float ms = a.part_ml[((unit0 + s) * kRows + r) * 2];
      const float w = ms == -INFINITY ? 0.f : exp2f(ms - mx);
      l += w * a.part_ml[((unit0 + s) * kRows + r) * 2 + 1];
      acc += w * a.part_o[(unit0 + s) * kRows * dh + r * dh + d];
    }
    const int rr = r0 + r, t = rr / group, h = g * group + rr % group;
    a.out[((int64_t)(t0 + t) * a.hq + h) * dh + d] = __float2bfloat16_rn(l > 0.f ? acc / l : 0.f);
  }
}

template <int DH, int KW, int NW = TmaDefault<DH>::kWarps, int NS = TmaDefault<DH>::kStages,
          int MINB = 2, int CHK = TmaDefault<DH>::kCh>
int launch_tma(TmaArgs& a, const CUtensorMap& km, const CUtensorMap& vm, int n_seqs,
               cudaStream_t s) {
  using Cfg = TmaCfg<DH, KW, NW, NS, CHK>;
  static_assert(MINB * (Cfg::kSmem + 1024) <= 228 * 1024, "CTAs per SM exceed shared memory");
  // The shared-memory opt-in is per device; remember it per device.
  static uint64_t attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(attr_set & bit)) {
    const cudaError_t e =
        cudaFuncSetAttribute(attn_tma_kernel<DH, KW, NW, NS, MINB, CHK>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
    if (e != cudaSuccess) return fail(MS_ERR_CUDA, "attn_tma: smem attribute: %s", cudaGetErrorString(e));
    attr_set |= bit;
  }
  dim3 grid(a.row_tiles * a.n_splits, a.hkv, n_seqs);
  launch_pdl(attn_tma_kernel<DH, KW, NW, NS, MINB, CHK>, grid, Cfg::kThreads, Cfg::kSmem, s, km, vm, a);
  MS_TRY(check_launch("attn_tma_kernel"));
  if (a.n_splits > 1) {
    launch_pdl(attn_tma_combine_kernel, dim3(a.row_tiles, a.hkv, n_seqs), 256, 0, s, a, DH);
    MS_TRY(check_launch("attn_tma_combine_kernel"));
  }
  return MS_OK;
}

// Layout by the batch's widest row tile.  dh 64: one warp per 16-row m-tile,
// each warp covering a whole 64-key chunk (no cross-warp merge), 2-3 stages,
// and as many CTAs per SM as shared memory and registers allow -- many
// independent TMA streams per SM keep more K/V bytes in flight than wide
// CTAs do (one layer of 256 sequences x 4 kv heads, contexts 512-2048: decode
// 8 rows 60 us, 5-token verify 40 rows 78 us).  dh 128 up to 32 rows: the
// same one-warp-per-m-tile layout at 3 CTAs per SM.  Wider dh-128 tiles: the
// default layout, the fewest m-tiles that cover the rows and the other warps
// splitting each chunk's keys.
template <int DH>
int launch_by_rows(TmaArgs& a, const CUtensorMap& km, const CUtensorMap& vm, int n_seqs,
                   int max_rows, cudaStream_t s) {
  const int mt = (min(max_rows, kRows) + 15) / 16;
  if constexpr (DH == 64) {
    switch (mt) {
      case 0:
      case 1: return launch_tma<DH, 64, 1, 2, 6, 64>(a, km, vm, n_seqs, s);
      case 2: return launch_tma<DH, 64, 2, 3, 4, 64>(a, km, vm, n_seqs, s);
      case 3: return launch_tma<DH, 64, 3, 2, 4, 64>(a, km, vm, n_seqs, s);
      default: return launch_tma<DH, 64, 4, 2, 3, 64>(a, km, vm, n_seqs, s);
    }
  }
  if constexpr (DH == 128) {
    // 8B-class heads (256 sequences x 8 kv heads, contexts 1024-3072): decode
    // 4 rows 320 us, 6-token verify 24 rows 340 us, both at the copy bandwidth.
    if (mt <= 1) return launch_tma<DH, 64, 1, 2, 3, 64>(a, km, vm, n_seqs, s);
    if (mt == 2) return launch_tma<DH, 64, 2, 2, 3, 64>(a, km, vm, n_seqs, s);
  }
  constexpr int kCh = TmaDefault<DH>::kCh, kW = TmaDefault<DH>::kWarps;
  if (mt <= 1) return launch_tma<DH, kCh / kW>(a, km, vm, n_seqs, s);
  if (mt == 2) return launch_tma<DH, 2 * kCh / kW>(a, km, vm, n_seqs, s);
  return launch_tma<DH, 4 * kCh / kW>(a, km, vm, n_seqs, s);
}

}  // namespace

bool attn_tma_supported(const ms_kv_cache& c, int hq) {
  const int bs = c.block_size;
  const bool pow2 = bs >= 8 && bs <= 64 && (bs & (bs - 1)) == 0;
  const int64_t rows = (int64_t)c.num_blocks * c.n_kv_heads * bs;
  return c.dtype == MS_DTYPE_BF16 && (c.d_head == 64 || c.d_head == 128) && pow2 &&
         hq % c.n_kv_heads == 0 && rows < (1ll << 31);
}

int paged_attention_tma(const void* q, int q_stride, const ms_kv_cache& c, int layer,
                        const ms_batch& bt, int hq, void* out, int max_context, void* scratch,
                        size_t scratch_bytes, cudaStream_t s, const int32_t* seq_order) {
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15 || q_stride % 8)
    return fail(MS_ERR_INVALID, "attn_tma: q/out must be 16-byte aligned");
  TmaArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_stride = q_stride;
  a.q_start = bt.q_start;
  a.context_lens = bt.context_lens;
  a.positions = bt.positions;
  a.tables = bt.block_tables;
  a.seq_order = seq_order;
  a.max_blocks = bt.max_blocks;
  a.bs = c.block_size;
  a.log2_bs = __builtin_ctz((unsigned)c.block_size);
  a.num_blocks = c.num_blocks;
  a.hq = hq;
  a.hkv = c.n_kv_heads;
  const int group = hq / c.n_kv_heads;
  attn_tc_plan(bt.max_q_len, group, max_context, bt.n_seqs, c.n_kv_heads, &a.row_tiles,
               &a.n_splits, &a.split_len);
  a.scale_log2 = kLog2e / sqrtf((float)c.d_head);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.err = device_error_word();
  const size_t need =
      attn_tc_scratch_bytes(bt.n_seqs, c.n_kv_heads, c.d_head, a.row_tiles, a.n_splits);
  if (need > scratch_bytes) {
    a.n_splits = 1;
    a.split_len = ((max_context + 63) / 64) * 64;
    if (a.split_len <= 0) a.split_len = 64;
  } else if (need > 0) {
    const size_t units = (size_t)bt.n_seqs * a.hkv * a.row_tiles * a.n_splits;
    a.part_o = static_cast<float*>(scratch);
    a.part_ml = a.part_o + units * kRows * c.d_head;
  }
  const int64_t rows = (int64_t)c.num_blocks * c.n_kv_heads * c.block_size;
  CUtensorMap km, vm;
  MS_TRY(pool_map(c.k_pool[layer], rows, c.d_head, c.block_size, &km));
  MS_TRY(pool_map(c.v_pool[layer], rows, c.d_head, c.block_size, &vm));
  const int max_rows = bt.max_q_len * group;
  if (c.d_head == 64) return launch_by_rows<64>(a, km, vm, bt.n_seqs, max_rows, s);
  return launch_by_rows<128>(a, km, vm, bt.n_seqs, max_rows, s);
}

}  // namespace ms
