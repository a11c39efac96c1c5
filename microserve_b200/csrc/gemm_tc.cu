// tcgen05 tensor-core GEMM for bf16 (sm_100a): C = A[M,K] * B[N,K]^T with
// float32 accumulation in tensor memory.  Persistent and warp-specialised.
//
// Grid: one CTA per SM (at most), 320 threads:
//   warp 0 lane 0  TMA producer: K-major 128B-swizzled A (128 x 64) and B
//                  (BN x 64, BN 64, 128 or 256) tiles into a 4-8 deep
//                  shared-memory ring;
//   warp 1         allocates 2 x BN TMEM columns (a double-buffered
//                  accumulator); lane 0 issues tcgen05.mma.cta_group::1
//                  .kind::f16 (M=128, N=BN, K=16), commits each stage back to
//                  the producer and each finished accumulator to the epilogue;
//   warps 2-9      epilogue: tcgen05.ld 32x32b (warp w reads TMEM lanes
//                  32*(w%4)..+31 = tile rows; warps w and w+4 split the
//                  columns), fused store / SwiGLU / residual / RoPE with
//                  the k, v cache write, through a shared-memory exchange
//                  that makes every global access whole 128-byte row
//                  segments, while the MMA warp fills the other accumulator.
// Work: output tiles are dealt round-robin to the CTAs; for the in-place
// residual GEMM (C += A B^T, R == C) the (tile, k-step) space is instead cut
// into equal contiguous ranges (stream-K) when the tiles are fewer than the
// SMs or A + B fit in L2, or whole tiles go first and only the tiles after
// the last full wave are cut (hybrid).  A piece that is a whole tile writes
// R + acc; a partial one is added into C with red.global.add, so small grids
// (o_proj/down at 1280 tokens: 80 tiles) keep every SM busy.  Partial sums
// then land in C in a hardware-chosen order, so those outputs can differ run
// to run by float rounding.
// A CTA's setup (barriers, TMEM) and, when B is constant (the forward's
// weights), its first stages' B loads run before the wait for the previous
// launch, so a CTA placed while that launch's last CTAs still run starts
// with its weights in flight.
// Loads are plain TMA tile loads of this GPU's memory (no multicast).  Every
// mbarrier wait is bounded (~2 s of SM clock); on expiry the CTA records
// kErrTimeout in the device error word, drains its own copies, frees its
// TMEM and returns.
#include <cuda.h>

#include <mutex>
#include <unordered_map>

#include "gemm.cuh"

namespace ms {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle atom row
constexpr int kEpiWarps = 8;  // warps 2..9: two per TMEM lane quarter
constexpr int kThreads = 32 * (2 + kEpiWarps);
constexpr int kStageRowBytes = 128;  // epilogue exchange: 32 rows x 128 B per warp
constexpr int kEpiBufBytes = 32 * kStageRowBytes;
constexpr int kEpiSmem = kEpiWarps * kEpiBufBytes;
constexpr int kNumSMs = 148;
constexpr long long kWaitCycles = 1ll << 32;  // ~2.2 s at 1.965 GHz
constexpr int kErrTimeout = 5;

template <int BN> struct TileCfg {
  static constexpr int kStages = BN == 64 ? 8 : (BN == 128 ? 6 : 4);
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kSmem =
      kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/ + kEpiSmem;
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
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
// Bounded wait: false on timeout or when another role has aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int* err) {
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
// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), sm100 descriptor version 1.
__device__ __forceinline__ uint64_t sdesc(uint32_t addr) {
  uint64_t d = (uint64_t)((addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;            // LBO (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;  // SBO
  d |= (uint64_t)1 << 46;            // version
  d |= (uint64_t)2 << 61;            // SWIZZLE_128B
  return d;
}
// Instruction descriptor, kind::f16: D f32, A/B bf16, both K-major, M=128.
template <int BN> __device__ __forceinline__ uint32_t idesc() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
         ((uint32_t)(BM >> 4) << 24);
}
__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t id,
                                     uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(id), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}
// tcgen05.ld of 32 (or 16) columns without the wait: the registers hold the
// values only after tmem_wait_ld(), so several loads can share one wait.
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  tmem_ld32_nowait(taddr, r);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// Two 32-column loads, one wait.
__device__ __forceinline__ void tmem_ld32x2(uint32_t ta, float (&va)[32], uint32_t tb,
                                            float (&vb)[32]) {
  uint32_t ra[32], rb[32];
  tmem_ld32_nowait(ta, ra);
  tmem_ld32_nowait(tb, rb);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    va[i] = __uint_as_float(ra[i]);
    vb[i] = __uint_as_float(rb[i]);
  }
}
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// Two 16-column loads, one wait.
__device__ __forceinline__ void tmem_ld16x2(uint32_t ta, float (&va)[16], uint32_t tb,
                                            float (&vb)[16]) {
  uint32_t ra[16], rb[16];
  tmem_ld16_nowait(ta, ra);
  tmem_ld16_nowait(tb, rb);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    va[i] = __uint_as_float(ra[i]);
    vb[i] = __uint_as_float(rb[i]);
  }
}
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ void red_add4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

// ---- epilogue stores through a per-warp shared-memory exchange --------------
// tcgen05.ld 32x32b gives each thread one accumulator row, so stores made
// straight from registers touch 32 rows (32 cache lines) per warp
// instruction and the epilogue runs at the load/store unit's line rate (a
// 128 x 256 f32 tile took ~5 us).  Instead each epilogue warp owns a 4 KB
// buffer of 32 rows x 128 bytes: the thread holding row r writes its
// 128-byte row segment, 16-byte chunk j at position j ^ (r & 7) (the eight
// lanes of each 128-bit phase hit distinct banks, on both sides); read back
// in 8 steps, step i gives lane l chunk (l & 7) of row 4 i + (l >> 3), so
// every warp-wide global access covers four whole 128-byte row segments.
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t x, uint32_t y, uint32_t z,
                                             uint32_t w) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(x), "r"(y), "r"(z),
               "r"(w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void stage_row(uint32_t buf, int lane, const uint32_t (&w)[32]) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
    st_shared_v4(buf + lane * kStageRowBytes + ((j ^ (lane & 7)) << 4), w[4 * j], w[4 * j + 1],
                 w[4 * j + 2], w[4 * j + 3]);
}
__device__ __forceinline__ uint4 staged_chunk(uint32_t buf, int r, int j) {
  return ld_shared_v4(buf + r * kStageRowBytes + ((j ^ (r & 7)) << 4));
}
// SwiGLU of 32 accumulator columns laid out [16g, 16g+8) gate, [16g+8,
// 16g+16) up (g = 0, 1): 16 bf16 outputs in 8 words.  silu(x) = x / (1 +
// e^-x) with the fast exponential and division intrinsics (the result is
// rounded to bf16).
__device__ __forceinline__ void swiglu16(const float (&v)[32], uint32_t* w) {
#pragma unroll
  for (int g = 0; g < 2; ++g) {
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      const float g0 = v[16 * g + j], g1 = v[16 * g + j + 1];
      const float u0 = v[16 * g + 8 + j], u1 = v[16 * g + 8 + j + 1];
      const float s0 = __fdividef(g0, 1.f + __expf(-g0)) * u0;
      const float s1 = __fdividef(g1, 1.f + __expf(-g1)) * u1;
      w[4 * g + j / 2] = pack_bf16(s0, s1);
    }
  }
}

// One warp's share of a finished BN-column accumulator: rows row0 .. row0+31
// (TMEM lanes at `base`), the 128-byte row segments u = half, half + 2, ...
// of the tile.  A segment is 32 input columns for f32 outputs, 64 for bf16
// and 128 for SwiGLU (64 bf16 outputs).  kEpiResidual with `reduce` adds
// into C with vector reductions (C already holds the residual); without it
// C = R + acc.
template <int BN, int EPI, typename TC>
__device__ __forceinline__ void epilogue_tile(uint32_t base, uint32_t buf, int lane, int half,
                                              int row0, int M, int n0, int64_t ldc, TC* C,
                                              const float* R, bool reduce) {
  constexpr int U = EPI == kEpiSwiGLU ? 128 : (sizeof(TC) == 2 ? 64 : 32);
  static_assert(BN % U == 0, "tile width");
#pragma unroll 1
  for (int u = half; u < BN / U; u += 2) {
    uint32_t w[32];
    if constexpr (EPI == kEpiSwiGLU) {
#pragma unroll
      for (int h = 0; h < 4; h += 2) {  // two loads per wait
        float v0[32], v1[32];
        tmem_ld32x2(base + u * U + 32 * h, v0, base + u * U + 32 * (h + 1), v1);
        swiglu16(v0, w + 8 * h);
        swiglu16(v1, w + 8 * (h + 1));
      }
    } else if constexpr (sizeof(TC) == 2) {
      float v0[32], v1[32];
      tmem_ld32x2(base + u * U, v0, base + u * U + 32, v1);
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        w[k] = pack_bf16(v0[2 * k], v0[2 * k + 1]);
        w[16 + k] = pack_bf16(v1[2 * k], v1[2 * k + 1]);
      }
    } else {
      float v[32];
      tmem_ld32(base + u * U, v);
#pragma unroll
      for (int k = 0; k < 32; ++k) w[k] = __float_as_uint(v[k]);
    }
    const int j = lane & 7;
    // the residual rows this lane adds, all loads issued before the exchange
    float4 res[EPI == kEpiResidual ? 8 : 1];
    if constexpr (EPI == kEpiResidual) {
      if (!reduce) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int m = row0 + 4 * i + (lane >> 3);
          res[i] = m < M ? *reinterpret_cast<const float4*>(R + (int64_t)m * ldc + n0 + u * U +
                                                            4 * j)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
    stage_row(buf, lane, w);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = 4 * i + (lane >> 3);
      const uint4 x = staged_chunk(buf, r, j);
      const int m = row0 + r;
      if (m >= M) continue;
      if constexpr (EPI == kEpiSwiGLU) {
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(C) + (int64_t)m * ldc +
                             (n0 + u * U) / 2 + 8 * j;
        *reinterpret_cast<uint4*>(out) = x;
      } else if constexpr (EPI == kEpiResidual) {
        const int64_t off = (int64_t)m * ldc + n0 + u * U + 4 * j;
        float* out = reinterpret_cast<float*>(C) + off;
        const float4 a = make_float4(__uint_as_float(x.x), __uint_as_float(x.y),
                                     __uint_as_float(x.z), __uint_as_float(x.w));
        if (reduce) {
          red_add4(out, a.x, a.y, a.z, a.w);
        } else {
          const float4 r4 = res[i];
          *reinterpret_cast<float4*>(out) =
              make_float4(r4.x + a.x, r4.y + a.y, r4.z + a.z, r4.w + a.w);
        }
      } else if constexpr (sizeof(TC) == 4) {
        *reinterpret_cast<uint4*>(reinterpret_cast<float*>(C) + (int64_t)m * ldc + n0 + u * U +
                                  4 * j) = x;
      } else {
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(C) + (int64_t)m * ldc + n0 +
                                  u * U + 8 * j) = x;
      }
    }
    __syncwarp();
  }
}

// kEpiRopeKV: rows row0 .. row0+31 of a BN-column tile of the qkv
// projection.  Every head lies inside one tile (dh divides BN and the tile
// start); the thread holding row m rotates the two halves of a head
// (columns j and j + dh/2) together.  Values are rounded to bf16 first and
// the rotation is the same arithmetic as rope_kv_write's, so q and the cache
// get the bits the separate kernels would write.  q goes to its row of the
// qkv buffer, k and v to the cache at the row's slot (pool layout
// (num_blocks, kv heads, block_size, dh)).  The two epilogue warps of a TMEM
// lane quarter take alternate heads (`half_warps` 0 or 1).  Each head's
// 32-column slice pair (128 bytes of bf16 per row) goes through the warp's
// exchange buffer, so the stores cover whole row segments.
// What the epilogue of one row needs before its accumulator is ready: the
// row's position and cache slot, and (d_head 64) its 32 cos/sin pairs, read
// while the MMAs still run.  Loading the cos/sin per 16 columns after each
// TMEM load made every step wait a full L2 round trip (a 1280 x 2560 verify
// qkv epilogue took 7.7 us).
struct RopeRow {
  int pos, slot;
  float cs[32], sn[32];
};
__device__ __forceinline__ void rope_row_load(const RopeKv& rk, int m, int M, int* err,
                                              RopeRow& r) {
  r.pos = 0;
  r.slot = -1;
  if (m < M) {
    r.pos = rk.positions[m];
    if (r.pos < 0 || r.pos >= rk.max_pos) {
      raise_device_error(err, kErrPosition);
      r.pos = 0;
    }
    r.slot = rk.slots[m];
  }
  if (rk.dh == 64) {
    const float4* c4 = reinterpret_cast<const float4*>(rk.cos_t + (int64_t)r.pos * 32);
    const float4* s4 = reinterpret_cast<const float4*>(rk.sin_t + (int64_t)r.pos * 32);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 c = c4[i], sv = s4[i];
      r.cs[4 * i] = c.x;
      r.cs[4 * i + 1] = c.y;
      r.cs[4 * i + 2] = c.z;
      r.cs[4 * i + 3] = c.w;
      r.sn[4 * i] = sv.x;
      r.sn[4 * i + 1] = sv.y;
      r.sn[4 * i + 2] = sv.z;
      r.sn[4 * i + 3] = sv.w;
    }
  }
}

// Writes a head's staged 32-row slice (exchange chunks 0-3: columns j ..
// j + 31 of the head's first half, 4-7: the same of its second half) to q's
// rows of the qkv buffer or to the cache at each row's slot; every lane
// stores whole 16-byte chunks, four rows per warp instruction.
// `crow`: this lane's row in the cache pool for kv head 0, block * hkv * bs +
// offset in block (-1: no valid slot).  q heads need no slot, so their
// rows skip the shuffle (the branch is uniform over the warp).
__device__ __forceinline__ void rope_store_rows(uint32_t buf, int lane, int row0, int M, int n0,
                                                int hc, int head, int j, int crow,
                                                const RopeKv& rk, __nv_bfloat16* qkv,
                                                int64_t ldc) {
  const int dh = rk.dh, half = dh >> 1;
  const int jj = lane & 7;
  const int col = jj < 4 ? j + 8 * jj : half + j + 8 * (jj - 4);
  if (head < rk.hq) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = 4 * i + (lane >> 3);
      const uint4 x = staged_chunk(buf, r, jj);
      const int mr = row0 + r;
      if (mr < M) *reinterpret_cast<uint4*>(qkv + (int64_t)mr * ldc + n0 + hc + col) = x;
    }
    return;
  }
  const bool is_k = head < rk.hq + rk.hkv;
  const int kh = head - rk.hq - (is_k ? 0 : rk.hkv);
  __nv_bfloat16* pool = (is_k ? rk.kpool : rk.vpool) + (int64_t)kh * rk.bs * dh + col;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = 4 * i + (lane >> 3);
    const uint4 x = staged_chunk(buf, r, jj);
    const int crow_r = __shfl_sync(0xffffffffu, crow, r);
    if (row0 + r >= M || crow_r < 0) continue;
    *reinterpret_cast<uint4*>(pool + (int64_t)crow_r * dh) = x;
  }
}

template <int BN>
__device__ __forceinline__ void rope_kv_rows(uint32_t base, uint32_t buf, int lane, int row0,
                                             int M, int n0, int half_warps, const RopeKv& rk,
                                             __nv_bfloat16* qkv, int64_t ldc, int* err,
                                             const RopeRow& rr) {
  const int dh = rk.dh, half = dh >> 1;
  const int m = row0 + lane;
  const bool live = m < M;
  const int pos = rr.pos, slot = rr.slot;
  const int blk = slot >= 0 ? slot / rk.bs : 0;
  const bool slot_ok = slot >= 0 && blk < rk.num_blocks;
  // the row's place in the pool (num_blocks, hkv, bs, dh) for kv head 0
  const int crow = slot_ok ? blk * rk.hkv * rk.bs + (slot - blk * rk.bs) : -1;
  // d_head 128: cos/sin of the row's position read as float4 per head
  const float* cos_row = rk.cos_t + (int64_t)pos * half;
  const float* sin_row = rk.sin_t + (int64_t)pos * half;
#pragma unroll 1
  for (int j = 0; j < half; j += 32) {
#pragma unroll 1
    for (int hc = half_warps * dh; hc < BN; hc += 2 * dh) {
      const int head = (n0 + hc) / dh;
      const bool rotate = head < rk.hq + rk.hkv;
#pragma unroll
      for (int sub = 0; sub < 2; ++sub) {  // 16 columns of each half at a time
        // words 0-7: columns j + 16 sub .. of the first half, 8-15: of the
        // second; they go to the row's exchange chunks 2 sub, 2 sub + 1 and
        // 4 + 2 sub, 5 + 2 sub
        uint32_t w[16];
        float a[16], b[16];
        tmem_ld16x2(base + hc + j + 16 * sub, a, base + hc + half + j + 16 * sub, b);
        if (rotate) {
#pragma unroll
          for (int i4 = 0; i4 < 4; ++i4) {
            const int c = j + 16 * sub + 4 * i4;
            float4 cv, sv;
            if (half == 32) {  // preloaded (j is 0)
              const int k = 16 * sub + 4 * i4;
              cv = make_float4(rr.cs[k], rr.cs[k + 1], rr.cs[k + 2], rr.cs[k + 3]);
              sv = make_float4(rr.sn[k], rr.sn[k + 1], rr.sn[k + 2], rr.sn[k + 3]);
            } else {
              cv = make_float4(0.f, 0.f, 0.f, 0.f);
              sv = cv;
              if (live) {
                cv = *reinterpret_cast<const float4*>(cos_row + c);
                sv = *reinterpret_cast<const float4*>(sin_row + c);
              }
            }
            const float cc[4] = {cv.x, cv.y, cv.z, cv.w}, ss[4] = {sv.x, sv.y, sv.z, sv.w};
            // the accumulators rounded to bf16 two at a time (each element
            // rounds to nearest on its own, as the one-value conversion does)
            float pv[4], qv[4];
#pragma unroll
            for (int e = 0; e < 4; e += 2) {
              const float2 pa = __bfloat1622float2(__floats2bfloat162_rn(a[4 * i4 + e],
                                                                         a[4 * i4 + e + 1]));
              const float2 qb = __bfloat1622float2(__floats2bfloat162_rn(b[4 * i4 + e],
                                                                         b[4 * i4 + e + 1]));
              pv[e] = pa.x;
              pv[e + 1] = pa.y;
              qv[e] = qb.x;
              qv[e + 1] = qb.y;
            }
            float r1[4], r2[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float p = pv[e], q = qv[e];
              r1[e] = p * cc[e] - q * ss[e];
              r2[e] = q * cc[e] + p * ss[e];
            }
            w[2 * i4] = pack_bf16(r1[0], r1[1]);
            w[2 * i4 + 1] = pack_bf16(r1[2], r1[3]);
            w[8 + 2 * i4] = pack_bf16(r2[0], r2[1]);
            w[8 + 2 * i4 + 1] = pack_bf16(r2[2], r2[3]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            w[i] = pack_bf16(a[2 * i], a[2 * i + 1]);
            w[8 + i] = pack_bf16(b[2 * i], b[2 * i + 1]);
          }
        }
        const uint32_t rowb = buf + lane * kStageRowBytes;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = (q < 2 ? 2 * sub : 2 + 2 * sub) + q;  // 2s, 2s+1, 4+2s, 5+2s
          st_shared_v4(rowb + ((chunk ^ (lane & 7)) << 4), w[4 * q], w[4 * q + 1], w[4 * q + 2],
                       w[4 * q + 3]);
        }
      }
      if (live && head >= rk.hq && !slot_ok) raise_device_error(err, kErrSlot);
      __syncwarp();
      rope_store_rows(buf, lane, row0, M, n0, hc, head, j, crow, rk, qkv, ldc);
      __syncwarp();
    }
  }
}

// The sequence of (tile, k-begin, k-end) pieces one CTA works on.  Every role
// of the CTA walks the same sequence.
// Work modes: kSchedTiles deals whole output tiles round-robin; kSchedStreamK
// cuts the (tile, k-step) space into equal contiguous ranges; kSchedHybrid
// deals whole tiles while every worker gets one (the largest multiple of
// the worker count), then cuts the remaining tiles' k-steps stream-K.
constexpr int kSchedTiles = 0, kSchedStreamK = 1, kSchedHybrid = 2;

struct Schedule {
  int tiles, kiters, grid, cta, mode;
  int dp_tiles;        // tiles dealt whole
  int64_t it, it_end;  // stream-K range over the other tiles' (tile, k-step) space
  int next_tile;       // round-robin over the whole tiles

  __device__ void init(int tiles_, int kiters_, int mode_) {
    init(tiles_, kiters_, mode_, gridDim.x, blockIdx.x);
  }
  // `grid_` workers, this one `cta_` (a CTA, or a CTA pair of the 2-SM kernel)
  __device__ void init(int tiles_, int kiters_, int mode_, int grid_, int cta_) {
    tiles = tiles_;
    kiters = kiters_;
    grid = grid_;
    cta = cta_;
    mode = mode_;
    dp_tiles = mode == kSchedTiles ? tiles
                                   : (mode == kSchedHybrid ? (tiles / grid) * grid : 0);
    const int64_t base = (int64_t)dp_tiles * kiters;
    const int64_t total = (int64_t)(tiles - dp_tiles) * kiters;
    it = base + total * cta / grid;
    it_end = base + total * (cta + 1) / grid;
    next_tile = cta;
  }
  __device__ bool next(int& tile, int& k0, int& k1) {
    if (next_tile < dp_tiles) {
      tile = next_tile;
      k0 = 0;
      k1 = kiters;
      next_tile += grid;
      return true;
    }
    {
      if (it >= it_end) return false;
      tile = (int)(it / kiters);
      k0 = (int)(it - (int64_t)tile * kiters);
      const int64_t e = min(it_end, (int64_t)(tile + 1) * kiters);
      k1 = k0 + (int)(e - it);
      it = e;
      return true;
    }
  }
};

template <int BN, int EPI, typename TC>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a,
                   const __grid_constant__ CUtensorMap tmap_b, TC* __restrict__ C,
                   const float* __restrict__ R, int M, int N, int K, int64_t ldc, int sched_mode,
                   int* err, const RopeKv rk, int b_const) {
  using Cfg = TileCfg<BN>;
  constexpr int S = Cfg::kStages;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;
  unsigned char* smem = smem_raw + pad;
  const uint32_t sbase = raw + pad;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * S;
  const uint32_t tfull0 = full0 + 16 * S, tempty0 = tfull0 + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = (M + BM - 1) / BM;
  const int tiles = mt * (N / BN);
  const int kiters = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull0 + 8 * a, 1);
      mbar_init(tempty0 + 8 * a, kEpiWarps);  // one arrive per epilogue warp
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(2 * BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  Schedule sched;
  sched.init(tiles, kiters, sched_mode);
  int tile, k0, k1;

  // Everything above touches only this CTA's shared memory and TMEM, so it
  // ran before the wait for the previous kernel (programmatic dependent
  // launch).  When B is constant (model weights), the first stages' B tiles
  // are loaded before the wait too: a CTA placed on an SM while the previous
  // kernel's last CTAs still run elsewhere starts with its weights in flight.
  uint32_t npre = 0;
  if (b_const && warp == 0 && lane == 0) {
    Schedule pre = sched;
    int pt, pk0, pk1;
    while (npre < (uint32_t)S && pre.next(pt, pk0, pk1)) {
      const int pn0 = (pt / mt) * BN;
      for (int k = pk0; k < pk1 && npre < (uint32_t)S; ++k, ++npre) {
        const uint32_t dst = sbase + npre * Cfg::kStageBytes;
        mbar_expect_tx(full0 + 8 * npre, Cfg::kStageBytes);
        tma_load_2d(dst + Cfg::kABytes, &tmap_b, full0 + 8 * npre, k * BK, pn0);
      }
    }
  }
  pdl_enter();

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer ----
      uint32_t q = 0;
      bool alive = true;
      while (alive && sched.next(tile, k0, k1)) {
        const int m0 = (tile % mt) * BM, n0 = (tile / mt) * BN;
        for (int k = k0; k < k1; ++k, ++q) {
          const uint32_t s = q % S;
          if (q >= (uint32_t)S &&
              !mbar_wait(empty0 + 8 * s, ((q / S) - 1) & 1, abort_flag, err)) {
            alive = false;
            break;
          }
          const uint32_t a_dst = sbase + s * Cfg::kStageBytes;
          if (q >= npre) {  // the first npre stages already hold their B tile
            mbar_expect_tx(full0 + 8 * s, Cfg::kStageBytes);
            tma_load_2d(a_dst + Cfg::kABytes, &tmap_b, full0 + 8 * s, k * BK, n0);
          }
          tma_load_2d(a_dst, &tmap_a, full0 + 8 * s, k * BK, m0);
        }
      }
      if (*abort_flag) {  // drain this thread's loads before leaving
        const long long t0 = clock64();
        for (uint32_t j = q > (uint32_t)S ? q - S : 0; j < q; ++j)
          while (!mbar_try_wait(full0 + 8 * (j % S), (j / S) & 1) && clock64() - t0 < kWaitCycles) {
          }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer ----
      const uint32_t id = idesc<BN>();
      uint32_t q = 0, seg = 0;
      bool alive = true;
      while (alive && sched.next(tile, k0, k1)) {
        const uint32_t a = seg & 1, u = seg >> 1;
        if (u >= 1 && !mbar_wait(tempty0 + 8 * a, (u - 1) & 1, abort_flag, err)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + a * BN;
        for (int k = k0; k < k1; ++k, ++q) {
          const uint32_t s = q % S;
          if (!mbar_wait(full0 + 8 * s, (q / S) & 1, abort_flag, err)) {
            alive = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a_addr = sbase + s * Cfg::kStageBytes;
          const uint32_t b_addr = a_addr + Cfg::kABytes;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma(d, sdesc(a_addr + kk * 32), sdesc(b_addr + kk * 32), id, (k > k0) || (kk > 0));
          umma_commit(empty0 + 8 * s);
        }
        if (!alive) break;
        umma_commit(tfull0 + 8 * a);
        ++seg;
      }
    }
  } else {
    // ---- epilogue warps 2..9: lane quarter warp % 4, column half (warp - 2) / 4 ----
    const int row_group = warp & 3;  // TMEM lanes 32*row_group .. +31
    const int half = (warp - 2) >> 2;
    const uint32_t buf = sbase + S * Cfg::kStageBytes + 256 + (warp - 2) * kEpiBufBytes;
    uint32_t seg = 0;
    while (sched.next(tile, k0, k1)) {
      // a piece that is a whole tile has no co-contributor: C = R + acc
      const bool reduce = EPI == kEpiResidual && (k0 > 0 || k1 < kiters);
      const uint32_t a = seg & 1, u = seg >> 1;
      const int m0 = (tile % mt) * BM, n0 = (tile / mt) * BN;
      const int row0 = m0 + row_group * 32;
      RopeRow rr;
      if constexpr (EPI == kEpiRopeKV) rope_row_load(rk, row0 + lane, M, err, rr);
      if (!mbar_wait(tfull0 + 8 * a, u & 1, abort_flag, err)) break;
      __syncwarp();
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t base = tmem + a * BN + ((uint32_t)(row_group * 32) << 16);
      if constexpr (EPI == kEpiRopeKV) {
        rope_kv_rows<BN>(base, buf, lane, row0, M, n0, half, rk,
                         reinterpret_cast<__nv_bfloat16*>(C), ldc, err, rr);
      } else {
        epilogue_tile<BN, EPI, TC>(base, buf, lane, half, row0, M, n0, ldc, static_cast<TC*>(C), R,
                                   reduce);
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty0 + 8 * a);
      ++seg;
    }
  }
  __syncwarp();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN));
  }
}

// ---- 2-SM variant (cta_group::2) ------------------------------------------------------
// A cluster of two CTAs on two SMs computes 256 x 256 output tiles with
// tcgen05.mma.cta_group::2 (M = 256): CTA r of the pair holds rows
// [128 r, 128 r + 128) of the A tile and rows [128 r, 128 r + 128) of the B
// tile (the tile's output columns) in its shared memory, and its TMEM holds
// output rows 128 r .. 128 r + 127 for all 256 columns.  Per k-step an SM
// loads 32 KB (16 KB of A, 16 KB of B) for the work a 1-SM 128 x 256 tile
// needs 48 KB for: the operand feed from L2, which bounds the 1-SM kernel at
// K = 2048 (about 45 B per SM-cycle against the 88 B a k-step's MMAs would
// take), carries two thirds of the bytes per FLOP.
//   warp 0 lane 0, both CTAs: TMA loads of its own A and B halves
//     (cp.async.bulk.tensor ... .cta_group::2, plain tile loads of this GPU's
//     memory), completing on the leader CTA's "full" barrier, whose expected
//     byte count (both halves of both CTAs) the leader posts;
//   warp 1: both CTAs allocate 512 TMEM columns (two 256-column
//     accumulators) with cta_group::2; lane 0 of the leader issues the MMAs
//     and commits each stage to both CTAs' "empty" barriers and each finished
//     accumulator to both CTAs' "tfull" barriers (a commit with the pair's
//     CTA mask: a completion signal, not a data load);
//   warps 2-9, both CTAs: the epilogue of their 128 rows, then an arrive on
//     the leader's "tempty" barrier (16 arrivals free an accumulator).
// Tiles (or stream-K pieces) are dealt to CTA pairs; both CTAs of a pair
// walk the same schedule.  Waits are bounded as in the 1-SM kernel; the
// pair meets at a cluster barrier before any cross-CTA signal and again
// before TMEM is released and the CTAs exit.
constexpr int kStages2 = 6;
constexpr int kHalf2 = 128 * BK * 2;       // one CTA's A or B half of a k-step (16 KB)
constexpr int kStage2 = 2 * kHalf2;        // per CTA and stage
constexpr int kSmem2 = kStages2 * kStage2 + 1024 + 256 + kEpiSmem;
static_assert(kSmem2 <= 227 * 1024, "shared memory per CTA");
constexpr int kBN2 = 256;                  // tile columns (each CTA holds 128 rows of B)

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The shared::cluster address of this CTA's shared variable `addr` in CTA `rank`.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t caddr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(caddr)
               : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::
          : "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map,
                                                 uint32_t leader_bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void umma_pair(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t id,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(id), "r"(accumulate)
      : "memory");
}
// Arrive on the barrier at shared offset `bar` in both CTAs of the pair once
// the MMAs this thread issued so far have completed (a commit to the CTA
// mask 0b11; no data moves).
__device__ __forceinline__ void umma_pair_commit_both(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"((uint16_t)0x3)
      : "memory");
}

template <int EPI, typename TC>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmap_a,
                    const __grid_constant__ CUtensorMap tmap_b, TC* __restrict__ C,
                    const float* __restrict__ R, int M, int N, int K, int64_t ldc, int stream_k,
                    int* err, int b_const) {
  constexpr int S = kStages2;
  constexpr int BN = kBN2;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;
  unsigned char* smem = smem_raw + pad;
  const uint32_t sbase = raw + pad;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * kStage2);
  const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * S;
  const uint32_t tfull0 = full0 + 16 * S, tempty0 = tfull0 + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int mt = (M + 2 * BM - 1) / (2 * BM);  // 256-row tiles
  const int tiles = mt * (N / BN);
  const int kiters = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull0 + 8 * a, 1);
      mbar_init(tempty0 + 8 * a, 2 * kEpiWarps);  // every epilogue warp of both CTAs
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(2 * BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any signal crosses
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  Schedule sched;
  sched.init(tiles, kiters, stream_k, gridDim.x / 2, blockIdx.x / 2);
  int tile, k0, k1;

  // As in the 1-SM kernel: the setup above ran before the wait for the
  // previous kernel, and with constant weights so do the first stages' B
  // loads (both CTAs walk the same schedule, so npre agrees; the leader
  // posts each stage's byte count).
  uint32_t npre = 0;
  if (b_const && warp == 0 && lane == 0) {
    const uint32_t leader_full0 = cluster_addr(full0, 0);
    Schedule pre = sched;
    int pt, pk0, pk1;
    while (npre < (uint32_t)S && pre.next(pt, pk0, pk1)) {
      const int pn0 = (pt / mt) * BN + (int)rank * (BN / 2);
      for (int k = pk0; k < pk1 && npre < (uint32_t)S; ++k, ++npre) {
        const uint32_t dst = sbase + npre * kStage2;
        if (rank == 0) mbar_expect_tx(full0 + 8 * npre, 2 * kStage2);
        tma_load_2d_pair(dst + kHalf2, &tmap_b, leader_full0 + 8 * npre, k * BK, pn0);
      }
    }
  }
  pdl_enter();

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer (both CTAs) ----
      const uint32_t leader_full0 = cluster_addr(full0, 0);
      uint32_t q = 0;
      bool alive = true;
      while (alive && sched.next(tile, k0, k1)) {
        const int m0 = (tile % mt) * 2 * BM + (int)rank * BM;
        const int n0 = (tile / mt) * BN + (int)rank * (BN / 2);
        for (int k = k0; k < k1; ++k, ++q) {
          const uint32_t s = q % S;
          if (q >= (uint32_t)S &&
              !mbar_wait(empty0 + 8 * s, ((q / S) - 1) & 1, abort_flag, err)) {
            alive = false;
            break;
          }
          const uint32_t dst = sbase + s * kStage2;
          if (q >= npre) {  // the first npre stages already hold their B halves
            if (rank == 0) mbar_expect_tx(full0 + 8 * s, 2 * kStage2);
            tma_load_2d_pair(dst + kHalf2, &tmap_b, leader_full0 + 8 * s, k * BK, n0);
          }
          tma_load_2d_pair(dst, &tmap_a, leader_full0 + 8 * s, k * BK, m0);
        }
      }
      if (*abort_flag && rank == 0) {  // every load of the pair completes on these barriers
        const long long t0 = clock64();
        for (uint32_t j = q > (uint32_t)S ? q - S : 0; j < q; ++j)
          while (!mbar_try_wait(full0 + 8 * (j % S), (j / S) & 1) && clock64() - t0 < kWaitCycles) {
          }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---- MMA issuer (leader CTA) ----
      const uint32_t id = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                          ((uint32_t)((2 * BM) >> 4) << 24);
      uint32_t q = 0, seg = 0;
      bool alive = true;
      while (alive && sched.next(tile, k0, k1)) {
        const uint32_t a = seg & 1, u = seg >> 1;
        if (u >= 1 && !mbar_wait(tempty0 + 8 * a, (u - 1) & 1, abort_flag, err)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + a * BN;
        for (int k = k0; k < k1; ++k, ++q) {
          const uint32_t s = q % S;
          if (!mbar_wait(full0 + 8 * s, (q / S) & 1, abort_flag, err)) {
            alive = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a_addr = sbase + s * kStage2;
          const uint32_t b_addr = a_addr + kHalf2;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_pair(d, sdesc(a_addr + kk * 32), sdesc(b_addr + kk * 32), id,
                      (k > k0) || (kk > 0));
          umma_pair_commit_both(empty0 + 8 * s);
        }
        if (!alive) break;
        umma_pair_commit_both(tfull0 + 8 * a);
        ++seg;
      }
    }
  } else {
    // ---- epilogue warps 2..9 (both CTAs): rows 128 * rank + 32 * (warp % 4) + lane,
    // column half (warp - 2) / 4 ----
    const int row_group = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t buf = sbase + S * kStage2 + 256 + (warp - 2) * kEpiBufBytes;
    const bool reduce = EPI == kEpiResidual && stream_k;
    const uint32_t leader_tempty0 = cluster_addr(tempty0, 0);
    uint32_t seg = 0;
    while (sched.next(tile, k0, k1)) {
      const uint32_t a = seg & 1, u = seg >> 1;
      if (!mbar_wait(tfull0 + 8 * a, u & 1, abort_flag, err)) break;
      __syncwarp();
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int row0 = (tile % mt) * 2 * BM + (int)rank * BM + row_group * 32;
      const int n0 = (tile / mt) * BN;
      const uint32_t base = tmem + a * BN + ((uint32_t)(row_group * 32) << 16);
      epilogue_tile<BN, EPI, TC>(base, buf, lane, half, row0, M, n0, ldc, static_cast<TC*>(C), R,
                                 reduce);
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(leader_tempty0 + 8 * a);
      ++seg;
    }
  }
  __syncwarp();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  cluster_sync();  // no CTA leaves while the pair's MMAs or signals may reach it
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN));
  }
}

// ---- host side ------------------------------------------------------------------------
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

struct MapKey {
  const void* ptr;
  int rows, cols, box_rows, dev;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && box_rows == o.box_rows &&
           dev == o.dev;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.ptr) ^ ((size_t)k.rows << 1) ^ ((size_t)k.cols << 21) ^
           ((size_t)k.box_rows << 41) ^ ((size_t)k.dev << 53);
  }
};

// A row-major (rows x cols) bf16 matrix as a K-major 2-D tensor map with a
// (64 x box_rows) box and 128-byte swizzle.  Cached: weights and the
// forward's workspace keep their addresses from call to call.
int tensor_map(const void* ptr, int rows, int cols, int box_rows, CUtensorMap* out) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const MapKey key{ptr, rows, cols, box_rows, dev};
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return MS_OK;
  }
  EncodeFn enc = encode_fn();
  if (!enc) return fail(MS_ERR_CUDA, "gemm_tc: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUtensorMap map;
  const CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MS_ERR_CUDA, "gemm_tc: tensor map encode failed (%d)", (int)r);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, map);
  *out = map;
  return MS_OK;
}

template <int BN, int EPI, typename TC>
int launch_tc(const void* A, const void* B, void* C, const float* R, int M, int N, int K,
              int64_t ldc, int mode, cudaStream_t s, const RopeKv& rk = RopeKv{},
              bool b_const = false) {
  CUtensorMap ta, tb;
  MS_TRY(tensor_map(A, M, K, BM, &ta));
  MS_TRY(tensor_map(B, N, K, BN, &tb));
  using Cfg = TileCfg<BN>;
  auto kern = gemm_tc_kernel<BN, EPI, TC>;
  // the shared-memory opt-in is per device
  static uint64_t attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set & (1ull << (dev & 63)))) {
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
    if (e != cudaSuccess) return fail(MS_ERR_CUDA, "gemm_tc: smem attribute: %s", cudaGetErrorString(e));
    attr_set |= 1ull << (dev & 63);
  }
  const int tiles = ((M + BM - 1) / BM) * (N / BN);
  const int kiters = (K + BK - 1) / BK;
  int grid = mode == kSchedStreamK ? (int)std::min<int64_t>((int64_t)tiles * kiters, kNumSMs)
                                    : std::min(tiles, kNumSMs);
  if (grid < 1) grid = 1;
  launch_pdl(kern, grid, kThreads, Cfg::kSmem, s, ta, tb, static_cast<TC*>(C), R, M, N, K, ldc,
             mode, device_error_word(), rk, b_const ? 1 : 0);
  return check_launch("gemm_tc_kernel");
}

template <int EPI, typename TC>
int launch_tc2(const void* A, const void* B, void* C, const float* R, int M, int N, int K,
               int64_t ldc, bool stream_k, cudaStream_t s, bool b_const) {
  CUtensorMap ta, tb;
  MS_TRY(tensor_map(A, M, K, BM, &ta));
  MS_TRY(tensor_map(B, N, K, kBN2 / 2, &tb));
  auto kern = gemm_tc2_kernel<EPI, TC>;
  static uint64_t attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set & (1ull << (dev & 63)))) {
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem2);
    if (e != cudaSuccess) return fail(MS_ERR_CUDA, "gemm_tc2: smem attribute: %s", cudaGetErrorString(e));
    attr_set |= 1ull << (dev & 63);
  }
  const int tiles = ((M + 2 * BM - 1) / (2 * BM)) * (N / kBN2);
  const int kiters = (K + BK - 1) / BK;
  // Pairs are placed within a GPC: as many as can be resident at once (at
  // most one CTA per SM), so the persistent grid is a single wave.
  static int max_pairs[64] = {};
  if (max_pairs[dev & 63] == 0) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(kNumSMs);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmem2;
    int n = 0;
    const cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    if (e != cudaSuccess || n < 1) {
      (void)cudaGetLastError();
      n = kNumSMs / 2;
    }
    max_pairs[dev & 63] = std::min(n, kNumSMs / 2);
  }
  const int pairs_max = max_pairs[dev & 63];
  int pairs = stream_k ? (int)std::min<int64_t>((int64_t)tiles * kiters, pairs_max)
                       : std::min(tiles, pairs_max);
  if (pairs < 1) pairs = 1;
  launch_pdl(kern, 2 * pairs, kThreads, kSmem2, s, ta, tb, static_cast<TC*>(C), R, M, N, K, ldc,
             stream_k ? kSchedStreamK : kSchedTiles, device_error_word(), b_const ? 1 : 0);
  return check_launch("gemm_tc2_kernel");
}

// Which tcgen05 kernel: 0 = by shape, 1 = one CTA per tile, 2 = CTA pairs
// (ms_gemm_set_policy; for measurements and tests).
int g_gemm_policy = 0;

// CTA pairs by shape: the wide store GEMMs (the lm_head: 1280 x 32000 x 2048
// 140 -> 128 us, 256 x 32000 x 2048 40 -> 37 us with the staged epilogue).
// The verify-sized SwiGLU GEMM is 3% faster alone on pairs (1280 x 11264 x
// 2048: 44.0 -> 42.6 us) but a round was not (6.29 against 6.27 ms);
// elsewhere the pairs measured slower (stream-K residual pieces twice as
// large on half as many workers, qkv, the M = 256 projections).
bool use_pairs(int M, int N, int epi) {
  if (g_gemm_policy == 1 || epi == kEpiRopeKV || N % kBN2 != 0) return false;
  if (g_gemm_policy == 2) return true;
  return epi == kEpiStore && N >= 16384 && M >= 2 * BM;
}

// Tile width: 256 columns when N allows it and there are enough tiles to go
// around, else 128.
bool use_bn256(int M, int N, bool stream_k) {
  if (N % 256 != 0) return false;
  const int mt = (M + BM - 1) / BM;
  // Stream-K pieces each add a whole tile into C: with at most two row tiles
  // (a draft pass) 128-wide tiles halve those reductions (draft o_proj
  // 16.9 -> 12.8 us, down 19.3 -> 16.4 us); taller GEMMs keep 256.
  if (stream_k) return mt > 2;
  return mt * (N / 256) >= kNumSMs / 2;
}

template <int EPI, typename TC>
int launch_any(const void* A, const void* B, void* C, const float* R, int M, int N, int K,
               int64_t ldc, int mode, cudaStream_t s, bool b_const) {
  if (use_bn256(M, N, mode == kSchedStreamK))
    return launch_tc<256, EPI, TC>(A, B, C, R, M, N, K, ldc, mode, s, RopeKv{}, b_const);
  return launch_tc<128, EPI, TC>(A, B, C, R, M, N, K, ldc, mode, s, RopeKv{}, b_const);
}

}  // namespace

int gemm_qkv_rope(const void* A, const void* W, void* qkv, int M, int N, int K, const RopeKv& rk,
                  cudaStream_t s, bool weights_const) {
  if ((rk.dh != 64 && rk.dh != 128) || N != (rk.hq + 2 * rk.hkv) * rk.dh ||
      !gemm_tc_supported(M, N, K, N, MS_DTYPE_BF16, kEpiStore) ||
      ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(W) |
        reinterpret_cast<uintptr_t>(qkv)) & 15))
    return MS_ERR_UNSUPPORTED;
  ProfScope prof(kClsGemm, s);
  if (use_bn256(M, N, false))
    return launch_tc<256, kEpiRopeKV, __nv_bfloat16>(A, W, qkv, nullptr, M, N, K, N, kSchedTiles,
                                                     s, rk, weights_const);
  // Few rows (a draft pass: M 256 gives 40 tiles of 128 columns, each CTA
  // streaming 1 MB of operands through a feed-bound k-loop): one head of 64
  // columns per tile while that still fits in one wave, so twice the CTAs
  // share the operand feed.
  if (rk.dh == 64 && ((M + BM - 1) / BM) * (N / 64) <= kNumSMs)
    return launch_tc<64, kEpiRopeKV, __nv_bfloat16>(A, W, qkv, nullptr, M, N, K, N, kSchedTiles,
                                                    s, rk, weights_const);
  return launch_tc<128, kEpiRopeKV, __nv_bfloat16>(A, W, qkv, nullptr, M, N, K, N, kSchedTiles, s,
                                                   rk, weights_const);
}

bool gemm_tc_supported(int M, int N, int K, int64_t ldc, int c_dtype, int epi) {
  if (M <= 0 || K % 8 != 0 || N % 128 != 0) return false;
  if (epi == kEpiResidual && c_dtype != MS_DTYPE_F32) return false;
  const int64_t align = (epi == kEpiSwiGLU || c_dtype == MS_DTYPE_BF16) ? 8 : 4;
  return ldc % align == 0;
}

int gemm_tc(const void* A, const void* B, void* C, const float* R, int M, int N, int K, int64_t ldc,
            int c_dtype, int epi, cudaStream_t s, bool weights_const) {
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B) |
       reinterpret_cast<uintptr_t>(C)) & 15)
    return fail(MS_ERR_INVALID, "gemm_tc: operands must be 16-byte aligned");
  if (use_pairs(M, N, epi)) {
    if (epi == kEpiSwiGLU)
      return launch_tc2<kEpiSwiGLU, __nv_bfloat16>(A, B, C, R, M, N, K, ldc, false, s,
                                                   weights_const);
    if (epi == kEpiResidual) {
      const bool in_place = static_cast<const void*>(R) == C;
      const int tiles2 = ((M + 2 * BM - 1) / (2 * BM)) * (N / kBN2);
      const double ab_bytes = 2.0 * ((double)M + (double)N) * (double)K;
      const bool stream_k = in_place && (tiles2 < kNumSMs / 2 || ab_bytes <= 64.0 * (1 << 20));
      return launch_tc2<kEpiResidual, float>(A, B, C, R, M, N, K, ldc, stream_k, s,
                                            weights_const);
    }
    if (c_dtype == MS_DTYPE_F32)
      return launch_tc2<kEpiStore, float>(A, B, C, R, M, N, K, ldc, false, s, weights_const);
    return launch_tc2<kEpiStore, __nv_bfloat16>(A, B, C, R, M, N, K, ldc, false, s, weights_const);
  }
  if (epi == kEpiSwiGLU)
    return launch_any<kEpiSwiGLU, __nv_bfloat16>(A, B, C, R, M, N, K, ldc, kSchedTiles, s,
                                                 weights_const);
  if (epi == kEpiResidual) {
    // In place (C += A B^T): stream-K with reductions into C when the tiles
    // are fewer than the SMs or A + B fit in L2.  Otherwise whole tiles first
    // (the CTAs stay near the same k-step: stream-K's scattered k offsets
    // keep the whole of A and B live at once, and at M 1536, K 14336
    // (160 MB) that re-read DRAM ~7 times), then stream-K over the tiles
    // left after the last whole wave, whose A and B fit in L2 (8B down, 192
    // tiles: 195 -> 144 us, the second wave no longer on 44 SMs alone).
    const bool in_place = static_cast<const void*>(R) == C;
    const int tiles256 = ((M + BM - 1) / BM) * (N / 256);
    const double ab_bytes = 2.0 * ((double)M + (double)N) * (double)K;
    int mode = kSchedTiles;
    if (in_place) {
      if (N % 256 != 0 || tiles256 < kNumSMs || ab_bytes <= 64.0 * (1 << 20))
        mode = kSchedStreamK;
      else if (tiles256 % kNumSMs != 0)
        mode = kSchedHybrid;
    }
    return launch_any<kEpiResidual, float>(A, B, C, R, M, N, K, ldc, mode, s, weights_const);
  }
  if (c_dtype == MS_DTYPE_F32)
    return launch_any<kEpiStore, float>(A, B, C, R, M, N, K, ldc, kSchedTiles, s, weights_const);
  return launch_any<kEpiStore, __nv_bfloat16>(A, B, C, R, M, N, K, ldc, kSchedTiles, s,
                                              weights_const);
}

}  // namespace ms

extern "C" int ms_gemm_set_policy(int policy) {
  if (policy < 0 || policy > 2) return ms::fail(MS_ERR_INVALID, "ms_gemm_set_policy: %d", policy);
  ms::g_gemm_policy = policy;
  return MS_OK;
}
