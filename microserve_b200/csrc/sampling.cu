// Sampling kernels: one CTA per vocabulary row (K8) or per request (K9).
//
// A row is processed the way reference sampling.py:17-74 does it
// (temperature -> top-k -> top-p -> softmax) but without sorting:
//   * top-k: radix select of the k-th largest value over the float bits
//     (4 passes of 8 bits, per-warp histograms in shared memory); keep x >= it
//     (ties keep more, as apply_top_k does);
//   * top-p: radix descent on probability mass to the "crossing" value, the
//     first value in descending order whose inclusive cumulative mass reaches
//     top_p; keep x >= it (apply_top_p keeps the crossing token);
//   * draws: inverse CDF in vocabulary order on unnormalised weights with a
//     Philox uniform (u * total), instead of torch.multinomial's CPU stream.
// The row is staged in shared memory when it fits, otherwise every pass
// re-reads it from global memory (L2-resident after the first pass).
#include <cfloat>
#include <cmath>

#include <cooperative_groups.h>

#include "common.cuh"

namespace ms {
namespace {

namespace cg = cooperative_groups;

constexpr int kMaxStagedV = 40960;  // 160 KB of float32 in shared memory
constexpr int kHistBins = 256;

__device__ __forceinline__ uint32_t fkey(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float kfloat(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

// Shared scratch used by every row routine.  `hist` holds one 256-bin
// histogram per warp (ints or floats), `red` small reduction slots.
struct RowSmem {
  float* stage;  // V floats when staged, else nullptr
  uint32_t* hist;
  float* red;       // 64 floats
  double* red_d;    // 64 doubles
  int* red_i;       // 64 ints
};

// Distribution over one row.  mode 0: logits (x = raw / T, p = exp(x-m)/z
// for x >= thresh); mode 1: probabilities as stored; mode 2: one-hot.
struct Dist {
  const float* row;
  int mode;
  bool divide;  // apply temperature when reading (row not pre-divided)
  float temp;
  float m, thresh, z, inv_z;
  int argmax;

  __device__ __forceinline__ float x(int i) const {
    const float v = row[i];
    return divide ? __fdiv_rn(v, temp) : v;
  }
  // Unnormalised weight, the quantity the inverse CDF walks.
  __device__ __forceinline__ float weight(int i) const {
    if (mode == 1) return row[i];
    if (mode == 2) return i == argmax ? 1.f : 0.f;
    const float xv = x(i);
    return xv >= thresh ? __expf(xv - m) : 0.f;
  }
  __device__ __forceinline__ float prob(int i) const {
    if (mode == 1) return row[i];
    if (mode == 2) return i == argmax ? 1.f : 0.f;
    const float xv = x(i);
    return xv >= thresh ? __expf(xv - m) * inv_z : 0.f;
  }
  // prob(i) from the row's value v = row[i] already loaded.
  __device__ __forceinline__ float prob_of(float v, int i) const {
    if (mode == 1) return v;
    if (mode == 2) return i == argmax ? 1.f : 0.f;
    const float xv = divide ? __fdiv_rn(v, temp) : v;
    return xv >= thresh ? __expf(xv - m) * inv_z : 0.f;
  }
};

// The rejection residual max(0, p - q) over n elements whose p values come
// from the staged x values xs[0, n) (p in mode 0 or 2, row indices lo + j);
// q is read from global memory at qrow[0, n).  The residual replaces xs
// (each thread overwrites only what it has just read); returns this
// thread's partial sum.  Four float4 loads of q per thread are in flight at
// once: the pass is bound by the latency of those loads.
__device__ float residual_pass(float* xs, int n, int lo, const Dist& pv, const Dist& qv,
                               const float* __restrict__ qrow) {
  auto pval = [&](float x, int i) {
    if (pv.mode == 2) return i == pv.argmax ? 1.f : 0.f;
    return x >= pv.thresh ? __expf(x - pv.m) * pv.inv_z : 0.f;
  };
  float part = 0.f;
  const bool vec = (reinterpret_cast<uintptr_t>(qrow) & 15) == 0;
  const int n4 = vec ? n >> 2 : 0;
  const float4* q4 = reinterpret_cast<const float4*>(qrow);
  float4* x4 = reinterpret_cast<float4*>(xs);
  for (int base = threadIdx.x; base < n4; base += 4 * blockDim.x) {
    float4 qa[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + u * blockDim.x;
      qa[u] = i < n4 ? __ldg(q4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + u * blockDim.x;
      if (i < n4) {
        const float4 xa = x4[i];
        const int g = lo + 4 * i;
        float4 o;
        o.x = fmaxf(pval(xa.x, g) - qv.prob_of(qa[u].x, g), 0.f);
        o.y = fmaxf(pval(xa.y, g + 1) - qv.prob_of(qa[u].y, g + 1), 0.f);
        o.z = fmaxf(pval(xa.z, g + 2) - qv.prob_of(qa[u].z, g + 2), 0.f);
        o.w = fmaxf(pval(xa.w, g + 3) - qv.prob_of(qa[u].w, g + 3), 0.f);
        x4[i] = o;
        part += (o.x + o.y) + (o.z + o.w);
      }
    }
  }
  for (int j = (n4 << 2) + threadIdx.x; j < n; j += blockDim.x) {
    const float r = fmaxf(pval(xs[j], lo + j) - qv.prob_of(__ldg(qrow + j), lo + j), 0.f);
    xs[j] = r;
    part += r;
  }
  return part;
}

// ---- block reductions with broadcast ---------------------------------------
__device__ float block_sum_b(float v, RowSmem& sm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) sm.red[warp] = v;
  __syncthreads();
  float t = lane < nw ? sm.red[lane] : 0.f;
  return warp_sum(t);
}

// Max with first-index tie break.
__device__ void block_argmax(float v, int idx, RowSmem& sm, float& out_v, int& out_i) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
  __syncthreads();
  if (lane == 0) {
    sm.red[warp] = v;
    sm.red_i[warp] = idx;
  }
  __syncthreads();
  v = lane < nw ? sm.red[lane] : -INFINITY;
  idx = lane < nw ? sm.red_i[lane] : 0x7fffffff;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
  out_v = v;
  out_i = idx;
}

// Pass over the row computing max and first argmax of x.
__device__ void row_argmax(const Dist d, int V, RowSmem& sm, float& m, int& am) {
  float best = -INFINITY;
  int bi = 0x7fffffff;
#pragma unroll 4
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = d.x(i);
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
  block_argmax(best, bi, sm, m, am);
  if (am == 0x7fffffff) am = 0;  // all NaN: degenerate, pick index 0
}

// Clears the per-warp histograms.
__device__ __forceinline__ void hist_clear(RowSmem& sm) {
  const int n = (blockDim.x >> 5) * kHistBins;
  for (int i = threadIdx.x; i < n; i += blockDim.x) sm.hist[i] = 0u;
  __syncthreads();
}

// Sums the per-warp histograms into bins [0,256) of warp 0's histogram.
template <bool kFloat>
__device__ __forceinline__ void hist_reduce(RowSmem& sm) {
  __syncthreads();
  const int nw = blockDim.x >> 5;
  for (int b = threadIdx.x; b < kHistBins; b += blockDim.x) {
    if (kFloat) {
      float s = 0.f;
      for (int w = 0; w < nw; ++w) s += __uint_as_float(sm.hist[w * kHistBins + b]);
      sm.hist[b] = __float_as_uint(s);
    } else {
      uint32_t s = 0;
      for (int w = 0; w < nw; ++w) s += sm.hist[w * kHistBins + b];
      sm.hist[b] = s;
    }
  }
  __syncthreads();
}

// Warp 0 walks the 256 reduced bins from the top and finds the first bin at
// which `above + bin >= target` (counts or masses).  Returns through smem:
// red_i[0] = bin (-1 if none), red[0]/red_i[1] = amount strictly above it.
template <bool kFloat>
__device__ void hist_find_from_top(RowSmem& sm, float target_f, uint32_t target_u) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    // lane l owns bins [255-8l-7, 255-8l], walked from the top.
    float sf = 0.f;
    uint32_t su = 0;
    float vf[8];
    uint32_t vu[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int b = 255 - 8 * lane - j;
      if (kFloat) {
        vf[j] = __uint_as_float(sm.hist[b]);
        sf += vf[j];
      } else {
        vu[j] = sm.hist[b];
        su += vu[j];
      }
    }
    // inclusive prefix over lanes (lane 0 = top bins)
    float incf = sf;
    uint32_t incu = su;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float tf = __shfl_up_sync(0xffffffffu, incf, o);
      const uint32_t tu = __shfl_up_sync(0xffffffffu, incu, o);
      if (lane >= o) {
        incf += tf;
        incu += tu;
      }
    }
    const bool hit = kFloat ? (incf >= target_f) : (incu >= target_u);
    const unsigned ballot = __ballot_sync(0xffffffffu, hit);
    if (ballot == 0u) {
      if (lane == 0) {
        sm.red_i[0] = -1;
        sm.red[0] = incf;  // total (unused)
      }
    } else {
      const int first = __ffs(ballot) - 1;
      if (lane == first) {
        float af = incf - sf;
        uint32_t au = incu - su;
        int bin = 255 - 8 * lane - 7;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const bool h = kFloat ? (af + vf[j] >= target_f) : (au + vu[j] >= target_u);
          if (h) {
            bin = 255 - 8 * lane - j;
            break;
          }
          af += kFloat ? vf[j] : 0.f;
          au += kFloat ? 0u : vu[j];
        }
        sm.red_i[0] = bin;
        sm.red[0] = af;
        sm.red_i[1] = (int)au;
      }
    }
  }
  __syncthreads();
}

// k-th largest x over the row (1 <= k <= V), exact.
__device__ float radix_kth_largest(const Dist d, int V, int k, RowSmem& sm) {
  uint32_t prefix = 0, mask = 0;
  uint32_t k_rem = (uint32_t)k;
  const int warp = threadIdx.x >> 5;
  for (int shift = 24; shift >= 0; shift -= 8) {
    hist_clear(sm);
    uint32_t* h = sm.hist + warp * kHistBins;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const uint32_t key = fkey(d.x(i));
      if ((key & mask) == prefix) atomicAdd(&h[(key >> shift) & 255u], 1u);
    }
    hist_reduce<false>(sm);
    hist_find_from_top<false>(sm, 0.f, k_rem);
    const int bin = sm.red_i[0];
    const uint32_t above = (uint32_t)sm.red_i[1];
    __syncthreads();
    if (bin < 0) break;  // cannot happen for 1 <= k <= V; keeps everything
    prefix |= (uint32_t)bin << shift;
    mask |= 255u << shift;
    k_rem -= above;
  }
  if (mask != 0xffffffffu) return -INFINITY;
  return kfloat(prefix);
}

// The top-p crossing value: first x in descending order whose inclusive
// cumulative probability reaches top_p.  Returns -inf if it never does.
__device__ float radix_top_p(const Dist d, int V, float top_p, RowSmem& sm) {
  uint32_t prefix = 0, mask = 0;
  float above_total = 0.f;
  const int warp = threadIdx.x >> 5;
  for (int shift = 24; shift >= 0; shift -= 8) {
    hist_clear(sm);
    uint32_t* h = sm.hist + warp * kHistBins;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float xv = d.x(i);
      if (xv < d.thresh) continue;
      const uint32_t key = fkey(xv);
      if ((key & mask) == prefix) {
        const float p = __expf(xv - d.m) * d.inv_z;
        atomicAdd(reinterpret_cast<float*>(&h[(key >> shift) & 255u]), p);
      }
    }
    hist_reduce<true>(sm);
    hist_find_from_top<true>(sm, top_p - above_total, 0u);
    const int bin = sm.red_i[0];
    const float above = sm.red[0];
    __syncthreads();
    if (bin < 0) return -INFINITY;
    prefix |= (uint32_t)bin << shift;
    mask |= 255u << shift;
    above_total += above;
  }
  return kfloat(prefix);
}

// ---- linear-bin selection -------------------------------------------------
// Values are binned by their distance below the row maximum, bin =
// floor((max - x) * 64) clamped to kLinBins-1: one pass with little atomic
// contention (logits spread over many bins, unlike their exponent bits), a
// block scan to find the bin holding the k-th largest value / the top-p
// crossing value, then an exact choice among that bin's candidates, ranked
// in shared memory (value descending, index ascending).  A bin with more
// than kCand candidates (flat or tied rows) falls back to the radix
// routines above.
//
// Top-p bin masses use two 32-bit integer atomics per element (shared-memory
// float and 64-bit atomics are much slower): a count, and the deficit
// 1 - e * 2^(b/64 log2 e) of the element's mass e = exp(x - max) against the
// bin's upper edge, in 2^-22 fixed point.  A bin's mass is then
// exp(-b/64) * (count - deficit * 2^-22), exact to about 2^-22 per element,
// and every sum fits 32 bits for up to 65536 elements per bin.
constexpr int kLinBins = 2048;
constexpr int kCand = 512;
constexpr float kBinsPerUnit = 64.f;
constexpr float kDefScale = 4194304.f;  // 2^22
// shared words: counts, deficits, candidate keys (u64), ranked keys (u64)
constexpr int kLinWords = 2 * kLinBins + 4 * kCand;

__device__ __forceinline__ int lin_bin(float m, float x) {
  const float t = (m - x) * kBinsPerUnit;
  return t < (float)(kLinBins - 1) ? (int)t : kLinBins - 1;
}
// The element's deficit against its bin's upper edge, fixed point.
__device__ __forceinline__ uint32_t lin_deficit(float m, float x, int b) {
  if (b >= kLinBins - 1) return 0u;
  const float r = __expf((x - m) + (float)b * (1.f / kBinsPerUnit));
  return __float2uint_rn(fmaxf(1.f - r, 0.f) * kDefScale);
}
__device__ __forceinline__ float lin_bin_mass(const uint32_t* Hc, const uint32_t* Hd, int b) {
  const float cnt = (float)Hc[b] - (float)Hd[b] * (1.f / kDefScale);
  return cnt * __expf(-(float)b * (1.f / kBinsPerUnit));
}

// Block-wide search over the kLinBins bins for the first bin whose inclusive
// prefix (counts when Hd is null, masses otherwise) reaches `target`.
// Returns the bin (-1 if none) and the amount in the bins before it.
__device__ int lin_find(const uint32_t* Hc, const uint32_t* Hd, double target, RowSmem& sm,
                        double& before) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int per = kLinBins / blockDim.x;
  const int b0 = threadIdx.x * per;
  double own = 0.0;
  for (int j = 0; j < per; ++j)
    own += Hd ? (double)lin_bin_mass(Hc, Hd, b0 + j) : (double)Hc[b0 + j];
  double inc = own;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += t;
  }
  __syncthreads();
  if (lane == 31) sm.red_d[warp] = inc;
  if (threadIdx.x == 0) sm.red_i[48] = -1;
  __syncthreads();
  double wb = 0.0;
  for (int w = 0; w < warp && w < nw; ++w) wb += sm.red_d[w];
  const double ex = wb + inc - own;  // before this thread's bins
  if (ex < target && ex + own >= target) {
    double a = ex;
    for (int j = 0; j < per; ++j) {
      const double h = Hd ? (double)lin_bin_mass(Hc, Hd, b0 + j) : (double)Hc[b0 + j];
      if (a + h >= target) {
        sm.red_i[48] = b0 + j;
        sm.red_d[48] = a;
        break;
      }
      a += h;
    }
  }
  __syncthreads();
  const int bin = sm.red_i[48];
  before = sm.red_d[48];
  __syncthreads();
  return bin;
}

// Gathers the sort keys (value descending, index ascending) of the kept
// elements in `bin`; returns their number (may exceed kCand: caller falls
// back).
__device__ int lin_gather(const Dist d, int V, int bin, unsigned long long* keys, RowSmem& sm) {
  if (threadIdx.x == 0) sm.red_i[50] = 0;
  __syncthreads();
  auto note = [&](float xv, int i) {
    if (xv >= d.thresh && lin_bin(d.m, xv) == bin) {
      const int slot = atomicAdd(&sm.red_i[50], 1);
      if (slot < kCand) keys[slot] = ((unsigned long long)fkey(xv) << 32) | (uint32_t)~(uint32_t)i;
    }
  };
  if (!d.divide && (reinterpret_cast<uintptr_t>(d.row) & 15) == 0) {
    const float4* r4 = reinterpret_cast<const float4*>(d.row);
    const int n4 = V >> 2;
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
      const float4 v = r4[i];
      note(v.x, 4 * i);
      note(v.y, 4 * i + 1);
      note(v.z, 4 * i + 2);
      note(v.w, 4 * i + 3);
    }
    for (int i = (n4 << 2) + threadIdx.x; i < V; i += blockDim.x) note(d.row[i], i);
  } else {
#pragma unroll 4
    for (int i = threadIdx.x; i < V; i += blockDim.x) note(d.x(i), i);
  }
  __syncthreads();
  const int n = sm.red_i[50];
  __syncthreads();
  return n;
}

// Ranks keys[0, n) (distinct) and writes them to `sorted` in descending
// order: rank = number of larger keys, one candidate per thread.
__device__ void rank_keys_desc(const unsigned long long* keys, unsigned long long* sorted, int n) {
  for (int c = threadIdx.x; c < n; c += blockDim.x) {
    const unsigned long long kc = keys[c];
    int r0 = 0, r1 = 0, r2 = 0, r3 = 0;
    int j = 0;
    for (; j + 4 <= n; j += 4) {
      r0 += keys[j] > kc;
      r1 += keys[j + 1] > kc;
      r2 += keys[j + 2] > kc;
      r3 += keys[j + 3] > kc;
    }
    for (; j < n; ++j) r0 += keys[j] > kc;
    sorted[(r0 + r1) + (r2 + r3)] = kc;
  }
  __syncthreads();
}

// k-th largest value (ties keep more).  ok=false: use the radix routine.
__device__ float linear_kth(const Dist d, int V, int k, RowSmem& sm, bool& ok) {
  uint32_t* Hc = sm.hist;
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(sm.hist + 2 * kLinBins);
  unsigned long long* sorted = keys + kCand;
  for (int i = threadIdx.x; i < kLinBins; i += blockDim.x) Hc[i] = 0u;
  __syncthreads();
  for (int i = threadIdx.x; i < V; i += blockDim.x) atomicAdd(&Hc[lin_bin(d.m, d.x(i))], 1u);
  __syncthreads();
  double before;
  const int bin = lin_find(Hc, nullptr, (double)k, sm, before);
  ok = false;
  if (bin < 0) return -INFINITY;
  const int n = lin_gather(d, V, bin, keys, sm);  // d.thresh is -inf here
  if (n > kCand || n == 0) return -INFINITY;
  const int rank = k - (int)before;  // 1-based rank wanted inside the bin
  if (rank < 1 || rank > n) return -INFINITY;
  rank_keys_desc(keys, sorted, n);
  const float v = kfloat((uint32_t)(sorted[rank - 1] >> 32));
  __syncthreads();
  ok = true;
  return v;
}

// Top-p on the mass bins built by row_stats: returns the crossing value --
// the first value in descending order whose inclusive mass reaches `target`
// (top_p times the kept total) -- and the mass kept at and above it.
// ok=false: use the radix routine.
__device__ float linear_top_p(const Dist d, int V, double target, RowSmem& sm, bool& ok,
                              double& z_keep) {
  const uint32_t* Hc = sm.hist;
  const uint32_t* Hd = sm.hist + kLinBins;
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(sm.hist + 2 * kLinBins);
  unsigned long long* sorted = keys + kCand;
  double before;
  const int bin = lin_find(Hc, Hd, target, sm, before);
  ok = false;
  if (bin < 0 || bin >= kLinBins - 1 || Hc[bin] > 65536u) return -INFINITY;
  const int n = lin_gather(d, V, bin, keys, sm);
  if (n > kCand || n == 0) return -INFINITY;
  rank_keys_desc(keys, sorted, n);
  // inclusive prefix of the ranked candidates' exact masses, one per thread
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int c = threadIdx.x;
  const float xc = c < n ? kfloat((uint32_t)(sorted[c] >> 32)) : -INFINITY;
  const double e = c < n ? (double)__expf(xc - d.m) : 0.0;
  double inc = e;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += t;
  }
  if (lane == 31) sm.red_d[warp] = inc;
  if (threadIdx.x == 0) sm.red_i[51] = -1;
  __syncthreads();
  double wb = before;
  for (int w = 0; w < warp && w < nw; ++w) wb += sm.red_d[w];
  const double cum = wb + inc;  // mass at and above candidate c
  if (c < n && cum - e < target && cum >= target) sm.red_i[51] = c;
  __syncthreads();
  const int cross = sm.red_i[51];
  if (cross < 0) {  // rounding found no crossing: radix fallback
    __syncthreads();
    return -INFINITY;
  }
  const float cut = kfloat((uint32_t)(sorted[cross] >> 32));
  // kept mass: through the last candidate equal to the cut (ties kept)
  if (c < n && xc == cut && (c + 1 == n || kfloat((uint32_t)(sorted[c + 1] >> 32)) < cut))
    sm.red_d[49] = cum;
  __syncthreads();
  z_keep = sm.red_d[49];
  __syncthreads();
  ok = true;
  return cut;
}

__device__ __forceinline__ bool linear_ok(int V) {
  return V >= 4096 && kLinBins % blockDim.x == 0 && (int)blockDim.x >= kCand;
}

// Fills d.m / d.argmax (unless have_max), d.thresh, d.z, d.inv_z for a
// logits row (mode 0).  The kept-mass total and the top-p mass bins come out
// of one pass; the top-p kept mass is derived from the bins and candidates.
__device__ void row_stats(Dist& dref, int V, int top_k, float top_p, RowSmem& sm, bool have_max) {
  Dist d = dref;  // register copy for the hot loops
  if (!have_max) {
    float m0;
    int am;
    row_argmax(d, V, sm, m0, am);
    d.m = m0;
    d.argmax = am;
  }
  const float m = d.m;
  d.thresh = -INFINITY;
  const bool lin = linear_ok(V);
  if (top_k > 0 && top_k < V) {
    bool ok = false;
    float kth = -INFINITY;
    if (lin) kth = linear_kth(d, V, top_k, sm, ok);
    d.thresh = ok ? kth : radix_kth_largest(d, V, top_k, sm);
  }
  const bool want_p = top_p < 1.f;
  const bool hist = want_p && lin;
  uint32_t* Hc = sm.hist;
  uint32_t* Hd = sm.hist + kLinBins;
  if (hist) {
    for (int i = threadIdx.x; i < 2 * kLinBins; i += blockDim.x) Hc[i] = 0u;
    __syncthreads();
  }
  float zl = 0.f;
  {
    const float thresh = d.thresh;
    auto note = [&](float xv) {
      if (xv >= thresh) {
        zl += __expf(xv - m);
        if (hist) {
          const int b = lin_bin(m, xv);
          atomicAdd(&Hc[b], 1u);
          atomicAdd(&Hd[b], lin_deficit(m, xv, b));
        }
      }
    };
    if (!d.divide && (reinterpret_cast<uintptr_t>(d.row) & 15) == 0) {
      // staged / pre-divided rows: two float4 loads ahead of the atomics
      const float4* r4 = reinterpret_cast<const float4*>(d.row);
      const int n4 = V >> 2;
      int i = threadIdx.x;
      for (; i + (int)blockDim.x < n4; i += 2 * blockDim.x) {
        const float4 a = r4[i], b = r4[i + blockDim.x];
        note(a.x);
        note(a.y);
        note(a.z);
        note(a.w);
        note(b.x);
        note(b.y);
        note(b.z);
        note(b.w);
      }
      for (; i < n4; i += blockDim.x) {
        const float4 a = r4[i];
        note(a.x);
        note(a.y);
        note(a.z);
        note(a.w);
      }
      for (int j = (n4 << 2) + threadIdx.x; j < V; j += blockDim.x) note(d.row[j]);
    } else {
#pragma unroll 4
      for (int j = threadIdx.x; j < V; j += blockDim.x) note(d.x(j));
    }
  }
  d.z = block_sum_b(zl, sm);
  d.inv_z = 1.f / d.z;
  if (!want_p) {
    dref = d;
    return;
  }
  float cut = -INFINITY;
  bool done = false;
  if (1.f >= top_p * d.z) {
    cut = m;  // the maximum alone already covers top_p
  } else if (hist) {
    double z_keep = d.z;
    bool ok = false;
    const float c = linear_top_p(d, V, (double)top_p * (double)d.z, sm, ok, z_keep);
    if (ok) {
      if (c > d.thresh) {
        d.thresh = c;
        d.z = (float)z_keep;
        d.inv_z = 1.f / d.z;
      }
      done = true;
    }
  }
  if (!done && cut == -INFINITY) cut = radix_top_p(d, V, top_p, sm);
  if (!done && cut > d.thresh) {
    d.thresh = cut;
    zl = 0.f;
#pragma unroll 4
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float xv = d.x(i);
      if (xv >= d.thresh) zl += __expf(xv - m);
    }
    d.z = block_sum_b(zl, sm);
    d.inv_z = 1.f / d.z;
  }
  dref = d;
}

// Inverse-CDF draw over weights w(i) in vocabulary order: the first index
// whose running sum exceeds u * total.  Falls back to the last positive
// weight when rounding leaves the target past the end.
//
// Warp w owns a contiguous segment of the row, walked in chunks of 4 * 32
// elements (element c0 + 32k + lane in slot k of a lane, so loads are
// conflict-free).  Pass 1 (cdf_totals): each lane sums its elements, one
// butterfly gives the warp's total, kept in red_d[warp] with the warp's last
// positive index in red_i[warp].  Pass 2 (cdf_search): only the warp holding
// the target re-walks its segment, skipping whole chunks by their totals, and
// scans inside the one chunk that crosses.  The two passes are separate so a
// cluster can place the target between them.
__device__ __forceinline__ void cdf_segment(int V, int& s0, int& s1) {
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int seg = (V + nw - 1) / nw;
  seg = (seg + 127) & ~127;
  s0 = min(V, warp * seg);
  s1 = min(V, s0 + seg);
}

// Pass 1: returns the total weight and the last positive index (-1: none).
template <typename W>
__device__ void cdf_totals(const W& w, int V, RowSmem& sm, double& total, int& glast) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int s0, s1;
  cdf_segment(V, s0, s1);
  float lsum = 0.f;
  int last = -1;
  for (int c0 = s0; c0 < s1; c0 += 4 * 128) {
    float v[4][4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int i = c0 + 128 * q + 32 * k + lane;
        v[q][k] = i < s1 ? w(i) : 0.f;
      }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      lsum += (v[q][0] + v[q][1]) + (v[q][2] + v[q][3]);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (v[q][k] > 0.f) last = max(last, c0 + 128 * q + 32 * k + lane);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
  __syncthreads();  // earlier users of red_* are done
  if (lane == 0) {
    sm.red_d[warp] = (double)lsum;
    sm.red_i[warp] = last;
  }
  if (threadIdx.x == 0) sm.red_i[40] = -1;
  __syncthreads();
  total = 0.0;
  glast = -1;
  for (int k = 0; k < nw; ++k) {
    total += sm.red_d[k];
    glast = max(glast, sm.red_i[k]);
  }
}

// Pass 2, after cdf_totals with nothing in between touching red_*: the index
// where the running sum, starting at `base`, first exceeds `target`; the
// crossing warp's last positive index when rounding finds none inside it; -1
// when the target lies in no warp's range.
template <typename W>
__device__ int cdf_search(const W& w, int V, double base, double target, RowSmem& sm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int s0, s1;
  cdf_segment(V, s0, s1);
  auto chunk = [&](int c0, float (&v)[4]) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = c0 + 32 * k + lane;
      v[k] = i < s1 ? w(i) : 0.f;
    }
  };
  double before = base;
  for (int k = 0; k < warp; ++k) before += sm.red_d[k];
  const double wtot = sm.red_d[warp];
  const int last = sm.red_i[warp];
  if (wtot > 0.0 && before <= target && target < before + wtot) {
    double run = before;
    int found = last;  // rounding: the segment's last positive weight
    bool done = false;
    for (int c0 = s0; c0 < s1 && !done; c0 += 4 * 128) {
      float v[4][4], t[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        chunk(c0 + 128 * q, v[q]);
        t[q] = (v[q][0] + v[q][1]) + (v[q][2] + v[q][3]);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int q = 0; q < 4; ++q) t[q] += __shfl_xor_sync(0xffffffffu, t[q], o);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (done) break;
        if (run + (double)t[q] <= target) {
          run += (double)t[q];
          continue;
        }
        // crossing chunk: slot by slot, an inclusive lane scan of each
        const int cq = c0 + 128 * q;
        int hit = -1, lp = -1;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float incl = v[q][k];
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
          }
          const unsigned hb =
              __ballot_sync(0xffffffffu, v[q][k] > 0.f && run + (double)incl > target);
          if (v[q][k] > 0.f) lp = cq + 32 * k + lane;
          if (hit < 0 && hb) hit = cq + 32 * k + (__ffs(hb) - 1);
          run += (double)__shfl_sync(0xffffffffu, incl, 31);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) lp = max(lp, __shfl_xor_sync(0xffffffffu, lp, o));
        // rounding inside the chunk: its last positive weight
        found = hit >= 0 ? hit : (lp >= 0 ? lp : found);
        done = true;
      }
    }
    if (lane == 0) sm.red_i[40] = found;
  }
  __syncthreads();
  const int res = sm.red_i[40];
  __syncthreads();
  return res;
}

template <typename W>
__device__ int inverse_cdf(const W& w, int V, float u, RowSmem& sm) {
  double total;
  int glast;
  cdf_totals(w, V, sm, total, glast);
  int res = cdf_search(w, V, 0.0, (double)u * total, sm);
  if (res < 0) res = glast;
  if (res < 0) res = 0;
  return res;
}

// Histogram area (32-bit words): per-warp radix histograms or the linear
// bins and candidate keys, whichever is larger.
__host__ __device__ constexpr int hist_words(int nw) {
  return nw * kHistBins > kLinWords ? nw * kHistBins : kLinWords;
}

__device__ void setup_smem(RowSmem& sm, int V, bool stage) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int nw = blockDim.x >> 5;
  unsigned char* p = smem_raw;
  sm.red_d = reinterpret_cast<double*>(p);
  p += 64 * sizeof(double);
  sm.red = reinterpret_cast<float*>(p);
  p += 64 * sizeof(float);
  sm.red_i = reinterpret_cast<int*>(p);
  p += 64 * sizeof(int);
  sm.hist = reinterpret_cast<uint32_t*>(p);
  p += (size_t)hist_words(nw) * sizeof(uint32_t);
  sm.stage = stage ? reinterpret_cast<float*>(p) : nullptr;
  (void)V;
}

size_t smem_bytes(int threads, int V, bool stage) {
  size_t b = 64 * sizeof(double) + 64 * sizeof(float) + 64 * sizeof(int) +
             (size_t)hist_words(threads / 32) * sizeof(uint32_t);
  if (stage) b += (size_t)V * sizeof(float);
  return b;
}

// Loads a logits row into a Dist: staged (pre-divided by T) when it fits.
// Loads a logits row into a Dist: staged in shared memory (pre-divided by T)
// when it fits, computing the row max and first argmax on the way (returns
// true); otherwise the Dist reads global memory (returns false).
__device__ bool load_logits(Dist& d, const float* row, int V, float temp, RowSmem& sm) {
  d.mode = 0;
  d.temp = temp;
  if (sm.stage == nullptr) {
    d.row = row;
    d.divide = temp != 1.f;
    return false;
  }
  __syncthreads();  // previous users of the stage are done
  const bool div = temp != 1.f;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  auto note = [&](float v, int i) {
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  };
  if ((reinterpret_cast<uintptr_t>(row) & 15) == 0) {
    // float4 loads, 8 in flight per thread
    const float4* r4 = reinterpret_cast<const float4*>(row);
    float4* s4 = reinterpret_cast<float4*>(sm.stage);
    const int n4 = V >> 2;
    for (int base = threadIdx.x; base < n4; base += 8 * blockDim.x) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = base + u * blockDim.x;
        v[u] = i < n4 ? __ldg(r4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = base + u * blockDim.x;
        if (i < n4) {
          float4 w = v[u];
          if (div) {
            w.x = __fdiv_rn(w.x, temp);
            w.y = __fdiv_rn(w.y, temp);
            w.z = __fdiv_rn(w.z, temp);
            w.w = __fdiv_rn(w.w, temp);
          }
          s4[i] = w;
          note(w.x, 4 * i);
          note(w.y, 4 * i + 1);
          note(w.z, 4 * i + 2);
          note(w.w, 4 * i + 3);
        }
      }
    }
    for (int i = (n4 << 2) + threadIdx.x; i < V; i += blockDim.x) {
      const float v = __ldg(row + i);
      const float x = div ? __fdiv_rn(v, temp) : v;
      sm.stage[i] = x;
      note(x, i);
    }
  } else {
#pragma unroll 8
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float v = __ldg(row + i);
      const float x = div ? __fdiv_rn(v, temp) : v;
      sm.stage[i] = x;
      note(x, i);
    }
  }
  d.row = sm.stage;
  d.divide = false;
  float m;
  int am;
  block_argmax(best, bi, sm, m, am);  // its barriers also publish the stage
  d.m = m;
  d.argmax = am == 0x7fffffff ? 0 : am;
  return true;
}

// ---- K8: one draw per row ----------------------------------------------------
struct SampleArgs {
  const float* logits;
  int64_t stride;
  int V;
  const ms_sampling_params* params;
  const int32_t* pidx;
  uint32_t lane_id;
  int32_t* tokens;
  float* probs;
  ms_row_stats* stats;
  int32_t* scatter_dst;
  const int32_t* scatter_idx;
};

// Row r drawn by one CTA (staged in shared memory when sm.stage is set).
__device__ __forceinline__ void sample_row_body(const SampleArgs& a, int r, RowSmem& sm) {
  const float* __restrict__ logits = a.logits;
  const int64_t stride = a.stride;
  const int V = a.V;
  const uint32_t lane_id = a.lane_id;
  int32_t* __restrict__ tokens = a.tokens;
  float* __restrict__ probs = a.probs;
  ms_row_stats* __restrict__ stats = a.stats;
  int32_t* scatter_dst = a.scatter_dst;
  const int32_t* __restrict__ scatter_idx = a.scatter_idx;
  const ms_sampling_params P = a.params[a.pidx ? a.pidx[r] : r];
  const float* row = logits + (int64_t)r * stride;
  Dist d;
  int token;
  if (P.temperature == 0.f) {
    d.row = row;
    d.mode = 0;
    d.divide = false;
    d.temp = 1.f;
    float m;
    int am;
    row_argmax(d, V, sm, m, am);
    d.mode = 2;
    d.argmax = am;
    d.m = m;
    d.thresh = m;
    d.z = 1.f;
    token = am;
  } else {
    const bool have_max = load_logits(d, row, V, P.temperature, sm);
    row_stats(d, V, P.top_k, P.top_p < 1.f ? P.top_p : 1.f, sm, have_max);
    const float u = philox_uniform(P.seed, P.step, lane_id);
    const Dist dv = d;
    token = inverse_cdf([dv](int i) { return dv.weight(i); }, V, u, sm);
  }
  if (threadIdx.x == 0) {
    tokens[r] = token;
    if (stats) stats[r] = ms_row_stats{d.m, d.thresh, d.z, d.argmax};
    if (scatter_dst && scatter_idx) scatter_dst[scatter_idx[r]] = token;
  }
  if (probs) {
    float* out = probs + (int64_t)r * V;
    for (int i = threadIdx.x; i < V; i += blockDim.x) out[i] = d.prob(i);
  }
}

__global__ void __launch_bounds__(1024, 1) sample_rows_kernel(SampleArgs a, int stage) {
  pdl_enter();
  RowSmem sm;
  setup_smem(sm, a.V, stage != 0);
  sample_row_body(a, blockIdx.x, sm);
}

// ---- K9: fused accept / resample / bonus, one CTA per request ---------------
struct AcceptArgs {
  const float* target;
  int64_t tstride;
  int target_probs;  // 1: target rows are probabilities
  const float* draft;
  int64_t dstride;
  const ms_row_stats* dstats;
  int draft_probs;  // 1: draft rows are probabilities
  const int32_t* proposals;
  const ms_sampling_params* params;  // nullable in probability mode
  const float* accept_u;             // explicit uniforms (nullable)
  const float* draw_u;
  int gamma, V;
  int32_t* out_tokens;
  int32_t* out_nacc;
  int* err;
};

// Request b of B, processed by one CTA (target rows staged when sm.stage is set).
__device__ __forceinline__ void accept_body(const AcceptArgs& a, int b, int B, RowSmem& sm) {
  const int V = a.V, G = a.gamma;
  ms_sampling_params P;
  if (a.params) {
    P = a.params[b];
  } else {
    P.temperature = 1.f;
    P.top_p = 1.f;
    P.top_k = 0;
    P.seed = 0;
    P.step = 0;
  }
  const bool greedy = a.params && P.temperature == 0.f;
  const float top_p = P.top_p < 1.f ? P.top_p : 1.f;
  int32_t* out = a.out_tokens + (int64_t)b * (G + 1);

  // Builds the target distribution for position i.
  auto target_dist = [&](int i, Dist& p) {
    const float* row = a.target + (int64_t)(b * (G + 1) + i) * a.tstride;
    if (a.target_probs) {
      p.row = row;
      p.mode = 1;
      p.divide = false;
      return;
    }
    if (greedy) {
      p.row = row;
      p.mode = 0;
      p.divide = false;
      p.temp = 1.f;
      float m;
      int am;
      row_argmax(p, V, sm, m, am);
      p.mode = 2;
      p.argmax = am;
      return;
    }
    const bool have_max = load_logits(p, row, V, P.temperature, sm);
    row_stats(p, V, P.top_k, top_p, sm, have_max);
  };
  // Builds the draft distribution for position i (never staged).
  auto draft_dist = [&](int i, Dist& q) {
    const int r = i * B + b;  // position-major: row of (b, i)
    const float* row = a.draft + (int64_t)r * a.dstride;
    q.row = row;
    if (a.draft_probs) {
      q.mode = 1;
      q.divide = false;
      return;
    }
    q.temp = greedy ? 1.f : P.temperature;
    q.divide = !greedy && P.temperature != 1.f;
    if (a.dstats) {
      const ms_row_stats s = a.dstats[r];
      q.m = s.max;
      q.thresh = s.thresh;
      q.z = s.z;
      q.inv_z = 1.f / s.z;
      q.argmax = s.argmax;
      q.mode = greedy ? 2 : 0;
      return;
    }
    q.mode = 0;
    if (greedy) {
      float m;
      int am;
      row_argmax(q, V, sm, m, am);
      q.mode = 2;
      q.argmax = am;
      return;
    }
    row_stats(q, V, P.top_k, top_p, sm, false);
  };

  for (int i = 0; i < G; ++i) {
    Dist p, q;
    target_dist(i, p);
    draft_dist(i, q);
    int x = a.proposals[i * B + b];
    if (x < 0 || x >= V) {
      if (threadIdx.x == 0) raise_device_error(a.err, kErrToken);
      x = 0;
    }
    const float px = p.prob(x);
    const float qx = q.prob(x);
    const float ratio = fminf(__fdiv_rn(px, fmaxf(qx, 1e-10f)), 1.f);
    const float u = a.accept_u ? a.accept_u[i * B + b]
                               : philox_uniform(P.seed, P.step, MS_LANE_ACCEPT + i);
    if (u < ratio) {
      if (threadIdx.x == 0) out[i] = x;
      continue;
    }
    // Rejected: draw from normalise(max(0, p - q)), or from p if that is ~0.
    // With the target row staged, the residual replaces it in shared memory
    // (each thread overwrites only the entries it has just read), so the
    // draw walks shared memory instead of evaluating both rows again.
    const Dist pv = p, qv = q;
    const bool in_smem = p.mode == 0 && sm.stage != nullptr && p.row == sm.stage;
    float part = 0.f;
    if (in_smem) {
      part = residual_pass(sm.stage, V, 0, pv, qv, qv.row);
    } else {
#pragma unroll 4
      for (int j = threadIdx.x; j < V; j += blockDim.x) part += fmaxf(pv.prob(j) - qv.prob(j), 0.f);
    }
    const float total = block_sum_b(part, sm);  // its barriers also publish the residual
    const float u2 = a.draw_u ? a.draw_u[b] : philox_uniform(P.seed, P.step, MS_LANE_RESAMPLE);
    int tok;
    if (total <= 1e-9f) {
      if (in_smem) {  // the residual overwrote p's staged row: stage it again
        Dist again;
        load_logits(again, a.target + (int64_t)(b * (G + 1) + i) * a.tstride, V, P.temperature, sm);
      }
      tok = inverse_cdf([pv](int j) { return pv.prob(j); }, V, u2, sm);
    } else if (in_smem) {
      const float* res = sm.stage;
      tok = inverse_cdf([res](int j) { return res[j]; }, V, u2, sm);
    } else {
      tok = inverse_cdf([pv, qv](int j) { return fmaxf(pv.prob(j) - qv.prob(j), 0.f); }, V, u2, sm);
    }
    if (threadIdx.x == 0) {
      out[i] = tok;
      a.out_nacc[b] = i;
    }
    return;
  }
  // Every proposal survived: the bonus token comes from p[gamma].
  Dist p;
  target_dist(G, p);
  const float u2 = a.draw_u ? a.draw_u[b] : philox_uniform(P.seed, P.step, MS_LANE_RESAMPLE);
  const Dist pv = p;
  const int tok = inverse_cdf([pv](int j) { return pv.weight(j); }, V, u2, sm);
  if (threadIdx.x == 0) {
    out[G] = tok;
    a.out_nacc[b] = G;
  }
}

__global__ void __launch_bounds__(1024, 1) spec_accept_kernel(AcceptArgs a, int stage) {
  pdl_enter();
  RowSmem sm;
  setup_smem(sm, a.V, stage != 0);
  accept_body(a, blockIdx.x, gridDim.x, sm);
}

// ---- cluster sampling: one thread-block cluster per row or request -------------
// A cluster of C CTAs shares a row: CTA k stages the slice [k*S, k*S + S) of
// the row, divided by the temperature, in its own shared memory, so the row
// is read from global memory once and every later pass is a shared-memory
// pass over V/C elements on C SMs.  Row-wide quantities (maximum, kept mass,
// mass bins, candidates, draw totals) are combined through distributed shared
// memory: every CTA publishes its part, all pass a cluster barrier, and every
// CTA reads all parts in rank order and combines them the same way.  Every
// CTA therefore reaches the same decisions and passes the same barriers.
//
// Top-p uses the linear mass bins of the single-CTA path summed over the
// cluster (CTA k sums bins [k*nb/C, (k+1)*nb/C) over all CTAs and writes the
// sums into every CTA), then, when the crossing bin holds more than kClCand
// elements, a second level of kSubBins sub-bins inside it.  Top-k rows, and
// rows whose crossing sub-bin still holds too many elements (flat or tied
// rows), are left to CTA 0 running the single-CTA code on global memory.
constexpr int kClThreads = 256;
constexpr int kClCand = 512;
constexpr int kSubBins = 256;
constexpr int kClMinV = kMaxStagedV + 1;  // rows one CTA can stage stay on one CTA
constexpr int kClMaxSlice = 32768;   // floats of one CTA's slice
// 32-bit words: region A = local bins (counts, deficits) + local candidate
// keys; region B = combined bin masses + counts.
constexpr int kClRegionA = 2 * kLinBins + 2 * kClCand;
constexpr int kClRegionB = 2 * kLinBins;
constexpr size_t kClFixedBytes = 64 * sizeof(double) + 64 * sizeof(float) + 64 * sizeof(int) +
                                 16 * sizeof(unsigned long long) +
                                 (size_t)(kClRegionA + kClRegionB) * sizeof(uint32_t);
static_assert(kClFixedBytes % 16 == 0, "the slice must start 16-byte aligned");
static_assert(kClRegionA >= (kClThreads / 32) * kHistBins, "single-CTA radix histograms");
static_assert(kLinBins % kClThreads == 0 && kSubBins % kClThreads == 0, "bins per thread");

struct ClSmem {
  RowSmem row;               // red_*; row.hist = region A (single-CTA code); row.stage = null
  unsigned long long* xch;   // two sets of 8 exchange words, used alternately
  uint32_t* hc;              // region A: local bin counts
  uint32_t* hd;              // region A: local bin deficits
  unsigned long long* kl;    // region A: this CTA's candidate keys
  unsigned long long* km;    // over hc once the bins are combined: every CTA's candidates
  unsigned long long* ks;    // over hc: the candidates ranked
  float* hm;                 // region B: combined bin masses
  uint32_t* hn;              // region B: combined bin counts (candidate prefix masses later)
  float* xs;                 // the slice
};

__device__ __forceinline__ void cl_setup(ClSmem& s) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* p = smem_raw;
  s.row.red_d = reinterpret_cast<double*>(p);
  p += 64 * sizeof(double);
  s.row.red = reinterpret_cast<float*>(p);
  p += 64 * sizeof(float);
  s.row.red_i = reinterpret_cast<int*>(p);
  p += 64 * sizeof(int);
  s.xch = reinterpret_cast<unsigned long long*>(p);
  p += 16 * sizeof(unsigned long long);
  uint32_t* A = reinterpret_cast<uint32_t*>(p);
  p += (size_t)kClRegionA * sizeof(uint32_t);
  uint32_t* Bw = reinterpret_cast<uint32_t*>(p);
  p += (size_t)kClRegionB * sizeof(uint32_t);
  s.row.hist = A;
  s.row.stage = nullptr;
  s.hc = A;
  s.hd = A + kLinBins;
  s.kl = reinterpret_cast<unsigned long long*>(A + 2 * kLinBins);
  s.km = reinterpret_cast<unsigned long long*>(A);
  s.ks = s.km + kClCand;
  s.hm = reinterpret_cast<float*>(Bw);
  s.hn = Bw + kLinBins;
  s.xs = reinterpret_cast<float*>(p);
}

__device__ __forceinline__ void cl_sync() { cg::this_cluster().sync(); }
template <typename T>
__device__ __forceinline__ T* cl_map(T* p, int rank) {
  return cg::this_cluster().map_shared_rank(p, (unsigned int)rank);
}

// Exchange state: the CTA's rank, the cluster size and which word set is next.
// A set written at exchange k was last read before the barrier of exchange
// k-1, so alternating two sets needs one barrier per exchange.
template <int C>
struct ClX {
  int rank, par;
  __device__ __forceinline__ unsigned long long* slot(ClSmem& s) const { return s.xch + 8 * par; }
};

// Stages [lo, lo + n) of `row` (divided by temp when div) into xs and returns
// the slice's maximum and first argmax (row index) to every thread.
__device__ void cl_stage(const float* __restrict__ row, int lo, int n, float temp, bool div,
                         float* xs, RowSmem& sm, float& m, int& am) {
  float best = -INFINITY;
  int bi = 0x7fffffff;
  auto note = [&](float v, int i) {
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  };
  const float* src = row + lo;
  if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    const float4* r4 = reinterpret_cast<const float4*>(src);
    float4* s4 = reinterpret_cast<float4*>(xs);
    const int n4 = n >> 2;
    for (int base = threadIdx.x; base < n4; base += 8 * blockDim.x) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = base + u * blockDim.x;
        v[u] = i < n4 ? __ldg(r4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = base + u * blockDim.x;
        if (i < n4) {
          float4 w = v[u];
          if (div) {
            w.x = __fdiv_rn(w.x, temp);
            w.y = __fdiv_rn(w.y, temp);
            w.z = __fdiv_rn(w.z, temp);
            w.w = __fdiv_rn(w.w, temp);
          }
          s4[i] = w;
          note(w.x, lo + 4 * i);
          note(w.y, lo + 4 * i + 1);
          note(w.z, lo + 4 * i + 2);
          note(w.w, lo + 4 * i + 3);
        }
      }
    }
    for (int i = (n4 << 2) + threadIdx.x; i < n; i += blockDim.x) {
      const float v = __ldg(src + i);
      const float x = div ? __fdiv_rn(v, temp) : v;
      xs[i] = x;
      note(x, lo + i);
    }
  } else {
#pragma unroll 8
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const float v = __ldg(src + i);
      const float x = div ? __fdiv_rn(v, temp) : v;
      xs[i] = x;
      note(x, lo + i);
    }
  }
  block_argmax(best, bi, sm, m, am);  // its barriers also publish the slice
}

// Row maximum and first argmax from every CTA's slice result.
template <int C>
__device__ void cl_argmax(ClSmem& s, ClX<C>& x, float mloc, int aloc, float& m, int& am) {
  unsigned long long* slot = x.slot(s);
  if (threadIdx.x == 0) {
    slot[0] = __float_as_uint(mloc);
    slot[1] = (uint32_t)aloc;
  }
  cl_sync();
  float best = -INFINITY;
  int bi = 0x7fffffff;
#pragma unroll
  for (int r = 0; r < C; ++r) {
    const unsigned long long* rs = cl_map(slot, r);
    const float v = __uint_as_float((uint32_t)rs[0]);
    const int i = (int)(uint32_t)rs[1];
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
  x.par ^= 1;
  m = best;
  am = bi == 0x7fffffff ? 0 : bi;
}

// Sum of every CTA's (block-uniform) float, in rank order.
template <int C>
__device__ float cl_sum(ClSmem& s, ClX<C>& x, float v) {
  unsigned long long* slot = x.slot(s);
  if (threadIdx.x == 0) slot[0] = __float_as_uint(v);
  cl_sync();
  float t = 0.f;
#pragma unroll
  for (int r = 0; r < C; ++r) t += __uint_as_float((uint32_t)cl_map(slot, r)[0]);
  x.par ^= 1;
  return t;
}

// The slice's kept mass sum exp(x - m) over x >= thresh; with kBins, also
// the linear mass bins (counts and deficits) of those elements.
template <bool kBins>
__device__ float cl_mass_pass(const float* xs, int n, float m, float thresh, ClSmem& s) {
  if (kBins) {
    for (int i = threadIdx.x; i < 2 * kLinBins; i += blockDim.x) s.hc[i] = 0u;
    __syncthreads();
  }
  float zl = 0.f;
  auto note = [&](float xv) {
    if (xv >= thresh) {
      zl += __expf(xv - m);
      if (kBins) {
        const int b = lin_bin(m, xv);
        atomicAdd(&s.hc[b], 1u);
        atomicAdd(&s.hd[b], lin_deficit(m, xv, b));
      }
    }
  };
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  const int n4 = n >> 2;
  int i = threadIdx.x;
  for (; i + (int)blockDim.x < n4; i += 2 * blockDim.x) {
    const float4 a = x4[i], b = x4[i + blockDim.x];
    note(a.x);
    note(a.y);
    note(a.z);
    note(a.w);
    note(b.x);
    note(b.y);
    note(b.z);
    note(b.w);
  }
  for (; i < n4; i += blockDim.x) {
    const float4 a = x4[i];
    note(a.x);
    note(a.y);
    note(a.z);
    note(a.w);
  }
  for (int j = (n4 << 2) + threadIdx.x; j < n; j += blockDim.x) note(xs[j]);
  return block_sum_b(zl, s.row);  // its barriers also complete the bins
}

// Second-level bins of the elements in first-level bin b1: sub-bin
// floor(frac(t) * kSubBins) of t = (m - x) * kBinsPerUnit, with deficits
// against the sub-bin's upper edge, in hc / hd [0, kSubBins).
__device__ __forceinline__ int sub_bin(float m, float x, int b1) {
  const float t = (m - x) * kBinsPerUnit;
  const int s = (int)((t - (float)b1) * (float)kSubBins);
  return s < kSubBins - 1 ? s : kSubBins - 1;
}
__device__ void cl_sub_pass(const float* xs, int n, float m, int b1, ClSmem& s) {
  for (int i = threadIdx.x; i < kSubBins; i += blockDim.x) {
    s.hc[i] = 0u;
    s.hd[i] = 0u;
  }
  __syncthreads();
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const float xv = xs[j];
    if (xv >= -INFINITY && lin_bin(m, xv) == b1) {
      const int sb = sub_bin(m, xv, b1);
      const float edge = (float)b1 + (float)sb * (1.f / kSubBins);
      const float r = __expf((xv - m) + edge * (1.f / kBinsPerUnit));
      atomicAdd(&s.hc[sb], 1u);
      atomicAdd(&s.hd[sb], __float2uint_rn(fmaxf(1.f - r, 0.f) * kDefScale));
    }
  }
  __syncthreads();
}

// After a cluster barrier that follows every CTA's bin pass: CTA `rank` sums
// bins [rank*nb/C, (rank+1)*nb/C) over all CTAs and writes the mass and count
// of each into every CTA's hm / hn.  Bin b's upper edge lies (e0 + b * ew) /
// kBinsPerUnit below the maximum.  Ends with a cluster barrier.
template <int C>
__device__ void cl_combine_bins(ClSmem& s, const ClX<C>& x, int nb, float e0, float ew) {
  const int per = nb / C;
  for (int j = threadIdx.x; j < per; j += blockDim.x) {
    const int b = x.rank * per + j;
    double acc = 0.0;
    uint32_t cnt = 0;
#pragma unroll
    for (int r = 0; r < C; ++r) {
      const uint32_t c = cl_map(s.hc, r)[b];
      const uint32_t d = cl_map(s.hd, r)[b];
      cnt += c;
      acc += (double)c - (double)d * (1.0 / kDefScale);
    }
    const float mass = (float)acc * __expf(-(e0 + (float)b * ew) * (1.f / kBinsPerUnit));
#pragma unroll
    for (int r = 0; r < C; ++r) {
      cl_map(s.hm, r)[b] = mass;
      cl_map(s.hn, r)[b] = cnt;
    }
  }
  cl_sync();
}

// First bin of hm[0, nb) whose inclusive mass prefix, starting at `base`,
// reaches `target` (-1 if none); `before` = the prefix before that bin.
__device__ int cl_find(const float* hm, int nb, double base, double target, RowSmem& sm,
                       double& before) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int per = nb / blockDim.x;
  const int b0 = threadIdx.x * per;
  double own = 0.0;
  for (int j = 0; j < per; ++j) own += (double)hm[b0 + j];
  double inc = own;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += t;
  }
  __syncthreads();
  if (lane == 31) sm.red_d[warp] = inc;
  if (threadIdx.x == 0) sm.red_i[48] = -1;
  __syncthreads();
  double wb = base;
  for (int w = 0; w < warp && w < nw; ++w) wb += sm.red_d[w];
  const double ex = wb + inc - own;
  if (ex < target && ex + own >= target) {
    double a = ex;
    for (int j = 0; j < per; ++j) {
      const double h = (double)hm[b0 + j];
      if (a + h >= target) {
        sm.red_i[48] = b0 + j;
        sm.red_d[48] = a;
        break;
      }
      a += h;
    }
  }
  __syncthreads();
  const int bin = sm.red_i[48];
  before = sm.red_d[48];
  __syncthreads();
  return bin;
}

// This slice's candidates: elements in bin b1 (and sub-bin sb when sb >= 0),
// as sort keys in kl (the first kClCand of them); returns their number.
__device__ int cl_gather(const float* xs, int n, int lo, float m, int b1, int sb, ClSmem& s) {
  if (threadIdx.x == 0) s.row.red_i[50] = 0;
  __syncthreads();
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const float xv = xs[j];
    if (xv >= -INFINITY && lin_bin(m, xv) == b1 && (sb < 0 || sub_bin(m, xv, b1) == sb)) {
      const int slot = atomicAdd(&s.row.red_i[50], 1);
      if (slot < kClCand)
        s.kl[slot] = ((unsigned long long)fkey(xv) << 32) | (uint32_t)~(uint32_t)(lo + j);
    }
  }
  __syncthreads();
  const int cnt = s.row.red_i[50];
  __syncthreads();
  return cnt;
}

// The top-p crossing among the ranked candidates ks[0, n), their exact
// masses accumulated from `before`: the cut value and the mass kept at and
// above it (ties kept).  False when rounding finds no crossing.
__device__ bool cl_cross(ClSmem& s, int n, float m, double before, double target, float& cut,
                         double& z_keep) {
  RowSmem& sm = s.row;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  double* cum_of = reinterpret_cast<double*>(s.hn);  // n <= kClCand doubles
  if (threadIdx.x == 0) sm.red_i[51] = 0x7fffffff;
  double carry = before;
  for (int base = 0; base < n; base += blockDim.x) {
    const int c = base + threadIdx.x;
    const float xc = c < n ? kfloat((uint32_t)(s.ks[c] >> 32)) : -INFINITY;
    const double e = c < n ? (double)__expf(xc - m) : 0.0;
    double inc = e;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double t = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += t;
    }
    __syncthreads();
    if (lane == 31) sm.red_d[warp] = inc;
    __syncthreads();
    double wb = carry, all = carry;
    for (int w = 0; w < nw; ++w) {
      if (w < warp) wb += sm.red_d[w];
      all += sm.red_d[w];
    }
    const double cum = wb + inc;
    if (c < n) {
      cum_of[c] = cum;
      if (cum - e < target && cum >= target) atomicMin(&sm.red_i[51], c);
    }
    carry = all;
  }
  __syncthreads();
  const int cross = sm.red_i[51];
  if (cross >= n) {
    __syncthreads();
    return false;
  }
  cut = kfloat((uint32_t)(s.ks[cross] >> 32));
  for (int c = cross + threadIdx.x; c < n; c += blockDim.x) {
    const float xc = kfloat((uint32_t)(s.ks[c] >> 32));
    if (xc == cut && (c + 1 == n || kfloat((uint32_t)(s.ks[c + 1] >> 32)) < cut))
      sm.red_d[49] = cum_of[c];
  }
  __syncthreads();
  z_keep = sm.red_d[49];
  __syncthreads();
  return true;
}

// Fills d.thresh, d.z, d.inv_z of a staged logits row (temperature > 0, no
// top-k) whose d.m is the row maximum.  Returns false when the row needs the
// single-CTA path; the answer is the same in every CTA of the cluster.
template <int C>
__device__ bool cl_row_stats(Dist& d, float top_p, int n, int lo, ClSmem& s, ClX<C>& x) {
  const float m = d.m;
  d.thresh = -INFINITY;
  const bool want_p = top_p < 1.f;
  const float zloc = want_p ? cl_mass_pass<true>(s.xs, n, m, -INFINITY, s)
                            : cl_mass_pass<false>(s.xs, n, m, -INFINITY, s);
  d.z = cl_sum(s, x, zloc);  // its barrier also completes every CTA's bins
  d.inv_z = 1.f / d.z;
  if (!want_p) return true;
  if (1.f >= top_p * d.z) {  // the maximum alone already covers top_p
    d.thresh = m;
    d.z = cl_sum(s, x, cl_mass_pass<false>(s.xs, n, m, m, s));
    d.inv_z = 1.f / d.z;
    return true;
  }
  const double target = (double)top_p * (double)d.z;
  cl_combine_bins(s, x, kLinBins, 0.f, 1.f);
  double before;
  const int b1 = cl_find(s.hm, kLinBins, 0.0, target, s.row, before);
  if (b1 < 0 || b1 >= kLinBins - 1) return false;
  int sb = -1;
  if (s.hn[b1] > (uint32_t)kClCand) {
    cl_sub_pass(s.xs, n, m, b1, s);
    cl_sync();  // every CTA's sub-bins are complete; hm / hn have been read
    cl_combine_bins(s, x, kSubBins, (float)b1, 1.f / kSubBins);
    double before2;
    sb = cl_find(s.hm, kSubBins, before, target, s.row, before2);
    if (sb < 0 || s.hn[sb] > (uint32_t)kClCand) return false;
    before = before2;
  }
  const int nloc = cl_gather(s.xs, n, lo, m, b1, sb, s);
  unsigned long long* slot = x.slot(s);
  if (threadIdx.x == 0) slot[0] = (uint32_t)nloc;
  cl_sync();
  int cnt[8], total = 0;
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    cnt[r] = r < C ? (int)cl_map(slot, r)[0] : 0;
    total += cnt[r];
  }
  x.par ^= 1;
  if (total > kClCand || total == 0) return false;
  int off = 0;
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    if (r < C) {
      const unsigned long long* rk = cl_map(s.kl, r);
      for (int j = threadIdx.x; j < cnt[r]; j += blockDim.x) s.km[off + j] = rk[j];
      off += cnt[r];
    }
  }
  __syncthreads();
  rank_keys_desc(s.km, s.ks, total);
  float cut;
  double zk;
  if (!cl_cross(s, total, m, before, target, cut, zk)) return false;
  if (cut > d.thresh) {
    d.thresh = cut;
    d.z = (float)zk;
    d.inv_z = 1.f / d.z;
  }
  return true;
}

// Inverse-CDF draw over the cluster: slice totals, a rank-order exchange that
// places u * total in one CTA (the owner), then the owner's in-slice search.
// Ends every DSMEM use with a cluster barrier, so CTAs may exit afterwards.
// `mine` tells the one CTA that holds the drawn token.
template <int C, typename W>
__device__ void cl_draw(const W& w, int n, int lo, float u, ClSmem& s, ClX<C>& x, int& tok,
                        bool& mine) {
  double tot;
  int last;
  cdf_totals(w, n, s.row, tot, last);
  unsigned long long* slot = x.slot(s);
  if (threadIdx.x == 0) {
    slot[0] = (unsigned long long)__double_as_longlong(tot);
    slot[1] = (uint32_t)(last >= 0 ? lo + last : -1);
  }
  cl_sync();
  double T[8];
  double total = 0.0;
  int glast = -1;
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    T[r] = 0.0;
    if (r < C) {
      const unsigned long long* rs = cl_map(slot, r);
      T[r] = __longlong_as_double((long long)rs[0]);
      total += T[r];
      glast = max(glast, (int)(uint32_t)rs[1]);
    }
  }
  x.par ^= 1;
  cl_sync();  // every CTA has read every slot: no DSMEM access after this
  const double target = (double)u * total;
  int owner = -1;
  double obase = 0.0, before = 0.0;
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    if (r < C) {
      if (owner < 0 && T[r] > 0.0 && before <= target && target < before + T[r]) {
        owner = r;
        obase = before;
      }
      before += T[r];
    }
  }
  mine = false;
  tok = 0;
  if (owner == x.rank) {
    int idx = cdf_search(w, n, obase, target, s.row);
    if (idx < 0) idx = last;
    tok = idx >= 0 ? lo + idx : (glast >= 0 ? glast : 0);
    mine = true;
  } else if (owner < 0 && x.rank == 0) {
    tok = glast >= 0 ? glast : 0;
    mine = true;
  }
}

// The single-CTA paths for rows the cluster leaves to CTA 0 (shared memory
// set up without a staged row: they read global memory).
__device__ __noinline__ void sample_row_single(SampleArgs a, int r, RowSmem sm) {
  sample_row_body(a, r, sm);
}
__device__ __noinline__ void accept_single(AcceptArgs a, int b, int B, RowSmem sm) {
  accept_body(a, b, B, sm);
}

template <int C>
__device__ __forceinline__ ClX<C> cl_begin(int S, int V, int& lo, int& n) {
  ClX<C> x;
  x.rank = (int)cg::this_cluster().block_rank();
  x.par = 0;
  lo = min(V, x.rank * S);
  n = min(V, lo + S) - lo;
  return x;
}

// ---- K8 on a cluster per row ----------------------------------------------------
template <int C>
__global__ void __cluster_dims__(C, 1, 1) __launch_bounds__(kClThreads, 2)
    sample_cluster_kernel(SampleArgs a, int S) {
  pdl_enter();
  ClSmem s;
  cl_setup(s);
  const int V = a.V;
  int lo, n;
  ClX<C> x = cl_begin<C>(S, V, lo, n);
  const int r = blockIdx.x / C;
  const ms_sampling_params P = a.params[a.pidx ? a.pidx[r] : r];
  const bool greedy = P.temperature == 0.f;
  if (!greedy && P.top_k > 0 && P.top_k < V) {  // top-k: CTA 0 alone, no cluster barrier
    if (x.rank == 0) sample_row_single(a, r, s.row);
    return;
  }
  const float temp = greedy ? 1.f : P.temperature;
  const float* row = a.logits + (int64_t)r * a.stride;
  float mloc;
  int aloc;
  cl_stage(row, lo, n, temp, !greedy && temp != 1.f, s.xs, s.row, mloc, aloc);
  Dist d;
  d.row = row;
  d.mode = 0;
  d.divide = false;
  d.temp = temp;
  cl_argmax(s, x, mloc, aloc, d.m, d.argmax);
  int tok;
  bool mine;
  if (greedy) {
    cl_sync();  // every CTA has read every slot
    d.mode = 2;
    d.thresh = d.m;
    d.z = 1.f;
    d.inv_z = 1.f;
    tok = d.argmax;
    mine = x.rank == 0;
  } else {
    if (!cl_row_stats(d, P.top_p < 1.f ? P.top_p : 1.f, n, lo, s, x)) {
      cl_sync();  // nobody reads this cluster's shared memory any more
      if (x.rank == 0) sample_row_single(a, r, s.row);
      return;
    }
    const float u = philox_uniform(P.seed, P.step, a.lane_id);
    const float* xs = s.xs;
    const float m = d.m, th = d.thresh;
    cl_draw([xs, m, th](int j) { const float v = xs[j]; return v >= th ? __expf(v - m) : 0.f; }, n,
            lo, u, s, x, tok, mine);
  }
  if (threadIdx.x == 0) {
    if (mine) {
      a.tokens[r] = tok;
      if (a.scatter_dst && a.scatter_idx) a.scatter_dst[a.scatter_idx[r]] = tok;
    }
    if (x.rank == 0 && a.stats) a.stats[r] = ms_row_stats{d.m, d.thresh, d.z, d.argmax};
  }
  if (a.probs) {
    float* out = a.probs + (int64_t)r * V + lo;
    const float* xs = s.xs;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
      float pr;
      if (d.mode == 2) {
        pr = lo + j == d.argmax ? 1.f : 0.f;
      } else {
        const float v = xs[j];
        pr = v >= d.thresh ? __expf(v - d.m) * d.inv_z : 0.f;
      }
      out[j] = pr;
    }
  }
}

// ---- K9 on a cluster per request ------------------------------------------------
// Target rows staged slice-wise; draft rows come with their statistics
// (ms_row_stats from the draft draws) and are read from global memory.
template <int C>
__global__ void __cluster_dims__(C, 1, 1) __launch_bounds__(kClThreads, 2)
    accept_cluster_kernel(AcceptArgs a, int S) {
  pdl_enter();
  ClSmem s;
  cl_setup(s);
  const int V = a.V, G = a.gamma;
  int lo, n;
  ClX<C> x = cl_begin<C>(S, V, lo, n);
  const int B = gridDim.x / C;
  const int b = blockIdx.x / C;
  const ms_sampling_params P = a.params[b];
  const bool greedy = P.temperature == 0.f;
  if (!greedy && P.top_k > 0 && P.top_k < V) {  // top-k: CTA 0 alone, no cluster barrier
    if (x.rank == 0) accept_single(a, b, B, s.row);
    return;
  }
  const float top_p = P.top_p < 1.f ? P.top_p : 1.f;
  const float temp = greedy ? 1.f : P.temperature;
  const bool div = !greedy && temp != 1.f;
  int32_t* out = a.out_tokens + (int64_t)b * (G + 1);
  const bool lead = x.rank == 0 && threadIdx.x == 0;

  // Target distribution of position i, staged; false: the single-CTA path.
  auto target_dist = [&](int i, Dist& p) -> bool {
    const float* row = a.target + (int64_t)(b * (G + 1) + i) * a.tstride;
    float mloc;
    int aloc;
    cl_stage(row, lo, n, temp, div, s.xs, s.row, mloc, aloc);
    p.row = row;
    p.divide = div;
    p.temp = temp;
    cl_argmax(s, x, mloc, aloc, p.m, p.argmax);
    if (greedy) {
      p.mode = 2;
      return true;
    }
    p.mode = 0;
    return cl_row_stats(p, top_p, n, lo, s, x);
  };
  const float* xs = s.xs;

  for (int i = 0; i < G; ++i) {
    Dist p;
    if (!target_dist(i, p)) {
      cl_sync();  // nobody reads this cluster's shared memory any more
      if (x.rank == 0) accept_single(a, b, B, s.row);
      return;
    }
    const int r = i * B + b;  // position-major: row of (b, i)
    const ms_row_stats st = a.dstats[r];
    Dist q;
    q.row = a.draft + (int64_t)r * a.dstride;
    q.temp = temp;
    q.divide = div;
    q.m = st.max;
    q.thresh = st.thresh;
    q.z = st.z;
    q.inv_z = 1.f / st.z;
    q.argmax = st.argmax;
    q.mode = greedy ? 2 : 0;
    int tokx = a.proposals[i * B + b];
    if (tokx < 0 || tokx >= V) {
      if (lead) raise_device_error(a.err, kErrToken);
      tokx = 0;
    }
    const float px = p.prob(tokx);
    const float qx = q.prob(tokx);
    const float ratio = fminf(__fdiv_rn(px, fmaxf(qx, 1e-10f)), 1.f);
    const float u = a.accept_u ? a.accept_u[i * B + b]
                               : philox_uniform(P.seed, P.step, MS_LANE_ACCEPT + i);
    if (u < ratio) {
      if (lead) out[i] = tokx;
      continue;
    }
    // Rejected: draw from normalise(max(0, p - q)), or from p if that is ~0;
    // the residual replaces the staged slice.
    const Dist pv = p, qv = q;
    const float part = residual_pass(s.xs, n, lo, pv, qv, qv.row + lo);
    const float total = cl_sum(s, x, block_sum_b(part, s.row));
    const float u2 = a.draw_u ? a.draw_u[b] : philox_uniform(P.seed, P.step, MS_LANE_RESAMPLE);
    int tok;
    bool mine;
    if (total <= 1e-9f) {  // the residual overwrote p's slice: stage it again
      float ml;
      int al;
      cl_stage(pv.row, lo, n, temp, div, s.xs, s.row, ml, al);
      cl_draw([xs, pv, lo](int j) {
                if (pv.mode == 2) return lo + j == pv.argmax ? 1.f : 0.f;
                const float v = xs[j];
                return v >= pv.thresh ? __expf(v - pv.m) * pv.inv_z : 0.f;
              },
              n, lo, u2, s, x, tok, mine);
    } else {
      cl_draw([xs](int j) { return xs[j]; }, n, lo, u2, s, x, tok, mine);
    }
    if (threadIdx.x == 0) {
      if (mine) out[i] = tok;
      if (x.rank == 0) a.out_nacc[b] = i;
    }
    return;
  }
  // Every proposal survived: the bonus token comes from p[gamma].
  Dist p;
  if (!target_dist(G, p)) {
    cl_sync();
    if (x.rank == 0) accept_single(a, b, B, s.row);
    return;
  }
  if (greedy) {
    cl_sync();  // every CTA has read every slot
    if (lead) {
      out[G] = p.argmax;
      a.out_nacc[b] = G;
    }
    return;
  }
  const float u2 = a.draw_u ? a.draw_u[b] : philox_uniform(P.seed, P.step, MS_LANE_RESAMPLE);
  const float m = p.m, th = p.thresh;
  int tok;
  bool mine;
  cl_draw([xs, m, th](int j) { const float v = xs[j]; return v >= th ? __expf(v - m) : 0.f; }, n,
          lo, u2, s, x, tok, mine);
  if (threadIdx.x == 0) {
    if (mine) out[G] = tok;
    if (x.rank == 0) a.out_nacc[b] = G;
  }
}

// Cluster shape for a vocabulary: C CTAs of S (a multiple of 4) floats each;
// 0 when the row is better served by one CTA.
int cl_shape(int V, int& S) {
  if (V < kClMinV) return 0;
  const int C = V <= 65536 ? 4 : 8;
  S = ((V + C - 1) / C + 3) & ~3;
  return S <= kClMaxSlice ? C : 0;
}
size_t cl_smem(int S) { return kClFixedBytes + (size_t)S * sizeof(float); }

// Sets the kernel's shared-memory size and checks (once per kernel and size)
// that a cluster of that shape can be resident; false: use the single-CTA
// kernel.
template <typename K>
bool cl_prepare(K kernel, int C, size_t smem) {
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  static thread_local const void* seen_fn[4] = {nullptr, nullptr, nullptr, nullptr};
  static thread_local size_t seen_smem[4] = {0, 0, 0, 0};
  static thread_local bool seen_ok[4] = {false, false, false, false};
  static thread_local int next = 0;
  for (int i = 0; i < 4; ++i)
    if (seen_fn[i] == (const void*)kernel && seen_smem[i] == smem) return seen_ok[i];
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(C, 1, 1);
  cfg.blockDim = dim3(kClThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  int clusters = 0;
  const bool ok =
      cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) == cudaSuccess && clusters >= 1;
  if (!ok) (void)cudaGetLastError();
  seen_fn[next] = (const void*)kernel;
  seen_smem[next] = smem;
  seen_ok[next] = ok;
  next = (next + 1) & 3;
  return ok;
}

// Launches K8 / K9 on clusters when the vocabulary suits them; returns
// MS_ERR_UNSUPPORTED (nothing launched) otherwise.
int launch_sample_cluster(const SampleArgs& a, int n_rows, cudaStream_t st) {
  int S = 0;
  const int C = cl_shape(a.V, S);
  if (C == 0) return MS_ERR_UNSUPPORTED;
  const size_t smem = cl_smem(S);
  if (C == 4) {
    if (!cl_prepare(sample_cluster_kernel<4>, 4, smem)) return MS_ERR_UNSUPPORTED;
    launch_pdl(sample_cluster_kernel<4>, n_rows * 4, kClThreads, smem, st, a, S);
  } else {
    if (!cl_prepare(sample_cluster_kernel<8>, 8, smem)) return MS_ERR_UNSUPPORTED;
    launch_pdl(sample_cluster_kernel<8>, n_rows * 8, kClThreads, smem, st, a, S);
  }
  return check_launch("sample_cluster_kernel");
}

int launch_accept_cluster(const AcceptArgs& a, int B, cudaStream_t st) {
  if (a.target_probs || a.draft_probs || !a.dstats || !a.params) return MS_ERR_UNSUPPORTED;
  int S = 0;
  const int C = cl_shape(a.V, S);
  if (C == 0) return MS_ERR_UNSUPPORTED;
  const size_t smem = cl_smem(S);
  if (C == 4) {
    if (!cl_prepare(accept_cluster_kernel<4>, 4, smem)) return MS_ERR_UNSUPPORTED;
    launch_pdl(accept_cluster_kernel<4>, B * 4, kClThreads, smem, st, a, S);
  } else {
    if (!cl_prepare(accept_cluster_kernel<8>, 8, smem)) return MS_ERR_UNSUPPORTED;
    launch_pdl(accept_cluster_kernel<8>, B * 8, kClThreads, smem, st, a, S);
  }
  return check_launch("accept_cluster_kernel");
}

int row_threads(int V) {
  int t = ((V / 16) + 31) & ~31;
  if (t < 128) t = 128;
  if (t > 512) t = 512;
  return t;
}

// K8 at large vocabularies: 32 warps per SM hide the shared-memory and
// atomic latency of the row passes (256 rows x 32000: 69 -> 57 us with top-p,
// 46 -> 36 us without, against 512 threads).
int sample_threads(int V) { return V >= 16384 ? 1024 : row_threads(V); }
// K9 likewise (256 requests x gamma 4 x 32000, top-p 0.9: 257 -> 223 us).
int accept_threads(int V) { return V >= 16384 ? 1024 : row_threads(V); }

int launch_accept(AcceptArgs a, int B, void* stream) {
  a.err = device_error_word();
  const int threads = accept_threads(a.V);
  const bool stage = a.V <= kMaxStagedV && !a.target_probs;
  const size_t smem = smem_bytes(threads, a.V, stage);
  cudaError_t e = cudaFuncSetAttribute(spec_accept_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return fail(MS_ERR_CUDA, "spec_accept: smem attribute: %s", cudaGetErrorString(e));
  ProfScope prof(kClsAccept, as_stream(stream));
  const int rc = launch_accept_cluster(a, B, as_stream(stream));
  if (rc != MS_ERR_UNSUPPORTED) return rc;
  launch_pdl(spec_accept_kernel, B, threads, smem, as_stream(stream), a, stage ? 1 : 0);
  return check_launch("spec_accept_kernel");
}

}  // namespace
}  // namespace ms

using namespace ms;

extern "C" int ms_sample(const float* logits, int64_t row_stride, int n_rows, int vocab,
                         const ms_sampling_params* params, const int32_t* pidx, int lane,
                         int32_t* tokens, float* probs, ms_row_stats* stats, int32_t* scatter_dst,
                         const int32_t* scatter_idx, void* stream) {
  MS_REQUIRE(n_rows >= 0 && vocab > 0, "ms_sample: bad sizes rows=%d vocab=%d", n_rows, vocab);
  if (n_rows == 0) return MS_OK;
  MS_REQUIRE(logits && params && tokens, "ms_sample: null pointer");
  MS_REQUIRE(row_stride >= vocab, "ms_sample: row_stride < vocab");
  const int threads = sample_threads(vocab);
  const bool stage = vocab <= kMaxStagedV;
  const size_t smem = smem_bytes(threads, vocab, stage);
  cudaError_t e = cudaFuncSetAttribute(sample_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return fail(MS_ERR_CUDA, "ms_sample: smem attribute: %s", cudaGetErrorString(e));
  ProfScope prof(kClsSample, as_stream(stream));
  const SampleArgs a{logits, row_stride, vocab, params, pidx, (uint32_t)lane, tokens, probs, stats,
                     scatter_dst, scatter_idx};
  const int rc = launch_sample_cluster(a, n_rows, as_stream(stream));
  if (rc != MS_ERR_UNSUPPORTED) return rc;
  launch_pdl(sample_rows_kernel, n_rows, threads, smem, as_stream(stream), a, stage ? 1 : 0);
  return check_launch("sample_rows_kernel");
}

extern "C" int ms_spec_accept(const float* target_logits, int64_t target_stride,
                              const float* draft_rows, int64_t draft_stride,
                              const ms_row_stats* draft_stats, int draft_probs_mode,
                              const int32_t* proposals, const ms_sampling_params* params,
                              int n_requests, int gamma, int vocab, int32_t* out_tokens,
                              int32_t* out_num_accepted, void* stream) {
  MS_REQUIRE(n_requests >= 0 && gamma >= 1 && vocab > 0, "ms_spec_accept: bad sizes");
  if (n_requests == 0) return MS_OK;
  MS_REQUIRE(target_logits && draft_rows && proposals && params && out_tokens && out_num_accepted,
             "ms_spec_accept: null pointer");
  MS_REQUIRE(target_stride >= vocab && draft_stride >= vocab, "ms_spec_accept: stride < vocab");
  AcceptArgs a{};
  a.target = target_logits;
  a.tstride = target_stride;
  a.target_probs = 0;
  a.draft = draft_rows;
  a.dstride = draft_stride;
  a.dstats = draft_stats;
  a.draft_probs = draft_probs_mode ? 1 : 0;
  a.proposals = proposals;
  a.params = params;
  a.gamma = gamma;
  a.V = vocab;
  a.out_tokens = out_tokens;
  a.out_nacc = out_num_accepted;
  return launch_accept(a, n_requests, stream);
}

extern "C" int ms_verify_probs(const float* target_probs, const float* draft_probs,
                               const int32_t* proposals, const float* accept_u, const float* draw_u,
                               int n_requests, int gamma, int vocab, int32_t* out_tokens,
                               int32_t* out_num_accepted, void* stream) {
  MS_REQUIRE(n_requests >= 0 && gamma >= 1 && vocab > 0, "ms_verify_probs: bad sizes");
  if (n_requests == 0) return MS_OK;
  MS_REQUIRE(target_probs && draft_probs && proposals && accept_u && draw_u && out_tokens &&
                 out_num_accepted,
             "ms_verify_probs: null pointer");
  AcceptArgs a{};
  a.target = target_probs;
  a.tstride = vocab;
  a.target_probs = 1;
  a.draft = draft_probs;
  a.dstride = vocab;
  a.draft_probs = 1;
  a.proposals = proposals;
  a.params = nullptr;
  a.accept_u = accept_u;
  a.draw_u = draw_u;
  a.gamma = gamma;
  a.V = vocab;
  a.out_tokens = out_tokens;
  a.out_nacc = out_num_accepted;
  return launch_accept(a, n_requests, stream);
}
