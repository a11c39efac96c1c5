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

#include "common.cuh"

namespace ms {
namespace {

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
};

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
// conflict-free).  Pass 1: each lane sums its elements, one butterfly gives
// the warp's total, and a block scan places the warps.  Pass 2: only the
// warp holding the target re-walks its segment, skipping whole chunks by
// their totals, and scans inside the one chunk that crosses.
template <typename W>
__device__ int inverse_cdf(const W& w, int V, float u, RowSmem& sm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int seg = (V + nw - 1) / nw;
  seg = (seg + 127) & ~127;
  const int s0 = min(V, warp * seg), s1 = min(V, s0 + seg);
  auto chunk = [&](int c0, float (&v)[4]) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = c0 + 32 * k + lane;
      v[k] = i < s1 ? w(i) : 0.f;
    }
  };
  // pass 1: lane sums (four independent chunks at a time), one butterfly
  float lsum = 0.f;
  int last = -1;
  for (int c0 = s0; c0 < s1; c0 += 4 * 128) {
    float v[4][4];
#pragma unroll
    for (int q = 0; q < 4; ++q) chunk(c0 + 128 * q, v[q]);
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
  const double wtot = (double)lsum;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
  __syncthreads();  // earlier users of red_* are done
  if (lane == 0) {
    sm.red_d[warp] = wtot;
    sm.red_i[warp] = last;
  }
  if (threadIdx.x == 0) sm.red_i[40] = -1;
  __syncthreads();
  double before = 0.0, total = 0.0;
  int glast = -1;
  for (int k = 0; k < nw; ++k) {
    const double t = sm.red_d[k];
    if (k < warp) before += t;
    total += t;
    glast = max(glast, sm.red_i[k]);
  }
  const double target = (double)u * total;
  if (wtot > 0.0 && before <= target && target < before + wtot) {
    // pass 2 (the target's warp): chunk totals four at a time, skip whole
    // chunks, scan inside the one that crosses
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
  int res = sm.red_i[40];
  if (res < 0) res = glast;
  if (res < 0) res = 0;
  __syncthreads();
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
__global__ void __launch_bounds__(512, 1) sample_rows_kernel(const float* __restrict__ logits, int64_t stride, int V,
                                   const ms_sampling_params* __restrict__ params,
                                   const int32_t* __restrict__ pidx, uint32_t lane_id,
                                   int32_t* __restrict__ tokens, float* __restrict__ probs,
                                   ms_row_stats* __restrict__ stats, int32_t* scatter_dst,
                                   const int32_t* __restrict__ scatter_idx, int stage) {
  pdl_enter();
  RowSmem sm;
  setup_smem(sm, V, stage != 0);
  const int r = blockIdx.x;
  const ms_sampling_params P = params[pidx ? pidx[r] : r];
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

__global__ void __launch_bounds__(512, 1) spec_accept_kernel(AcceptArgs a, int stage) {
  pdl_enter();
  RowSmem sm;
  setup_smem(sm, a.V, stage != 0);
  const int b = blockIdx.x;
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
    const int r = i * (int)gridDim.x + b;  // position-major: row of (b, i)
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
    int x = a.proposals[i * (int)gridDim.x + b];
    if (x < 0 || x >= V) {
      if (threadIdx.x == 0) raise_device_error(a.err, kErrToken);
      x = 0;
    }
    const float px = p.prob(x);
    const float qx = q.prob(x);
    const float ratio = fminf(__fdiv_rn(px, fmaxf(qx, 1e-10f)), 1.f);
    const float u = a.accept_u ? a.accept_u[i * (int)gridDim.x + b]
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
      float* res = sm.stage;
#pragma unroll 4
      for (int j = threadIdx.x; j < V; j += blockDim.x) {
        const float r = fmaxf(pv.prob(j) - qv.prob(j), 0.f);
        res[j] = r;
        part += r;
      }
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

int row_threads(int V) {
  int t = ((V / 16) + 31) & ~31;
  if (t < 128) t = 128;
  if (t > 512) t = 512;
  return t;
}

int launch_accept(AcceptArgs a, int B, void* stream) {
  a.err = device_error_word();
  const int threads = row_threads(a.V);
  const bool stage = a.V <= kMaxStagedV && !a.target_probs;
  const size_t smem = smem_bytes(threads, a.V, stage);
  cudaError_t e = cudaFuncSetAttribute(spec_accept_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return fail(MS_ERR_CUDA, "spec_accept: smem attribute: %s", cudaGetErrorString(e));
  ProfScope prof(kClsAccept, as_stream(stream));
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
  const int threads = row_threads(vocab);
  const bool stage = vocab <= kMaxStagedV;
  const size_t smem = smem_bytes(threads, vocab, stage);
  cudaError_t e = cudaFuncSetAttribute(sample_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return fail(MS_ERR_CUDA, "ms_sample: smem attribute: %s", cudaGetErrorString(e));
  ProfScope prof(kClsSample, as_stream(stream));
  launch_pdl(sample_rows_kernel, n_rows, threads, smem, as_stream(stream),
      logits, row_stride, vocab, params, pidx, (uint32_t)lane, tokens, probs, stats, scatter_dst,
      scatter_idx, stage ? 1 : 0);
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
