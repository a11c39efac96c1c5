// Per-token kernels of the paged forward: embedding + RMSNorm, RMSNorm,
// RoPE with the K/V cache write, and the cache write/gather used by the
// PagedKVCache API.
//
// Pool layout per layer: [num_blocks][n_kv_heads][block_size][d_head], so one
// (block, kv head) tile of block_size x d_head is contiguous in HBM.
#include "common.cuh"
#include "model_kernels.cuh"

namespace ms {
namespace {

// One warp per row.  y = x * (1/sqrt(mean(x^2) + eps)) * w, float32 math
// (reference model.py:77-79).
template <typename TY>
__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                               TY* __restrict__ y, const int32_t* __restrict__ row_idx, int n_rows,
                               int dim, float eps) {
  pdl_enter();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n_rows) return;
  const int src = row_idx ? row_idx[warp] : warp;
  const float* xr = x + (int64_t)src * dim;
  float ss = 0.f;
  for (int i = lane; i < dim; i += 32) {
    const float v = xr[i];
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  const float r = 1.f / sqrtf(ss / (float)dim + eps);
  TY* yr = y + (int64_t)warp * dim;
  for (int i = lane; i < dim; i += 32) yr[i] = from_f<TY>(xr[i] * r * w[i]);
}

// Vectorised RMSNorm for dim % 4 == 0 and dim <= 4 * 128 * kVec: one
// 128-thread CTA per row, the row held in registers (one read of x).
constexpr int kNormThreads = 128;
constexpr int kVec = 8;  // float4 per thread -> dim up to 4096
template <typename TY>
__global__ void __launch_bounds__(kNormThreads)
    rmsnorm_vec_kernel(const float* __restrict__ x, const float* __restrict__ w, TY* __restrict__ y,
                       const int32_t* __restrict__ row_idx, int dim, float eps, int w_const) {
  __shared__ float red[kNormThreads / 32];
  const int n4 = dim >> 2;
  // Constant norm weights (a model's) are read while the kernel that writes
  // x still runs, before the launch wait; other weights after it.
  const float4* wr = reinterpret_cast<const float4*>(w);
  float4 g[kVec];
  auto load_w = [&]() {
#pragma unroll
    for (int k = 0; k < kVec; ++k) {
      const int i = threadIdx.x + k * kNormThreads;
      g[k] = i < n4 ? wr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  if (w_const) load_w();
  pdl_enter();
  if (!w_const) load_w();
  const int row = blockIdx.x;
  const int src = row_idx ? row_idx[row] : row;
  const float4* xr = reinterpret_cast<const float4*>(x + (int64_t)src * dim);
  float4 v[kVec];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kVec; ++k) {
    const int i = threadIdx.x + k * kNormThreads;
    v[k] = i < n4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    ss = fmaf(v[k].x, v[k].x, fmaf(v[k].y, v[k].y, fmaf(v[k].z, v[k].z, fmaf(v[k].w, v[k].w, ss))));
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  ss = red[0] + red[1] + red[2] + red[3];
  const float r = 1.f / sqrtf(ss / (float)dim + eps);
  TY* yr = y + (int64_t)row * dim;
#pragma unroll
  for (int k = 0; k < kVec; ++k) {
    const int i = threadIdx.x + k * kNormThreads;
    if (i >= n4) break;
    const float a = v[k].x * r * g[k].x, b = v[k].y * r * g[k].y, c = v[k].z * r * g[k].z,
                d = v[k].w * r * g[k].w;
    if constexpr (sizeof(TY) == 4) {
      reinterpret_cast<float4*>(yr)[i] = make_float4(a, b, c, d);
    } else {
      const __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
      uint2 pk;
      pk.x = *reinterpret_cast<const uint32_t*>(&lo);
      pk.y = *reinterpret_cast<const uint32_t*>(&hi);
      reinterpret_cast<uint2*>(yr)[i] = pk;
    }
  }
}

// x[t] = embed[ids[t]] (float32 residual stream), y[t] = rmsnorm(x[t]) * w.
template <typename TW>
__global__ void embed_rmsnorm_kernel(const TW* __restrict__ embed, const int32_t* __restrict__ ids,
                                     int n_tokens, int vocab, int dim, const float* __restrict__ w,
                                     float eps, float* __restrict__ x, TW* __restrict__ y,
                                     int* __restrict__ err) {
  pdl_enter();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n_tokens) return;
  int id = ids[warp];
  if (id < 0 || id >= vocab) {
    if (lane == 0) raise_device_error(err, kErrToken);
    id = 0;
  }
  const TW* er = embed + (int64_t)id * dim;
  float* xr = x + (int64_t)warp * dim;
  float ss = 0.f;
  for (int i = lane; i < dim; i += 32) {
    const float v = to_f(er[i]);
    xr[i] = v;
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  const float r = 1.f / sqrtf(ss / (float)dim + eps);
  TW* yr = y + (int64_t)warp * dim;
  for (int i = lane; i < dim; i += 32) yr[i] = from_f<TW>(to_f(er[i]) * r * w[i]);
}

// bf16 rows with dim % 256 == 0 (<= 4096): one warp per token, 16-byte
// loads, the row kept in registers between the sum of squares and the
// scaled write (one read of the embedding row).
constexpr int kEmbedChunks = 16;  // 8-element chunks per lane: dim <= 32 * 8 * 16
constexpr int kEmbedWarps = 4;
__global__ void __launch_bounds__(kEmbedWarps * 32)
    embed_rmsnorm_vec_kernel(const __nv_bfloat16* __restrict__ embed,
                             const int32_t* __restrict__ ids, int n_tokens, int vocab, int dim,
                             const float* __restrict__ w, float eps, float* __restrict__ x,
                             __nv_bfloat16* __restrict__ y, int* __restrict__ err) {
  pdl_enter();
  const int tok = blockIdx.x * kEmbedWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (tok >= n_tokens) return;
  int id = ids[tok];
  if (id < 0 || id >= vocab) {
    if (lane == 0) raise_device_error(err, kErrToken);
    id = 0;
  }
  const uint4* er = reinterpret_cast<const uint4*>(embed + (int64_t)id * dim);
  const int nc = dim >> 8;
  uint4 raw[kEmbedChunks];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kEmbedChunks; ++c) {
    if (c < nc) {
      raw[c] = er[c * 32 + lane];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[c]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h[e]);
        ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
      }
    }
  }
  ss = warp_sum(ss);
  const float r = 1.f / sqrtf(ss / (float)dim + eps);
  float4* xr = reinterpret_cast<float4*>(x + (int64_t)tok * dim);
  uint4* yr = reinterpret_cast<uint4*>(y + (int64_t)tok * dim);
  const float4* wr = reinterpret_cast<const float4*>(w);
#pragma unroll
  for (int c = 0; c < kEmbedChunks; ++c) {
    if (c < nc) {
      const int q = c * 32 + lane;  // chunk of 8 elements
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[c]);
      float v[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h[e]);
        v[2 * e] = f.x;
        v[2 * e + 1] = f.y;
      }
      xr[2 * q] = make_float4(v[0], v[1], v[2], v[3]);
      xr[2 * q + 1] = make_float4(v[4], v[5], v[6], v[7]);
      const float4 g0 = wr[2 * q], g1 = wr[2 * q + 1];
      const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162 b =
            __floats2bfloat162_rn(v[2 * e] * r * g[2 * e], v[2 * e + 1] * r * g[2 * e + 1]);
        o[e] = *reinterpret_cast<const uint32_t*>(&b);
      }
      yr[q] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

__device__ __forceinline__ int64_t pool_offset(int slot, int g, int d, int bs, int hkv, int dh,
                                               int num_blocks, bool& ok) {
  const int blk = slot / bs, off = slot - blk * bs;
  ok = slot >= 0 && blk < num_blocks;
  return (((int64_t)blk * hkv + g) * bs + off) * dh + d;
}

// One CTA per token: rotate q and k heads in place (half-split rotation,
// reference model.py:104-113) and scatter k, v into the layer's pools.
template <typename T>
__global__ void rope_kv_kernel(T* __restrict__ qkv, const int32_t* __restrict__ positions,
                               const int32_t* __restrict__ slots, const float* __restrict__ cos_t,
                               const float* __restrict__ sin_t, int max_pos, int hq, int hkv,
                               int dh, int bs, int num_blocks, T* __restrict__ kpool,
                               T* __restrict__ vpool, int* __restrict__ err) {
  pdl_enter();
  const int t = blockIdx.x;
  const int width = (hq + 2 * hkv) * dh;
  T* row = qkv + (int64_t)t * width;
  int pos = positions[t];
  if (pos < 0 || pos >= max_pos) {
    if (threadIdx.x == 0) raise_device_error(err, kErrPosition);
    pos = 0;
  }
  const int slot = slots[t];
  const int half = dh / 2;
  const float* c = cos_t + (int64_t)pos * half;
  const float* s = sin_t + (int64_t)pos * half;
  // rotations: q heads then k heads
  const int n_rot = (hq + hkv) * half;
  for (int idx = threadIdx.x; idx < n_rot; idx += blockDim.x) {
    const int h = idx / half, i = idx - h * half;
    T* hp = row + h * dh;
    const float x1 = to_f(hp[i]), x2 = to_f(hp[i + half]);
    const float r1 = x1 * c[i] - x2 * s[i];
    const float r2 = x2 * c[i] + x1 * s[i];
    if (h < hq) {
      hp[i] = from_f<T>(r1);
      hp[i + half] = from_f<T>(r2);
    } else {
      const int g = h - hq;
      bool ok;
      const int64_t o1 = pool_offset(slot, g, i, bs, hkv, dh, num_blocks, ok);
      if (!ok) {
        raise_device_error(err, kErrSlot);
        continue;
      }
      kpool[o1] = from_f<T>(r1);
      kpool[o1 + half] = from_f<T>(r2);
    }
  }
  const int n_v = hkv * dh;
  const T* vrow = row + (hq + hkv) * dh;
  for (int idx = threadIdx.x; idx < n_v; idx += blockDim.x) {
    const int g = idx / dh, d = idx - g * dh;
    bool ok;
    const int64_t o = pool_offset(slot, g, d, bs, hkv, dh, num_blocks, ok);
    if (!ok) {
      raise_device_error(err, kErrSlot);
      continue;
    }
    vpool[o] = vrow[idx];
  }
}

// Vectorised rope_kv for bf16 with d_head % 16 == 0: a task is 8 rotation
// pairs of one q/k head (two 16-byte loads, cos/sin as float4) or 8 values of
// one v head; kRopeTokens tokens per CTA.  Same arithmetic as rope_kv_kernel.
constexpr int kRopeTokens = 4;
__global__ void __launch_bounds__(128)
    rope_kv_vec_kernel(__nv_bfloat16* __restrict__ qkv, const int32_t* __restrict__ positions,
                       const int32_t* __restrict__ slots, const float* __restrict__ cos_t,
                       const float* __restrict__ sin_t, int max_pos, int n_tokens, int hq, int hkv,
                       int dh, int bs, int num_blocks, __nv_bfloat16* __restrict__ kpool,
                       __nv_bfloat16* __restrict__ vpool, int* __restrict__ err) {
  pdl_enter();
  const int width = (hq + 2 * hkv) * dh;
  const int half = dh / 2, hc = half / 8, vc = dh / 8;
  const int n_rot = (hq + hkv) * hc, per_token = n_rot + hkv * vc;
  for (int idx = threadIdx.x; idx < kRopeTokens * per_token; idx += blockDim.x) {
    const int tl = idx / per_token, task = idx - tl * per_token;
    const int t = blockIdx.x * kRopeTokens + tl;
    if (t >= n_tokens) break;
    __nv_bfloat16* row = qkv + (int64_t)t * width;
    const int slot = slots[t];
    if (task < n_rot) {
      int pos = positions[t];
      if (pos < 0 || pos >= max_pos) {
        raise_device_error(err, kErrPosition);
        pos = 0;
      }
      const int h = task / hc, i0 = (task - h * hc) * 8;
      __nv_bfloat16* hp = row + h * dh;
      const uint4 a = *reinterpret_cast<const uint4*>(hp + i0);
      const uint4 b = *reinterpret_cast<const uint4*>(hp + half + i0);
      const float4* c4 = reinterpret_cast<const float4*>(cos_t + (int64_t)pos * half + i0);
      const float4* s4 = reinterpret_cast<const float4*>(sin_t + (int64_t)pos * half + i0);
      const float4 ca = c4[0], cb = c4[1], sa = s4[0], sb = s4[1];
      const float c[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
      const float sn[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
      const __nv_bfloat162* x1 = reinterpret_cast<const __nv_bfloat162*>(&a);
      const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&b);
      uint4 o1, o2;
      __nv_bfloat162* r1 = reinterpret_cast<__nv_bfloat162*>(&o1);
      __nv_bfloat162* r2 = reinterpret_cast<__nv_bfloat162*>(&o2);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 p = __bfloat1622float2(x1[j]), q = __bfloat1622float2(x2[j]);
        const int k0 = 2 * j, k1 = 2 * j + 1;
        r1[j] = __floats2bfloat162_rn(p.x * c[k0] - q.x * sn[k0], p.y * c[k1] - q.y * sn[k1]);
        r2[j] = __floats2bfloat162_rn(q.x * c[k0] + p.x * sn[k0], q.y * c[k1] + p.y * sn[k1]);
      }
      if (h < hq) {
        *reinterpret_cast<uint4*>(hp + i0) = o1;
        *reinterpret_cast<uint4*>(hp + half + i0) = o2;
      } else {
        bool ok;
        const int64_t o = pool_offset(slot, h - hq, i0, bs, hkv, dh, num_blocks, ok);
        if (!ok) {
          raise_device_error(err, kErrSlot);
          continue;
        }
        *reinterpret_cast<uint4*>(kpool + o) = o1;
        *reinterpret_cast<uint4*>(kpool + o + half) = o2;
      }
    } else {
      const int vt = task - n_rot, g = vt / vc, d0 = (vt - g * vc) * 8;
      bool ok;
      const int64_t o = pool_offset(slot, g, d0, bs, hkv, dh, num_blocks, ok);
      if (!ok) {
        raise_device_error(err, kErrSlot);
        continue;
      }
      *reinterpret_cast<uint4*>(vpool + o) =
          *reinterpret_cast<const uint4*>(row + (hq + hkv) * dh + g * dh + d0);
    }
  }
}

template <typename T>
__global__ void kv_write_kernel(const int32_t* __restrict__ slots, int n_tokens,
                                const float* __restrict__ keys, const float* __restrict__ values,
                                int hkv, int dh, int bs, int num_blocks, T* __restrict__ kpool,
                                T* __restrict__ vpool, int* __restrict__ err) {
  pdl_enter();
  const int t = blockIdx.x;
  const int slot = slots[t];
  for (int idx = threadIdx.x; idx < hkv * dh; idx += blockDim.x) {
    const int g = idx / dh, d = idx - g * dh;
    bool ok;
    const int64_t o = pool_offset(slot, g, d, bs, hkv, dh, num_blocks, ok);
    if (!ok) {
      raise_device_error(err, kErrSlot);
      continue;
    }
    kpool[o] = from_f<T>(keys[(int64_t)t * hkv * dh + idx]);
    vpool[o] = from_f<T>(values[(int64_t)t * hkv * dh + idx]);
  }
}

// keys/values out: (B, max_context, hkv, dh) float32; key j of sequence b
// lives at slot table[b][j / bs] * bs + j % bs.
template <typename T>
__global__ void kv_gather_kernel(const int32_t* __restrict__ tables, int max_blocks,
                                 int max_context, int hkv, int dh, int bs, int num_blocks,
                                 const T* __restrict__ kpool, const T* __restrict__ vpool,
                                 float* __restrict__ keys, float* __restrict__ values,
                                 int* __restrict__ err) {
  pdl_enter();
  const int j = blockIdx.x, b = blockIdx.y;
  int blk = tables[(int64_t)b * max_blocks + j / bs];
  if (blk < 0 || blk >= num_blocks) {
    if (threadIdx.x == 0) raise_device_error(err, kErrBlock);
    blk = 0;
  }
  const int slot = blk * bs + j % bs;
  float* ko = keys + ((int64_t)b * max_context + j) * hkv * dh;
  float* vo = values + ((int64_t)b * max_context + j) * hkv * dh;
  for (int idx = threadIdx.x; idx < hkv * dh; idx += blockDim.x) {
    const int g = idx / dh, d = idx - g * dh;
    bool ok;
    const int64_t o = pool_offset(slot, g, d, bs, hkv, dh, num_blocks, ok);
    ko[idx] = to_f(kpool[o]);
    vo[idx] = to_f(vpool[o]);
  }
}

}  // namespace

int rmsnorm(const float* x, const float* w, void* y, const int32_t* row_idx, int n_rows, int dim,
            float eps, int dtype, cudaStream_t s, bool w_const) {
  if (n_rows == 0) return MS_OK;
  ProfScope prof(kClsNorm, s);
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
                         reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  if (dim % 4 == 0 && dim <= 4 * kNormThreads * kVec && aligned) {
    if (dtype == MS_DTYPE_F32)
      launch_pdl(rmsnorm_vec_kernel<float>, n_rows, kNormThreads, 0, s, x, w, static_cast<float*>(y),
                 row_idx, dim, eps, w_const ? 1 : 0);
    else if (dtype == MS_DTYPE_BF16)
      launch_pdl(rmsnorm_vec_kernel<__nv_bfloat16>, n_rows, kNormThreads, 0, s,
          x, w, static_cast<__nv_bfloat16*>(y), row_idx, dim, eps, w_const ? 1 : 0);
    else
      return fail(MS_ERR_UNSUPPORTED, "rmsnorm: dtype %d", dtype);
    return check_launch("rmsnorm_vec_kernel");
  }
  const int blocks = ceil_div(n_rows, 8);
  if (dtype == MS_DTYPE_F32)
    launch_pdl(rmsnorm_kernel<float>, blocks, 256, 0, s, x, w, static_cast<float*>(y), row_idx, n_rows, dim,
                                                 eps);
  else if (dtype == MS_DTYPE_BF16)
    launch_pdl(rmsnorm_kernel<__nv_bfloat16>, blocks, 256, 0, s, x, w, static_cast<__nv_bfloat16*>(y),
                                                         row_idx, n_rows, dim, eps);
  else
    return fail(MS_ERR_UNSUPPORTED, "rmsnorm: dtype %d", dtype);
  return check_launch("rmsnorm_kernel");
}

int embed_rmsnorm(const void* embed, const int32_t* ids, int n_tokens, int vocab, int dim,
                  const float* w, float eps, float* x, void* y, int dtype, cudaStream_t s) {
  if (n_tokens == 0) return MS_OK;
  ProfScope prof(kClsNorm, s);
  const bool aligned = ((reinterpret_cast<uintptr_t>(embed) | reinterpret_cast<uintptr_t>(w) |
                         reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  if (dtype == MS_DTYPE_BF16 && aligned && dim % 256 == 0 && dim <= 32 * 8 * kEmbedChunks) {
    launch_pdl(embed_rmsnorm_vec_kernel, ceil_div(n_tokens, kEmbedWarps), kEmbedWarps * 32, 0, s,
               static_cast<const __nv_bfloat16*>(embed), ids, n_tokens, vocab, dim, w, eps, x,
               static_cast<__nv_bfloat16*>(y), device_error_word());
    return check_launch("embed_rmsnorm_vec_kernel");
  }
  const int blocks = ceil_div(n_tokens, 8);
  if (dtype == MS_DTYPE_F32)
    launch_pdl(embed_rmsnorm_kernel<float>, blocks, 256, 0, s, static_cast<const float*>(embed), ids,
                                                       n_tokens, vocab, dim, w, eps, x,
                                                       static_cast<float*>(y), device_error_word());
  else if (dtype == MS_DTYPE_BF16)
    launch_pdl(embed_rmsnorm_kernel<__nv_bfloat16>, blocks, 256, 0, s,
        static_cast<const __nv_bfloat16*>(embed), ids, n_tokens, vocab, dim, w, eps, x,
        static_cast<__nv_bfloat16*>(y), device_error_word());
  else
    return fail(MS_ERR_UNSUPPORTED, "embed_rmsnorm: dtype %d", dtype);
  return check_launch("embed_rmsnorm_kernel");
}

int rope_kv_write(void* qkv, const int32_t* positions, const int32_t* slots, const float* cos_t,
                  const float* sin_t, int max_pos, int n_tokens, int hq, int hkv, int dh,
                  const ms_kv_cache& cache, int layer, int dtype, cudaStream_t s) {
  if (n_tokens == 0) return MS_OK;
  ProfScope prof(kClsNorm, s);
  const int threads = 128;
  if (dtype == MS_DTYPE_F32)
    launch_pdl(rope_kv_kernel<float>, n_tokens, threads, 0, s,
        static_cast<float*>(qkv), positions, slots, cos_t, sin_t, max_pos, hq, hkv, dh,
        cache.block_size, cache.num_blocks, static_cast<float*>(cache.k_pool[layer]),
        static_cast<float*>(cache.v_pool[layer]), device_error_word());
  else if (dtype == MS_DTYPE_BF16 && dh % 16 == 0 &&
           (reinterpret_cast<uintptr_t>(qkv) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(cos_t) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(sin_t) & 15) == 0) {
    launch_pdl(rope_kv_vec_kernel, ceil_div(n_tokens, kRopeTokens), threads, 0, s,
        static_cast<__nv_bfloat16*>(qkv), positions, slots, cos_t, sin_t, max_pos, n_tokens, hq,
        hkv, dh, cache.block_size, cache.num_blocks,
        static_cast<__nv_bfloat16*>(cache.k_pool[layer]),
        static_cast<__nv_bfloat16*>(cache.v_pool[layer]), device_error_word());
    return check_launch("rope_kv_vec_kernel");
  } else if (dtype == MS_DTYPE_BF16)
    launch_pdl(rope_kv_kernel<__nv_bfloat16>, n_tokens, threads, 0, s,
        static_cast<__nv_bfloat16*>(qkv), positions, slots, cos_t, sin_t, max_pos, hq, hkv, dh,
        cache.block_size, cache.num_blocks, static_cast<__nv_bfloat16*>(cache.k_pool[layer]),
        static_cast<__nv_bfloat16*>(cache.v_pool[layer]), device_error_word());
  else
    return fail(MS_ERR_UNSUPPORTED, "rope_kv_write: dtype %d", dtype);
  return check_launch("rope_kv_kernel");
}

int validate_cache(const ms_kv_cache* c, int layer) {
  MS_REQUIRE(c != nullptr, "null ms_kv_cache");
  MS_REQUIRE(c->k_pool && c->v_pool, "ms_kv_cache: null pool arrays");
  MS_REQUIRE(layer >= 0 && layer < c->n_layers, "layer %d out of range [0,%d)", layer, c->n_layers);
  MS_REQUIRE(c->k_pool[layer] && c->v_pool[layer], "ms_kv_cache: null pool for layer %d", layer);
  MS_REQUIRE(c->block_size > 0 && c->num_blocks > 0 && c->n_kv_heads > 0 && c->d_head > 0,
             "ms_kv_cache: bad geometry");
  return MS_OK;
}

}  // namespace ms

using namespace ms;

extern "C" int ms_rmsnorm(const float* x, const float* w, void* y, const int32_t* row_idx,
                          int n_rows, int dim, float eps, int dtype, void* stream) {
  MS_REQUIRE(n_rows >= 0 && dim > 0, "ms_rmsnorm: bad sizes");
  MS_REQUIRE(n_rows == 0 || (x && w && y), "ms_rmsnorm: null pointer");
  return rmsnorm(x, w, y, row_idx, n_rows, dim, eps, dtype, as_stream(stream));
}

extern "C" int ms_kv_write(const ms_kv_cache* cache, int layer, const int32_t* slots,
                           int n_tokens, const float* keys, const float* values, void* stream) {
  MS_TRY(validate_cache(cache, layer));
  MS_REQUIRE(n_tokens >= 0, "ms_kv_write: n_tokens < 0");
  if (n_tokens == 0) return MS_OK;
  MS_REQUIRE(slots && keys && values, "ms_kv_write: null pointer");
  const ms_kv_cache& c = *cache;
  cudaStream_t s = as_stream(stream);
  if (c.dtype == MS_DTYPE_F32)
    launch_pdl(kv_write_kernel<float>, n_tokens, 128, 0, s, slots, n_tokens, keys, values, c.n_kv_heads,
                                                    c.d_head, c.block_size, c.num_blocks,
                                                    static_cast<float*>(c.k_pool[layer]),
                                                    static_cast<float*>(c.v_pool[layer]),
                                                    device_error_word());
  else if (c.dtype == MS_DTYPE_BF16)
    launch_pdl(kv_write_kernel<__nv_bfloat16>, n_tokens, 128, 0, s,
        slots, n_tokens, keys, values, c.n_kv_heads, c.d_head, c.block_size, c.num_blocks,
        static_cast<__nv_bfloat16*>(c.k_pool[layer]), static_cast<__nv_bfloat16*>(c.v_pool[layer]),
        device_error_word());
  else
    return fail(MS_ERR_UNSUPPORTED, "ms_kv_write: dtype %d", c.dtype);
  return check_launch("kv_write_kernel");
}

extern "C" int ms_kv_gather(const ms_kv_cache* cache, int layer, const int32_t* block_tables,
                            int n_seqs, int max_blocks, int max_context, float* keys,
                            float* values, void* stream) {
  MS_TRY(validate_cache(cache, layer));
  MS_REQUIRE(n_seqs >= 0 && max_context >= 0 && max_blocks > 0, "ms_kv_gather: bad sizes");
  if (n_seqs == 0 || max_context == 0) return MS_OK;
  MS_REQUIRE(block_tables && keys && values, "ms_kv_gather: null pointer");
  const ms_kv_cache& c = *cache;
  MS_REQUIRE((int64_t)max_blocks * c.block_size >= max_context,
             "ms_kv_gather: max_context %d beyond the table (%d blocks of %d)", max_context,
             max_blocks, c.block_size);
  dim3 grid(max_context, n_seqs);
  cudaStream_t s = as_stream(stream);
  if (c.dtype == MS_DTYPE_F32)
    launch_pdl(kv_gather_kernel<float>, grid, 128, 0, s, block_tables, max_blocks, max_context,
                                                 c.n_kv_heads, c.d_head, c.block_size,
                                                 c.num_blocks,
                                                 static_cast<const float*>(c.k_pool[layer]),
                                                 static_cast<const float*>(c.v_pool[layer]), keys,
                                                 values, device_error_word());
  else if (c.dtype == MS_DTYPE_BF16)
    launch_pdl(kv_gather_kernel<__nv_bfloat16>, grid, 128, 0, s,
        block_tables, max_blocks, max_context, c.n_kv_heads, c.d_head, c.block_size, c.num_blocks,
        static_cast<const __nv_bfloat16*>(c.k_pool[layer]),
        static_cast<const __nv_bfloat16*>(c.v_pool[layer]), keys, values, device_error_word());
  else
    return fail(MS_ERR_UNSUPPORTED, "ms_kv_gather: dtype %d", c.dtype);
  return check_launch("kv_gather_kernel");
}
