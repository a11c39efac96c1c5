// Shared helpers for the microserve_b200 kernels (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdio>
#include <string>
#include <utility>

#include "../../include/microserve_b200.h"

namespace ms {

// ---- host-side status plumbing -------------------------------------------
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
extern std::atomic<uint64_t> g_launches;
// Checks the launch just issued; counts it.
int check_launch(const char* what);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ---- programmatic dependent launch -------------------------------------------
// Every kernel of this library begins with pdl_enter(): it waits until the
// previous kernel on the stream has completed and its writes are visible
// (griddepcontrol.wait), then allows the next launch to begin
// (griddepcontrol.launch_dependents).  Launched with launch_pdl, a kernel's
// CTAs are scheduled while its predecessor's last CTAs still run and start
// the moment it completes, so back-to-back launches lose no launch latency.
// Nothing the previous kernels write is read or written before the wait, so
// ordering is the stream's.  (The tcgen05 GEMM calls it after its CTA-local
// setup -- barriers, TMEM -- and, for constant weights, after issuing its
// first weight tiles.)  Launched without the attribute, the wait returns at
// once.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  // A failure is recorded as the thread's last error; check_launch reports it.
  (void)cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---- live per-kernel-class timing (ms_profile_start / ms_profile_stop) -----
// While a class is selected, every launch of that class is bracketed by a
// pair of CUDA events on its own stream; stop() sums the elapsed times.
enum KernelClass : int {
  kClsNone = 0,
  kClsGemm = 1,
  kClsAttention = 2,
  kClsSample = 3,
  kClsAccept = 4,
  kClsNorm = 5,
};
struct ProfScope {
  ProfScope(int cls, cudaStream_t s);
  ~ProfScope();
  bool active;
  cudaStream_t stream;
  int slot;
};

#define MS_REQUIRE(cond, ...)                              \
  do {                                                     \
    if (!(cond)) return ::ms::fail(MS_ERR_INVALID, __VA_ARGS__); \
  } while (0)

#define MS_TRY(expr)               \
  do {                             \
    int _rc = (expr);              \
    if (_rc != MS_OK) return _rc;  \
  } while (0)

// ---- device-side error word ----------------------------------------------
// Bounds checks on metadata record the first failing code in a per-device
// word and skip the access instead of faulting.  Kernels receive the word's
// address (device_error_word(), resolved once per device).
int* device_error_word();
enum DeviceError : int {
  kErrNone = 0,
  kErrSlot = 1,      // slot id outside the pool
  kErrBlock = 2,     // block id outside the pool
  kErrToken = 3,     // token id outside the vocabulary
  kErrPosition = 4,  // position beyond the RoPE table
};
__device__ __forceinline__ void raise_device_error(int* err, int code) {
  atomicCAS(err, 0, code);
}

// ---- element conversion ----------------------------------------------------
__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// ---- reductions -------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum; `red` must hold >= 32 floats. All threads get the result.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nwarps ? red[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

// ---- Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers:
// as easy as 1, 2, 3", SC'11) ------------------------------------------------
// Counter (lane, 0, step_lo, step_hi), key (seed_lo, seed_hi).  The uniform is
// the top 24 bits of the first output word scaled by 2^-24, so it is exact in
// float32 and lies in [0, 1).
__host__ __device__ __forceinline__ void philox_round(uint32_t& c0, uint32_t& c1, uint32_t& c2,
                                                      uint32_t& c3, uint32_t k0, uint32_t k1) {
  const uint64_t p0 = (uint64_t)0xD2511F53u * c0;
  const uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
  const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
  const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
  const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
  c0 = n0;
  c1 = lo1;
  c2 = n2;
  c3 = lo0;
}

__host__ __device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
  uint32_t c0 = c.x, c1 = c.y, c2 = c.z, c3 = c.w;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r > 0) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    philox_round(c0, c1, c2, c3, k0, k1);
  }
  return make_uint4(c0, c1, c2, c3);
}

__host__ __device__ __forceinline__ float philox_uniform(uint64_t seed, uint64_t step, uint32_t lane) {
  const uint4 r = philox4x32_10(make_uint4(lane, 0u, (uint32_t)step, (uint32_t)(step >> 32)),
                                (uint32_t)seed, (uint32_t)(seed >> 32));
  return (float)(r.x >> 8) * (1.0f / 16777216.0f);
}

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

}  // namespace ms
