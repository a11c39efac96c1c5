// Status reporting, launch accounting, device error word and Philox uniforms.
#include <cstdarg>
#include <cstring>
#include <vector>

#include "common.cuh"

namespace ms {

static thread_local char t_last_error[512] = "";
std::atomic<uint64_t> g_launches{0};
static __device__ int g_device_error = 0;

int* device_error_word() {
  static int* cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (cached[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    cached[dev] = static_cast<int*>(p);
  }
  return cached[dev];
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MS_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return MS_OK;
}

// ---- live per-class timing -------------------------------------------------
static int g_prof_class = kClsNone;
static std::vector<cudaEvent_t> g_prof_events;  // pairs: [2i] start, [2i+1] end
static int g_prof_used = 0;

ProfScope::ProfScope(int cls, cudaStream_t s) : active(false), stream(s), slot(-1) {
  if (g_prof_class == kClsNone || cls != g_prof_class) return;
  if ((int)g_prof_events.size() < 2 * (g_prof_used + 1)) {
    cudaEvent_t a, b;
    if (cudaEventCreate(&a) != cudaSuccess) return;
    if (cudaEventCreate(&b) != cudaSuccess) {
      cudaEventDestroy(a);
      return;
    }
    g_prof_events.push_back(a);
    g_prof_events.push_back(b);
  }
  slot = g_prof_used++;
  active = cudaEventRecord(g_prof_events[2 * slot], s) == cudaSuccess;
}

ProfScope::~ProfScope() {
  if (active) cudaEventRecord(g_prof_events[2 * slot + 1], stream);
}

__global__ void philox_uniforms_kernel(const uint64_t* seeds, const uint64_t* steps, int n,
                                       uint32_t lane, float* out) {
  pdl_enter();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = philox_uniform(seeds[i], steps[i], lane);
}

}  // namespace ms

using namespace ms;

extern "C" int ms_version(void) { return 1; }

extern "C" const char* ms_last_error(void) { return t_last_error; }

extern "C" uint64_t ms_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" int ms_device_error(void* stream, int32_t* out_code) {
  MS_REQUIRE(out_code != nullptr, "ms_device_error: null out_code");
  int host = 0;
  cudaStream_t s = as_stream(stream);
  cudaError_t e = cudaMemcpyFromSymbolAsync(&host, g_device_error, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fail(MS_ERR_CUDA, "ms_device_error: %s", cudaGetErrorString(e));
  *out_code = host;
  if (host != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return fail(MS_ERR_CUDA, "ms_device_error: %s", cudaGetErrorString(e));
  }
  return MS_OK;
}

extern "C" int ms_profile_start(int kernel_class) {
  MS_REQUIRE(kernel_class >= kClsNone && kernel_class <= kClsNorm, "ms_profile_start: class %d",
             kernel_class);
  g_prof_class = kernel_class;
  g_prof_used = 0;
  return MS_OK;
}

extern "C" int ms_profile_stop(double* total_ms, int64_t* launches) {
  MS_REQUIRE(total_ms && launches, "ms_profile_stop: null output");
  double total = 0.0;
  for (int i = 0; i < g_prof_used; ++i) {
    cudaError_t e = cudaEventSynchronize(g_prof_events[2 * i + 1]);
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, g_prof_events[2 * i], g_prof_events[2 * i + 1]);
    if (e != cudaSuccess) return fail(MS_ERR_CUDA, "ms_profile_stop: %s", cudaGetErrorString(e));
    total += ms;
  }
  *total_ms = total;
  *launches = g_prof_used;
  g_prof_class = kClsNone;
  g_prof_used = 0;
  return MS_OK;
}

extern "C" int ms_philox_uniforms(const uint64_t* seeds, const uint64_t* steps, int n, int lane,
                                  float* out, void* stream) {
  MS_REQUIRE(n >= 0, "ms_philox_uniforms: n < 0");
  if (n == 0) return MS_OK;
  MS_REQUIRE(seeds && steps && out, "ms_philox_uniforms: null pointer");
  launch_pdl(philox_uniforms_kernel, ceil_div(n, 256), 256, 0, as_stream(stream), seeds, steps, n,
                                                                          (uint32_t)lane, out);
  return check_launch("ms_philox_uniforms");
}
