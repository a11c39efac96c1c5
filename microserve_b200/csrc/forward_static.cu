// ms_forward_static_scratch: the paged forward with its scratch memory in an
// array compiled into this library, for callers that cannot allocate device
// memory themselves.
//
// ms_forward needs a workspace (residual stream, normalised activations,
// q/k/v, attention output, SwiGLU activations, logit-row activations) that
// its caller allocates.  A host that binds only this C ABI through a foreign
// function interface and owns no CUDA allocator, or a serving loop that must
// not call cudaMalloc once it is running (cudaMalloc can synchronise the
// device and fail under memory pressure), can use this entry point instead:
// the workspace is g_forward_scratch below, kStaticScratchBytes per device,
// held by every GPU that loads the library until the process exits.
//
// Host code cannot use g_forward_scratch's name as a device address (in host
// code it names a host-side stand-in).  The first call on each device, with
// that device current, resolves the real address with cudaGetSymbolAddress
// and caches it; make that first call before any stream capture.  Every call
// on a device shares the one array and leaves the last call's contents in it
// (the forward writes every scratch byte it reads, so nothing needs
// clearing), and calls whose kernels overlap on the GPU -- two streams, or
// two threads -- race on it.
#include <atomic>

#include "common.cuh"

namespace {

constexpr size_t kStaticScratchBytes = size_t(16) << 20;  // 16 MiB per device
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_forward_scratch[kStaticScratchBytes];

// One resolved address per device.  Two host threads making their first call
// on the same device may both resolve it; they store the same value, and the
// atomic makes that well defined.
std::atomic<void*> g_scratch_cache[kMaxDevices];

int scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return ms::fail(MS_ERR_CUDA, "ms_forward_static_scratch: cudaGetDevice: %s",
                    cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return ms::fail(MS_ERR_UNSUPPORTED, "ms_forward_static_scratch: device %d", dev);
  void* p = g_scratch_cache[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    e = cudaGetSymbolAddress(&p, g_forward_scratch);
    if (e != cudaSuccess || p == nullptr)
      return ms::fail(MS_ERR_CUDA, "ms_forward_static_scratch: cudaGetSymbolAddress: %s",
                      cudaGetErrorString(e));
    g_scratch_cache[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return MS_OK;
}

}  // namespace

extern "C" int ms_forward_static_scratch(const ms_model* model, const ms_kv_cache* cache,
                                         const ms_batch* batch, const int32_t* logit_rows,
                                         int n_logit_rows, float* logits,
                                         int64_t logits_row_stride, void* stream) {
  MS_REQUIRE(model != nullptr && batch != nullptr, "ms_forward_static_scratch: null model/batch");
  MS_REQUIRE(batch->n_tokens >= 0, "ms_forward_static_scratch: n_tokens < 0");
  const int rows = logit_rows ? n_logit_rows : batch->n_tokens;
  const size_t need = ms_forward_workspace_size(model, batch->n_tokens, rows);
  if (need > kStaticScratchBytes)
    return ms::fail(MS_ERR_TOO_LARGE,
                    "ms_forward_static_scratch: this batch needs %zu bytes of scratch but the "
                    "built-in array holds %zu (16 MiB); split the batch or call ms_forward "
                    "with a caller-provided workspace",
                    need, kStaticScratchBytes);
  void* scratch = nullptr;
  MS_TRY(scratch_address(&scratch));
  return ms_forward(model, cache, batch, logit_rows, n_logit_rows, logits, logits_row_stride,
                    scratch, kStaticScratchBytes, stream);
}
