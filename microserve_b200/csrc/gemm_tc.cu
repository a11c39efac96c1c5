// tcgen05 tensor-core GEMM for bf16 (sm_100a).  Not wired in yet: every
// bf16 shape currently takes the CUDA-core kernel.
#include "gemm.cuh"

namespace ms {

bool gemm_tc_supported(int, int, int, int64_t, int, int) { return false; }

int gemm_tc(const void*, const void*, void*, const float*, int, int, int, int64_t, int, int,
            cudaStream_t) {
  return fail(MS_ERR_UNSUPPORTED, "gemm_tc: not available");
}

}  // namespace ms
