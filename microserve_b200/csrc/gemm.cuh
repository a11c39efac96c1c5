// GEMM entry points shared by the forward pass.
#pragma once
#include "common.cuh"

namespace ms {

enum Epilogue : int {
  kEpiStore = 0,     // C = acc
  kEpiResidual = 1,  // C(float) = R(float) + acc   (R may alias C)
  kEpiSwiGLU = 2,    // C[:, 8g+j] = silu(acc[:, 16g+j]) * acc[:, 16g+8+j]
  kEpiRopeKV = 3,    // qkv projection: RoPE on q and k, q into C, k and v into the cache
};

// What the RoPE / cache-write epilogue needs (the rope_kv_write arguments).
struct RopeKv {
  const int32_t* positions;
  const int32_t* slots;
  const float* cos_t;
  const float* sin_t;
  int max_pos, hq, hkv, dh, bs, num_blocks;
  __nv_bfloat16* kpool;
  __nv_bfloat16* vpool;
};
// The qkv GEMM with RoPE and the cache write in its epilogue (bf16, d_head 64
// or 128, tensor-core shapes): replaces gemm_dispatch(kEpiStore) followed by
// rope_kv_write.  Returns MS_ERR_UNSUPPORTED when the shape does not apply.
// weights_const: W is never written by the kernels before it (model weights),
// so its first tiles may be loaded before the previous launch completes.
int gemm_qkv_rope(const void* A, const void* W, void* qkv, int M, int N, int K, const RopeKv& rk,
                  cudaStream_t s, bool weights_const = false);

// C = A[M,K] * B[N,K]^T; picks the tensor-core kernel when it applies.
// C and R rows are ldc elements apart (ldc >= output columns).
// weights_const as for gemm_qkv_rope, for B.
int gemm_dispatch(const void* A, const void* B, void* C, const float* R, int M, int N, int K,
                  int64_t ldc, int ab_dtype, int c_dtype, int epi, cudaStream_t s,
                  bool weights_const = false);
int gemm_simt(const void* A, const void* B, void* C, const float* R, int M, int N, int K,
              int64_t ldc, int ab_dtype, int c_dtype, int epi, cudaStream_t s);
// tcgen05 bf16 kernel (gemm_tc.cu).
bool gemm_tc_supported(int M, int N, int K, int64_t ldc, int c_dtype, int epi);
int gemm_tc(const void* A, const void* B, void* C, const float* R, int M, int N, int K,
            int64_t ldc, int c_dtype, int epi, cudaStream_t s, bool weights_const = false);

}  // namespace ms
