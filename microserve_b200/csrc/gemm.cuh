// GEMM entry points shared by the forward pass.
#pragma once
#include "common.cuh"

namespace ms {

enum Epilogue : int {
  kEpiStore = 0,     // C = acc
  kEpiResidual = 1,  // C(float) = R(float) + acc   (R may alias C)
  kEpiSwiGLU = 2,    // C[:, 8g+j] = silu(acc[:, 16g+j]) * acc[:, 16g+8+j]
};

// C = A[M,K] * B[N,K]^T; picks the tensor-core kernel when it applies.
// C and R rows are ldc elements apart (ldc >= output columns).
int gemm_dispatch(const void* A, const void* B, void* C, const float* R, int M, int N, int K,
                  int64_t ldc, int ab_dtype, int c_dtype, int epi, cudaStream_t s);
int gemm_simt(const void* A, const void* B, void* C, const float* R, int M, int N, int K,
              int64_t ldc, int ab_dtype, int c_dtype, int epi, cudaStream_t s);
// tcgen05 bf16 kernel (gemm_tc.cu).
bool gemm_tc_supported(int M, int N, int K, int64_t ldc, int c_dtype, int epi);
int gemm_tc(const void* A, const void* B, void* C, const float* R, int M, int N, int K,
            int64_t ldc, int c_dtype, int epi, cudaStream_t s);

}  // namespace ms
