// CUDA-core GEMM: C = A * B^T with float32 accumulation (torch Linear).
//
// Used for the float32 models (the verify pass of a d_model=128 char model is
// a few MFLOP: launch latency, not arithmetic, bounds it) and as the generic
// fallback for bf16 shapes the tensor-core kernel does not tile.  64x64 output
// tile, k-step 16, 256 threads with a 4x4 register micro-tile; the finished
// tile goes through shared memory so every epilogue stores coalesced rows.
#include "common.cuh"
#include "gemm.cuh"

namespace ms {
namespace {

constexpr int BM = 64, BN = 64, BK = 16;

template <typename TA, typename TC>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const TA* __restrict__ A,
                                                       const TA* __restrict__ B,
                                                       TC* __restrict__ C,
                                                       const float* __restrict__ R, int M, int N,
                                                       int K, int64_t ldc, int epilogue) {
  pdl_enter();
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  __shared__ float Cs[BM][BN + 1];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += BK) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int idx = tid + e * 256;  // 0..1023
      const int r = idx >> 4, c = idx & 15;
      const int gk = k0 + c;
      const int gm = m0 + r, gn = n0 + r;
      As[c][r] = (gm < M && gk < K) ? to_f(A[(int64_t)gm * K + gk]) : 0.f;
      Bs[c][r] = (gn < N && gk < K) ? to_f(B[(int64_t)gn * K + gk]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) Cs[ty * 4 + i][tx * 4 + j] = acc[i][j];
  __syncthreads();
  if (epilogue == kEpiSwiGLU) {
    // Columns [16g, 16g+8) are gate, [16g+8, 16g+16) up; output column 8g+j.
    const int NO = N / 2;
    for (int idx = tid; idx < BM * (BN / 2); idx += 256) {
      const int r = idx / (BN / 2), oc = idx % (BN / 2);
      const int g = oc >> 3, j = oc & 7;
      const int gm = m0 + r, gon = n0 / 2 + oc;
      if (gm < M && gon < NO) {
        const float gate = Cs[r][16 * g + j], up = Cs[r][16 * g + 8 + j];
        const float silu = gate / (1.f + expf(-gate));
        C[(int64_t)gm * ldc + gon] = from_f<TC>(silu * up);
      }
    }
  } else {
    for (int idx = tid; idx < BM * BN; idx += 256) {
      const int r = idx / BN, c = idx % BN;
      const int gm = m0 + r, gn = n0 + c;
      if (gm < M && gn < N) {
        float v = Cs[r][c];
        if (epilogue == kEpiResidual) v += R[(int64_t)gm * ldc + gn];
        C[(int64_t)gm * ldc + gn] = from_f<TC>(v);
      }
    }
  }
}

template <typename TA, typename TC>
int launch_simt(const void* A, const void* B, void* C, const float* R, int M, int N, int K,
                int64_t ldc, int epi, cudaStream_t s) {
  dim3 grid(ceil_div(N, BN), ceil_div(M, BM));
  launch_pdl(gemm_simt_kernel<TA, TC>, grid, 256, 0, s, static_cast<const TA*>(A),
                                                static_cast<const TA*>(B), static_cast<TC*>(C),
                                                R, M, N, K, ldc, epi);
  return check_launch("gemm_simt_kernel");
}

}  // namespace

int gemm_simt(const void* A, const void* B, void* C, const float* R, int M, int N, int K,
              int64_t ldc, int ab_dtype, int c_dtype, int epi, cudaStream_t s) {
  if (epi == kEpiResidual && c_dtype != MS_DTYPE_F32)
    return fail(MS_ERR_UNSUPPORTED, "gemm: residual epilogue writes float32 only");
  if (ab_dtype == MS_DTYPE_F32 && c_dtype == MS_DTYPE_F32)
    return launch_simt<float, float>(A, B, C, R, M, N, K, ldc, epi, s);
  if (ab_dtype == MS_DTYPE_BF16 && c_dtype == MS_DTYPE_F32)
    return launch_simt<__nv_bfloat16, float>(A, B, C, R, M, N, K, ldc, epi, s);
  if (ab_dtype == MS_DTYPE_BF16 && c_dtype == MS_DTYPE_BF16)
    return launch_simt<__nv_bfloat16, __nv_bfloat16>(A, B, C, R, M, N, K, ldc, epi, s);
  if (ab_dtype == MS_DTYPE_F32 && c_dtype == MS_DTYPE_BF16)
    return launch_simt<float, __nv_bfloat16>(A, B, C, R, M, N, K, ldc, epi, s);
  return fail(MS_ERR_UNSUPPORTED, "gemm: dtype pair %d/%d", ab_dtype, c_dtype);
}

int gemm_dispatch(const void* A, const void* B, void* C, const float* R, int M, int N, int K,
                  int64_t ldc, int ab_dtype, int c_dtype, int epi, cudaStream_t s,
                  bool weights_const) {
  if (M == 0 || N == 0) return MS_OK;
  if (epi == kEpiSwiGLU && (N % 16) != 0)
    return fail(MS_ERR_UNSUPPORTED, "gemm: SwiGLU needs N %% 16 == 0 (got %d)", N);
  const int64_t out_cols = epi == kEpiSwiGLU ? N / 2 : N;
  if (ldc <= 0) ldc = out_cols;
  if (ldc < out_cols) return fail(MS_ERR_INVALID, "gemm: ldc %lld < %lld", (long long)ldc,
                                  (long long)out_cols);
  ProfScope prof(kClsGemm, s);
  if (ab_dtype == MS_DTYPE_BF16 && gemm_tc_supported(M, N, K, ldc, c_dtype, epi))
    return gemm_tc(A, B, C, R, M, N, K, ldc, c_dtype, epi, s, weights_const);
  return gemm_simt(A, B, C, R, M, N, K, ldc, ab_dtype, c_dtype, epi, s);
}

}  // namespace ms

using namespace ms;

extern "C" int ms_gemm(const void* A, const void* B, void* C, const float* R, int M, int N, int K,
                       int64_t ldc, int ab_dtype, int c_dtype, int epilogue, void* stream) {
  MS_REQUIRE(M >= 0 && N >= 0 && K > 0, "ms_gemm: bad sizes M=%d N=%d K=%d", M, N, K);
  MS_REQUIRE(A && B && C, "ms_gemm: null pointer");
  MS_REQUIRE(epilogue >= 0 && epilogue <= 2, "ms_gemm: unknown epilogue %d", epilogue);
  MS_REQUIRE(epilogue != kEpiResidual || R != nullptr, "ms_gemm: residual epilogue needs R");
  return gemm_dispatch(A, B, C, R, M, N, K, ldc, ab_dtype, c_dtype, epilogue, as_stream(stream));
}
