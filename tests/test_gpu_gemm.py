"""ms_gemm (tcgen05 tensor cores for bf16 shapes with N % 128 == 0, CUDA cores
otherwise) against a float32 torch reference of the same bf16 operands."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _gemm(A, B, C, R, M, N, K, ldc, ab, c, epi) -> None:
    from microserve_b200 import _lib

    _lib.call("ms_gemm", A.data_ptr(), B.data_ptr(), C.data_ptr(), _lib.ptr(R), M, N, K, ldc, ab, c,
              epi, _lib.stream_ptr())
    torch.cuda.synchronize()


def _ref(A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    return A.float() @ B.float().T


@pytest.fixture(params=[1, 2], ids=["one_cta_per_tile", "cta_pairs"], autouse=True)
def policy(request):
    """Every case on both tcgen05 kernels: one CTA per 128 x 256 tile, and CTA
    pairs (cta_group::2, 256 x 256 tiles) wherever N allows."""
    from microserve_b200 import _lib

    _lib.call("ms_gemm_set_policy", request.param)
    yield request.param
    _lib.call("ms_gemm_set_policy", 0)


# (1536, 4096, 8192) and (1500, 3328, 8192): more 256-wide tiles than SMs but not a
# whole number of waves, and A + B over 64 MB, so the in-place residual runs whole
# tiles, then stream-K over the rest
SHAPES = [(1, 128, 64), (77, 256, 520), (128, 128, 2048), (300, 384, 200), (1280, 2560, 2048),
          (256, 1024, 5632), (600, 512, 192), (1280, 2048, 5632), (2048, 2048, 2048),
          (1536, 4096, 8192), (1500, 3328, 8192)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_store_bf16_and_f32(M: int, N: int, K: int) -> None:
    from microserve_b200 import _lib

    g = torch.Generator(device=DEV).manual_seed(M * 7 + N + K)
    A = torch.randn(M, K, device=DEV, generator=g).bfloat16()
    B = (torch.randn(N, K, device=DEV, generator=g) * 0.05).bfloat16()
    want = _ref(A, B)
    scale = want.abs().max().item() + 1e-6
    C = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    _gemm(A, B, C, None, M, N, K, 0, _lib.DTYPE_BF16, _lib.DTYPE_BF16, 0)
    torch.testing.assert_close(C.float(), want, rtol=1e-2, atol=1e-2 * scale)
    # float32 output with a row stride wider than N (the logits layout)
    ldc = N + 64
    Cf = torch.full((M, ldc), float("nan"), dtype=torch.float32, device=DEV)
    _gemm(A, B, Cf, None, M, N, K, ldc, _lib.DTYPE_BF16, _lib.DTYPE_F32, 0)
    torch.testing.assert_close(Cf[:, :N], want, rtol=1e-3, atol=1e-4 * scale)
    assert torch.isnan(Cf[:, N:]).all()


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_residual_epilogue(M: int, N: int, K: int) -> None:
    from microserve_b200 import _lib

    g = torch.Generator(device=DEV).manual_seed(M + N * 3 + K)
    A = torch.randn(M, K, device=DEV, generator=g).bfloat16()
    B = (torch.randn(N, K, device=DEV, generator=g) * 0.05).bfloat16()
    X = torch.randn(M, N, device=DEV, generator=g)
    want = X + _ref(A, B)
    Y = torch.full_like(X, float("nan"))
    _gemm(A, B, Y, X, M, N, K, 0, _lib.DTYPE_BF16, _lib.DTYPE_F32, 1)  # y = x + A B^T
    torch.testing.assert_close(Y, want, rtol=1e-3, atol=1e-3 * want.abs().max().item())
    _gemm(A, B, X, X, M, N, K, 0, _lib.DTYPE_BF16, _lib.DTYPE_F32, 1)  # in place: x += A B^T
    torch.testing.assert_close(X, want, rtol=1e-3, atol=1e-3 * want.abs().max().item())


@pytest.mark.parametrize("M,N,K", [(5, 256, 128), (130, 1024, 2048), (1280, 11264, 2048)])
def test_swiglu_epilogue(M: int, N: int, K: int) -> None:
    from microserve_b200 import _lib
    from microserve_b200.model import interleave_gate_up

    g = torch.Generator(device=DEV).manual_seed(N + K)
    A = torch.randn(M, K, device=DEV, generator=g).bfloat16()
    gate = (torch.randn(N // 2, K, device=DEV, generator=g) * 0.05).bfloat16()
    up = (torch.randn(N // 2, K, device=DEV, generator=g) * 0.05).bfloat16()
    W = interleave_gate_up(gate, up).contiguous()
    gf, uf = _ref(A, gate), _ref(A, up)
    want = torch.nn.functional.silu(gf) * uf
    C = torch.empty(M, N // 2, dtype=torch.bfloat16, device=DEV)
    _gemm(A, W, C, None, M, N, K, 0, _lib.DTYPE_BF16, _lib.DTYPE_BF16, 2)
    torch.testing.assert_close(C.float(), want, rtol=2e-2, atol=2e-2 * want.abs().max().item())
    assert _lib.device_error() == 0
