"""The tcgen05 GEMM against an fp32 torch product of the same bf16 operands, in every operand
orientation, at ragged and at step shapes (fp32 accumulation: differences come only from the
summation order and the output rounding)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(a, b_t, bias=None):
    r = a.float() @ b_t.float().t()
    return r if bias is None else r + bias.float()


def _check(out, ref, out_dtype):
    if out_dtype == torch.float32:
        torch.testing.assert_close(out, ref, rtol=1e-3, atol=1e-3)
    else:
        torch.testing.assert_close(out.float(), ref, rtol=1.6e-2, atol=1e-2)


@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_gemm_orientations(cuda, a_t, b_t, out_dtype):
    from hackathon_b200.gemm import device_error, gemm
    torch.manual_seed(0)
    M, N, K = 384, 512, 320
    a = torch.randn(K, M, device=cuda).to(torch.bfloat16).t() if a_t else \
        torch.randn(M, K, device=cuda).to(torch.bfloat16)
    b = torch.randn(K, N, device=cuda).to(torch.bfloat16).t() if b_t else \
        torch.randn(N, K, device=cuda).to(torch.bfloat16)
    out = gemm(a, b, out_dtype=out_dtype)
    device_error()
    _check(out, _ref(a, b), out_dtype)


@pytest.mark.parametrize("shape", [(1, 1, 1), (127, 255, 63), (129, 257, 65), (200, 1000, 96),
                                   (1000, 136, 2048)])
def test_gemm_ragged_edges(cuda, shape):
    from hackathon_b200.gemm import device_error, gemm
    M, N, K = shape
    torch.manual_seed(1)
    # leading dims padded to a multiple of 8 elements (16-byte rows), views cut to the shape
    lda, ldb = (K + 7) // 8 * 8, (K + 7) // 8 * 8
    a = torch.randn(M, lda, device=cuda).to(torch.bfloat16)[:, :K]
    b = torch.randn(N, ldb, device=cuda).to(torch.bfloat16)[:, :K]
    bias = torch.randn(N, device=cuda)
    out = gemm(a, b, out_dtype=torch.float32, bias=bias)
    device_error()
    _check(out, _ref(a, b, bias), torch.float32)


@pytest.mark.parametrize("shape", [(16384, 3584, 3584), (4096, 18944, 3584),
                                   (4096, 3584, 18944)])
def test_gemm_step_shapes(cuda, shape):
    """7B projection shapes (x W^T) against cuBLAS-free fp32 reference on a row sample."""
    from hackathon_b200.gemm import device_error, gemm
    M, N, K = shape
    g = torch.Generator(device=cuda).manual_seed(2)
    a = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    b = (torch.randn(N, K, device=cuda, generator=g) * 0.02).to(torch.bfloat16)
    out = gemm(a, b, out_dtype=torch.bfloat16)
    device_error()
    rows = torch.tensor([0, 1, 127, 128, M // 2, M - 1], device=cuda)
    ref = a[rows].float() @ b.float().t()
    torch.testing.assert_close(out[rows].float(), ref, rtol=1.6e-2, atol=2e-2)


def test_gemm_rejects_misaligned_rows(cuda):
    from hackathon_b200.gemm import gemm
    a = torch.randn(64, 67, device=cuda).to(torch.bfloat16)   # 134-byte rows
    b = torch.randn(64, 67, device=cuda).to(torch.bfloat16)
    with pytest.raises(RuntimeError, match="16"):
        gemm(a, b)
