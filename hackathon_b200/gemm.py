"""bf16 GEMM on the tcgen05 kernel (C-ABI qb_gemm_bf16), for the contractions of the step."""

import torch

from . import _lib


def _operand(t):
    """(tensor, leading dim, mn_major) of a 2-D operand that is row-major or a transposed view."""
    if t.stride(-1) == 1:
        return t, t.stride(0), False
    if t.stride(0) == 1:
        return t, t.stride(1), True
    t = t.contiguous()
    return t, t.stride(0), False


def gemm(a, b_t, out=None, out_dtype=torch.bfloat16, bias=None):
    """out[M, N] = a[M, K] @ b_t[N, K].T (+ bias) with fp32 accumulation.

    `a` and `b_t` are bf16; each may be row-major or the transpose view of a row-major tensor
    (read as MN-major, no copy)."""
    _lib.require_cuda(a, b_t, what="gemm")
    if a.dtype != torch.bfloat16 or b_t.dtype != torch.bfloat16:
        raise TypeError("gemm: bf16 operands only")
    M, K = a.shape
    N, K2 = b_t.shape
    if K != K2:
        raise ValueError(f"gemm: inner dimensions differ ({K} vs {K2})")
    a, lda, a_mn = _operand(a)
    b_t, ldb, b_mn = _operand(b_t)
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    if bias is not None:
        bias = bias.float().contiguous()
    _lib.call("qb_gemm_bf16", a.data_ptr(), lda, int(a_mn), b_t.data_ptr(), ldb, int(b_mn),
              out.data_ptr(), out.stride(0), _lib.tag(out.dtype), _lib.ptr(bias), M, N, K,
              _lib.stream(a.device), work=(0, 2 * M * N * K))
    return out


def device_error():
    """Raises if a tensor-core kernel on this device gave up a bounded wait (synchronises)."""
    _lib.call("qb_device_error", _lib.stream())
