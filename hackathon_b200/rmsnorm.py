"""Qwen2RMSNorm forward + backward on the sm_100a row kernels (API of solution/rmsnorm.py).

    y  = w * round_x(x * r),  r = 1/sqrt(mean(x^2) + eps)      (rmsnorm.py:25-39)
    dx = r * (g - x * r^2 * mean(g*x)),  g = dy * w              (rmsnorm.py:43-55)
round_x rounds through x's dtype (the original's `.to(input_dtype)`); the weight is frozen, so
there is no dw. The output dtype is promote(weight, x), as in Qwen2RMSNorm.
"""

import torch

from . import _common, _lib, ops  # noqa: F401 - ops registers the custom operators


def fwd_into(x2, w, y, rstd, eps):
    """qb_rmsnorm_fwd over the rows of x2 [M, N] into y [M, N] (its own dtype) and rstd [M]."""
    _lib.require_cuda(x2, w, what="rmsnorm")
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    w = w if w.is_contiguous() else w.contiguous()
    M, N = x2.shape
    _lib.call("qb_rmsnorm_fwd", x2.data_ptr(), _lib.tag(x2.dtype), x2.stride(0), w.data_ptr(),
              _lib.tag(w.dtype), y.data_ptr(), _lib.tag(y.dtype), y.stride(0), rstd.data_ptr(),
              M, N, float(eps), _lib.stream(x2.device),
              work=(M * N * (x2.element_size() + y.element_size()) + M * 4, 0))


def bwd_into(dy2, x2, w, rstd, dx):
    """qb_rmsnorm_bwd: dx [M, N] (its own dtype) from dy2, the saved x2 and rstd."""
    if dy2.stride(-1) != 1:
        dy2 = dy2.contiguous()
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    w = w if w.is_contiguous() else w.contiguous()
    M, N = x2.shape
    _lib.call("qb_rmsnorm_bwd", dy2.data_ptr(), _lib.tag(dy2.dtype), dy2.stride(0),
              x2.data_ptr(), _lib.tag(x2.dtype), x2.stride(0), w.data_ptr(), _lib.tag(w.dtype),
              rstd.data_ptr(), dx.data_ptr(), _lib.tag(dx.dtype), dx.stride(0), M, N,
              _lib.stream(dy2.device),
              work=(M * N * (dy2.element_size() + 2 * x2.element_size()) + M * 4, 0))


class CudaRMSNorm:
    """Qwen2RMSNorm on the row kernels (rmsnorm.py:62-96): the custom op qlora_b200::rmsnorm,
    whose registered backward is qlora_b200::rmsnorm_bwd (dx; the weight is frozen)."""

    @staticmethod
    def apply(x, weight, eps, out_dtype):
        _lib.require_cuda(x, weight, what="rmsnorm")
        return torch.ops.qlora_b200.rmsnorm(x, weight, float(eps), out_dtype)[0]


# The reference's class name is part of its API; no Triton runs behind it here.
TritonRMSNorm = CudaRMSNorm


def rmsnorm(x, weight, eps):
    """Same result and dtype as Qwen2RMSNorm.forward (weight * x_normed.to(x.dtype))."""
    out_dtype = torch.promote_types(weight.dtype, x.dtype)
    return CudaRMSNorm.apply(x, weight, eps, out_dtype)


def patch():
    """Qwen2RMSNorm.forward through `rmsnorm` for what the kernels take (rmsnorm.py:99-115): a
    CUDA 1-D frozen weight over the last dimension of a float CUDA input."""
    from transformers.models.qwen2 import modeling_qwen2 as m

    def build(original):
        def forward(self, hidden_states):
            w = getattr(self, "weight", None)
            if (_common.on_gpu(hidden_states, w) and w.dim() == 1 and not w.requires_grad
                    and hidden_states.shape[-1] == w.shape[0]
                    and hidden_states.dtype in (torch.float32, torch.float16, torch.bfloat16)):
                return rmsnorm(hidden_states, w, self.variance_epsilon)
            return original(self, hidden_states)
        return forward

    _common.install(m.Qwen2RMSNorm, "forward", build)
