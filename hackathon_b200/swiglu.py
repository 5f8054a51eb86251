"""Fused SwiGLU, silu(gate) * up, forward and backward (API of solution/swiglu.py)."""

import torch

from . import _lib


class SwiGLU(torch.autograd.Function):
    """silu(gate) * up in one launch each way (swiglu.py:40-61)."""

    @staticmethod
    def forward(ctx, gate, up):
        _lib.require_cuda(gate, up, what="swiglu")
        gate = gate.contiguous()
        up = up.to(gate.dtype).contiguous()
        out = torch.empty_like(gate)
        _lib.call("qb_swiglu_fwd", gate.data_ptr(), up.data_ptr(), out.data_ptr(),
                  _lib.tag(gate.dtype), gate.numel(), _lib.stream(gate.device),
                  work=(3 * gate.numel() * gate.element_size(), 0))
        ctx.save_for_backward(gate, up)
        return out

    @staticmethod
    def backward(ctx, grad):
        gate, up = ctx.saved_tensors
        grad = grad.to(gate.dtype).contiguous()
        dgate, dup = torch.empty_like(gate), torch.empty_like(up)
        _lib.call("qb_swiglu_bwd", grad.data_ptr(), gate.data_ptr(), up.data_ptr(),
                  dgate.data_ptr(), dup.data_ptr(), _lib.tag(gate.dtype), gate.numel(),
                  _lib.stream(gate.device), work=(5 * gate.numel() * gate.element_size(), 0))
        return dgate, dup


def swiglu(gate, up):
    return SwiGLU.apply(gate, up)


def patch_qwen2_mlp():
    """Sends Qwen2MLP.forward through the fused kernel (swiglu.py:68-81)."""
    from transformers.models.qwen2 import modeling_qwen2

    original = modeling_qwen2.Qwen2MLP.forward
    if getattr(original, "_solution_patch", False):
        return

    def forward(self, x):
        act = getattr(getattr(self, "config", None), "hidden_act", "silu")
        if act != "silu" or not x.is_cuda:
            return original(self, x)
        return self.down_proj(swiglu(self.gate_proj(x), self.up_proj(x)))

    forward._solution_patch = True
    modeling_qwen2.Qwen2MLP.forward = forward
