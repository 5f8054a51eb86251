"""Fused SwiGLU, silu(gate) * up, forward and backward (API of solution/swiglu.py)."""

import torch

from . import _common, _lib, ops  # noqa: F401 - ops registers the custom operators


def fwd_into(gate, up, out):
    """qb_swiglu_fwd: out = silu(gate) * up, all contiguous and of one dtype."""
    _lib.require_cuda(gate, up, what="swiglu")
    _lib.call("qb_swiglu_fwd", gate.data_ptr(), up.data_ptr(), out.data_ptr(),
              _lib.tag(gate.dtype), gate.numel(), _lib.stream(gate.device),
              work=(3 * gate.numel() * gate.element_size(), 0))


def bwd_into(grad, gate, up, dgate, dup):
    """qb_swiglu_bwd: (dgate, dup) of silu(gate) * up, all contiguous and of one dtype."""
    _lib.call("qb_swiglu_bwd", grad.data_ptr(), gate.data_ptr(), up.data_ptr(),
              dgate.data_ptr(), dup.data_ptr(), _lib.tag(gate.dtype), gate.numel(),
              _lib.stream(gate.device), work=(5 * gate.numel() * gate.element_size(), 0))


class SwiGLU:
    """silu(gate) * up in one launch each way (swiglu.py:40-61): the custom op
    qlora_b200::swiglu, whose registered backward is qlora_b200::swiglu_bwd."""

    @staticmethod
    def apply(gate, up):
        _lib.require_cuda(gate, up, what="swiglu")
        return torch.ops.qlora_b200.swiglu(gate, up)


def swiglu(gate, up):
    return SwiGLU.apply(gate, up)


def patch_qwen2_mlp():
    """Qwen2MLP.forward with the fused SwiGLU between its projections (swiglu.py:68-81), for a
    silu MLP on a CUDA input."""
    from transformers.models.qwen2 import modeling_qwen2 as m

    def build(original):
        def forward(self, x):
            act = getattr(getattr(self, "config", None), "hidden_act", "silu")
            if act == "silu" and x.is_cuda:
                return self.down_proj(swiglu(self.gate_proj(x), self.up_proj(x)))
            return original(self, x)
        return forward

    _common.install(m.Qwen2MLP, "forward", build)
