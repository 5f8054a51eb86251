"""Small helpers shared by the ops and the patches (mirrors solution/_common.py:6-25)."""

import torch


def on_gpu(*tensors):
    """True when every argument is a CUDA tensor. Every patch checks this first and hands other
    inputs (CPU tensors, meta tensors, fakes) to the unpatched upstream code."""
    return all(isinstance(t, torch.Tensor) and t.is_cuda for t in tensors)


def autocast_dtype():
    """The dtype CUDA matmuls run in right now: the autocast dtype when autocast is on, else None."""
    if torch.is_autocast_enabled("cuda"):
        return torch.get_autocast_dtype("cuda")
    return None


def round_mode(dtype):
    """0: keep fp32, 1: round through fp16, 2: round through bf16 (the kernels' dtype tags)."""
    if dtype == torch.float16:
        return 1
    if dtype == torch.bfloat16:
        return 2
    return 0
