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


PATCH_MARK = "_qlora_b200_patch"


def install(owner, name, build):
    """Replaces owner.<name> by build(original) once: the replacement carries PATCH_MARK and the
    original as __wrapped__, so a second call (and apply() run twice) leaves it alone. Every
    patch of this package goes through here; each replacement hands the inputs its kernels do
    not take to `original` unchanged. Returns the function now installed."""
    current = getattr(owner, name)
    if getattr(current, PATCH_MARK, False):
        return current
    replacement = build(current)
    setattr(replacement, PATCH_MARK, True)
    replacement.__wrapped__ = current
    setattr(owner, name, replacement)
    return replacement
