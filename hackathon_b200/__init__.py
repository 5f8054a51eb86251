"""qlora_b200: a B200 (sm_100a) CUDA kernel suite for the Qwen2.5 QLoRA training step.

A drop-in for the Python API of the reference package `solution/` (imoshka2009-lab/hackathon):

  nf4.py            dequantize_nf4, NF4Linear, linear4bit, quantize_nf4     NF4 + double quant
  rmsnorm.py        rmsnorm, TritonRMSNorm (= CudaRMSNorm), patch()         fwd + bwd
  rope.py           TritonRoPE (= CudaRoPE = RoPEFunction), patch()         fwd + bwd, q and k
  swiglu.py         swiglu, SwiGLU, patch_qwen2_mlp()                       fwd + bwd
  lora.py           DropoutCast, ScaledAdd, patch()                         Philox dropout
  cross_entropy.py  fused_causal_lm_loss, FusedLinearCrossEntropy, patch()  chunked linear CE
  fused_ce.py       fused_head_loss, FusedLinearCE, ce_rows                 earlier CE API

Every op calls hand-written sm_100a kernels through the C-ABI of libqlora_b200.so
(include/qlora_b200.h); none has a CPU path. `apply()` installs the patches on transformers /
peft / trl classes, as the reference's apply() does (solution/__init__.py:17-34).
"""

PATCHES = ("rmsnorm", "rope", "cross_entropy", "lora")

_applied = set()


def apply(include_example=True):
    """Installs every patch (idempotent). Call before the model and trainer are built."""
    from importlib import import_module

    for name in PATCHES:
        if name not in _applied:
            import_module(f"{__name__}.{name}").patch()
            _applied.add(name)
    if include_example and "swiglu" not in _applied:
        from .swiglu import patch_qwen2_mlp

        patch_qwen2_mlp()
        _applied.add("swiglu")
