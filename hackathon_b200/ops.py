"""The suite's ops as PyTorch custom operators (torch.library, namespace `qlora_b200`).

Each op runs this package's sm_100a kernels through the C-ABI on the current stream, has a fake
(meta) implementation, so FakeTensor tracing and torch.compile see its output shapes without
running it, and - where it is differentiable - a registered autograd formula built from the
suite's own backward ops. The reference's autograd.Function class names (NF4Linear,
TritonRMSNorm, TritonRoPE, SwiGLU, DropoutCast, ScaledAdd, FusedLinearCrossEntropy,
FusedLinearCE) are thin aliases whose `apply` calls these ops.

    op                      computes                                          backward
    nf4_dequant             W from NF4 bytes + double-quantised scales        (frozen)
    nf4_linear              x W^T + b, W rebuilt from NF4                     nf4_linear_dgrad
    nf4_linear_dgrad        dy W
    rmsnorm                 (y, rstd) of Qwen2RMSNorm                         rmsnorm_bwd
    rmsnorm_bwd             dx
    rope                    rotate-half RoPE of q and k (or its transpose)    rope (transpose)
    swiglu                  silu(gate) * up                                   swiglu_bwd
    swiglu_bwd              (dgate, dup)
    dropout_scale           Philox dropout (reference stream) * scale, cast   dropout_scale
    scaled_add              base + lo * scaling                               dropout_scale
    gemm                    a @ b_t^T, fp32 accumulation (the LoRA products)  gemm
    linear_ce               per-row CE loss, entropy, argmax of h W^T and the
                            per-row gradient of the loss (logits never whole) dh_rows * g

No op has a CPU kernel: called on CPU tensors they raise (device_types="cuda").
"""

from typing import Optional

import torch
from torch import Tensor

NS = "qlora_b200"


def _op(name, **kw):
    return torch.library.custom_op(f"{NS}::{name}", mutates_args=(), device_types="cuda", **kw)


# ------------------------------------------------------------------------------------------
# NF4


@_op("nf4_dequant")
def nf4_dequant(packed: Tensor, absmax: Tensor, code2: Optional[Tensor],
                absmax2: Optional[Tensor], offset: float, blocksize: int, blocksize2: int,
                rows: int, cols: int, dtype: torch.dtype) -> Tensor:
    from .nf4 import dequant_into
    out = torch.empty((rows, cols), dtype=dtype, device=packed.device)
    dequant_into(out, packed, absmax, code2, absmax2, offset, blocksize, blocksize2)
    return out


@nf4_dequant.register_fake
def _(packed, absmax, code2, absmax2, offset, blocksize, blocksize2, rows, cols, dtype):
    return packed.new_empty((rows, cols), dtype=dtype)


@_op("nf4_linear")
def nf4_linear(x: Tensor, packed: Tensor, absmax: Tensor, code2: Optional[Tensor],
               absmax2: Optional[Tensor], offset: float, blocksize: int, blocksize2: int,
               out_features: int, in_features: int, bias: Optional[Tensor]) -> Tensor:
    from .nf4 import fused_ok, nf4_linear_fwd, state_of
    qs = state_of(absmax, code2, absmax2, offset, blocksize, blocksize2, out_features,
                  in_features)
    if fused_ok(x, qs):    # bf16: the weight is rebuilt inside the tcgen05 GEMM
        return nf4_linear_fwd(x, packed, qs, bias)
    w = nf4_dequant(packed, absmax, code2, absmax2, offset, blocksize, blocksize2,
                    out_features, in_features, x.dtype)
    return torch.nn.functional.linear(x, w, bias)


@nf4_linear.register_fake
def _(x, packed, absmax, code2, absmax2, offset, blocksize, blocksize2, out_features,
      in_features, bias):
    return x.new_empty((*x.shape[:-1], out_features))


@_op("nf4_linear_dgrad")
def nf4_linear_dgrad(dy: Tensor, packed: Tensor, absmax: Tensor, code2: Optional[Tensor],
                     absmax2: Optional[Tensor], offset: float, blocksize: int, blocksize2: int,
                     out_features: int, in_features: int) -> Tensor:
    from . import nf4
    qs = nf4.state_of(absmax, code2, absmax2, offset, blocksize, blocksize2, out_features,
                      in_features)
    if nf4.fused_ok(dy, qs):
        return nf4.nf4_linear_dgrad(dy, packed, qs)
    w = nf4_dequant(packed, absmax, code2, absmax2, offset, blocksize, blocksize2,
                    out_features, in_features, dy.dtype)
    return torch.matmul(dy, w)


@nf4_linear_dgrad.register_fake
def _(dy, packed, absmax, code2, absmax2, offset, blocksize, blocksize2, out_features,
      in_features):
    return dy.new_empty((*dy.shape[:-1], in_features))


def _nf4_linear_setup(ctx, inputs, output):
    (_, packed, absmax, code2, absmax2, offset, bs, bs2, out_f, in_f, _) = inputs
    ctx.save_for_backward(packed, absmax, code2, absmax2)
    ctx.meta = (offset, bs, bs2, out_f, in_f)


def _nf4_linear_backward(ctx, grad):
    packed, absmax, code2, absmax2 = ctx.saved_tensors
    dx = None
    if ctx.needs_input_grad[0]:
        dx = nf4_linear_dgrad(grad, packed, absmax, code2, absmax2, *ctx.meta)
    return dx, None, None, None, None, None, None, None, None, None, None


nf4_linear.register_autograd(_nf4_linear_backward, setup_context=_nf4_linear_setup)


# ------------------------------------------------------------------------------------------
# RMSNorm


@_op("rmsnorm")
def rmsnorm(x: Tensor, weight: Tensor, eps: float,
            out_dtype: torch.dtype) -> tuple[Tensor, Tensor]:
    from .rmsnorm import fwd_into
    x2 = x.reshape(-1, x.shape[-1])
    y = torch.empty(x2.shape, dtype=out_dtype, device=x.device)
    rstd = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device)
    fwd_into(x2, weight, y, rstd, eps)
    return y.view(x.shape), rstd


@rmsnorm.register_fake
def _(x, weight, eps, out_dtype):
    rows = x.numel() // x.shape[-1]
    return x.new_empty(x.shape, dtype=out_dtype), x.new_empty((rows,), dtype=torch.float32)


@_op("rmsnorm_bwd")
def rmsnorm_bwd(dy: Tensor, x: Tensor, weight: Tensor, rstd: Tensor) -> Tensor:
    from .rmsnorm import bwd_into
    x2 = x.reshape(-1, x.shape[-1])
    dx = torch.empty(x2.shape, dtype=x.dtype, device=x.device)
    bwd_into(dy.reshape(x2.shape), x2, weight, rstd, dx)
    return dx.view(x.shape)


@rmsnorm_bwd.register_fake
def _(dy, x, weight, rstd):
    return x.new_empty(x.shape)


def _rmsnorm_setup(ctx, inputs, output):
    x, weight, _, _ = inputs
    ctx.save_for_backward(x, weight, output[1])
    ctx.mark_non_differentiable(output[1])


def _rmsnorm_backward(ctx, dy, _drstd):
    x, weight, rstd = ctx.saved_tensors
    return rmsnorm_bwd(dy, x, weight, rstd), None, None, None


rmsnorm.register_autograd(_rmsnorm_backward, setup_context=_rmsnorm_setup)


# ------------------------------------------------------------------------------------------
# RoPE


def _unit_last(t):
    return t if t.stride(-1) == 1 else t.contiguous()


@_op("rope")
def rope(q: Tensor, k: Tensor, cos: Tensor, sin: Tensor, transpose: bool, q_dtype: torch.dtype,
         k_dtype: torch.dtype) -> tuple[Tensor, Tensor]:
    """Outputs keep the inputs' layout (q, k may be (B, H, S, D) views of (B, S, H, D))."""
    from .rope import apply_into
    q, k = _unit_last(q), _unit_last(k)
    q_out = torch.empty_like(q, dtype=q_dtype)
    k_out = torch.empty_like(k, dtype=k_dtype)
    apply_into(q, k, cos, sin, q_out, k_out, transpose)
    return q_out, k_out


@rope.register_fake
def _(q, k, cos, sin, transpose, q_dtype, k_dtype):
    q, k = _unit_last(q), _unit_last(k)
    return torch.empty_like(q, dtype=q_dtype), torch.empty_like(k, dtype=k_dtype)


def _rope_setup(ctx, inputs, output):
    q, k, cos, sin, transpose, _, _ = inputs
    ctx.save_for_backward(cos, sin)
    ctx.transpose, ctx.dtypes = transpose, (q.dtype, k.dtype)


def _rope_backward(ctx, gq, gk):
    cos, sin = ctx.saved_tensors
    if gk.dtype != gq.dtype:
        gk = gk.to(gq.dtype)
    dq, dk = rope(gq, gk, cos, sin, not ctx.transpose, *ctx.dtypes)
    return dq, dk, None, None, None, None, None


rope.register_autograd(_rope_backward, setup_context=_rope_setup)


# ------------------------------------------------------------------------------------------
# SwiGLU


@_op("swiglu")
def swiglu(gate: Tensor, up: Tensor) -> Tensor:
    from .swiglu import fwd_into
    g = gate.contiguous()
    u = up.to(g.dtype).contiguous()
    out = torch.empty_like(g)
    fwd_into(g, u, out)
    return out


@swiglu.register_fake
def _(gate, up):
    return torch.empty_like(gate, memory_format=torch.contiguous_format)


@_op("swiglu_bwd")
def swiglu_bwd(grad: Tensor, gate: Tensor, up: Tensor) -> tuple[Tensor, Tensor]:
    from .swiglu import bwd_into
    g = gate.contiguous()
    u = up.to(g.dtype).contiguous()
    dg, du = torch.empty_like(g), torch.empty_like(u)
    bwd_into(grad.to(g.dtype).contiguous(), g, u, dg, du)
    return dg, du


@swiglu_bwd.register_fake
def _(grad, gate, up):
    return (torch.empty_like(gate, memory_format=torch.contiguous_format),
            torch.empty_like(gate, memory_format=torch.contiguous_format))


def _swiglu_setup(ctx, inputs, output):
    gate, up = inputs
    ctx.save_for_backward(gate, up)
    ctx.up_dtype = up.dtype


def _swiglu_backward(ctx, grad):
    gate, up = ctx.saved_tensors
    dg, du = swiglu_bwd(grad, gate, up)
    return dg, du if du.dtype == ctx.up_dtype else du.to(ctx.up_dtype)


swiglu.register_autograd(_swiglu_backward, setup_context=_swiglu_setup)


# ------------------------------------------------------------------------------------------
# LoRA dropout-cast and scaled add


@_op("dropout_scale")
def dropout_scale(x: Tensor, p: float, seed: int, scale: float, out_dtype: torch.dtype) -> Tensor:
    from .lora import dropout_scale_into
    out = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    dropout_scale_into(x, out, p, seed, scale)
    return out


@dropout_scale.register_fake
def _(x, p, seed, scale, out_dtype):
    return x.new_empty(x.shape, dtype=out_dtype)


def _dropout_setup(ctx, inputs, output):
    x, p, seed, scale, _ = inputs
    ctx.args = (p, seed, scale, x.dtype)


def _dropout_backward(ctx, g):
    return dropout_scale(g, *ctx.args), None, None, None, None


dropout_scale.register_autograd(_dropout_backward, setup_context=_dropout_setup)


@_op("scaled_add")
def scaled_add(base: Tensor, lo: Tensor, scaling: float) -> Tensor:
    from .lora import scaled_add_into
    out = torch.empty(base.shape, dtype=torch.promote_types(base.dtype, lo.dtype),
                      device=base.device)
    scaled_add_into(base, lo, out, scaling)
    return out


@scaled_add.register_fake
def _(base, lo, scaling):
    return base.new_empty(base.shape, dtype=torch.promote_types(base.dtype, lo.dtype))


def _scaled_add_setup(ctx, inputs, output):
    base, lo, scaling = inputs
    ctx.scaling, ctx.dtypes = scaling, (base.dtype, lo.dtype)


def _scaled_add_backward(ctx, g):
    base_dtype, lo_dtype = ctx.dtypes
    d_base = g if g.dtype == base_dtype else g.to(base_dtype)
    return d_base, dropout_scale(g, 0.0, 0, ctx.scaling, lo_dtype), None


scaled_add.register_autograd(_scaled_add_backward, setup_context=_scaled_add_setup)


# ------------------------------------------------------------------------------------------
# GEMM (the LoRA products: xd A^T, V = g (s B), dA = V^T xd, dB = s g^T U)


@_op("gemm")
def gemm(a: Tensor, b_t: Tensor, out_dtype: torch.dtype) -> Tensor:
    from .gemm import gemm as run
    return run(a, b_t, out_dtype=out_dtype)


@gemm.register_fake
def _(a, b_t, out_dtype):
    return a.new_empty((a.shape[0], b_t.shape[0]), dtype=out_dtype)


def _gemm_setup(ctx, inputs, output):
    a, b_t, _ = inputs
    ctx.save_for_backward(a, b_t)


def _gemm_backward(ctx, g):
    a, b_t = ctx.saved_tensors
    g16 = g if g.dtype == torch.bfloat16 else g.to(torch.bfloat16)
    da = gemm(g16, b_t.t(), a.dtype) if ctx.needs_input_grad[0] else None
    db = gemm(g16.t(), a.t(), b_t.dtype) if ctx.needs_input_grad[1] else None
    return da, db, None


gemm.register_autograd(_gemm_backward, setup_context=_gemm_setup)


# ------------------------------------------------------------------------------------------
# Linear cross-entropy


@_op("linear_ce")
def linear_ce(hidden: Tensor, weight: Tensor, target: Tensor, chunk_rows: int,
              with_grad: bool) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    from .cross_entropy import linear_ce_rows
    return linear_ce_rows(hidden, weight, target, chunk_rows, with_grad)


@linear_ce.register_fake
def _(hidden, weight, target, chunk_rows, with_grad):
    n, h = hidden.shape
    f32 = torch.float32
    return (hidden.new_empty((n,), dtype=f32), hidden.new_empty((n,), dtype=f32),
            hidden.new_empty((n,), dtype=torch.int64),
            hidden.new_empty((n if with_grad else 0, h), dtype=f32))


def _linear_ce_setup(ctx, inputs, output):
    ctx.save_for_backward(output[3])
    ctx.hidden_dtype = inputs[0].dtype
    ctx.mark_non_differentiable(output[1], output[2], output[3])


def _linear_ce_backward(ctx, g_loss, _g_entropy, _g_pred, _g_dh):
    (dh_rows,) = ctx.saved_tensors
    if dh_rows.shape[0] != g_loss.shape[0]:
        raise RuntimeError("qlora_b200::linear_ce: backward through a call made without the "
                           "gradient (with_grad=False)")
    grad = dh_rows * g_loss.float()[:, None]
    return grad.to(ctx.hidden_dtype), None, None, None, None


linear_ce.register_autograd(_linear_ce_backward, setup_context=_linear_ce_setup)


def ops():
    """Every op of the namespace (for checks such as torch.library.opcheck)."""
    return {name: getattr(torch.ops.qlora_b200, name) for name in (
        "nf4_dequant", "nf4_linear", "nf4_linear_dgrad", "rmsnorm", "rmsnorm_bwd", "rope",
        "swiglu", "swiglu_bwd", "dropout_scale", "scaled_add", "gemm", "linear_ce")}
