"""Rotary position embedding for q and k in one launch, forward and backward (API of
solution/rope.py).

With halves (x1, x2), (c1, c2), (s1, s2) of the last dimension:
    forward:  o1 = x1*c1 - x2*s1        o2 = x2*c2 + x1*s2
    backward: d1 = g1*c1 + g2*s2        d2 = g2*c2 - g1*s1
(the general form: it stays right when the two halves of cos/sin differ). q and k may be
(B, H, S, D) views of (B, S, H, D) buffers; outputs keep the input strides (empty_like), as the
original element-wise ops do.
"""

import torch

from . import _common, _lib


def _launch(q, k, cos, sin, q_out, k_out, backward):
    B, HQ, S, D = q.shape
    HK = k.shape[1]
    # the kernel reads cos/sin at b * stride(0) + s * stride(1): the tables must cover every
    # (b, s) it visits (a batch-broadcast table comes in expanded, batch stride 0)
    for t in (cos, sin):
        if t.dim() != 3 or t.shape[0] != B or t.shape[1] < S or t.shape[2] != D:
            raise ValueError(f"rope: table {tuple(t.shape)} does not cover (B, S, D) = "
                             f"({B}, {S}, {D})")
    if q.dtype != k.dtype or q_out.dtype != k_out.dtype or cos.dtype != sin.dtype:
        raise TypeError("rope: q/k, q_out/k_out and cos/sin must share dtypes")
    if cos.stride() != sin.stride():  # the kernel walks both with one set of strides
        cos, sin = cos.contiguous(), sin.contiguous()
    _lib.call("qb_rope_qk", q.data_ptr(), k.data_ptr(), q_out.data_ptr(), k_out.data_ptr(),
              cos.data_ptr(), sin.data_ptr(), _lib.tag(q.dtype), _lib.tag(q_out.dtype),
              _lib.tag(cos.dtype), B, HQ, HK, S, D, _lib.strides3(q), _lib.strides3(k),
              _lib.strides3(q_out), _lib.strides3(k_out), cos.stride(0), cos.stride(1),
              int(backward), _lib.stream(q.device),
              work=((HQ + HK) * B * S * D * (q.element_size() + q_out.element_size())
                    + 2 * S * D * cos.element_size(), 0))


def rope_rows(x2, cos, sin, backward=False):
    """RoPE (or its transpose) on a projection output laid out as rows of tokens: x2 [B*S, H*D]
    bf16 with row m the token at position m % S, cos/sin [S, D]. Returns a new [B*S, H*D]."""
    S, D = cos.shape
    T, F = x2.shape
    if cos.shape != sin.shape or T % S or F % D:
        raise ValueError(f"rope_rows: rows {T} x {F} do not tile by cos/sin {tuple(cos.shape)}")
    B = T // S
    q = x2.contiguous().view(B, S, F // D, D).transpose(1, 2)          # (B, H, S, D) view
    out = torch.empty((T, F), dtype=x2.dtype, device=x2.device)
    qo = out.view(B, S, F // D, D).transpose(1, 2)
    # one table for every sequence of the batch: batch stride 0, as CudaRoPE passes it
    c, s = cos[None].expand(B, S, D), sin[None].expand(B, S, D)
    _launch(q, q[:, :0], c, s, qo, qo[:, :0], backward)
    return out


def _unit_last(t):
    return t if t.stride(-1) == 1 else t.contiguous()


class CudaRoPE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, cos, sin):
        _lib.require_cuda(q, k, cos, sin, what="rope")
        B, _, S, _ = q.shape
        q, k = _unit_last(q), _unit_last(k)
        cos = _unit_last(cos).expand(B, S, -1)   # (B or 1, S, D) -> (B, S, D), stride 0 on B
        sin = _unit_last(sin).expand(B, S, -1)
        q_out = torch.empty_like(q, dtype=torch.promote_types(q.dtype, cos.dtype))
        k_out = torch.empty_like(k, dtype=torch.promote_types(k.dtype, cos.dtype))
        _launch(q, k, cos, sin, q_out, k_out, backward=False)
        ctx.save_for_backward(cos, sin)  # the backward needs no activations
        ctx.q_dtype, ctx.k_dtype = q.dtype, k.dtype
        return q_out, k_out

    @staticmethod
    def backward(ctx, dq_out, dk_out):
        cos, sin = ctx.saved_tensors
        dq_out, dk_out = _unit_last(dq_out), _unit_last(dk_out)
        if dq_out.dtype != dk_out.dtype:
            dk_out = dk_out.to(dq_out.dtype)
        dq = torch.empty_like(dq_out, dtype=ctx.q_dtype)
        dk = torch.empty_like(dk_out, dtype=ctx.k_dtype)
        _launch(dq_out, dk_out, cos, sin, dq, dk, backward=True)
        return dq, dk, None, None


# The reference's class name (rope.py:82) and the alias its stale test imports
# (test_kernels.py:79).
TritonRoPE = CudaRoPE
RoPEFunction = CudaRoPE


def _supported(q, k, cos, sin, unsqueeze_dim):
    if not _common.on_gpu(q, k, cos, sin) or unsqueeze_dim != 1:
        return False
    if q.dim() != 4 or k.dim() != 4 or cos.dim() != 3 or sin.shape != cos.shape:
        return False
    B, _, S, D = q.shape
    if k.shape[0] != B or k.shape[2] != S or k.shape[3] != D or D % 2 or (D & (D - 1)):
        return False
    if cos.shape[0] not in (1, B) or cos.shape[1] != S or cos.shape[2] != D:
        return False
    if q.dtype != k.dtype:
        return False
    return not (cos.requires_grad or sin.requires_grad)


def patch():
    """Sends modeling_qwen2.apply_rotary_pos_emb through CudaRoPE when the inputs fit
    (rope.py:120-135)."""
    from transformers.models.qwen2 import modeling_qwen2 as m

    original = m.apply_rotary_pos_emb
    if getattr(original, "_solution_patch", False):
        return

    def apply_rotary_pos_emb(q, k, cos, sin, *args, **kwargs):
        unsqueeze_dim = kwargs.get("unsqueeze_dim", args[0] if args else 1)
        if len(args) > 1 or set(kwargs) - {"unsqueeze_dim"} or \
                not _supported(q, k, cos, sin, unsqueeze_dim):
            return original(q, k, cos, sin, *args, **kwargs)
        return CudaRoPE.apply(q, k, cos, sin)

    apply_rotary_pos_emb._solution_patch = True
    m.apply_rotary_pos_emb = apply_rotary_pos_emb
