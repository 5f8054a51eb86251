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

from . import _common, _lib, ops  # noqa: F401 - ops registers the custom operators


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


def apply_into(q, k, cos, sin, q_out, k_out, transpose):
    """RoPE (transpose=False) or its transpose on q [B, HQ, S, D] and k [B, HK, S, D] (unit last
    stride, any other strides) into q_out / k_out; cos/sin (B or 1, >= S, D)."""
    _lib.require_cuda(q, k, cos, sin, what="rope")
    B = q.shape[0]
    cos = _unit_last(cos).expand(B, cos.shape[1], -1)   # (B or 1, S, D) -> (B, S, D)
    sin = _unit_last(sin).expand(B, sin.shape[1], -1)
    _launch(q, k, cos, sin, q_out, k_out, transpose)


class CudaRoPE:
    """Rotate-half RoPE of q and k in one launch (rope.py:82-104): the custom op qlora_b200::rope,
    whose registered backward is the same op with the transposed rotation. Outputs are in
    promote(q, cos) / promote(k, cos) and keep q's / k's layout."""

    @staticmethod
    def apply(q, k, cos, sin):
        _lib.require_cuda(q, k, cos, sin, what="rope")
        return torch.ops.qlora_b200.rope(q, k, cos, sin, False,
                                         torch.promote_types(q.dtype, cos.dtype),
                                         torch.promote_types(k.dtype, cos.dtype))


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
    """modeling_qwen2.apply_rotary_pos_emb through CudaRoPE for the calls `_supported` admits
    (rope.py:120-135); anything else, extra arguments included, goes to the original."""
    from transformers.models.qwen2 import modeling_qwen2 as m

    def build(original):
        def apply_rotary_pos_emb(q, k, cos, sin, *args, **kwargs):
            dim = kwargs.get("unsqueeze_dim", args[0] if args else 1)
            if len(args) <= 1 and set(kwargs) <= {"unsqueeze_dim"} and \
                    _supported(q, k, cos, sin, dim):
                return CudaRoPE.apply(q, k, cos, sin)
            return original(q, k, cos, sin, *args, **kwargs)
        return apply_rotary_pos_emb

    _common.install(m, "apply_rotary_pos_emb", build)
