"""The qlora_b200 custom operators without a GPU: every op is registered with a fake (meta)
implementation that gives its outputs' shapes and dtypes under FakeTensorMode - what
torch.compile and FakeTensor tracing see - the differentiable ones carry an autograd formula, and
a CPU tensor reaches no kernel: the op raises (there is no CPU path)."""

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import hackathon_b200.ops as qops

BF = torch.bfloat16


def _fake_calls():
    """(op name, args, output shapes) for every op; the tensors are meta tensors that the test
    turns into CUDA fake tensors of the same shape, dtype and strides."""
    c = dict(device="meta")
    e = lambda *s, dtype=BF: torch.empty(*s, dtype=dtype, **c)  # noqa: E731
    f32, u8, i64 = torch.float32, torch.uint8, torch.int64
    nf4 = (e(256 * 512 // 2, 1, dtype=u8), e(256 * 512 // 64, dtype=u8), e(256, dtype=f32),
           e(8, dtype=f32), 0.01, 64, 256)
    q = e(2, 16, 4, 128).transpose(1, 2)          # (B, H, S, D) view of (B, S, H, D)
    k = e(2, 16, 2, 128).transpose(1, 2)
    return [
        ("nf4_dequant", nf4 + (256, 512, BF), [(256, 512)]),
        ("nf4_linear", (e(3, 5, 512),) + nf4 + (256, 512, None), [(3, 5, 256)]),
        ("nf4_linear_dgrad", (e(3, 5, 256),) + nf4 + (256, 512), [(3, 5, 512)]),
        ("rmsnorm", (e(3, 5, 64), e(64), 1e-6, BF), [(3, 5, 64), (15,)]),
        ("rmsnorm_bwd", (e(3, 5, 64), e(3, 5, 64), e(64), e(15, dtype=f32)), [(3, 5, 64)]),
        ("rope", (q, k, e(1, 16, 128), e(1, 16, 128), False, BF, BF),
         [(2, 4, 16, 128), (2, 2, 16, 128)]),
        ("swiglu", (e(8, 96), e(8, 96)), [(8, 96)]),
        ("swiglu_bwd", (e(8, 96), e(8, 96), e(8, 96)), [(8, 96), (8, 96)]),
        ("dropout_scale", (e(8, 96), 0.1, 1234, 1 / 0.9, f32), [(8, 96)]),
        ("scaled_add", (e(8, 96), e(8, 96, dtype=f32), 2.0), [(8, 96)]),
        ("gemm", (e(64, 32), e(48, 32), f32), [(64, 48)]),
        ("linear_ce", (e(10, 64), e(300, 64), e(10, dtype=i64), 4, True),
         [(10,), (10,), (10,), (10, 64)]),
    ]


def test_every_op_is_registered():
    assert set(qops.ops()) == {name for name, _, _ in _fake_calls()}


@pytest.mark.parametrize("name,args,shapes", _fake_calls(), ids=[c[0] for c in _fake_calls()])
def test_fake_implementation_gives_the_output_shapes(name, args, shapes):
    with FakeTensorMode():
        args = tuple(torch.empty_strided(a.shape, a.stride(), dtype=a.dtype, device="cuda")
                     if isinstance(a, torch.Tensor) else a for a in args)
        out = getattr(torch.ops.qlora_b200, name)(*args)
    outs = out if isinstance(out, (tuple, list)) else (out,)
    assert [tuple(o.shape) for o in outs] == shapes
    assert all(o.device.type == "cuda" for o in outs)


def test_rope_outputs_keep_the_strided_layout_under_fake_tensors():
    with FakeTensorMode():
        q = torch.empty(2, 16, 4, 128, dtype=BF, device="cuda").transpose(1, 2)
        k = torch.empty(2, 16, 2, 128, dtype=BF, device="cuda").transpose(1, 2)
        c = torch.empty(1, 16, 128, dtype=BF, device="cuda")
        qo, ko = torch.ops.qlora_b200.rope(q, k, c, c, False, BF, BF)
    assert qo.stride() == q.stride() and ko.stride() == k.stride()


def test_differentiable_ops_have_a_backward_on_meta_tensors():
    """The registered autograd formulas run on meta tensors (through their own ops' fakes): the
    gradients have the inputs' shapes and dtypes."""
    m = dict(dtype=BF, device="meta")
    x = torch.empty(6, 64, requires_grad=True, **m)
    y, _ = torch.ops.qlora_b200.rmsnorm(x, torch.empty(64, **m), 1e-6, BF)
    (gx,) = torch.autograd.grad(y.sum(), x)
    assert gx.shape == x.shape
    a = torch.empty(32, 16, requires_grad=True, **m)
    b = torch.empty(8, 16, requires_grad=True, **m)
    ga, gb = torch.autograd.grad(torch.ops.qlora_b200.gemm(a, b, BF).sum(), (a, b))
    assert ga.shape == a.shape and gb.shape == b.shape
    h = torch.empty(10, 64, requires_grad=True, **m)
    t = torch.empty(10, dtype=torch.int64, device="meta")
    loss = torch.ops.qlora_b200.linear_ce(h, torch.empty(300, 64, **m), t, 4, True)[0]
    (gh,) = torch.autograd.grad(loss.sum(), h)
    assert gh.shape == h.shape and gh.dtype == BF
    g = torch.empty(8, 96, requires_grad=True, **m)
    dg, du = torch.autograd.grad(torch.ops.qlora_b200.swiglu(g, g).sum(), (g, g))
    assert dg.shape == g.shape


def test_cpu_tensors_reach_no_kernel():
    with pytest.raises(NotImplementedError, match="CPU"):
        torch.ops.qlora_b200.swiglu(torch.ones(4, 8), torch.ones(4, 8))


def test_reference_class_names_call_the_ops():
    """The reference's autograd.Function names are thin aliases over the custom ops."""
    from hackathon_b200 import cross_entropy, fused_ce, lora, nf4, rmsnorm, rope, swiglu
    for cls in (nf4.NF4Linear, rmsnorm.TritonRMSNorm, rope.TritonRoPE, rope.RoPEFunction,
                swiglu.SwiGLU, lora.DropoutCast, lora.ScaledAdd,
                cross_entropy.FusedLinearCrossEntropy, fused_ce.FusedLinearCE):
        assert callable(cls.apply)
    with FakeTensorMode():
        x = torch.empty(4, 8, dtype=BF, device="cuda")
        assert swiglu.SwiGLU.apply(x, x).shape == (4, 8)
        assert lora.DropoutCast.apply(x, 0.1, 2 ** 63 + 5, torch.float32).dtype == torch.float32
        assert lora.ScaledAdd.apply(x, x, 2.0).shape == (4, 8)
