"""The NF4 x LoRA projection on both of its paths — "fused" (tcgen05, weight dequantised in
registers inside the GEMM) and "dequant" (transient bf16 weight, then the TMA-fed two-segment
GEMM) — against the same math on a materialised weight: dequantize_nf4 (bit-exact with the
reference kernel) then an fp32 product. Forward with bias and the LoRA term as extra K,
input-gradient with the LoRA term, at Qwen2.5 projection shapes and ragged token counts."""

import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [(512, 3584, 300), (3584, 3584, 1024), (256, 896, 77), (18944, 3584, 256),
          (3584, 18944, 256), (128, 128, 1)]
PATHS = ["fused", "dequant"]


def _setup(cuda, out_f, in_f, T, seed=0):
    from hackathon_b200.nf4 import dequantize_nf4, quantize_nf4
    g = torch.Generator(device=cuda).manual_seed(seed)
    w = (torch.randn(out_f, in_f, device=cuda, generator=g) * 0.02).to(torch.bfloat16)
    packed, st = quantize_nf4(w)
    wd = dequantize_nf4(packed, st, torch.bfloat16).float()
    x = torch.randn(T, in_f, device=cuda, generator=g).to(torch.bfloat16)
    return packed, st, wd, x, g


def _close(got, ref):
    torch.testing.assert_close(got.float(), ref, rtol=1.6e-2, atol=2e-2)


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("shape", SHAPES)
def test_fwd_matches_dequant_matmul(cuda, shape, path):
    from hackathon_b200.gemm import device_error
    from hackathon_b200.nf4 import nf4_linear_fwd
    out_f, in_f, T = shape
    packed, st, wd, x, g = _setup(cuda, out_f, in_f, T)
    bias = torch.randn(out_f, device=cuda, generator=g).to(torch.bfloat16)
    y = nf4_linear_fwd(x, packed, st, bias, path=path)
    device_error()
    _close(y, x.float() @ wd.t() + bias.float())


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("r", [16, 64])
@pytest.mark.parametrize("shape", [(512, 3584, 300), (3584, 3584, 1024), (256, 896, 77)])
def test_fwd_with_lora_as_extra_k(cuda, shape, r, path):
    from hackathon_b200.gemm import device_error
    from hackathon_b200.nf4 import nf4_linear_fwd
    out_f, in_f, T = shape
    packed, st, wd, x, g = _setup(cuda, out_f, in_f, T, seed=1)
    u = torch.randn(T, r, device=cuda, generator=g).to(torch.bfloat16)
    lb = (torch.randn(out_f, r, device=cuda, generator=g) * 0.05).to(torch.bfloat16)
    y = nf4_linear_fwd(x, packed, st, None, u, lb, path=path)
    device_error()
    _close(y, x.float() @ wd.t() + u.float() @ lb.float().t())


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("r", [0, 64])
def test_dgrad_matches_dequant_matmul(cuda, shape, r, path):
    from hackathon_b200.gemm import device_error
    from hackathon_b200.nf4 import nf4_linear_dgrad
    out_f, in_f, T = shape
    packed, st, wd, _, g = _setup(cuda, out_f, in_f, T, seed=2)
    dy = torch.randn(T, out_f, device=cuda, generator=g).to(torch.bfloat16)
    if r:
        v = torch.randn(T, r, device=cuda, generator=g).to(torch.bfloat16)
        la = (torch.randn(r, in_f, device=cuda, generator=g) * 0.05).to(torch.bfloat16)
        dx = nf4_linear_dgrad(dy, packed, st, v, la, path=path)
        ref = dy.float() @ wd + v.float() @ la.float()
    else:
        dx = nf4_linear_dgrad(dy, packed, st, path=path)
        ref = dy.float() @ wd
    device_error()
    _close(dx, ref)


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("shape", [(384, 256), (512, 3584), (256, 896)])
def test_weight_operand_is_bit_exact(cuda, shape, path):
    """With identity activations every output element is one weight times 1.0, accumulated
    exactly: both paths must reproduce dequantize_nf4's bf16 weights bit for bit (and
    dequantize_nf4 is bit-exact with the reference kernel)."""
    from hackathon_b200.gemm import device_error
    from hackathon_b200.nf4 import dequantize_nf4, nf4_linear_dgrad, nf4_linear_fwd, quantize_nf4
    out_f, in_f = shape
    g = torch.Generator(device=cuda).manual_seed(11)
    w = (torch.randn(out_f, in_f, device=cuda, generator=g) * 0.02).to(torch.bfloat16)
    packed, st = quantize_nf4(w)
    wd = dequantize_nf4(packed, st, torch.bfloat16)
    eye_in = torch.eye(in_f, device=cuda, dtype=torch.bfloat16)
    y = nf4_linear_fwd(eye_in, packed, st, path=path)            # y[t, o] = W[o, t]
    eye_out = torch.eye(out_f, device=cuda, dtype=torch.bfloat16)
    dx = nf4_linear_dgrad(eye_out, packed, st, path=path)        # dx[t, i] = W[t, i]
    device_error()
    assert torch.equal(y.view(torch.int16), wd.t().contiguous().view(torch.int16))
    assert torch.equal(dx.view(torch.int16), wd.view(torch.int16))


def test_nf4linear_autograd_fused_matches_unfused(cuda):
    """NF4Linear (the reference's autograd API) on bf16 takes the fused kernels; fp32 inputs take
    dequantize + matmul. Both agree."""
    from hackathon_b200.nf4 import NF4Linear, fused_ok
    packed, st, wd, x, g = _setup(cuda, 1024, 1536, 333, seed=3)
    assert fused_ok(x, st)
    bias = torch.randn(1024, device=cuda, generator=g).to(torch.bfloat16)
    xb = x.clone().requires_grad_()
    y = NF4Linear.apply(xb, packed, st, bias)
    gy = torch.randn_like(y)
    y.backward(gy)
    xf = x.float().requires_grad_()
    yf = NF4Linear.apply(xf, packed, st, bias.float())
    yf.backward(gy.float())
    _close(y, yf.detach())
    _close(xb.grad, xf.grad)


def test_long_token_counts_take_the_dequant_path(cuda):
    """At DEQUANT_GEMM_MIN_TOKENS and above the default path is the transient-weight GEMM; it
    agrees with the fused kernel on the same call (both fp32-accumulated: same tolerance), and the
    workspace is reused across projections of different shapes on one stream."""
    from hackathon_b200 import nf4
    from hackathon_b200.gemm import device_error
    T = nf4.DEQUANT_GEMM_MIN_TOKENS
    for out_f, in_f in [(256, 896), (896, 256)]:
        packed, st, wd, x, g = _setup(cuda, out_f, in_f, T, seed=5)
        u = torch.randn(T, 16, device=cuda, generator=g).to(torch.bfloat16)
        lb = (torch.randn(out_f, 16, device=cuda, generator=g) * 0.05).to(torch.bfloat16)
        y = nf4.nf4_linear_fwd(x, packed, st, None, u, lb)
        yf = nf4.nf4_linear_fwd(x, packed, st, None, u, lb, path="fused")
        dy = torch.randn(T, out_f, device=cuda, generator=g).to(torch.bfloat16)
        dx = nf4.nf4_linear_dgrad(dy, packed, st)
        dxf = nf4.nf4_linear_dgrad(dy, packed, st, path="fused")
        device_error()
        _close(y, yf.float())
        _close(dx, dxf.float())
        _close(y, x.float() @ wd.t() + u.float() @ lb.float().t())
