"""torch.library.opcheck on every qlora_b200 custom operator with real CUDA inputs: the schema
(no undeclared mutation or aliasing), the registered autograd formula, the fake implementation
against the real outputs (shapes, dtypes, strides), and AOT dispatch with dynamic shapes. The
values of the ops are checked against the oracle by the parity tests, which reach them through
the package's public functions."""

import pytest
import torch

pytestmark = pytest.mark.gpu

BF = torch.bfloat16


def _inputs(name, dev):
    from hackathon_b200.nf4 import quantize_nf4
    g = torch.Generator(device=dev).manual_seed(11)

    def r(*s, dtype=BF, grad=False, scale=1.0):
        t = (torch.randn(*s, device=dev, generator=g) * scale).to(dtype)
        return t.requires_grad_(grad)

    if name.startswith("nf4"):
        packed, st = quantize_nf4(r(256, 512, scale=0.02))
        nf4 = (packed, st.absmax, st.state2.code, st.state2.absmax, float(st.offset), 64, 256)
        if name == "nf4_dequant":
            return nf4 + (256, 512, BF)
        if name == "nf4_linear":
            return (r(3, 40, 512, grad=True),) + nf4 + (256, 512, r(256))
        return (r(3, 40, 256),) + nf4 + (256, 512)
    if name == "rmsnorm":
        return (r(3, 5, 64, grad=True), r(64), 1e-6, BF)
    if name == "rmsnorm_bwd":
        x = r(3, 5, 64)
        rstd = torch.rsqrt(x.float().pow(2).mean(-1) + 1e-6).reshape(-1)
        return (r(3, 5, 64), x, r(64), rstd)
    if name == "rope":
        q = r(2, 16, 4, 128).transpose(1, 2).detach().requires_grad_()
        k = r(2, 16, 2, 128).transpose(1, 2).detach().requires_grad_()
        return (q, k, r(1, 16, 128), r(1, 16, 128), False, BF, BF)
    if name == "swiglu":
        return (r(8, 96, grad=True), r(8, 96, grad=True))
    if name == "swiglu_bwd":
        return (r(8, 96), r(8, 96), r(8, 96))
    if name == "dropout_scale":
        return (r(8, 96, grad=True), 0.1, 1234, 1 / 0.9, torch.float32)
    if name == "scaled_add":
        return (r(8, 96, grad=True), r(8, 96, dtype=torch.float32, grad=True), 2.0)
    if name == "gemm":
        return (r(64, 32, grad=True), r(48, 32, grad=True), torch.float32)
    if name == "linear_ce":
        t = torch.randint(0, 300, (10,), device=dev, generator=g)
        t[3] = -100
        return (r(10, 64, grad=True), r(300, 64, scale=0.05), t, 4, True)
    raise KeyError(name)


NAMES = ("nf4_dequant", "nf4_linear", "nf4_linear_dgrad", "rmsnorm", "rmsnorm_bwd", "rope",
         "swiglu", "swiglu_bwd", "dropout_scale", "scaled_add", "gemm", "linear_ce")


@pytest.mark.parametrize("name", NAMES)
def test_opcheck(cuda, name):
    import hackathon_b200.ops as qops
    assert set(NAMES) == set(qops.ops())
    op = getattr(torch.ops.qlora_b200, name)
    torch.library.opcheck(op.default, _inputs(name, cuda))
