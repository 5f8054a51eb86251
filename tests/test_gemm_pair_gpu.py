"""The 2-SM (cta_group::2) GEMM kernel, which the launcher takes for launches with a 256 x 256
tile for every SM pair: forced on (QB_GEMM_PAIR=1, read once per process, hence the child
process) for small and ragged shapes too, with both B layouts, the LoRA segment and the residual
epilogue, against fp32 products."""

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

CHILD = r"""
import torch
from hackathon_b200.gemm import device_error, gemm, gemm2
dev = torch.device("cuda")
g = torch.Generator(device=dev).manual_seed(0)
def r(*s):
    return torch.randn(*s, device=dev, generator=g).to(torch.bfloat16)
for M, N, K in [(512, 512, 256), (300, 700, 200), (1024, 3584, 512)]:
    a, b = r(M, K), r(N, K)
    out = gemm(a, b, out_dtype=torch.float32)
    device_error()
    torch.testing.assert_close(out, a.float() @ b.float().t(), rtol=1e-3, atol=1e-3)
    bt = r(K, (N + 7) // 8 * 8)[:, :N].t()            # MN-major B, 16-byte rows
    out = gemm(a, bt, out_dtype=torch.float32)
    device_error()
    torch.testing.assert_close(out, a.float() @ bt.float().t(), rtol=1e-3, atol=1e-3)
    u, sb, res = r(M, 64), r(N, 64), r(M, N)
    out = gemm2(a, b, u, sb, residual=res)
    device_error()
    ref = res.float() + a.float() @ b.float().t() + u.float() @ sb.float().t()
    torch.testing.assert_close(out.float(), ref, rtol=1.6e-2, atol=5e-2)
print("pair ok")
"""


def test_pair_kernel_in_child_process():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, QB_GEMM_PAIR="1", PYTHONPATH=root)
    res = subprocess.run([sys.executable, "-c", CHILD], env=env, cwd=root, capture_output=True,
                         text=True, timeout=600)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    assert "pair ok" in res.stdout
