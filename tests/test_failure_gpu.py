"""The tensor-core kernels' failure path, exercised without a GPU fault: a wait that nothing
satisfies gives up after its limit, raises the device error flag, and the host reads
QB_ERR_TIMEOUT through qb_device_error; the flag is cleared and the context keeps working. The
launch monitor (pinned host memory the kernels write) names the site of the wait that gave up
and shows every traced launch finished, read with no CUDA call."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_context_survives(cuda):
    from hackathon_b200 import _lib
    from hackathon_b200.gemm import device_error, gemm
    lib = _lib.load()
    s = _lib.stream(cuda)
    assert lib.qb_device_error(s) == 0                      # nothing pending
    assert lib.qb_selftest_bounded_wait(20_000_000, s) == 0   # 20 ms wait, launched
    torch.cuda.synchronize()
    buf = ctypes.create_string_buffer(1024)
    assert lib.qb_monitor_report(cuda.index or 0, buf, len(buf)) == 0
    report = buf.value.decode()
    assert "last wait that gave up: site 99" in report, report
    assert "no CTA of these launches is running" in report, report
    assert lib.qb_device_error(s) == 4                      # QB_ERR_TIMEOUT
    assert b"site 99" in lib.qb_last_error()
    assert lib.qb_device_error(s) == 0                      # read-and-clear
    with pytest.raises(RuntimeError, match="bounded wait"):   # the Python surface raises
        lib.qb_selftest_bounded_wait(20_000_000, s)
        device_error()
    # the context still runs tensor-core work correctly
    a = torch.randn(256, 128, device=cuda).to(torch.bfloat16)
    b = torch.randn(384, 128, device=cuda).to(torch.bfloat16)
    out = gemm(a, b, out_dtype=torch.float32)
    device_error()
    torch.testing.assert_close(out, a.float() @ b.float().t(), rtol=1e-3, atol=1e-3)
    # ... and the monitor saw that GEMM's CTAs start and finish
    assert lib.qb_monitor_report(cuda.index or 0, buf, len(buf)) == 0
    report = buf.value.decode()
    assert "(last gemm_bf16)" in report and "no CTA of these launches is running" in report, \
        report
