"""The allocation-free double-quant entry point, for callers that cannot call cudaMalloc (code
inside an allocator's hooks, plugin hosts that own all device memory). It must give exactly what
the workspace-taking entry point gives, call after call, through the C-ABI.

This file is collected last on purpose: a run that stops at the first failure has run every
other test before this one."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(n_blocks, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    return torch.rand(n_blocks, device=dev, generator=g) * 0.05 + 0.001


def _with_workspace(lib, absmax, code2, bs2):
    from hackathon_b200 import _lib
    n = absmax.numel()
    q = torch.empty(n, dtype=torch.uint8, device=absmax.device)
    a2 = torch.empty((n + bs2 - 1) // bs2, dtype=torch.float32, device=absmax.device)
    off = torch.empty(1, dtype=torch.float32, device=absmax.device)
    ws = torch.empty(int(lib.qb_nf4_double_quant_workspace(n)), dtype=torch.uint8,
                     device=absmax.device)
    _lib.call("qb_nf4_double_quant", absmax.data_ptr(), n, bs2, code2.data_ptr(), q.data_ptr(),
              a2.data_ptr(), off.data_ptr(), ws.data_ptr(), _lib.stream(absmax.device))
    return q, a2, off


def _without_allocation(absmax, code2, bs2):
    from hackathon_b200 import _lib
    n = absmax.numel()
    q = torch.empty(n, dtype=torch.uint8, device=absmax.device)
    a2 = torch.empty((n + bs2 - 1) // bs2, dtype=torch.float32, device=absmax.device)
    off = torch.empty(1, dtype=torch.float32, device=absmax.device)
    _lib.call("qb_nf4_double_quant_noalloc", absmax.data_ptr(), n, bs2, code2.data_ptr(),
              q.data_ptr(), a2.data_ptr(), off.data_ptr(), _lib.stream(absmax.device))
    return q, a2, off


def test_noalloc_double_quant_matches_workspace_entry_point(cuda):
    from hackathon_b200 import _lib
    from hackathon_b200.nf4 import signed_dynamic_code
    lib = _lib.load()
    code2 = signed_dynamic_code().to(cuda)
    # two calls in a row with different inputs and sizes: the shared scratch keeps the last
    # call's contents, which must not leak into the next result
    for seed, n_blocks in ((0, 1_060_864), (1, 200_003)):
        absmax = _inputs(n_blocks, seed, cuda)
        want = _with_workspace(lib, absmax, code2, 256)
        got = _without_allocation(absmax, code2, 256)
        torch.cuda.synchronize()
        assert torch.equal(got[0], want[0]), seed          # codes: bit for bit
        assert torch.equal(got[1], want[1]), seed          # second-level scales
        assert torch.equal(got[2], want[2]), seed          # offset (mean)


def test_noalloc_double_quant_rejects_sizes_over_its_limit(cuda):
    from hackathon_b200 import _lib
    lib = _lib.load()
    limit = int(lib.qb_nf4_double_quant_noalloc_max_blocks())
    assert limit == 512 * 4096
    with pytest.raises(RuntimeError, match="static scratch limit"):
        _lib.call("qb_nf4_double_quant_noalloc", 1, limit + 1, 256, 1, 1, 1, 1, None)
