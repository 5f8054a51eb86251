import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (a B200) and the built library")
    config.addinivalue_line("markers", "slow: takes more than a few seconds")


def golden(name):
    """The arrays of tests/golden/<name>.npz (written by tests/golden/make_golden.py from the
    reference's own kernels)."""
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as f:
        return {k: f[k] for k in f.files}


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA GPU")
    from hackathon_b200 import _lib

    _lib.load()  # fails loudly when the library is not built
    return torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _tensor_core_error_flag(request):
    """After every GPU test: reads (and clears) the tensor-core kernels' error flag, so a kernel
    that gave up a bounded wait fails the test it ran in, with the wait's site, instead of making
    every later tensor-core launch of the session bail out."""
    yield
    if "cuda" not in request.fixturenames:
        return
    import torch

    from hackathon_b200 import _lib

    lib = _lib.load()
    if lib.qb_device_error(_lib.stream(torch.device("cuda:0"))) != 0:
        pytest.fail("a tensor-core kernel gave up a bounded wait in this test: "
                    + lib.qb_last_error().decode(errors="replace"))
