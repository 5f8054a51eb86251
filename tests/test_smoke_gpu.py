"""The entry point's smoke() on the GPU: the round trip a reviewer's first run makes (every
kernel family once against its CPU check, then one training step of the flagship model)."""

import pytest

pytestmark = pytest.mark.gpu


def test_graft_entry_smoke(cuda):
    import __graft_entry__ as entry
    entry.smoke()
