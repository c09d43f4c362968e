"""Shared pytest set-up: the ``gpu`` marker and import paths.

The product package ``tjkernels`` lives in ``tiktok-techjam-2026_b200/``;
the test-only oracle lives in ``oracle/`` at the repository root.
"""

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "tiktok-techjam-2026_b200"
for p in (str(ROOT), str(PKG_DIR)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line(
        "markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


import pytest  # noqa: E402


@pytest.fixture(autouse=True)
def _no_device_timeout(request):
    """After every GPU test: no kernel recorded a bounded-wait timeout.  The
    status word is sticky, so a wait that ran out inside a test whose outputs
    still happened to compare equal is caught at that test, not later."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch

    if not torch.cuda.is_available():
        return
    from tjkernels import kernels as K

    status = K.device_status(clear=True)
    assert status == 0, f"a kernel hit a bounded-wait timeout (device status {status})"
