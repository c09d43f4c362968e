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
