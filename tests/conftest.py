from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden" / "shift_golden.npz"
# the reference's own package, installed (not committed) by baseline/install_ref.py
REFERENCE_INSTALL = ROOT / "baseline" / "_ref"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built library")


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA (run with -m 'not gpu')")
    from marathon_b200 import _lib

    _lib.load()  # the native library must be there; no fallback
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def reference_pkg():
    """The reference's unmodified ``marathon`` package (for its gap-fill channel and planner).

    It is installed into ``baseline/_ref`` by ``baseline/install_ref.py``; the
    tests that need it skip, saying so, when it is not there.
    """
    if not (REFERENCE_INSTALL / "marathon" / "__init__.py").is_file():
        pytest.skip("the reference package is not installed: run "
                    "`python baseline/install_ref.py <reference checkout>`")
    if str(REFERENCE_INSTALL) not in sys.path:
        sys.path.insert(0, str(REFERENCE_INSTALL))
    import marathon

    return marathon
