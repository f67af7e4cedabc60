"""Shared test configuration.

Markers: `gpu` tests need a CUDA device (B200) and the built libm5b200.so;
everything else runs on CPU.  The repo root (oracle/) and the package
directory (m5kernels_b200/) are put on sys.path here.
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "m5-max-kernels_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and libm5b200.so")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return dict(np.load(ROOT / "tests" / "golden" / "reference_vectors.npz"))


@pytest.fixture(scope="session")
def rms_golden():
    import numpy as np

    return dict(np.load(ROOT / "tests" / "golden" / "rms_quant_vectors.npz"))
